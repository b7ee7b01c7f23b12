/*
 * oracle/tb_oracle.h — CPU restatement of Trailblaze's GGUF dequant semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs use it, and only as the checker.
 *
 * Semantics variants (see tb_oracle.c for the per-type citations):
 *   TBO_SEM_CUDA      the decode the reference's CUDA kernels compute
 *                     (layer4/tb_gguf_dequant.cu:89-332); for Q2_K, which has
 *                     no CUDA kernel there, layer4/tb_gguf.c:210-225.
 *                     This is the parity contract of the sm_100a library.
 *   TBO_SEM_GGUF_C    layer4/tb_gguf.c:109-371 as shipped (tb_gguf_dequant_row).
 *                     Differs from TBO_SEM_CUDA only for Q4_K (tb_gguf.c:163-168
 *                     scale unpack) and Q5_K (tb_gguf.c:139 min unpack, j >= 4).
 *   TBO_SEM_DISPATCH  src/tb_analog_dispatch.c scalar tier: Q4_K / Q3_K with the
 *                     CUDA scale unpack but d/dmin read as bf16
 *                     (tb_analog_dispatch.c:228-229, 266).  Used only to pin the
 *                     scale-unpack and nibble-order restatement against
 *                     tb_dot_q4k_scalar / tb_dot_q3k_scalar.
 *
 * Parity pinning: every TBO_SEM_GGUF_C decoder is checked bit for bit against
 * the reference's own tb_gguf_dequant_row (built from the reference sources
 * into oracle/_ref/), the TBO_SEM_DISPATCH decoders against the reference's
 * tb_dot_*_scalar, and the converters against tb_gguf.c's self-test
 * known-answer values (tb_gguf.c:995-1092).  See tests/test_oracle_pins.py.
 */
#ifndef TB_ORACLE_H
#define TB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { TBO_SEM_CUDA = 0, TBO_SEM_GGUF_C = 1, TBO_SEM_DISPATCH = 2 };

/* ggml qtype ids as used by the reference ABI (tb_gguf_dequant.cu:447-460). */
enum {
    TBO_F32 = 0, TBO_F16 = 1, TBO_Q4_0 = 2, TBO_Q8_0 = 8, TBO_Q2_K = 10,
    TBO_Q3_K = 11, TBO_Q4_K = 12, TBO_Q5_K = 13, TBO_Q6_K = 14, TBO_Q8_K = 15,
    TBO_IQ3_S = 21, TBO_BF16 = 30
};

/* Block geometry; returns 0 for an unknown qtype. */
int    tbo_qtype_geometry(int qtype, int *block_weights, int *block_bytes);
/* Bytes of one row of K weights (K a multiple of the block size), 0 on error. */
size_t tbo_row_bytes(int qtype, int K);

float  tbo_h2f(uint16_t h);   /* reference fp16 converter, subnormal quirk kept */
float  tbo_bf2f(uint16_t b);

/* Dequantise one block (block_weights floats).  Returns 1 on success. */
int tbo_dequant_block(int qtype, int sem, const uint8_t *blk, float *out);

/* Dequantise M rows of K weights into out[M*K].  Returns 1 on success. */
int tbo_dequant_rows(int qtype, int sem, const void *W, int M, int K, float *out);

/* y[m] = sum_k w[m,k]*x[k] with w from tbo_dequant_rows and fp64 accumulation. */
int tbo_matvec_f64(int qtype, int sem, const void *W, int M, int K,
                   const float *x, double *y);

/* Same product with the reference CPU loop's own arithmetic: fp32, sequential
 * `acc += w[k]*x[k]` with separate multiply and add (tb_gguf.c:411-417). */
int tbo_matvec_f32_seq(int qtype, int sem, const void *W, int M, int K,
                       const float *x, float *y);

#ifdef __cplusplus
}
#endif
#endif
