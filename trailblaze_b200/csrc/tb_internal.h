// tb_internal.h — declarations shared between the library's translation units.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

namespace tb {

// An NVTX range over a scope (a kernel family's host-side launch or a blocking
// call), named per family, e.g. "tb.matvec", "tb.decode.step"; free when no
// profiler is attached (NVTX3 is header-only and injected by the tool).
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};

// Fused transforms of the matvec's input and output (see tb_cuda_matvec_fused_dev).
enum MvXMode : uint32_t { MV_X_PLAIN = 0, MV_X_RMSNORM = 1, MV_X_SWIGLU = 2 };
// MV_Y_SWIGLU_PAIRS: rows come in (gate, up) pairs; y[i] = silu(row 2i) * row 2i+1 (M/2 outputs)
enum MvYMode : uint32_t { MV_Y_PLAIN = 0, MV_Y_SWIGLU_PAIRS = 1 };
static constexpr int kMaxRanks = 8;   // tensor-parallel ranks at most

struct MvFuse {
    uint32_t xmode = MV_X_PLAIN;
    uint32_t ymode = MV_Y_PLAIN;
    const float *x2 = nullptr;    // SwiGLU: the up vector
    const float *nw = nullptr;    // RMSNorm: the norm weights
    float eps = 0.f;              // RMSNorm epsilon
    const float *res = nullptr;   // added to y when not null
    bool w_early = false;         // W is constant over the launch chain: stream it before the
                                  // programmatic-dependency wait
    // Tensor-parallel exchange over peer memory (unused when nsl / ny are 0),
    // through tagged slots: a slot element is one 64-bit word (tag << 32 |
    // float bits), stored and loaded whole (single-copy atomic), so a reader
    // that sees the tag it expects also sees the value, with no fence or
    // arrival counter in between.  Tags are (epoch * mul + add) mod 2^32 with
    // the device-side step count epoch: unique per step and exchange.
    // Input: x <- x + the nsl rows of xs ([nsl][K] tagged words, summed in row
    // order), each word waited for (bounded) until it carries tag
    // (*xs_epoch) * xs_mul + xs_add; CTA 0 also writes that x to xout when
    // not null.  Output: y[row] goes to ys[p][row] for the ny ranks p instead
    // of y, tagged (*y_epoch) * y_mul + y_add.
    const unsigned long long *xs = nullptr;
    const int *xs_epoch = nullptr;
    unsigned long long xs_mul = 0, xs_add = 0;
    float *xout = nullptr;
    uint32_t nsl = 0, ny = 0;
    unsigned long long *ys[kMaxRanks] = {};
    const int *y_epoch = nullptr;
    unsigned long long y_mul = 0, y_add = 0;
    // Expert groups (MoE; unused when ng is 0): ng matvecs of M rows
    // each in one launch, group g on its own CTAs.  Group g reads the
    // matrix W + e * w_stride bytes, e = ids[g] read on the device after the
    // dependency wait (ids produced by the previous kernel; e = g when ids is
    // null; e >= n_experts sets the error word and skips the group), x + g *
    // x_stride floats (0: one shared x) and writes y + g * y_stride floats.
    uint32_t ng = 0, n_experts = 0;
    const int *ids = nullptr;
    // With ng_dev (device memory, written by the previous kernel; requires
    // ids): only the first min(*ng_dev, ng) groups run, the grid split evenly
    // among them.
    const int *ng_dev = nullptr;
    unsigned long long w_stride = 0;
    uint32_t x_stride = 0, y_stride = 0;
};

// Activation arithmetic of the quantized matvec decoders.  FP32: x stays fp32
// (exact power-of-two prescaling), fp32 products and sums, like the reference
// (tb_gguf_dequant.cu:113-114); the default.  INT16: x rounded to 16-bit
// integers at a per-128-weight power-of-two scale, exact integer products and
// sums (dp4a); opt-in, narrower than the reference's fp32 arithmetic.
enum MvArith : int { MV_ARITH_FP32 = 0, MV_ARITH_INT16 = 1 };
// Sets the mode for later launches; returns the previous one (-1: bad mode).
int mv_set_arith(int mode);
int mv_get_arith();

// Launch the matvec d_y[M] = dequant(W) @ d_x[K] on `st`.  Returns 1 when the
// launch was issued, 0 for unsupported arguments or a launch error.
int mv_launch(const void *W, int qtype, int M, int K, const float *d_x, float *d_y,
              cudaStream_t st, int *d_err, int num_sms, uint32_t wait_limit,
              const MvFuse *fuse = nullptr);

// Launch the prefill GEMM C[T][N] = A[T][K] (bf16) x dequant(W)[N][K]^T on the
// tensor cores (tb_qgemm.cu).  Returns 1 when launched, 0 for unsupported shapes.
int qg_launch(const void *W, int qtype, int N, int K, const void *A, int T, float *C, cudaStream_t st, int *d_err,
              int num_sms, uint32_t wait_limit);

// Launch the top-k / nucleus sampler of one logits vector (tb_sample.cu):
// *d_token = the chosen index for the uniform variate u in [0, 1).  top_k > 0:
// top-k (k >= vocab: nucleus with p = 0.95); top_k = 0: nucleus with top_p.
// With d_u (the decode graph): u = d_u[*d_u_idx], then *d_pos and *d_u_idx
// each advance by one.
// Tensor parallelism (the decode step's sampler on a rank): before reading the
// logits, wait (bounded) until *ctr >= (*epoch + 1) * per_step, the arrivals of
// every rank's logits slice; after the pick, *epoch += 1 (the step count).
struct SmpTP {
    const unsigned long long *ctr = nullptr;
    int *epoch = nullptr;
    unsigned long long per_step = 0;
    uint32_t wait_limit = 0;
};

// Device scratch of the two-stage top-k (kSmpPreCap candidates and a flag;
// the flag starts at 0 and every call leaves it at 0).  Without it, or when
// the top k is too large a share of the vocabulary, top-k runs in one CTA.
static constexpr int kSmpPreCap = 160 * 256;
struct SmpScratch {
    float *cv = nullptr;    // [kSmpPreCap] candidate logits
    int *ci = nullptr;      // [kSmpPreCap] their vocabulary indices
    int *nonfin = nullptr;  // set when a slice held a non-finite logit
};

int sample_launch(const float *d_logits, int vocab, int top_k, float top_p, float temperature, float u,
                  int *d_token, int *d_err, cudaStream_t st, const float *d_u = nullptr, int *d_u_idx = nullptr,
                  int *d_pos = nullptr, const SmpTP *tp = nullptr, const SmpScratch *scr = nullptr);

// Launch the bit-exact dequantisation of M rows of K weights into d_out.
int dq_launch(const void *W, int qtype, int M, int K, float *d_out, int sem, cudaStream_t st);

// Dequantise row d_token[i] of a [vocab x K] table into row i of d_out, for
// i < n (zeros for a token outside [0, vocab)); programmatic-dependent-launch
// aware.
int dq_embed_launch(const void *W, int qtype, int vocab, int K, const int *d_token, float *d_out,
                    cudaStream_t st, int n = 1);

// Batched prefill (tb_prefill.cu): one layer of T prompt tokens (padded to
// Tp, a multiple of 16), the projections on the tcgen05 GEMM.
struct PfLayer {
    const void *wqkv, *wo, *wgu, *wd;
    int qkv_qt, o_qt, gu_qt, d_qt;
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
    float *kc, *vc;   // the layer's K and V cache, [n_kv_heads][max_ctx][128]
};
struct PfShape {
    int hidden, n_heads, n_kv_heads, ffn_dim, max_ctx, quirks;
    float eps, rope_base;
};
struct PfBufs {   // [Tp] rows each
    float *X, *QKV, *Y, *GU;
    void *A, *AO, *ACT;   // bf16: [Tp][hidden], [Tp][n_heads * 128], [Tp][ffn_dim]
};
// True when the prefill GEMM takes an N x K tensor of this type.
bool pf_supported(int qtype, int N, int K);
// One layer over the chunk's rows of X (positions pos0 .. pos0 + T - 1);
// stream-ordered.  1 = launched.
int pf_layer(const PfLayer &w, const PfShape &c, const PfBufs &b, int pos0, int T, int Tp, cudaStream_t st,
             int *err, int sms);

// Shape of the decode step (tb_decode.cu); mirrors tb_dec_config.
struct DecConfig {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_ctx;
    float rope_base, norm_eps;
    int quirks;
};

// Raise a kernel's dynamic shared-memory limit once per device.
bool smem_attr_once(const void *kernel, int bytes);

}  // namespace tb
