/*
 * include/tb_gguf_dequant.h — C ABI of libtb_cuda_sm100.so, the B200 (sm_100a)
 * GGUF K-quant dequant x fp32 matrix-vector library.
 *
 * Part 1 is a drop-in for Trailblaze's layer4/tb_gguf_dequant.h:19-43: the
 * same eight symbols with the same argument meaning, return codes and
 * ownership, so layer4/tb_gguf.c and layer4/tb_infer.c built with -DTB_CUDA
 * link against this library unchanged.  Part 2 adds stream-ordered
 * device-pointer entry points that have no reference counterpart.  Part 3
 * is the batch-1 decode step built on the matvec (a GPU form of
 * layer4/tb_infer.c's tb_infer_decode).
 *
 * Conventions (shared with the reference):
 *   - int returns are 1 = success, 0 = failure (the caller may fall back);
 *     pointer returns are NULL on failure.  Nothing in the library aborts.
 *   - qtype ids are ggml's: 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 10 Q2_K, 11 Q3_K,
 *     12 Q4_K, 13 Q5_K, 14 Q6_K, 15 Q8_K, 21 IQ3_S (decoded as Q3_K, as the
 *     reference does), 30 BF16.
 *   - W is M rows of K weights, each row exactly K/block_weights blocks of
 *     raw GGUF bytes, rows contiguous.  K must be a multiple of the
 *     block size (256 for K-quants, 32 for Q4_0/Q8_0, 1 for F32/F16/BF16);
 *     other K are rejected with 0 (the reference truncates silently).
 *   - Results: y[m] = sum_k dequant(W)[m,k] * x[k] with fp32 x, fp32
 *     products and fp32 accumulation (the default; tb_cuda_set_matvec_arith
 *     selects an opt-in narrower integer form); dequantisation follows the
 *     reference CUDA kernels bit for bit (tb_gguf_dequant.cu:89-332), and
 *     Q2_K follows tb_gguf.c:210-225.
 *   - The library computes on the GPU only.  There is no CPU fallback inside
 *     it: the caller's own fallback (tb_gguf.c:449-451) stays where it is.
 */
#ifndef TB_GGUF_DEQUANT_B200_H
#define TB_GGUF_DEQUANT_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ───────────── Part 1: the reference ABI (tb_gguf_dequant.h:19-43) ───────── */

/* Replaces tb_gguf_dequant.h:19 / tb_gguf_dequant.cu:388-400.  Binds the
 * calling thread's current CUDA device (device 0 unless the host selected
 * another), creates the library stream and staging buffers.  1 = ok. */
int   tb_cuda_init(void);

/* Replaces tb_gguf_dequant.h:22 / .cu:411-416.  Allocates byte_count bytes of
 * HBM and copies host_data into it synchronously; the host keeps ownership of
 * host_data.  Returns the device pointer or NULL. */
void *tb_cuda_upload_tensor(const void *host_data, size_t byte_count);

/* Replaces tb_gguf_dequant.h:23 / .cu:418.  NULL-safe. */
void  tb_cuda_free_tensor(void *d_ptr);

/* Replaces tb_gguf_dequant.h:27 / .cu:403-409.  Copies x into the library's
 * device-resident activation buffer.  A following tb_cuda_matvec_device call
 * with x_host == NULL uses it, so one upload serves every matvec of a step
 * (the reference declares this but never reads the buffer).  1 = ok. */
int   tb_cuda_upload_x(const float *x_host, int K);

/* Replaces tb_gguf_dequant.h:31 / .cu:420.  The argument is the reference's
 * `const TBOscSnapshot *` (a pointer, so the ABI is identical); it is accepted
 * and ignored.  Launch geometry never depends on it (the reference's
 * oscillator-driven grid skips rows, tb_gguf_dequant.cu:378-384). */
void  tb_cuda_set_snap(const void *snap);

/* Replaces tb_gguf_dequant.h:36-37 / .cu:422-472.  Blocking: copies x_host
 * (K floats; NULL = the buffer from tb_cuda_upload_x) to the device, runs the
 * matvec on W_device (device pointer, any byte alignment, e.g. an expert's
 * row offset into a packed tensor), and copies M floats into out_host.
 * 1 = out_host filled; 0 = unsupported qtype/shape or a CUDA error. */
int   tb_cuda_matvec_device(const void *W_device, int qtype, int M, int K,
                            const float *x_host, float *out_host);

/* Replaces tb_gguf_dequant.h:40 / .cu:474-476.  Waits for all library work. */
void  tb_cuda_sync_all(void);

/* Replaces tb_gguf_dequant.h:43 / .cu:478-486.  Frees staging buffers and the
 * stream; safe to call twice; tb_cuda_init may be called again afterwards. */
void  tb_cuda_cleanup(void);

/* ───────────── Part 2: additive entry points (no reference counterpart) ─── */

/* Stream-ordered matvec on device pointers: d_y[M] = dequant(W_dev) @ d_x[K].
 * No host synchronisation; `stream` is a cudaStream_t (NULL = legacy default
 * stream).  Returns 1 if the launch was issued, 0 on bad arguments or a launch
 * error.  Device-side failures (a bounded wait that ran out) are reported by
 * tb_cuda_last_error().  The tb_gguf_tensor_matvec call site
 * (tb_gguf.c:444-451) and the MoE expert call sites (tb_infer.c:810-816) map
 * onto this with d_data (+ a byte offset) as W_dev. */
int   tb_cuda_matvec_dev(const void *W_dev, int qtype, int M, int K,
                         const float *d_x, float *d_y, void *stream);

/* The matvec with the decode step's neighbours fused in (no reference
 * counterpart; the unfused ops are layer1/tb_tensor.c:194-199 tb_rms_norm,
 * layer4/tb_infer.c:130-135 tb_swiglu and the residual adds of
 * tb_infer.c:731, 876).  The input is transformed on the fly:
 *   xmode 0: x                      (d_x2, d_norm_w unused)
 *   xmode 1: x[k] * rms * d_norm_w[k], rms = 1/sqrt(sum(x^2)/K + eps)
 *   xmode 2: silu(x[k]) * d_x2[k],  silu(g) = g / (1 + e^-g)
 * and the output:
 *   ymode 0: y[m] = (dequant(W) @ x')[m] + d_res[m] (d_res may be NULL)
 *   ymode 1: W's rows are (gate, up) pairs and y[i] = silu(row 2i . x') *
 *            (row 2i+1 . x'), M/2 outputs (M even, d_res must be NULL)
 * d_res may be d_y only if nothing else reads d_y meanwhile.  Stream-ordered
 * like tb_cuda_matvec_dev.  1 = issued. */
int   tb_cuda_matvec_fused_dev(const void *W_dev, int qtype, int M, int K,
                               const float *d_x, float *d_y, int xmode, const float *d_x2,
                               const float *d_norm_w, float eps, const float *d_res,
                               int ymode, void *stream);

/* Expert matvecs on a packed expert tensor (the MoE call sites of
 * layer4/tb_infer.c:797-816, which run one tb_gguf_dequant_matvec per selected
 * expert on a row offset of blk.N.ffn_*_exps), all selected experts in one
 * launch.  W_dev is n_experts matrices of M x K, back to back.  For
 * g < n_sel, expert e = d_ids[g] (device memory, read by the kernel, so a
 * router kernel earlier in the stream may write it; d_ids NULL: e = g):
 *   d_y[g * y_stride + m] = (dequant(W_e) @ d_x[g * x_stride ...])[m]
 * x_stride = 0 shares one x.  ymode 1 applies SwiGLU to (gate, up) row pairs
 * as in tb_cuda_matvec_fused_dev (M/2 outputs per expert).  An id outside
 * [0, n_experts) skips its expert and sets the error word (2).
 * Stream-ordered.  1 = issued. */
int   tb_cuda_matvec_experts_dev(const void *W_dev, int qtype, int M, int K, int n_experts,
                                 const int *d_ids, int n_sel, const float *d_x, int x_stride,
                                 float *d_y, int y_stride, int ymode, void *stream);

/* Sampling of one logits vector on the device (replaces layer1/tb_tensor.c:
 * 411-540 tb_sample_top_k / tb_sample_top_p for a caller whose logits are in
 * device memory).  u in [0, 1) is the uniform variate the reference draws with
 * rand() / (RAND_MAX + 1.0f).  top_k > 0: top-k at temperature (k >= vocab:
 * nucleus with p = 0.95, as the reference); top_k = 0: nucleus sampling with
 * top_p in (0, 1].  Writes the chosen index to *d_token; stream-ordered.
 * top_k <= 2048 (when < vocab).  Non-finite logits set the error word (2)
 * and write 0.  A small top_k (at most 256, at least 8 slices of 4 k logits)
 * runs in two launches through a candidate buffer the library allocates on
 * the first top-k call and shares between calls: calls that overlap on the
 * GPU (different streams) must not both use it.  1 = issued. */
int   tb_cuda_sample_dev(const float *d_logits, int vocab, int top_k, float top_p, float temperature,
                         float u, int *d_token, void *stream);

/* Bit-exact dequantisation of M rows of K weights into d_out[M*K] (fp32),
 * stream-ordered.  sem = 0 gives the reference CUDA-kernel semantics (the
 * parity contract); sem = 1 gives layer4/tb_gguf.c's shipped decoders, which
 * differ for Q4_K (tb_gguf.c:163-168) and Q5_K (tb_gguf.c:139).  1 = issued. */
int   tb_cuda_dequant_dev(const void *W_dev, int qtype, int M, int K,
                          float *d_out, int sem, void *stream);

/* Block geometry of a qtype: weights and bytes per block.  1 = known qtype. */
int   tb_cuda_qtype_info(int qtype, int *block_weights, int *block_bytes);

/* Synchronises the device, then returns and clears the library's device error
 * word: 0 = none, 1 = a pipeline wait ran out of its iteration limit,
 * 2 = a CUDA runtime error was seen by a blocking call. */
int   tb_cuda_last_error(void);

/* Number of matvec / dequant kernel launches the library has issued since
 * load (a host-side counter, for launch accounting in benchmarks). */
unsigned long long tb_cuda_launch_count(void);

/* Library build identifier, e.g. "tb_cuda_sm100 1.1 sm_100a". */
const char *tb_cuda_version(void);

/* Activation arithmetic of the quantized matvecs (every qtype except F32, F16
 * and BF16, which always compute in fp32), for all later launches of the
 * process, the decode step's included (a decoder keeps the kernels its CUDA
 * graph was captured with):
 *   TB_MATVEC_ARITH_FP32 (0, the default): x stays fp32 and every product and
 *     sum is an fp32 operation, as in the reference's kernels
 *     (tb_gguf_dequant.cu:113-114).  Scales are factored out of each
 *     sub-block's sum, and x is prescaled by exact powers of two, so the
 *     result differs from the reference's only by fp32 rounding order.
 *   TB_MATVEC_ARITH_INT16 (1, opt-in): x is rounded to a 16-bit integer at a
 *     power-of-two scale shared by 128 consecutive activations (the exponent
 *     of their largest |x|), then products and sums are exact integer dp4a.
 *     Narrower than the reference's fp32 x: an activation 2^15 times smaller
 *     than the largest of its 128-slot rounds to zero.
 * Returns the previous mode, or -1 for an unknown mode (nothing changes).
 * Host-only: it launches nothing and needs no device. */
#define TB_MATVEC_ARITH_FP32  0
#define TB_MATVEC_ARITH_INT16 1
int   tb_cuda_set_matvec_arith(int mode);
/* The current mode (TB_MATVEC_ARITH_*). */
int   tb_cuda_get_matvec_arith(void);

/* No counterpart in the reference.  Blocking matvec like tb_cuda_matvec_device
 * (x_host must not be NULL), but it allocates nothing, not even on first use:
 * x, y and the device error word live in static device buffers of fixed size
 * (K <= 65536 floats of x, M <= 262144 floats of y), whose addresses are looked
 * up once per device.  Larger M or K are rejected with 0.  It runs on the
 * legacy default stream and copies straight from / to the caller's buffers.
 * The buffers are shared by every call on a device, so overlapping calls race:
 * this library serialises its own callers with its lock, and a caller must not
 * run two of these at once by any other route (e.g. two processes sharing a
 * context).  1 = out_host filled; 0 = bad arguments, oversize, or an error. */
int   tb_cuda_matvec_device_noalloc(const void *W_device, int qtype, int M, int K,
                                    const float *x_host, float *out_host);

/* Model upload into one device arena (replaces the per-tensor cudaMalloc and
 * synchronous pageable copy of layer4/tb_gguf.c:469-520 tb_gguf_cuda_upload_all
 * / tb_gguf_dequant.cu:411-416 tb_cuda_upload_tensor).  tb_cuda_arena_create
 * makes one device allocation of `bytes` on the current device; each upload
 * reserves the next 256-byte aligned range and copies the host bytes into it
 * unchanged, in 32 MB chunks through two pinned staging buffers so the host
 * copy of one chunk overlaps the DMA of the previous one.  Blocking; returns
 * the device pointer, NULL when the arena is full or a copy fails.  Any qtype
 * (Q2_K, F32, BF16 included): the bytes are not interpreted.
 *   _rows: rows [r_lo, r_hi) of a tensor of row_bytes-byte rows (a
 *          tensor-parallel rank's q/k/v heads, FFN row pairs or vocabulary);
 *   _cols: bytes [b_lo, b_hi) of each of the M rows, packed (a K slice on
 *          block boundaries: a rank's o / ffn_down columns), so a rank never
 *          holds the whole tensor on its device.
 * Thread-safe per arena; destroy frees everything the arena holds. */
void  *tb_cuda_arena_create(size_t bytes);
void  *tb_cuda_arena_upload(void *arena, const void *host, size_t n);
void  *tb_cuda_arena_upload_rows(void *arena, const void *host, size_t row_bytes, int r_lo, int r_hi);
void  *tb_cuda_arena_upload_cols(void *arena, const void *host, int M, size_t row_bytes, size_t b_lo,
                                 size_t b_hi);
size_t tb_cuda_arena_used(void *arena);
void   tb_cuda_arena_destroy(void *arena);

/* Prefill GEMM on the tensor cores (tcgen05, bf16 x bf16 -> fp32):
 * C_dev[T][N] = A_bf16_dev[T][K] x dequant(W_dev)[N][K]^T, row t of C being
 * the matvec of W with token t (the batched form of the reference's
 * token-by-token prefill, layer4/tb_infer.c:1071-1074).  The weights are
 * dequantised exactly (as tb_cuda_dequant_dev) and rounded to bf16 on the way
 * into shared memory.  qtype Q4_K or Q6_K; N a multiple of 128, K of 256;
 * T a multiple of 16 in [16, 512]; A and W 16-byte aligned and W's rows a
 * multiple of 16 bytes (always for Q4_K; K a multiple of 2048 for Q6_K).
 * Stream-ordered, no host synchronisation.  1 = launched, 0 = unsupported. */
int tb_cuda_qgemm_dev(const void *W_dev, int qtype, int N, int K, const void *A_bf16_dev, int T, float *C_dev,
                      void *stream);

/* ───────────── Part 3: the decode step (no reference counterpart) ────────────
 *
 * The GPU form of layer4/tb_infer.c:889-1050 tb_infer_decode for a dense
 * Qwen3-style model, built on the matvec.  Per token: embedding row; per layer
 * RMSNorm + QKV matvec, per-head QK-norm + RoPE + KV-cache append + attention
 * (layer1/tb_tensor.c:303-409), output projection + residual, RMSNorm +
 * gate/up matvec, SwiGLU + down matvec + residual; final RMSNorm + output
 * matvec; greedy argmax (tb_tensor.c:415-420).  One CUDA graph per token,
 * token and position kept on the device.
 *
 * quirks = 1 follows tb_layer_forward's order: RoPE before the per-head
 * QK-norm, and each K head rotated n_heads/n_kv_heads times
 * (tb_infer.c:665); quirks = 0 is the Qwen3 order (norm, then one rotation).
 * head_dim must be 128 and n_heads/n_kv_heads at most 8. */
typedef struct {
    int   n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_ctx;
    float rope_base, norm_eps;
    int   quirks;
} tb_dec_config;

/* One layer's device tensors.  w_qkv is the fused projection (rows: the
 * n_heads*head_dim q rows, then n_kv_heads*head_dim k rows, then v rows; the
 * reference's blk.N.attn_qkv layout, tb_infer.c:640-649); w_gate_up holds
 * the gate and up rows interleaved (row 2i = gate row i, row 2i+1 = up row i),
 * so that one matvec also applies SwiGLU.  Norm weights are fp32
 * device vectors; q_norm / k_norm may be NULL (no QK-norm).  The decoder keeps
 * the pointers; the caller keeps ownership. */
typedef struct {
    const void  *w_qkv;     int qkv_qtype;
    const void  *w_o;       int o_qtype;
    const void  *w_gate_up; int gate_up_qtype;
    const void  *w_down;    int down_qtype;
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
} tb_dec_layer;

/* Creates a decoder on the current device: the fp32 KV cache
 * (n_layers x n_kv_heads x max_ctx x head_dim, zeroed) and scratch vectors.
 * NULL on unsupported shapes or allocation failure. */
void  *tb_cuda_dec_create(const tb_dec_config *cfg);
int    tb_cuda_dec_set_layer(void *dec, int layer, const tb_dec_layer *w);
int    tb_cuda_dec_set_head(void *dec, const void *tok_embd, int embd_qtype, const float *out_norm,
                            const void *w_out, int out_qtype);
/* Device pointer of a layer's K (which = 0) or V (which = 1) cache,
 * [n_kv_heads][max_ctx][head_dim] fp32, e.g. to load a prefix. */
float *tb_cuda_dec_kv(void *dec, int layer, int which);
/* Copies positions [p0, p0 + n) of a layer's K (which = 0) or V (1) cache in
 * (to_device = 1, e.g. a prefix) or out (0); the other side, `host`, is
 * [n_kv_heads][n][head_dim] fp32 in host or device memory.  Blocking; the copy
 * runs on the decoder's own (non-blocking) stream, so device memory written
 * by work on another stream must be complete before the call.  1 = ok. */
int    tb_cuda_dec_kv_copy(void *dec, int layer, int which, int p0, int n, float *host, int to_device);
/* Batched prefill of a prompt (the reference prefills by one decode step per
 * prompt token, layer4/tb_infer.c:1071-1074): tokens[0..n) at positions
 * pos0 .. pos0 + n - 1 go through every layer together, in chunks of up to 512,
 * filling the K and V cache; the projections run on the tcgen05 GEMM
 * (tb_cuda_qgemm_dev: bf16 activations, weights dequantised exactly and
 * rounded to bf16), attention, norms and the residual stream in fp32.  Then
 * the last token's final norm, output matvec and greedy argmax:
 * *next_token, logits_host (may be NULL) its vocab logits; decoding continues
 * with tb_cuda_dec_generate(*next_token, pos0 + n, ...).  Dense single-device
 * decoder; every projection Q4_K or Q6_K with rows a multiple of 128, K of
 * 256 and row bytes of 16 (Q6_K: K a multiple of 2048).  Blocking.  1 = ok. */
int    tb_cuda_dec_prefill(void *dec, const int *tokens, int n, int pos0, int *next_token, float *logits_host);
/* One token at position pos: *next_token = greedy argmax; logits_host (may be
 * NULL) receives the vocab logits.  Blocking.  1 = ok. */
int    tb_cuda_dec_step(void *dec, int token, int pos, int *next_token, float *logits_host);
/* n tokens back to back from (token, pos), each step fed the previous argmax;
 * tokens_out (may be NULL) receives them, logits_host (may be NULL) the last
 * step's logits, device_ms (may be NULL) the device time of the n steps. */
int    tb_cuda_dec_generate(void *dec, int token, int pos, int n, int *tokens_out, float *logits_host,
                            float *device_ms);
/* Sampling instead of the greedy argmax (the choice of layer4/tb_infer.c:
 * 1031-1038): temperature < 0.01 greedy (the default); else top_k > 0 the
 * top-k sampler, top_k = 0 the nucleus of top_p (tb_cuda_sample_dev's rules,
 * inside the step's graph).  Under tensor or expert parallelism every rank
 * gathers the whole vocabulary's logits from the others over NVLink and
 * samples them with the same variate, so all ranks take the same token (each
 * rank must pass the same variates).  1 = ok. */
int    tb_cuda_dec_set_sampling(void *dec, float temperature, int top_k, float top_p);
/* tb_cuda_dec_generate with the variates: step i samples with u[i] in [0, 1)
 * (the reference's rand() / (RAND_MAX + 1.0f)).  Required while sampling is
 * set (tb_cuda_dec_step / _generate then fail); u is ignored when greedy. */
int    tb_cuda_dec_generate_u(void *dec, int token, int pos, int n, const float *u, int *tokens_out,
                              float *logits_host, float *device_ms);
/* Copies n floats of one of the last step's activation vectors to host:
 * which = 0 the hidden state after the last layer (hidden), 1 the state after
 * the last layer's attention block (hidden), 2 the last layer's q | k | v
 * before QK-norm and RoPE ((n_heads + 2 n_kv_heads) head_dim), 3 its attention
 * output (n_heads head_dim), 4 its SwiGLU activation (ffn_dim), 5 the logits
 * (vocab); for a routed decoder 6 the last layer's router logits (n_experts),
 * 7 its expert weights and 8 its expert ids (top_k; int32 bits in the float
 * slots), rank order, 9 the selected experts' SwiGLU activations (top_k x
 * ffn_dim, rank order; under expert parallelism this rank's selected experts,
 * local order), 10 the number of this rank's selected experts and 11 their
 * local indices (expert parallelism only; int32 bits).  Blocking.  1 = ok, 0
 * for an unknown vector, one this decoder does not have, or n past its size. */
int    tb_cuda_dec_read(void *dec, int which, float *host, int n);

/* Tensor parallelism over `world` GPUs (2, 4 or 8; one process per GPU), the
 * sharding of Megatron-style decode: rank r holds
 *   w_qkv      rows of its q heads [r NH/w, (r+1) NH/w), then of its k heads and
 *              its v heads (the same split of n_kv_heads), H columns;
 *   w_o        all H rows, the K columns of its q heads (K = NH/w * head_dim);
 *   w_gate_up  its FFN row pairs [r F/w, (r+1) F/w), interleaved gate_i, up_i;
 *   w_down     all H rows, the K columns [r F/w, (r+1) F/w);
 *   w_out      its vocabulary rows [r V/w, (r+1) V/w); tok_embd is whole;
 *   the norm weights whole.
 * The ranks exchange the o and down partials and the greedy pairs over NVLink
 * through peer stores into each other's exchange region (mapped with CUDA IPC;
 * no collective library).  Every rank must run the same steps: a rank that
 * stops makes the others' bounded waits run out (their call returns 0).
 * tb_cuda_dec_step / _generate return the same token on every rank; logits and
 * tb_cuda_dec_read vectors are this rank's; the KV cache holds its kv heads. */
void  *tb_cuda_dec_create_tp(const tb_dec_config *c, int rank, int world);
/* The 64-byte CUDA IPC handle of this rank's exchange region.  1 = ok. */
int    tb_cuda_dec_tp_handle(void *dec, void *handle_out);
/* Maps the other ranks' regions; handles = world x 64 bytes in rank order (as
 * gathered from every rank's tb_cuda_dec_tp_handle).  1 = ok. */
int    tb_cuda_dec_tp_connect(void *dec, const void *handles);

/* Mixture-of-experts decoder (replaces the routed FFN of layer4/tb_infer.c:
 * 753-850 and the router of tb_infer.c:351-374).  cfg->ffn_dim is the expert
 * FFN width F; every layer routes rmsnorm(x2) through its router to the top_k
 * of n_experts (<= 256) experts, weights = softmax renormalised over the
 * selected ones, x = x2 + sum of weight * expert SwiGLU FFN.  The experts are
 * ranked by probability, equal probabilities by lower index (the reference's
 * replace-the-minimum scan picks the same set except among exactly equal
 * probabilities).  One device. */
void  *tb_cuda_dec_create_moe(const tb_dec_config *cfg, int n_experts, int top_k);
/* A routed layer's FFN tensors (its attention tensors and norms come from
 * tb_cuda_dec_set_layer, whose w_gate_up / w_down are then ignored):
 * w_router [n_experts][hidden] (blk.N.ffn_gate_inp); w_gate_up_exps
 * [n_experts][2F][hidden], expert e's gate and up rows interleaved (row 2i =
 * gate row i of blk.N.ffn_gate_exps, row 2i+1 = up row i of
 * blk.N.ffn_up_exps); w_down_exps [n_experts][hidden][F]
 * (blk.N.ffn_down_exps).  1 = ok. */
/* Expert parallelism over `world` GPUs (one process per GPU; n_experts a
 * multiple of world, top_k <= 32): rank r holds experts [r E/w, (r+1) E/w),
 * its tb_cuda_dec_set_moe_layer tensors being those experts' rows
 * ([E/w][2F][hidden] and [E/w][hidden][F]) and the router whole.  Attention,
 * the output and the exchange are those of tb_cuda_dec_create_tp (rank r's q
 * heads [r NH/w, (r+1) NH/w); when world is a multiple of n_kv_heads, kv head
 * r / (world / n_kv_heads), its K and V cache held by that many ranks).  Each
 * layer every rank computes the same router top k, runs its own selected
 * experts on the whole grid, and sends its weighted share of the FFN output
 * to every rank over NVLink (peer stores, like the down partials); the next
 * layer adds the world shares in rank order.  Connected with
 * tb_cuda_dec_tp_handle / _tp_connect.  NULL on unsupported shapes. */
void  *tb_cuda_dec_create_moe_tp(const tb_dec_config *cfg, int n_experts, int top_k, int rank, int world);
int    tb_cuda_dec_set_moe_layer(void *dec, int layer, const void *w_router, int router_qtype,
                                 const void *w_gate_up_exps, int gate_up_qtype, const void *w_down_exps,
                                 int down_qtype);
void   tb_cuda_dec_destroy(void *dec);

#ifdef __cplusplus
}
#endif
#endif /* TB_GGUF_DEQUANT_B200_H */
