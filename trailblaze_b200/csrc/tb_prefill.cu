// tb_prefill.cu — batched prefill of a prompt for the dense decode step.
//
// The reference's prefill is a token-by-token decode loop
// (layer4/tb_infer.c:1071-1074: one tb_infer_decode per prompt token).  Here
// the prompt's T tokens go through every layer together, chunks of up to 512:
//
//   X[t]      = embedding row of token t                (k_embed_row, batched)
//   A         = bf16(rmsnorm(X) * attn_norm)            k_pf_norm
//   QKV       = A . Wqkv^T                              tcgen05 GEMM (tb_qgemm.cu)
//   q, k      : RoPE and per-head QK-norm in the reference's order, k and v
//               appended to the cache at pos0 + t       k_pf_qk
//   AO[t]     = causal attention of token t over cache positions 0 .. pos0+t
//                                                       k_pf_attn (fp32, CUDA cores)
//   X        += bf16(AO) . Wo^T
//   A         = bf16(rmsnorm(X) * ffn_norm)             k_pf_norm (the residual add fused)
//   GU        = A . Wgu^T  (gate / up rows interleaved)
//   ACT       = bf16(silu(gate) * up)                   k_pf_swiglu
//   X        += ACT . Wd^T
//
// After the last layer the last token's row is the decode step's residual x,
// and the final norm, output matvec and greedy argmax of the decode step give
// the next token (tb_decode.cu).  The GEMMs take bf16 activations and round
// the exactly dequantised weights to bf16, so prefill
// logits differ from a token-by-token fp32 decode by that rounding; the
// attention, norms and residual stream are fp32.  Every kernel is launched
// stream-ordered on the decoder's stream; nothing here waits on the host.
#include <cuda_bf16.h>

#include <cstdio>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

static constexpr int kHDp = 128;   // head_dim of the decode step

__device__ __forceinline__ float block_sum256(float v, float *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w];   // warp order: the same sum in every thread
    __syncthreads();
    return s;
}

// Row t (one CTA, 256 threads): X[t] += R[t] when R (written back), then
// A[t] = bf16(X[t] * rms * w), rms = 1/sqrt(sum(X^2)/H + eps)
// (layer1/tb_tensor.c:194-199).  Rows t >= T are padding: A = 0.
__global__ void __launch_bounds__(256) k_pf_norm(float *X, const float *R, const float *w, float eps, int H, int T,
                                                 __nv_bfloat16 *A)
{
    __shared__ float red[8];
    const int t = blockIdx.x;
    __nv_bfloat16 *a = A + static_cast<size_t>(t) * H;
    if (t >= T) {
        for (int i = threadIdx.x; i < H; i += 256) a[i] = __float2bfloat16_rn(0.f);
        return;
    }
    float *x = X + static_cast<size_t>(t) * H;
    const float *r = R ? R + static_cast<size_t>(t) * H : nullptr;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += 256) {
        float v = x[i];
        if (r) {
            v += r[i];
            x[i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    const float sc = 1.0f / sqrtf(block_sum256(ss, red) / static_cast<float>(H) + eps);
    for (int i = threadIdx.x; i < H; i += 256) a[i] = __float2bfloat16_rn(x[i] * sc * w[i]);
}

// RoPE angle of pair i at position pos (layer4/tb_infer.c:143-145), as the
// decode step computes it.
__device__ __forceinline__ float2 pf_rope_cs(int pos, int i, float base)
{
    const float theta = static_cast<float>(pos) / powf(base, 2.0f * static_cast<float>(i) / static_cast<float>(kHDp));
    return make_float2(cosf(theta), sinf(theta));
}

// grid (T, NH + NK), 128 threads (one per dimension).  Head hh < NH: query
// head hh of token t, rotated and normed in place in QKV.  Otherwise kv head
// j = hh - NH: its k rotated (quirks: once per query head that maps to it)
// and normed, then k and v appended to the cache at position pos0 + t
// (layer4/tb_infer.c:665-710 in the reference's order when quirks, else
// norm then one rotation).
__global__ void __launch_bounds__(kHDp) k_pf_qk(float *QKV, int qkv_dim, const float *qn, const float *kn, float *kc,
                                                float *vc, int pos0, int NH, int NK, int max_ctx, float eps,
                                                float base, int quirks)
{
    __shared__ float s[kHDp];
    __shared__ float red[4];
    const int t = blockIdx.x, hh = blockIdx.y, d = threadIdx.x;
    const int pos = pos0 + t;
    const bool isq = hh < NH;
    float *row = QKV + static_cast<size_t>(t) * qkv_dim;
    float *v = row + (isq ? hh : NH + (hh - NH)) * kHDp;
    const float *nw = isq ? qn : kn;
    const int times = isq ? 1 : (quirks ? NH / NK : 1);
    s[d] = v[d];
    __syncthreads();
    auto rope = [&]() {
        if (d < kHDp / 2) {
            const float2 cs = pf_rope_cs(pos, d, base);
            for (int u = 0; u < times; ++u) {
                const float a0 = s[2 * d], b0 = s[2 * d + 1];
                s[2 * d] = a0 * cs.x - b0 * cs.y;
                s[2 * d + 1] = a0 * cs.y + b0 * cs.x;
            }
        }
        __syncthreads();
    };
    auto norm = [&]() {
        if (!nw) return;
        float ss = s[d] * s[d];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        if ((d & 31) == 0) red[d >> 5] = ss;
        __syncthreads();
        const float sc = 1.0f / sqrtf((red[0] + red[1] + red[2] + red[3]) / static_cast<float>(kHDp) + eps);
        s[d] = s[d] * sc * nw[d];
        __syncthreads();
    };
    if (quirks) {
        rope();
        norm();
    } else {
        norm();
        rope();
    }
    if (isq) {
        v[d] = s[d];
    } else {
        const int j = hh - NH;
        const size_t off = (static_cast<size_t>(j) * max_ctx + pos) * kHDp + d;
        kc[off] = s[d];
        vc[off] = row[(NH + NK + j) * kHDp + d];
    }
}

// Causal attention, one warp per (token t, query head h), query head h using
// kv head h / (NH / NK) (layer1/tb_tensor.c:303-409): scores q . k * 1/sqrt(HD)
// over cache positions 0 .. pos0 + t, softmax, p . v.  Scores of 32 positions
// at a time (lane = position, q read from shared memory), a running maximum and
// sum (online softmax), p . v with lane = 4 dimensions.  Output bf16 (the next
// GEMM's operand).
__global__ void __launch_bounds__(256) k_pf_attn(const float *QKV, int qkv_dim, const float *kc, const float *vc,
                                                 int pos0, int T, int NH, int NK, int max_ctx, float scale,
                                                 __nv_bfloat16 *out)
{
    __shared__ __align__(16) float qsh[8][kHDp];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * 8 + warp;
    if (item >= T * NH) return;
    const int t = item / NH, h = item % NH, j = h / (NH / NK);
    const float *q = QKV + static_cast<size_t>(t) * qkv_dim + h * kHDp;
    reinterpret_cast<float4 *>(qsh[warp])[lane] = reinterpret_cast<const float4 *>(q)[lane];
    __syncwarp();
    const float *K = kc + static_cast<size_t>(j) * max_ctx * kHDp;
    const float *V = vc + static_cast<size_t>(j) * max_ctx * kHDp;
    const int n = pos0 + t + 1;
    float m = -1e38f, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p0 = 0; p0 < n; p0 += 32) {
        const int p = p0 + lane;
        float sc = -1e38f;
        if (p < n) {
            const float4 *kr = reinterpret_cast<const float4 *>(K + static_cast<size_t>(p) * kHDp);
            const float4 *qs = reinterpret_cast<const float4 *>(qsh[warp]);
            float dsum = 0.f;
#pragma unroll 8
            for (int i = 0; i < kHDp / 4; ++i) {
                const float4 a = __ldg(kr + i), b = qs[i];
                dsum = fmaf(a.x, b.x, dsum);
                dsum = fmaf(a.y, b.y, dsum);
                dsum = fmaf(a.z, b.z, dsum);
                dsum = fmaf(a.w, b.w, dsum);
            }
            sc = dsum * scale;
        }
        float cm = sc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xFFFFFFFFu, cm, o));
        const float mn = fmaxf(m, cm);
        const float corr = expf(m - mn);
        const float pr = p < n ? expf(sc - mn) : 0.f;
        float ps = pr;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, o);
        l = l * corr + ps;
        acc.x *= corr;
        acc.y *= corr;
        acc.z *= corr;
        acc.w *= corr;
        const int cnt = min(32, n - p0);
        for (int u = 0; u < cnt; ++u) {
            const float pu = __shfl_sync(0xFFFFFFFFu, pr, u);
            const float4 vv = __ldg(reinterpret_cast<const float4 *>(V + static_cast<size_t>(p0 + u) * kHDp) + lane);
            acc.x = fmaf(pu, vv.x, acc.x);
            acc.y = fmaf(pu, vv.y, acc.y);
            acc.z = fmaf(pu, vv.z, acc.z);
            acc.w = fmaf(pu, vv.w, acc.w);
        }
        m = mn;
    }
    const float inv = 1.0f / l;
    __nv_bfloat16 *o = out + static_cast<size_t>(t) * NH * kHDp + h * kHDp + 4 * lane;
    o[0] = __float2bfloat16_rn(acc.x * inv);
    o[1] = __float2bfloat16_rn(acc.y * inv);
    o[2] = __float2bfloat16_rn(acc.z * inv);
    o[3] = __float2bfloat16_rn(acc.w * inv);
}

// ACT[t][i] = bf16(silu(GU[t][2i]) * GU[t][2i+1]) (layer4/tb_infer.c:130-135;
// gate / up rows interleaved in the weights, so in the GEMM's columns).  Rows
// t >= T are padding: 0.
__global__ void __launch_bounds__(256) k_pf_swiglu(const float *GU, int F, int T, __nv_bfloat16 *act)
{
    const int t = blockIdx.y;
    for (int i = blockIdx.x * 256 + threadIdx.x; i < F; i += gridDim.x * 256) {
        float v = 0.f;
        if (t < T) {
            const float g = GU[static_cast<size_t>(t) * 2 * F + 2 * i];
            const float u = GU[static_cast<size_t>(t) * 2 * F + 2 * i + 1];
            v = (g / (1.0f + expf(-g))) * u;
        }
        act[static_cast<size_t>(t) * F + i] = __float2bfloat16_rn(v);
    }
}

// X[t] += Y[t] for t < T (the down projection's residual; the o projection's
// is fused into the next k_pf_norm).
__global__ void __launch_bounds__(256) k_pf_add(float *X, const float *Y, int H, int T)
{
    const size_t n = static_cast<size_t>(T) * H;
    for (size_t i = blockIdx.x * 256ull + threadIdx.x; i < n; i += gridDim.x * 256ull) X[i] += Y[i];
}

bool pf_supported(int qtype, int N, int K)
{
    if (qtype != QT_Q4_K && qtype != QT_Q6_K) return false;
    const Geom g = geom_of(qtype);
    const unsigned long long rb = static_cast<unsigned long long>(K / g.block_weights) * g.block_bytes;
    return N % 128 == 0 && K % 256 == 0 && rb % 16 == 0;
}

int pf_layer(const PfLayer &w, const PfShape &c, const PfBufs &b, int pos0, int T, int Tp, cudaStream_t st,
             int *err, int sms)
{
    const int H = c.hidden, NH = c.n_heads, NK = c.n_kv_heads, F = c.ffn_dim;
    const int QKV = (NH + 2 * NK) * kHDp;
    const uint32_t lim = 1u << 22;
    __nv_bfloat16 *A = static_cast<__nv_bfloat16 *>(b.A), *AO = static_cast<__nv_bfloat16 *>(b.AO);
    __nv_bfloat16 *ACT = static_cast<__nv_bfloat16 *>(b.ACT);
    k_pf_norm<<<Tp, 256, 0, st>>>(b.X, nullptr, w.attn_norm, c.eps, H, T, A);
    if (!qg_launch(w.wqkv, w.qkv_qt, QKV, H, b.A, Tp, b.QKV, st, err, sms, lim)) return 0;
    k_pf_qk<<<dim3(T, NH + NK), kHDp, 0, st>>>(b.QKV, QKV, w.q_norm, w.k_norm, w.kc, w.vc, pos0, NH, NK, c.max_ctx,
                                              c.eps, c.rope_base, c.quirks);
    // k_pf_qk reads qkv rows written by the GEMM and rewrites q in place: the
    // attention below reads q of its own token only
    if (Tp > T) cudaMemsetAsync(AO + static_cast<size_t>(T) * NH * kHDp, 0,
                                sizeof(__nv_bfloat16) * static_cast<size_t>(Tp - T) * NH * kHDp, st);
    k_pf_attn<<<(T * NH + 7) / 8, 256, 0, st>>>(b.QKV, QKV, w.kc, w.vc, pos0, T, NH, NK, c.max_ctx,
                                               1.0f / sqrtf(static_cast<float>(kHDp)), AO);
    if (!qg_launch(w.wo, w.o_qt, H, NH * kHDp, AO, Tp, b.Y, st, err, sms, lim)) return 0;
    k_pf_norm<<<Tp, 256, 0, st>>>(b.X, b.Y, w.ffn_norm, c.eps, H, T, A);
    if (!qg_launch(w.wgu, w.gu_qt, 2 * F, H, A, Tp, b.GU, st, err, sms, lim)) return 0;
    k_pf_swiglu<<<dim3((F + 255) / 256, Tp), 256, 0, st>>>(b.GU, F, T, ACT);
    if (!qg_launch(w.wd, w.d_qt, H, F, ACT, Tp, b.Y, st, err, sms, lim)) return 0;
    k_pf_add<<<(T * H + 255) / 256 < 4096 ? (T * H + 255) / 256 : 4096, 256, 0, st>>>(b.X, b.Y, H, T);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

}  // namespace tb
