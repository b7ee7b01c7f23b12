// tb_decode.cu — the batch-1 decode step around the matvecs, on sm_100a.
//
// GPU versions of the reference's per-token neighbours of the matvec
// (layer4/tb_infer.c:553-887 tb_layer_forward, :889-1050 tb_infer_decode):
//
//   * k_attn_decode: per-head QK-norm and RoPE (layer4/tb_infer.c:665-710,
//     tb_rope_apply :142-155), the KV-cache append and attention over the
//     cached positions (layer1/tb_tensor.c:303-409 tb_attention), split over
//     chunks of the context; the last CTA of each KV head combines the chunk
//     partials (no second launch);
//   * k_argmax_step: greedy sampling (tb_tensor.c:415-420 tb_sample_greedy)
//     and the advance of the device-side token / position;
//   * k_embed_row (tb_dequant.cu): the token's embedding row.
//
// RMSNorm (tb_tensor.c:194-199), SwiGLU (tb_infer.c:130-135) and the residual
// adds run inside the matvec kernel (tb_matvec.cu, MvFuse).  The Decoder
// below owns the KV cache and the scratch vectors and replays one CUDA graph
// per token; token and position live in device memory, so consecutive tokens
// need no host round trip.
//
// Reference order ("quirks" = 1, the default): RoPE is applied to q and k
// before the per-head RMSNorm, and each K head is rotated once for every query
// head h with h % NK == its index (tb_infer.c:665), i.e. NH/NK times.  Quirks =
// 0 gives the Qwen3 order: norm first, one rotation.
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

static constexpr int kHD = 128;            // head_dim supported by the attention kernel
static constexpr int kPS = kHD + 4;        // floats per chunk partial: o[HD], m, l, 2 pad (16-byte rows)
static constexpr int kAttnThreads = 256;

struct AttnArgs {
    const float *qkv;      // [NH*HD | NK*HD | NK*HD]: this token's q, k, v
    const float *qn, *kn;  // per-head RMSNorm weights [HD], or null (no QK-norm)
    float *kc, *vc;        // this layer's cache: [NK][max_ctx][HD] each
    const int *pos;        // device: position of this token (attends to 0..pos)
    float *part;           // [NH][nchunk][kPS]: o (unnormalised), m, l per chunk
    unsigned *count;       // [NK] chunk tickets; 0 on entry and left at 0
    float *out;            // [NH*HD]
    int *err;
    int NH, NK, max_ctx, nchunk, lmax, quirks;
    float eps, rope_base, scale;
};

// RoPE of one (even, odd) pair by the reference's angle (tb_infer.c:143-145).
__device__ __forceinline__ void rope_pair(float &a, float &b, int pos, int i, float base)
{
    const float theta = static_cast<float>(pos) / powf(base, 2.0f * static_cast<float>(i) / static_cast<float>(kHD));
    const float c = cosf(theta), s = sinf(theta);
    const float a0 = a, b0 = b;
    a = a0 * c - b0 * s;
    b = a0 * s + b0 * c;
}

// In-place per-head RMSNorm of hv[kHD] in shared memory by one warp
// (tb_infer.c:689-693: sc = 1/sqrtf(sum/HD + eps), x*sc*w).
__device__ __forceinline__ void head_norm_warp(float *hv, const float *w, float eps)
{
    const int lane = threadIdx.x & 31;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kHD / 32; ++j) {
        const float t = hv[lane + 32 * j];
        ss = fmaf(t, t, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float sc = 1.0f / sqrtf(ss / static_cast<float>(kHD) + eps);
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kHD / 32; ++j) {
        const int d = lane + 32 * j;
        hv[d] = hv[d] * sc * __ldg(w + d);
    }
    __syncwarp();
}

static constexpr int kVMax = 128;          // context positions per attention CTA at most
static constexpr int kKB = (kVMax + 7) / 8; // K rows held in registers per warp

__host__ __device__ inline size_t attn_smem_floats(int rep, int lmax)
{
    const size_t area = static_cast<size_t>(rep) * lmax > 8ull * rep * kHD ? static_cast<size_t>(rep) * lmax
                                                                           : 8ull * rep * kHD;
    return static_cast<size_t>(rep) * kHD + kHD + 32 + area + static_cast<size_t>(lmax) * kHD;
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

// grid (NK, nchunk), kAttnThreads threads, 2 CTAs per SM.  Shared memory
// (attn_smem_floats): q[rep][HD], k[HD], chunk statistics [32], a work area
// (the scores [rep][lmax], later the pass-2 partials [8][rep][HD] and the
// chunk weights), and the chunk's V rows [lmax][HD].
//
// Every load of the chunk is issued at the start: each warp's K rows into
// registers, every V row into shared memory with cp.async; q is rotated and
// normed meanwhile, so the DRAM latency is paid about once per CTA.
__global__ void __launch_bounds__(kAttnThreads, 2) k_attn_decode(const AttnArgs a)
{
    extern __shared__ __align__(16) float sm[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = kAttnThreads / 32;
    const int kh = blockIdx.x, c = blockIdx.y;
    const int rep = a.NH / a.NK;
    const int pos = *a.pos;
    const int total = pos + 1;
    const int L = (total + a.nchunk - 1) / a.nchunk;
    const int t0 = min(c * L, total), t1 = min(t0 + L, total);
    const bool owner = pos >= t0 && pos < t1;   // this chunk holds the new position

    float *qs = sm;                         // [rep][HD]
    float *ks = qs + rep * kHD;             // [HD]
    float *red = ks + kHD;                  // [32]: m, l per head; later 1/L per head
    float *sc = red + 32;                   // scores / pass-2 partials / chunk weights
    const size_t area = static_cast<size_t>(rep) * a.lmax > 8ull * rep * kHD ? static_cast<size_t>(rep) * a.lmax
                                                                             : 8ull * rep * kHD;
    float *vs = sc + area;                  // [lmax][HD]
    __shared__ int s_last;

    const float *kcache = a.kc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    float *kcw = a.kc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    float *vcache = a.vc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    const float *vnew = a.qkv + (a.NH + a.NK) * kHD + kh * kHD;

    // ---- every load of the chunk, issued up front ----
    for (int e = tid; e < (t1 - t0) * (kHD / 4); e += kAttnThreads)
        cp_async16(vs + 4 * e, vcache + static_cast<size_t>(t0) * kHD + 4 * e);
    asm volatile("cp.async.commit_group;" ::: "memory");
    float4 kv[kKB];
#pragma unroll
    for (int j = 0; j < kKB; ++j) {
        const int t = t0 + warp + j * nwarp;
        kv[j] = t < t1 ? __ldg(reinterpret_cast<const float4 *>(kcache + static_cast<size_t>(t) * kHD) + lane)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // ---- q (and, for the owner, k) of this KV head, normed and rotated ----
    const float *qsrc = a.qkv + kh * rep * kHD;
    for (int e = tid; e < rep * kHD; e += kAttnThreads) qs[e] = __ldg(qsrc + e);
    if (owner)
        for (int e = tid; e < kHD; e += kAttnThreads) ks[e] = __ldg(a.qkv + a.NH * kHD + kh * kHD + e);
    __syncthreads();
    auto rope_all = [&]() {
        for (int e = tid; e < rep * (kHD / 2); e += kAttnThreads) {
            const int h = e / (kHD / 2), i = e % (kHD / 2);
            rope_pair(qs[h * kHD + 2 * i], qs[h * kHD + 2 * i + 1], pos, i, a.rope_base);
        }
        if (owner) {
            // reference order: the K head is rotated once per query head mapped
            // to it by h % NK; the Qwen3 order rotates it once
            const int times = a.quirks ? a.NH / a.NK : 1;
            for (int i = tid; i < kHD / 2; i += kAttnThreads)
                for (int r = 0; r < times; ++r) rope_pair(ks[2 * i], ks[2 * i + 1], pos, i, a.rope_base);
        }
        __syncthreads();
    };
    auto norm_all = [&]() {
        if (a.qn)
            for (int h = warp; h < rep; h += nwarp) head_norm_warp(qs + h * kHD, a.qn, a.eps);
        if (owner && a.kn && warp == nwarp - 1) head_norm_warp(ks, a.kn, a.eps);
        __syncthreads();
    };
    if (a.quirks) {
        rope_all();
        norm_all();
    } else {
        norm_all();
        rope_all();
    }
    if (owner)   // append (tb_tensor.c:314-323); nothing else reads position pos now
        for (int e = tid; e < kHD; e += kAttnThreads) {
            kcw[static_cast<size_t>(pos) * kHD + e] = ks[e];
            vcache[static_cast<size_t>(pos) * kHD + e] = __ldg(vnew + e);
        }

    // ---- pass 1: scores; warp w holds the K rows of positions t0 + w + 8j ----
#pragma unroll
    for (int j = 0; j < kKB; ++j) {
        const int t = t0 + warp + j * nwarp;
        if (t >= t1) break;
        const float4 k4 = (t == pos && owner) ? reinterpret_cast<const float4 *>(ks)[lane] : kv[j];
        for (int h = 0; h < rep; ++h) {
            const float4 q = reinterpret_cast<const float4 *>(qs + h * kHD)[lane];
            float d = q.x * k4.x;
            d = fmaf(q.y, k4.y, d);
            d = fmaf(q.z, k4.z, d);
            d = fmaf(q.w, k4.w, d);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
            if (lane == 0) sc[h * a.lmax + (t - t0)] = d * a.scale;
        }
    }
    __syncthreads();

    // ---- softmax statistics of the chunk: one warp per head ----
    const int n = t1 - t0;
    for (int h = warp; h < rep; h += nwarp) {
        float m = -1e38f;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[h * a.lmax + j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        float l = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float p = expf(sc[h * a.lmax + j] - m);
            sc[h * a.lmax + j] = p;
            l += p;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
        if (lane == 0) {
            red[2 * h] = m;
            red[2 * h + 1] = l;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (owner)   // the new V row replaces the stale one copied from the cache
        for (int e = tid; e < kHD; e += kAttnThreads) vs[(pos - t0) * kHD + e] = __ldg(vnew + e);
    __syncthreads();

    // ---- pass 2: o[h][d] = sum_t p[h][t] * v[t][d]; thread = (dim quad, position lane) ----
    {
        const int dq = tid & 31, tl = tid >> 5;   // dims 4*dq..4*dq+3, positions t0 + tl + 8k
        float4 acc[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = tl; j < n; j += 8) {
            const float4 v = reinterpret_cast<const float4 *>(vs + j * kHD)[dq];
#pragma unroll
            for (int h = 0; h < 8; ++h) {
                if (h < rep) {
                    const float p = sc[h * a.lmax + j];
                    acc[h].x = fmaf(p, v.x, acc[h].x);
                    acc[h].y = fmaf(p, v.y, acc[h].y);
                    acc[h].z = fmaf(p, v.z, acc[h].z);
                    acc[h].w = fmaf(p, v.w, acc[h].w);
                }
            }
        }
        __syncthreads();   // scores no longer needed: reuse sc as [8][rep][HD] partials
        float4 *pr = reinterpret_cast<float4 *>(sc);
#pragma unroll
        for (int h = 0; h < 8; ++h)
            if (h < rep) pr[(tl * rep + h) * (kHD / 4) + dq] = acc[h];
        __syncthreads();
        for (int e = tid; e < rep * (kHD / 4); e += kAttnThreads) {
            const int h = e / (kHD / 4), q4 = e % (kHD / 4);
            float4 s = pr[h * (kHD / 4) + q4];
            for (int u = 1; u < 8; ++u) {
                const float4 t = pr[(u * rep + h) * (kHD / 4) + q4];
                s.x += t.x;
                s.y += t.y;
                s.z += t.z;
                s.w += t.w;
            }
            float *dst = a.part + (static_cast<size_t>(kh * rep + h) * a.nchunk + c) * kPS;
            reinterpret_cast<float4 *>(dst)[q4] = s;
            if (q4 == 0) {
                dst[kHD] = red[2 * h];
                dst[kHD + 1] = red[2 * h + 1];
            }
        }
    }

    // ---- the last chunk of this KV head combines all chunks ----
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.count + kh, 1u) == static_cast<unsigned>(a.nchunk) - 1u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // chunk weights w[h][u] = e^(m_u - M_h) and 1/L per head into shared memory,
    // then each output float4 is a weighted sum over the chunks
    float *wts = sc;                                  // [rep][nchunk]
    float *hm = red;                                  // [rep] 1/L
    const float *pk = a.part + static_cast<size_t>(kh * rep) * a.nchunk * kPS;
    for (int h = warp; h < rep; h += nwarp) {
        const float *ph = pk + static_cast<size_t>(h) * a.nchunk * kPS;
        float M = -1e38f;
        for (int u = lane; u < a.nchunk; u += 32) M = fmaxf(M, __ldcg(ph + u * kPS + kHD));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
        float Ls = 0.f;
        for (int u = lane; u < a.nchunk; u += 32) {
            const float w = expf(__ldcg(ph + u * kPS + kHD) - M);
            wts[h * a.nchunk + u] = w;
            Ls = fmaf(__ldcg(ph + u * kPS + kHD + 1), w, Ls);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xFFFFFFFFu, Ls, o);
        if (lane == 0) hm[h] = Ls > 0.f ? 1.0f / Ls : 0.f;
    }
    __syncthreads();
    constexpr int kCB = 8;
    for (int e = tid; e < rep * (kHD / 4); e += kAttnThreads) {   // one float4 of one head per thread
        const int h = e / (kHD / 4), q4 = e % (kHD / 4);
        const float *ph = pk + static_cast<size_t>(h) * a.nchunk * kPS;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int u0 = 0; u0 < a.nchunk; u0 += kCB) {
            float4 ob[kCB];
#pragma unroll
            for (int j = 0; j < kCB; ++j)
                ob[j] = u0 + j < a.nchunk ? __ldcg(reinterpret_cast<const float4 *>(ph + (u0 + j) * kPS) + q4)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kCB; ++j) {
                const float w = u0 + j < a.nchunk ? wts[h * a.nchunk + u0 + j] : 0.f;
                o.x = fmaf(ob[j].x, w, o.x);
                o.y = fmaf(ob[j].y, w, o.y);
                o.z = fmaf(ob[j].z, w, o.z);
                o.w = fmaf(ob[j].w, w, o.w);
            }
        }
        const float il = hm[h];
        reinterpret_cast<float4 *>(a.out + (kh * rep + h) * kHD)[q4] = make_float4(o.x * il, o.y * il, o.z * il, o.w * il);
    }
    if (tid == 0) a.count[kh] = 0u;   // ready for the next layer / token
}

// Greedy sampling (tb_tensor.c:415-420: the first index of the largest logit)
// and the step's advance: token <- argmax, pos <- pos + 1.  grid G CTAs of
// kArgThreads; the last CTA to finish reduces the G partial results.
static constexpr int kArgThreads = 512;

struct ArgBest {
    float v;
    int i;
};
__device__ __forceinline__ ArgBest better(ArgBest a, ArgBest b)
{
    return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}
__device__ __forceinline__ ArgBest warp_best(ArgBest b)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest t{__shfl_xor_sync(0xFFFFFFFFu, b.v, o), __shfl_xor_sync(0xFFFFFFFFu, b.i, o)};
        b = better(b, t);
    }
    return b;
}

__global__ void __launch_bounds__(kArgThreads) k_argmax_step(const float *logits, int n, float *pv, int *pi,
                                                              unsigned *count, int *token, int *pos)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ ArgBest sb[kArgThreads / 32];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, G = gridDim.x, c = blockIdx.x;
    const int lo = static_cast<int>((static_cast<long long>(n) * c) / G);
    const int hi = static_cast<int>((static_cast<long long>(n) * (c + 1)) / G);
    ArgBest b{-FLT_MAX, 0x7FFFFFFF};
    for (int i = lo + tid; i < hi; i += kArgThreads) b = better(b, ArgBest{__ldg(logits + i), i});
    b = warp_best(b);
    if (lane == 0) sb[warp] = b;
    __syncthreads();
    if (warp == 0) {
        b = lane < kArgThreads / 32 ? sb[lane] : ArgBest{-FLT_MAX, 0x7FFFFFFF};
        b = warp_best(b);
        if (lane == 0) {
            pv[c] = b.v;
            pi[c] = b.i;
            __threadfence();
            s_last = atomicAdd(count, 1u) == static_cast<unsigned>(G) - 1u;
        }
    }
    __syncthreads();
    if (!s_last || warp != 0) return;
    __threadfence();
    b = ArgBest{-FLT_MAX, 0x7FFFFFFF};
    for (int u = lane; u < G; u += 32) b = better(b, ArgBest{__ldcg(pv + u), __ldcg(pi + u)});
    b = warp_best(b);
    if (lane == 0) {
        *token = b.i == 0x7FFFFFFF ? 0 : b.i;
        *pos = *pos + 1;
        *count = 0u;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// Launch with programmatic stream serialization (kernels above wait on their
// predecessor with griddepcontrol.wait before touching global memory).
template <class... A>
static bool launch_pdl(void (*kern)(A...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A... args)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess;
}

struct DecLayer {
    const void *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
    int qkv_qt = -1, o_qt = -1, gu_qt = -1, d_qt = -1;
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
};

struct Decoder {
    DecConfig cfg{};
    int dev = 0, sms = 0, nchunk = 1, lmax = 1;
    DecLayer *layers = nullptr;
    const void *emb = nullptr, *lm = nullptr;
    int emb_qt = -1, lm_qt = -1;
    const float *out_norm = nullptr;
    cudaStream_t st = nullptr;
    cudaGraphExec_t gexec = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    int *err = nullptr;
    // device buffers
    float *x = nullptr, *x2 = nullptr, *qkv = nullptr, *att = nullptr, *gu = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr, *part = nullptr, *argv = nullptr;
    int *argi = nullptr, *tok = nullptr, *pos = nullptr, *hostio = nullptr;
    unsigned *counts = nullptr;   // [NK] attention tickets + [1] argmax ticket

    size_t kv_layer_floats() const
    {
        return static_cast<size_t>(cfg.n_kv_heads) * cfg.max_ctx * cfg.head_dim;
    }
    bool ready() const
    {
        if (!emb || !lm || !out_norm) return false;
        for (int l = 0; l < cfg.n_layers; ++l)
            if (!layers[l].wqkv || !layers[l].wo || !layers[l].wgu || !layers[l].wd || !layers[l].attn_norm ||
                !layers[l].ffn_norm)
                return false;
        return true;
    }
    bool enqueue(cudaStream_t s);
};

bool Decoder::enqueue(cudaStream_t s)
{
    const DecConfig &c = cfg;
    const int H = c.hidden, NH = c.n_heads, NK = c.n_kv_heads, HD = c.head_dim, F = c.ffn_dim;
    const int QKV = (NH + 2 * NK) * HD;
    const uint32_t lim = 1u << 22;
    if (!dq_embed_launch(emb, emb_qt, c.vocab, H, tok, x, s)) return false;
    for (int l = 0; l < c.n_layers; ++l) {
        const DecLayer &w = layers[l];
        MvFuse f;
        // q | k | v = Wqkv @ rmsnorm(x)
        f = MvFuse{};
        f.xmode = MV_X_RMSNORM;
        f.nw = w.attn_norm;
        f.eps = c.norm_eps;
        if (!mv_launch(w.wqkv, w.qkv_qt, QKV, H, x, qkv, s, err, sms, lim, &f)) return false;
        // attention (QK-norm, RoPE, cache append, split-context softmax)
        AttnArgs a{};
        a.qkv = qkv;
        a.qn = w.q_norm;
        a.kn = w.k_norm;
        a.kc = kc + static_cast<size_t>(l) * kv_layer_floats();
        a.vc = vc + static_cast<size_t>(l) * kv_layer_floats();
        a.pos = pos;
        a.part = part;
        a.count = counts;
        a.out = att;
        a.err = err;
        a.NH = NH;
        a.NK = NK;
        a.max_ctx = c.max_ctx;
        a.nchunk = nchunk;
        a.lmax = lmax;
        a.quirks = c.quirks;
        a.eps = c.norm_eps;
        a.rope_base = c.rope_base;
        a.scale = 1.0f / sqrtf(static_cast<float>(HD));
        const size_t smem = attn_smem_floats(NH / NK, lmax) * sizeof(float);
        if (!launch_pdl(k_attn_decode, dim3(NK, nchunk), dim3(kAttnThreads), smem, s, a)) return false;
        // x2 = x + Wo @ att
        f = MvFuse{};
        f.res = x;
        if (!mv_launch(w.wo, w.o_qt, H, NH * HD, att, x2, s, err, sms, lim, &f)) return false;
        // act = swiglu(gate, up), (gate | up) rows interleaved in Wgu, of rmsnorm(x2)
        f = MvFuse{};
        f.xmode = MV_X_RMSNORM;
        f.nw = w.ffn_norm;
        f.eps = c.norm_eps;
        f.ymode = MV_Y_SWIGLU_PAIRS;
        if (!mv_launch(w.wgu, w.gu_qt, 2 * F, H, x2, gu, s, err, sms, lim, &f)) return false;
        // x = x2 + Wd @ act
        f = MvFuse{};
        f.res = x2;
        if (!mv_launch(w.wd, w.d_qt, H, F, gu, x, s, err, sms, lim, &f)) return false;
    }
    MvFuse f;
    f.xmode = MV_X_RMSNORM;
    f.nw = out_norm;
    f.eps = c.norm_eps;
    if (!mv_launch(lm, lm_qt, c.vocab, H, x, logits, s, err, sms, lim, &f)) return false;
    const int G = sms;
    return launch_pdl(k_argmax_step, dim3(G), dim3(kArgThreads), 0, s, static_cast<const float *>(logits),
                      c.vocab, argv, argi, counts + NK, tok, pos);
}

static bool dec_ok(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return true;
    fprintf(stderr, "[tb_cuda] decoder: %s: %s\n", what, cudaGetErrorString(e));
    return false;
}

static void dec_free(Decoder *d)
{
    if (!d) return;
    if (d->gexec) cudaGraphExecDestroy(d->gexec);
    if (d->st) cudaStreamDestroy(d->st);
    if (d->ev0) cudaEventDestroy(d->ev0);
    if (d->ev1) cudaEventDestroy(d->ev1);
    void *bufs[] = {d->x, d->x2, d->qkv, d->att, d->gu, d->logits, d->kc, d->vc, d->part, d->argv,
                    d->argi, d->tok, d->pos, d->counts, d->err};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (d->hostio) cudaFreeHost(d->hostio);
    delete[] d->layers;
    delete d;
}

Decoder *dec_create(const DecConfig &c)
{
    if (c.n_layers <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim != kHD ||
        c.n_heads % c.n_kv_heads || c.n_heads / c.n_kv_heads > 8 || c.ffn_dim <= 0 || c.vocab <= 0 ||
        c.max_ctx <= 0) {
        fprintf(stderr, "[tb_cuda] decoder: unsupported configuration (head_dim must be %d, n_heads/n_kv_heads <= 8)\n", kHD);
        return nullptr;
    }
    Decoder *d = new Decoder;
    d->cfg = c;
    d->layers = new DecLayer[c.n_layers];
    cudaGetDevice(&d->dev);
    cudaDeviceGetAttribute(&d->sms, cudaDevAttrMultiProcessorCount, d->dev);
    // context chunks: about four attention CTAs per SM over all KV heads
    // context chunks: one wave of two attention CTAs per SM over all KV heads,
    // more if a chunk would exceed kVMax positions (its V rows live in shared memory)
    d->nchunk = (2 * d->sms) / c.n_kv_heads;
    if (d->nchunk < (c.max_ctx + kVMax - 1) / kVMax) d->nchunk = (c.max_ctx + kVMax - 1) / kVMax;
    if (d->nchunk < 1) d->nchunk = 1;
    d->lmax = (c.max_ctx + d->nchunk - 1) / d->nchunk;
    const int NH = c.n_heads, NK = c.n_kv_heads, HD = c.head_dim;
    const size_t kvf = static_cast<size_t>(c.n_layers) * d->kv_layer_floats();
    bool ok = dec_ok(cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking), "stream") &&
              dec_ok(cudaEventCreate(&d->ev0), "event") && dec_ok(cudaEventCreate(&d->ev1), "event") &&
              dec_ok(cudaMalloc(&d->x, sizeof(float) * c.hidden), "x") &&
              dec_ok(cudaMalloc(&d->x2, sizeof(float) * c.hidden), "x2") &&
              dec_ok(cudaMalloc(&d->qkv, sizeof(float) * (NH + 2 * NK) * HD), "qkv") &&
              dec_ok(cudaMalloc(&d->att, sizeof(float) * NH * HD), "att") &&
              dec_ok(cudaMalloc(&d->gu, sizeof(float) * 2 * static_cast<size_t>(c.ffn_dim)), "gate_up") &&
              dec_ok(cudaMalloc(&d->logits, sizeof(float) * static_cast<size_t>(c.vocab)), "logits") &&
              dec_ok(cudaMalloc(&d->kc, sizeof(float) * kvf), "k cache") &&
              dec_ok(cudaMalloc(&d->vc, sizeof(float) * kvf), "v cache") &&
              dec_ok(cudaMalloc(&d->part, sizeof(float) * NH * static_cast<size_t>(d->nchunk) * kPS), "partials") &&
              dec_ok(cudaMalloc(&d->argv, sizeof(float) * d->sms), "argmax") &&
              dec_ok(cudaMalloc(&d->argi, sizeof(int) * d->sms), "argmax") &&
              dec_ok(cudaMalloc(&d->tok, sizeof(int)), "token") && dec_ok(cudaMalloc(&d->pos, sizeof(int)), "pos") &&
              dec_ok(cudaMalloc(&d->counts, sizeof(unsigned) * (NK + 1)), "tickets") &&
              dec_ok(cudaMalloc(&d->err, sizeof(int)), "err") &&
              dec_ok(cudaMallocHost(&d->hostio, sizeof(int) * 4), "host io");
    if (ok) {
        ok = dec_ok(cudaMemset(d->counts, 0, sizeof(unsigned) * (NK + 1)), "memset") &&
             dec_ok(cudaMemset(d->err, 0, sizeof(int)), "memset") &&
             dec_ok(cudaMemset(d->kc, 0, sizeof(float) * kvf), "memset") &&
             dec_ok(cudaMemset(d->vc, 0, sizeof(float) * kvf), "memset");
        const size_t smem = attn_smem_floats(NH / NK, d->lmax) * sizeof(float);
        if (ok && smem > 48 * 1024)
            ok = dec_ok(cudaFuncSetAttribute(k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem)), "attention smem");
    }
    if (!ok) {
        dec_free(d);
        return nullptr;
    }
    return d;
}

// Captures the whole token step into one CUDA graph (once; shapes never
// change, token and position are read from device memory).
static bool dec_graph(Decoder *d)
{
    if (d->gexec) return true;
    if (!d->ready()) {
        fprintf(stderr, "[tb_cuda] decoder: weights not complete (set every layer and the head)\n");
        return false;
    }
    cudaGraph_t g = nullptr;
    if (!dec_ok(cudaStreamBeginCapture(d->st, cudaStreamCaptureModeThreadLocal), "begin capture")) return false;
    const bool ok = d->enqueue(d->st);
    const cudaError_t e = cudaStreamEndCapture(d->st, &g);
    if (!ok || e != cudaSuccess || !g) {
        fprintf(stderr, "[tb_cuda] decoder: graph capture failed (%s)\n", cudaGetErrorString(e));
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return false;
    }
    const bool inst = dec_ok(cudaGraphInstantiate(&d->gexec, g, 0), "graph instantiate");
    cudaGraphDestroy(g);
    return inst;
}

// Runs n tokens back to back from (token, pos): token_i+1 = argmax of step i.
// tokens[i] receives each generated token when not null; ms receives the device
// time of the n replays (CUDA events on the decoder's stream).
int dec_run(Decoder *d, int token, int pos, int n, int *tokens, float *logits_host, float *ms)
{
    if (!d || n <= 0 || token < 0 || token >= d->cfg.vocab || pos < 0 || pos + n > d->cfg.max_ctx) return 0;
    if (!dec_graph(d)) return 0;
    d->hostio[0] = token;
    d->hostio[1] = pos;
    if (!dec_ok(cudaMemcpyAsync(d->tok, &d->hostio[0], sizeof(int), cudaMemcpyHostToDevice, d->st), "token") ||
        !dec_ok(cudaMemcpyAsync(d->pos, &d->hostio[1], sizeof(int), cudaMemcpyHostToDevice, d->st), "pos"))
        return 0;
    cudaEventRecord(d->ev0, d->st);
    for (int i = 0; i < n; ++i) {
        if (!dec_ok(cudaGraphLaunch(d->gexec, d->st), "graph launch")) return 0;
        if (tokens)
            cudaMemcpyAsync(tokens + i, d->tok, sizeof(int), cudaMemcpyDeviceToHost, d->st);
    }
    cudaEventRecord(d->ev1, d->st);
    if (logits_host)
        cudaMemcpyAsync(logits_host, d->logits, sizeof(float) * d->cfg.vocab, cudaMemcpyDeviceToHost, d->st);
    int e = 0;
    cudaMemcpyAsync(&d->hostio[2], d->err, sizeof(int), cudaMemcpyDeviceToHost, d->st);
    if (!dec_ok(cudaStreamSynchronize(d->st), "step")) return 0;
    e = d->hostio[2];
    if (ms) cudaEventElapsedTime(ms, d->ev0, d->ev1);
    if (e) {
        fprintf(stderr, "[tb_cuda] decoder: device error %d\n", e);
        cudaMemsetAsync(d->err, 0, sizeof(int), d->st);
        cudaStreamSynchronize(d->st);
        return 0;
    }
    return 1;
}

}  // namespace tb

// ---------------------------------------------------------------------------
// C ABI (include/tb_gguf_dequant.h, part 3)
// ---------------------------------------------------------------------------
#include "../../include/tb_gguf_dequant.h"

extern "C" {

void *tb_cuda_dec_create(const tb_dec_config *c)
{
    if (!c) return nullptr;
    tb::DecConfig k{c->n_layers, c->hidden, c->n_heads, c->n_kv_heads, c->head_dim, c->ffn_dim,
                    c->vocab, c->max_ctx, c->rope_base, c->norm_eps, c->quirks};
    return tb::dec_create(k);
}

int tb_cuda_dec_set_layer(void *dec, int layer, const tb_dec_layer *w)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !w || layer < 0 || layer >= d->cfg.n_layers) return 0;
    for (int qt : {w->qkv_qtype, w->o_qtype, w->gate_up_qtype, w->down_qtype})
        if (!tb::geom_of(qt).block_weights) return 0;
    tb::DecLayer &l = d->layers[layer];
    l.wqkv = w->w_qkv;
    l.qkv_qt = w->qkv_qtype;
    l.wo = w->w_o;
    l.o_qt = w->o_qtype;
    l.wgu = w->w_gate_up;
    l.gu_qt = w->gate_up_qtype;
    l.wd = w->w_down;
    l.d_qt = w->down_qtype;
    l.attn_norm = w->attn_norm;
    l.ffn_norm = w->ffn_norm;
    l.q_norm = w->q_norm;
    l.k_norm = w->k_norm;
    if (d->gexec) {   // weights changed: capture again on the next step
        cudaGraphExecDestroy(d->gexec);
        d->gexec = nullptr;
    }
    return 1;
}

int tb_cuda_dec_set_head(void *dec, const void *tok_embd, int embd_qtype, const float *out_norm,
                         const void *w_out, int out_qtype)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !tok_embd || !out_norm || !w_out) return 0;
    if (!tb::geom_of(embd_qtype).block_weights || !tb::geom_of(out_qtype).block_weights) return 0;
    d->emb = tok_embd;
    d->emb_qt = embd_qtype;
    d->out_norm = out_norm;
    d->lm = w_out;
    d->lm_qt = out_qtype;
    if (d->gexec) {
        cudaGraphExecDestroy(d->gexec);
        d->gexec = nullptr;
    }
    return 1;
}

float *tb_cuda_dec_kv(void *dec, int layer, int which)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || layer < 0 || layer >= d->cfg.n_layers || (which != 0 && which != 1)) return nullptr;
    return (which ? d->vc : d->kc) + static_cast<size_t>(layer) * d->kv_layer_floats();
}

int tb_cuda_dec_kv_copy(void *dec, int layer, int which, int p0, int n, float *host, int to_device)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !host || layer < 0 || layer >= d->cfg.n_layers || (which != 0 && which != 1) || p0 < 0 || n <= 0 ||
        p0 + n > d->cfg.max_ctx)
        return 0;
    float *base = tb_cuda_dec_kv(dec, layer, which);
    const size_t hd = static_cast<size_t>(d->cfg.head_dim) * sizeof(float);
    // host [n_kv_heads][n][head_dim] <-> device [n_kv_heads][max_ctx][head_dim] at position p0
    float *dev = base + static_cast<size_t>(p0) * d->cfg.head_dim;
    const size_t dpitch = static_cast<size_t>(d->cfg.max_ctx) * hd, hpitch = static_cast<size_t>(n) * hd;
    // cudaMemcpyDefault: `host` may also be device memory (unified addressing)
    const cudaError_t e = to_device
        ? cudaMemcpy2DAsync(dev, dpitch, host, hpitch, hpitch, d->cfg.n_kv_heads, cudaMemcpyDefault, d->st)
        : cudaMemcpy2DAsync(host, hpitch, dev, dpitch, hpitch, d->cfg.n_kv_heads, cudaMemcpyDefault, d->st);
    if (!tb::dec_ok(e, "kv copy")) return 0;
    return tb::dec_ok(cudaStreamSynchronize(d->st), "kv copy sync") ? 1 : 0;
}

int tb_cuda_dec_generate(void *dec, int token, int pos, int n, int *tokens_out, float *logits_host,
                         float *device_ms)
{
    return tb::dec_run(static_cast<tb::Decoder *>(dec), token, pos, n, tokens_out, logits_host, device_ms);
}

int tb_cuda_dec_step(void *dec, int token, int pos, int *next_token, float *logits_host)
{
    return tb::dec_run(static_cast<tb::Decoder *>(dec), token, pos, 1, next_token, logits_host, nullptr);
}

void tb_cuda_dec_destroy(void *dec)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (d) cudaStreamSynchronize(d->st);
    tb::dec_free(d);
}

}  // extern "C"
