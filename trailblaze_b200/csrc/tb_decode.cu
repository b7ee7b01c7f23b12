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

// The reference's RoPE angle for pair i at position pos (tb_infer.c:143-145):
// theta = pos / base^(2i/HD); cos and sin of it.  Every rotation by pair i at
// this position uses the same angle, so it is computed once per launch.
__device__ __forceinline__ float2 rope_cs(int pos, int i, float base)
{
    const float theta = static_cast<float>(pos) / powf(base, 2.0f * static_cast<float>(i) / static_cast<float>(kHD));
    return make_float2(cosf(theta), sinf(theta));
}

// One rotation of the (even, odd) pair by (c, s) (tb_infer.c:146-153).
__device__ __forceinline__ void rope_rot(float &a, float &b, float2 cs)
{
    const float a0 = a, b0 = b;
    a = a0 * cs.x - b0 * cs.y;
    b = a0 * cs.y + b0 * cs.x;
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

// Sums 32 per-lane values over the warp, one sum per lane: on return lane l
// holds sum over all lanes of v[l].  Each step halves the values a lane keeps
// (it keeps the half selected by its lane bit and sends the other half to its
// partner), so the 32 sums take 31 shuffles instead of 32 x 5.
__device__ __forceinline__ float transpose_sum(float (&v)[32])
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
            const float send = up ? v[i] : v[i + off];
            const float keep = up ? v[i + off] : v[i];
            v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, off);
        }
    }
    return v[0];
}

static constexpr int kVMax = 128;            // context positions per attention CTA at most
static constexpr int kKB = kVMax / 8;        // K rows held in registers per warp

// Work area (floats) for the scores [rep][lmax], the pass-2 partials
// [8][rep][HD] and the combine's per-group state [256][8].
__host__ __device__ inline size_t attn_area_floats(int rep, int lmax)
{
    size_t area = static_cast<size_t>(rep) * lmax;
    if (area < 8ull * rep * kHD) area = 8ull * rep * kHD;
    if (area < 8ull * 256) area = 8ull * 256;
    return area;
}

__host__ __device__ inline size_t attn_smem_floats(int rep, int lmax)
{
    // q[rep][HD] | k[HD] | (cos, sin)[HD/2] | statistics [32] | area | V rows [lmax][HD]
    return static_cast<size_t>(rep) * kHD + kHD + kHD + 32 + attn_area_floats(rep, lmax) +
           static_cast<size_t>(lmax) * kHD;
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

__device__ __forceinline__ float dot4(float4 a, float4 b)
{
    float d = a.x * b.x;
    d = fmaf(a.y, b.y, d);
    d = fmaf(a.z, b.z, d);
    return fmaf(a.w, b.w, d);
}

// grid (NK, nchunk), kAttnThreads threads, 2 CTAs per SM; R2 = query heads per
// KV head rounded up to a power of two (1, 2, 4 or 8).  Shared memory
// (attn_smem_floats): q[rep][HD], k[HD], the RoPE (cos, sin) of the position,
// chunk statistics [32], the work area and the chunk's V rows [lmax][HD].
//
// This token's q, k and v are requested first, then the chunk's cached K and V
// rows (row pos, this step's, is never read from the cache), so q is rotated
// and normed while the cache rows stream in.  Each warp keeps its K rows in
// registers (positions t0 + warp + 8j); the V rows go to shared memory by
// cp.async.  Scores: each lane forms the partial dot products of its four
// dimensions for 32 (position, head) items and one transposed reduction turns
// them into 32 whole scores, one per lane.
template <int R2>
__global__ void __launch_bounds__(kAttnThreads, 2) k_attn_decode(const AttnArgs a)
{
    extern __shared__ __align__(16) float sm[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int nwarp = kAttnThreads / 32;
    const int kh = blockIdx.x, c = blockIdx.y;
    const int rep = a.NH / a.NK;
    const int pos = *a.pos;
    const int total = pos + 1;
    const int L = (total + a.nchunk - 1) / a.nchunk;
    const int t0 = min(c * L, total), t1 = min(t0 + L, total);
    const bool owner = pos >= t0 && pos < t1;   // this chunk holds the new position (its last)
    const int tc = min(t1, pos);                // cached rows of the chunk: [t0, tc)

    float *qs = sm;                                          // [rep][HD]
    float *ks = qs + rep * kHD;                              // [HD]
    float2 *csr = reinterpret_cast<float2 *>(ks + kHD);      // [HD/2] (cos, sin)
    float *red = ks + 2 * kHD;                               // [32]: m, l per head
    float *sc = red + 32;                                    // work area
    float *vs = sc + attn_area_floats(rep, a.lmax);          // [lmax][HD]
    __shared__ int s_last;

    const float *kcache = a.kc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    float *kcw = a.kc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    float *vcache = a.vc + static_cast<size_t>(kh) * a.max_ctx * kHD;

    // ---- this token's q (and, in the owner chunk, k and v), requested first:
    // behind the chunk's ~60 KB of cache rows they would arrive last ----
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 qv = z4, kn = z4, vn = z4;
    if (tid < rep * (kHD / 4)) qv = __ldcg(reinterpret_cast<const float4 *>(a.qkv + kh * rep * kHD) + tid);
    if (owner && tid < kHD / 4) {
        kn = __ldcg(reinterpret_cast<const float4 *>(a.qkv + (a.NH + kh) * kHD) + tid);
        vn = __ldcg(reinterpret_cast<const float4 *>(a.qkv + (a.NH + a.NK + kh) * kHD) + tid);
    }

    // ---- then the chunk's cached rows (row pos, this step's, is not read) ----
    for (int e = tid; e < (tc - t0) * (kHD / 4); e += kAttnThreads)
        cp_async16(vs + 4 * e, vcache + static_cast<size_t>(t0) * kHD + 4 * e);
    asm volatile("cp.async.commit_group;" ::: "memory");
    float4 kv[kKB];
#pragma unroll
    for (int j = 0; j < kKB; ++j) {
        const int t = t0 + warp + j * nwarp;
        kv[j] = t < tc ? __ldg(reinterpret_cast<const float4 *>(kcache + static_cast<size_t>(t) * kHD) + lane) : z4;
    }

    // ---- q and k normed and rotated in shared memory ----
    if (tid < rep * (kHD / 4)) reinterpret_cast<float4 *>(qs)[tid] = qv;
    if (owner && tid < kHD / 4) reinterpret_cast<float4 *>(ks)[tid] = kn;
    if (tid < kHD / 2) csr[tid] = rope_cs(pos, tid, a.rope_base);
    __syncthreads();
    auto rope_all = [&]() {
        for (int e = tid; e < rep * (kHD / 2); e += kAttnThreads) {
            const int h = e / (kHD / 2), i = e % (kHD / 2);
            rope_rot(qs[h * kHD + 2 * i], qs[h * kHD + 2 * i + 1], csr[i]);
        }
        if (owner && tid < kHD / 2) {
            // reference order: the K head is rotated once per query head mapped
            // to it by h % NK; the Qwen3 order rotates it once
            const int times = a.quirks ? rep : 1;
            const float2 r = csr[tid];
            for (int u = 0; u < times; ++u) rope_rot(ks[2 * tid], ks[2 * tid + 1], r);
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
    if (owner && tid < kHD / 4) {   // append (tb_tensor.c:314-323) and stage the new V row
        const float4 k4 = reinterpret_cast<const float4 *>(ks)[tid];
        reinterpret_cast<float4 *>(kcw + static_cast<size_t>(pos) * kHD)[tid] = k4;
        reinterpret_cast<float4 *>(vcache + static_cast<size_t>(pos) * kHD)[tid] = vn;
        reinterpret_cast<float4 *>(vs + (pos - t0) * kHD)[tid] = vn;
    }

    // ---- pass 1: scores ----
    float4 qr[R2];
#pragma unroll
    for (int h = 0; h < R2; ++h)
        qr[h] = h < rep ? reinterpret_cast<const float4 *>(qs + h * kHD)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (owner) {   // the new position's k replaces the (unloaded) cache row
        const float4 k4 = reinterpret_cast<const float4 *>(ks)[lane];
#pragma unroll
        for (int j = 0; j < kKB; ++j)
            if (t0 + warp + j * nwarp == pos) kv[j] = k4;
    }
    {
        constexpr int PP = 32 / R2;                // positions per 32 items
        constexpr int P = PP < kKB ? PP : kKB;     // of them backed by K rows
        constexpr int NG = kKB / P;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            if (t0 + warp + g * P * nwarp >= t1) break;   // warp-uniform
            float v[32];
#pragma unroll
            for (int p = 0; p < PP; ++p)
#pragma unroll
                for (int h = 0; h < R2; ++h) v[p * R2 + h] = p < P ? dot4(qr[h], kv[g * P + p]) : 0.f;
            const float d = transpose_sum(v);
            const int p = lane / R2, h = lane % R2;
            const int t = t0 + warp + (g * P + p) * nwarp;
            if (p < P && h < rep && t < t1) sc[h * a.lmax + (t - t0)] = d * a.scale;
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

    // ---- pass 2: o[h][d] = sum_t p[h][t] * v[t][d]; thread = (dim quad, position lane) ----
    {
        const int dq = tid & 31, tl = tid >> 5;   // dims 4*dq..4*dq+3, positions t0 + tl + 8k
        float4 acc[R2];
#pragma unroll
        for (int h = 0; h < R2; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = tl; j < n; j += 8) {
            const float4 v = reinterpret_cast<const float4 *>(vs + j * kHD)[dq];
#pragma unroll
            for (int h = 0; h < R2; ++h) {
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
        for (int h = 0; h < R2; ++h)
            if (h < rep) pr[(tl * rep + h) * (kHD / 4) + dq] = acc[h];
        __syncthreads();
        for (int e = tid; e < rep * (kHD / 4); e += kAttnThreads) {
            const int h = e / (kHD / 4), q4 = e % (kHD / 4);
            float4 s = pr[h * (kHD / 4) + q4];
#pragma unroll
            for (int u = 1; u < 8; ++u) {
                const float4 t = pr[(u * rep + h) * (kHD / 4) + q4];
                s.x += t.x;
                s.y += t.y;
                s.z += t.z;
                s.w += t.w;
            }
            float *dst = a.part + (static_cast<size_t>(kh * rep + h) * a.nchunk + c) * kPS;
            reinterpret_cast<float4 *>(dst)[q4] = s;
            if (q4 == 0) reinterpret_cast<float2 *>(dst + kHD)[0] = make_float2(red[2 * h], red[2 * h + 1]);
        }
    }

    // ---- the last chunk of this KV head combines all chunks ----
    __syncthreads();
    if (tid == 0) {   // release the partials (the barrier orders the CTA's writes before the fence)
        __threadfence();
        const bool last = atomicAdd(a.count + kh, 1u) == static_cast<unsigned>(a.nchunk) - 1u;
        if (last) __threadfence();
        s_last = last;
    }
    __syncthreads();
    if (!s_last) return;

    // thread = (output float4 (head, quad), chunk group); each thread merges its
    // chunks with a running maximum (online softmax), all loads of a batch of
    // kCB chunks in flight together; then the groups are merged in shared memory
    constexpr int NO = R2 * 32, NGc = kAttnThreads / NO, kCB = 10;
    const int o = tid % NO, grp = tid / NO, h = o >> 5, q4 = o & 31;
    float Mx = -1e38f, Ls = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (h < rep) {
        const float *ph = a.part + static_cast<size_t>(kh * rep + h) * a.nchunk * kPS;
        for (int u0 = grp; u0 < a.nchunk; u0 += NGc * kCB) {
            float mb[kCB], lb[kCB];
            float4 ob[kCB];
#pragma unroll
            for (int j = 0; j < kCB; ++j) {
                const int u = u0 + j * NGc;
                const float *pu = ph + static_cast<size_t>(u) * kPS;
                const bool ok = u < a.nchunk;
                ob[j] = ok ? __ldcg(reinterpret_cast<const float4 *>(pu) + q4) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float2 ml = ok ? __ldcg(reinterpret_cast<const float2 *>(pu + kHD)) : make_float2(-1e38f, 0.f);
                mb[j] = ml.x;
                lb[j] = ml.y;
            }
            float Mn = Mx;
#pragma unroll
            for (int j = 0; j < kCB; ++j) Mn = fmaxf(Mn, mb[j]);
            const float f = expf(Mx - Mn);
            acc = make_float4(acc.x * f, acc.y * f, acc.z * f, acc.w * f);
            Ls *= f;
#pragma unroll
            for (int j = 0; j < kCB; ++j) {
                const float w = expf(mb[j] - Mn);
                acc.x = fmaf(ob[j].x, w, acc.x);
                acc.y = fmaf(ob[j].y, w, acc.y);
                acc.z = fmaf(ob[j].z, w, acc.z);
                acc.w = fmaf(ob[j].w, w, acc.w);
                Ls = fmaf(lb[j], w, Ls);
            }
            Mx = Mn;
        }
    }
    if constexpr (NGc > 1) {
        float4 *gs = reinterpret_cast<float4 *>(sc);   // [NGc][NO][2] float4: (M, L, -, -), o
        gs[2 * (grp * NO + o)] = make_float4(Mx, Ls, 0.f, 0.f);
        gs[2 * (grp * NO + o) + 1] = acc;
        __syncthreads();
        if (grp == 0 && h < rep) {
#pragma unroll
            for (int g = 1; g < NGc; ++g) {
                const float4 ml = gs[2 * (g * NO + o)], og = gs[2 * (g * NO + o) + 1];
                const float Mn = fmaxf(Mx, ml.x);
                const float fa = expf(Mx - Mn), fg = expf(ml.x - Mn);
                acc = make_float4(acc.x * fa + og.x * fg, acc.y * fa + og.y * fg, acc.z * fa + og.z * fg,
                                  acc.w * fa + og.w * fg);
                Ls = Ls * fa + ml.y * fg;
                Mx = Mn;
            }
        }
    }
    if (grp == 0 && h < rep) {
        const float il = Ls > 0.f ? 1.0f / Ls : 0.f;
        reinterpret_cast<float4 *>(a.out + (kh * rep + h) * kHD)[q4] =
            make_float4(acc.x * il, acc.y * il, acc.z * il, acc.w * il);
    }
    if (tid == 0) a.count[kh] = 0u;   // ready for the next layer / token
}

static int attn_r2(int rep)
{
    return rep <= 1 ? 1 : rep <= 2 ? 2 : rep <= 4 ? 4 : 8;
}

static void (*attn_kernel(int rep))(const AttnArgs)
{
    switch (attn_r2(rep)) {
    case 1: return k_attn_decode<1>;
    case 2: return k_attn_decode<2>;
    case 4: return k_attn_decode<4>;
    default: return k_attn_decode<8>;
    }
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
        f.w_early = true;
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
        if (!launch_pdl(attn_kernel(NH / NK), dim3(NK, nchunk), dim3(kAttnThreads), smem, s, a)) return false;
        // x2 = x + Wo @ att
        f = MvFuse{};
        f.res = x;
        f.w_early = true;
        if (!mv_launch(w.wo, w.o_qt, H, NH * HD, att, x2, s, err, sms, lim, &f)) return false;
        // act = swiglu(gate, up), (gate | up) rows interleaved in Wgu, of rmsnorm(x2)
        f = MvFuse{};
        f.xmode = MV_X_RMSNORM;
        f.nw = w.ffn_norm;
        f.eps = c.norm_eps;
        f.ymode = MV_Y_SWIGLU_PAIRS;
        f.w_early = true;
        if (!mv_launch(w.wgu, w.gu_qt, 2 * F, H, x2, gu, s, err, sms, lim, &f)) return false;
        // x = x2 + Wd @ act
        f = MvFuse{};
        f.res = x2;
        f.w_early = true;
        if (!mv_launch(w.wd, w.d_qt, H, F, gu, x, s, err, sms, lim, &f)) return false;
    }
    MvFuse f;
    f.xmode = MV_X_RMSNORM;
    f.nw = out_norm;
    f.eps = c.norm_eps;
    f.w_early = true;
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
            ok = dec_ok(cudaFuncSetAttribute(attn_kernel(NH / NK), cudaFuncAttributeMaxDynamicSharedMemorySize,
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

int tb_cuda_dec_read(void *dec, int which, float *host, int n)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !host || n < 0) return 0;
    const tb::DecConfig &c = d->cfg;
    const float *src = nullptr;
    long long size = 0;
    switch (which) {
    case 0: src = d->x, size = c.hidden; break;
    case 1: src = d->x2, size = c.hidden; break;
    case 2: src = d->qkv, size = static_cast<long long>(c.n_heads + 2 * c.n_kv_heads) * c.head_dim; break;
    case 3: src = d->att, size = static_cast<long long>(c.n_heads) * c.head_dim; break;
    case 4: src = d->gu, size = c.ffn_dim; break;
    case 5: src = d->logits, size = c.vocab; break;
    default: return 0;
    }
    if (n > size) return 0;
    if (!tb::dec_ok(cudaMemcpyAsync(host, src, sizeof(float) * static_cast<size_t>(n), cudaMemcpyDeviceToHost, d->st),
                    "read"))
        return 0;
    return tb::dec_ok(cudaStreamSynchronize(d->st), "read sync") ? 1 : 0;
}

void tb_cuda_dec_destroy(void *dec)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (d) cudaStreamSynchronize(d->st);
    tb::dec_free(d);
}

}  // extern "C"
