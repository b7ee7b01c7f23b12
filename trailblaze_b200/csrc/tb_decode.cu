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
static constexpr int kAttnThreads = 512;

struct AttnArgs {
    const float *qkv;      // [NH*HD | NK*HD | NK*HD]: this token's q, k, v
    const float *qn, *kn;  // per-head RMSNorm weights [HD], or null (no QK-norm)
    float *kc, *vc;        // this layer's cache: [NK][max_ctx][HD] each
    const int *pos;        // device: position of this token (attends to 0..pos)
    float *part;           // [NH][nchunk][kPS]: o (unnormalised), m, l per chunk
    unsigned *count;       // [NK] chunk tickets; 0 on entry and left at 0
    float *out;            // [NH*HD]
    int *err;
    int NH, NK, max_ctx, nchunk, quirks;
    int krot;              // rotations of the new K row (quirks: the whole model's n_heads / n_kv_heads)
    float eps, rope_base, scale;
    uint32_t wait_limit;   // iterations of a bounded ring wait
    unsigned long long *stamp;   // TB_ATTN_STAMPS builds only: 16 device-clock stamps per CTA
};

#if TB_ATTN_STAMPS
#define ATT_STAMP(k)                                                                              \
    do {                                                                                          \
        if (a.stamp && threadIdx.x == 0) {                                                        \
            unsigned long long t_;                                                                \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                \
            a.stamp[(blockIdx.y * gridDim.x + blockIdx.x) * 16u + (k)] = t_;                      \
        }                                                                                         \
    } while (0)
#else
#define ATT_STAMP(k) \
    do {             \
    } while (0)
#endif

static constexpr uint32_t kAttnDrain = 1u << 26;   // bound of the drain after a failed wait

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
// (tb_infer.c:689-693: sc = 1/sqrtf(sum/HD + eps), x*sc*w); w is in shared
// memory too.
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
        hv[d] = hv[d] * sc * w[d];
    }
    __syncwarp();
}

// Sums V per-lane values (V a power of two, at most 32) over the warp: on return
// lane l holds the sum over all 32 lanes of v[l % V].  The first log2(V) steps
// transpose while they add (each lane keeps the half of its values selected by
// its lane bit and sends the other half to its partner), the rest are plain
// butterfly adds, so the V sums take V - 1 + (5 - log2 V) shuffles instead of
// 5 V.
template <int V>
__device__ __forceinline__ float transpose_sum(float (&v)[V])
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int off = V / 2; off >= 1; off >>= 1) {
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
            const float send = up ? v[i] : v[i + off];
            const float keep = up ? v[i + off] : v[i];
            v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, off);
        }
    }
    float r = v[0];
#pragma unroll
    for (int off = V; off < 32; off <<= 1) r += __shfl_xor_sync(0xFFFFFFFFu, r, off);
    return r;
}

// The chunk's cached rows stream through a ring of kNS stages by 1-D bulk
// copies that one thread issues: first the K rows of every block of kBP
// positions, then the V rows (2 nb loads for nb blocks).  The scores need only
// K and are cheap, so the K stages are released, and refilled with V rows,
// while the stream is still running.
static constexpr int kBP = 64;                                   // positions per load
static constexpr int kNS = 3;                                    // ring stages (5 and 6 measured no faster)
static constexpr uint32_t kStageBytes = kBP * kHD * sizeof(float);   // the K or V rows of a block
static constexpr int kPW = kBP / (kAttnThreads / 32);            // positions of a load per warp
static_assert(kPW * 8 <= 32 && kPW * (kAttnThreads / 32) == kBP, "a warp's (position, head) items fit its lanes");
static constexpr int kSmemCap = 232448;                          // 227 KB opt-in per CTA

__host__ __device__ inline int attn_r2(int rep)
{
    return rep <= 1 ? 1 : rep <= 2 ? 2 : rep <= 4 ? 4 : 8;
}

// Positions of the score buffer, a multiple of 4 so its rows stay 16-byte aligned.
__host__ __device__ inline int attn_lmax4(int lmax)
{
    return (lmax + 3) & ~3;
}

// Dynamic shared memory: ring [kNS][kBP][HD] | scores, then probabilities
// [lmax4][R2] | q[rep][HD] | k[HD] | new v[HD] | q-norm and k-norm weights
// [2][HD] | (cos, sin)[HD/2] | chunk statistics [32] | full barriers [kNS] |
// stage release counters [kNS] | last load issued per stage [kNS].  The ring
// doubles as scratch once every load is consumed.
__host__ __device__ inline size_t attn_smem_bytes(int rep, int lmax)
{
    return static_cast<size_t>(kNS) * kStageBytes +
           sizeof(float) * (static_cast<size_t>(attn_lmax4(lmax)) * attn_r2(rep) +
                            static_cast<size_t>(rep) * kHD + 5 * kHD + 32) +
           kNS * (sizeof(uint64_t) + 2 * sizeof(uint32_t));
}

__device__ __forceinline__ float dot4(float4 a, float4 b)
{
    float d = a.x * b.x;
    d = fmaf(a.y, b.y, d);
    d = fmaf(a.z, b.z, d);
    return fmaf(a.w, b.w, d);
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// R2 probabilities of one position (row of the [lmax4][R2] buffer).
template <int R2>
__device__ __forceinline__ void load_probs(const float *row, float (&p)[R2])
{
    if constexpr (R2 >= 4) {
#pragma unroll
        for (int i = 0; i < R2; i += 4) {
            const float4 t = reinterpret_cast<const float4 *>(row)[i / 4];
            p[i] = t.x;
            p[i + 1] = t.y;
            p[i + 2] = t.z;
            p[i + 3] = t.w;
        }
    } else if constexpr (R2 == 2) {
        const float2 t = reinterpret_cast<const float2 *>(row)[0];
        p[0] = t.x;
        p[1] = t.y;
    } else {
        p[0] = row[0];
    }
}

// grid (NK, nchunk), kAttnThreads threads, one CTA per SM; R2 = query heads
// per KV head rounded up to a power of two (1, 2, 4 or 8).
//
// Before the programmatic-dependency wait thread 0 starts the ring on the
// cached rows (written by earlier steps, and pos by the previous step's
// argmax: the q/k/v matvec ahead of this kernel lets it start only after its
// own dependency wait, so all of those are complete).  After the wait this
// token's q (and, in the chunk that owns pos, k and v) is loaded, rotated and
// normed while the rows stream in (row pos, this step's, is never read from
// the cache).  Warp w
// takes positions kPW w .. kPW w + kPW - 1 of every block:
//   scores   (K loads) each lane forms the partial dot products of its four
//            dimensions for the warp's (position, head) items; one transposed
//            reduction gives whole scores, lane l holding item l % (kPW R2);
//   softmax  (once, between the K and the V loads) warp h: maximum, sum and
//            probabilities of head h over the chunk;
//   p . V    (V loads) lane l: dimensions 4 l .. 4 l + 3, every head.
// The last warp done with a stage (a shared-memory counter) refills it with
// the load kNS further on.  The warps' o are summed in shared memory into the
// chunk's partial (o, m, l).
template <int R2>
__global__ void __launch_bounds__(kAttnThreads, 1) k_attn_decode(const AttnArgs a)
{
    extern __shared__ __align__(128) uint8_t smraw[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    ATT_STAMP(0);

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
    const int nb = (t1 - t0 + kBP - 1) / kBP;   // blocks of the chunk
    const int nl = 2 * nb;                      // loads: K rows of every block, then V rows
    const int lmax4 = attn_lmax4((a.max_ctx + a.nchunk - 1) / a.nchunk);

    uint8_t *ring = smraw;
    float *sc = reinterpret_cast<float *>(smraw + kNS * kStageBytes);   // [lmax4][R2]
    float *qs = sc + lmax4 * R2;                                         // [rep][HD]
    float *ks = qs + rep * kHD;                                          // [HD]
    float *vnw = ks + kHD;                                               // [HD]
    float *qnw = vnw + kHD;                                              // [HD]
    float *knw = qnw + kHD;                                              // [HD]
    float2 *csr = reinterpret_cast<float2 *>(knw + kHD);                 // [HD/2]
    float *red = reinterpret_cast<float *>(csr + kHD / 2);              // [32]: m, l per head
    uint64_t *full = reinterpret_cast<uint64_t *>(red + 32);             // [kNS]
    unsigned *cnt = reinterpret_cast<unsigned *>(full + kNS);            // [kNS] warps done with a stage
    int *iss = reinterpret_cast<int *>(cnt + kNS);                       // [kNS] last load issued
    __shared__ int s_last;

    const float *kcache = a.kc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    float *kcw = a.kc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    float *vcache = a.vc + static_cast<size_t>(kh) * a.max_ctx * kHD;
    const uint64_t pol = l2_evict_first_policy();

    // ---- the ring: load j (the K rows of block j for j < nb, else the V rows
    // of block j - nb) into stage j % kNS ----
    auto issue = [&](int j, int s) {   // one thread
        const int blk = j < nb ? j : j - nb;
        const int tb = t0 + blk * kBP;
        const int n = max(0, min(tb + kBP, tc) - tb);
        const uint32_t bytes = static_cast<uint32_t>(n) * kHD * sizeof(float);
        const uint32_t bar = smem_u32(full + s);
        mbar_expect_tx(bar, bytes);   // with n == 0 a plain arrival completes the phase
        if (n > 0)
            bulk_g2s(smem_u32(ring + static_cast<size_t>(s) * kStageBytes),
                     (j < nb ? kcache : vcache) + static_cast<size_t>(tb) * kHD, bytes, bar, pol);
    };
    if (tid == 0) {
        for (int u = 0; u < kNS; ++u) {
            mbar_init(smem_u32(full + u), 1);
            cnt[u] = 0u;
            iss[u] = u < nl ? u : -1;
        }
        fence_mbar_init();
        for (int u = 0; u < min(nl, kNS); ++u) issue(u, u);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    ATT_STAMP(1);
    // ---- this token's q (and, in the owner chunk, k and v) and the QK-norm weights ----
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 qv = z4, kn = z4, vn = z4, qnv = z4, knv = z4;
    if (a.qn && tid < kHD / 4) qnv = __ldg(reinterpret_cast<const float4 *>(a.qn) + tid);
    if (owner && a.kn && tid < kHD / 4) knv = __ldg(reinterpret_cast<const float4 *>(a.kn) + tid);
    if (tid < rep * (kHD / 4)) qv = __ldcg(reinterpret_cast<const float4 *>(a.qkv + kh * rep * kHD) + tid);
    if (owner && tid < kHD / 4) {
        kn = __ldcg(reinterpret_cast<const float4 *>(a.qkv + (a.NH + kh) * kHD) + tid);
        vn = __ldcg(reinterpret_cast<const float4 *>(a.qkv + (a.NH + a.NK + kh) * kHD) + tid);
    }

    // ---- q and k normed and rotated in shared memory ----
    if (tid < rep * (kHD / 4)) reinterpret_cast<float4 *>(qs)[tid] = qv;
    if (owner && tid < kHD / 4) {
        reinterpret_cast<float4 *>(ks)[tid] = kn;
        reinterpret_cast<float4 *>(vnw)[tid] = vn;
        reinterpret_cast<float4 *>(knw)[tid] = knv;
    }
    if (tid < kHD / 4) reinterpret_cast<float4 *>(qnw)[tid] = qnv;
    if (tid < 32) red[tid] = (tid & 1) ? 0.f : -1e38f;   // an empty chunk's statistics
    if (tid < kHD / 2) csr[tid] = rope_cs(pos, tid, a.rope_base);
    __syncthreads();
    auto rope_all = [&]() {
        for (int e = tid; e < rep * (kHD / 2); e += kAttnThreads) {
            const int h = e / (kHD / 2), i = e % (kHD / 2);
            rope_rot(qs[h * kHD + 2 * i], qs[h * kHD + 2 * i + 1], csr[i]);
        }
        if (owner && tid < kHD / 2) {
            // reference order: the K head is rotated once per query head mapped
            // to it by h % NK, counted over the whole model (a replicated kv head
            // has fewer query heads on this rank); the Qwen3 order rotates it once
            const int times = a.krot;
            const float2 r = csr[tid];
            for (int u = 0; u < times; ++u) rope_rot(ks[2 * tid], ks[2 * tid + 1], r);
        }
        __syncthreads();
    };
    auto norm_all = [&]() {
        if (a.qn)
            for (int h = warp; h < rep; h += nwarp) head_norm_warp(qs + h * kHD, qnw, a.eps);
        if (owner && a.kn && warp == nwarp - 1) head_norm_warp(ks, knw, a.eps);
        __syncthreads();
    };
    if (a.quirks) {
        rope_all();
        norm_all();
    } else {
        norm_all();
        rope_all();
    }
    if (owner && tid < kHD / 4) {   // append (tb_tensor.c:314-323); the ring never reads row pos
        reinterpret_cast<float4 *>(kcw + static_cast<size_t>(pos) * kHD)[tid] = reinterpret_cast<const float4 *>(ks)[tid];
        reinterpret_cast<float4 *>(vcache + static_cast<size_t>(pos) * kHD)[tid] = vn;
    }

    float4 qr[R2];
#pragma unroll
    for (int h = 0; h < R2; ++h)
        qr[h] = h < rep ? reinterpret_cast<const float4 *>(qs + h * kHD)[lane] : z4;
    const float4 kn4 = owner ? reinterpret_cast<const float4 *>(ks)[lane] : z4;
    const float4 vn4 = owner ? reinterpret_cast<const float4 *>(vnw)[lane] : z4;

    ATT_STAMP(2);
    // ---- the loads: scores from the K rows, the softmax once, p . V from the V rows ----
    constexpr int V = kPW * R2;   // (position, head) items of a warp per block
    float4 acc[R2];
#pragma unroll
    for (int h = 0; h < R2; ++h) acc[h] = z4;
    bool fail = false;
    int s = 0;
    uint32_t par = 0;
    for (int j = 0; j < nl; ++j) {
        if (j == nb) {
            // every score of the chunk is in sc: maximum, probabilities and sum
            // of each head over the chunk, one warp per head
            ATT_STAMP(3);
            __syncthreads();
            const int n = t1 - t0;
            if (warp < rep) {
                const int h = warp;
                float m = -1e38f;
                for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[t * R2 + h]);
                m = warp_max(m);
                float l = 0.f;
                for (int t = lane; t < n; t += 32) {
                    const float p = expf(sc[t * R2 + h] - m);
                    sc[t * R2 + h] = p;
                    l += p;
                }
                l = warp_sum(l);
                if (lane == 0) {
                    red[2 * h] = m;
                    red[2 * h + 1] = l;
                }
            }
            __syncthreads();
            ATT_STAMP(4);
        }
        // a warp whose wait ran out stops consuming (and releasing) loads; the
        // others' waits then run out as well, nothing refills the ring
        fail = fail || !__all_sync(0xFFFFFFFFu, mbar_wait_bounded(smem_u32(full + s), par, a.err, a.wait_limit));
        if (!fail) {
            const float *R = reinterpret_cast<const float *>(ring + static_cast<size_t>(s) * kStageBytes);
            const int blk = j < nb ? j : j - nb;
            const int tb = t0 + blk * kBP;
            const int nv = min(kBP, t1 - tb);   // positions of this block
            if (j < nb) {
                float v[V];
#pragma unroll
                for (int p = 0; p < kPW; ++p) {
                    const int pl = warp * kPW + p;
                    const float4 k4 = (tb + pl == pos) ? kn4 : reinterpret_cast<const float4 *>(R + pl * kHD)[lane];
#pragma unroll
                    for (int h = 0; h < R2; ++h) v[p * R2 + h] = dot4(qr[h], k4);
                }
                const float d = transpose_sum<V>(v);
                const int it = lane % V, p = it / R2, h = it % R2;
                const int pl = warp * kPW + p;
                if (lane < V && h < rep && pl < nv) sc[(blk * kBP + pl) * R2 + h] = d * a.scale;
            } else {
#pragma unroll
                for (int p = 0; p < kPW; ++p) {
                    const int pl = warp * kPW + p;
                    if (pl < nv) {
                        const float4 v4 = (tb + pl == pos) ? vn4 : reinterpret_cast<const float4 *>(R + pl * kHD)[lane];
                        float pr[R2];
                        load_probs<R2>(sc + (blk * kBP + pl) * R2, pr);
#pragma unroll
                        for (int h = 0; h < R2; ++h)
                            if (h < rep) {
                                acc[h].x = fmaf(pr[h], v4.x, acc[h].x);
                                acc[h].y = fmaf(pr[h], v4.y, acc[h].y);
                                acc[h].z = fmaf(pr[h], v4.z, acc[h].z);
                                acc[h].w = fmaf(pr[h], v4.w, acc[h].w);
                            }
                    }
                }
            }
            // the last warp done with this stage refills it with load j + kNS
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                if (atomicAdd(cnt + s, 1u) == static_cast<unsigned>(nwarp) - 1u) {
                    cnt[s] = 0u;
                    __threadfence_block();
                    if (j + kNS < nl) {
                        fence_proxy_async_smem();
                        issue(j + kNS, s);
                        iss[s] = j + kNS;
                    }
                }
            }
        }
        if (++s == kNS) {
            s = 0;
            par ^= 1u;
        }
    }
    if (__syncthreads_or(fail)) {
        // let the copies still in flight land before the ring is reused
        // (bounded; only a stage's last load can be in flight) and hand in an
        // empty partial so the tickets stay consistent; the error word is set
        if (tid == 0)
            for (int u = 0; u < kNS; ++u)
                if (iss[u] >= 0) mbar_wait_bounded(smem_u32(full + u), (iss[u] / kNS) & 1u, nullptr, kAttnDrain);
#pragma unroll
        for (int h = 0; h < R2; ++h) acc[h] = z4;
        if (tid < 16) red[tid] = (tid & 1) ? 0.f : -1e38f;
    }
    __syncthreads();   // every load consumed (or drained): the ring is free
    ATT_STAMP(5);

    // ---- the chunk's partial: o summed over the warps, m and l per head ----
    {
        float4 *pr4 = reinterpret_cast<float4 *>(ring);   // [nwarp][rep][HD/4]
#pragma unroll
        for (int h = 0; h < R2; ++h)
            if (h < rep) pr4[(warp * rep + h) * (kHD / 4) + lane] = acc[h];
        __syncthreads();
        for (int e = tid; e < rep * (kHD / 4); e += kAttnThreads) {
            const int h = e / (kHD / 4), q4 = e % (kHD / 4);
            float4 so = pr4[h * (kHD / 4) + q4];
            for (int u = 1; u < nwarp; ++u) {
                const float4 t = pr4[(u * rep + h) * (kHD / 4) + q4];
                so.x += t.x;
                so.y += t.y;
                so.z += t.z;
                so.w += t.w;
            }
            float *dst = a.part + (static_cast<size_t>(kh * rep + h) * a.nchunk + c) * kPS;
            reinterpret_cast<float4 *>(dst)[q4] = so;
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
    ATT_STAMP(6);
    if (!s_last) return;

    // thread = (output float4 (head, quad), chunk group); each thread merges its
    // chunks with a running maximum (online softmax), all loads of a batch of
    // kCB chunks in flight together; then the groups are merged in shared memory
    constexpr int NO = R2 * 32, NGc = kAttnThreads / NO, kCB = 8;
    const int o = tid % NO, grp = tid / NO, h = o >> 5, q4 = o & 31;
    float Mx = -1e38f, Ls = 0.f;
    float4 oc = make_float4(0.f, 0.f, 0.f, 0.f);
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
            oc = make_float4(oc.x * f, oc.y * f, oc.z * f, oc.w * f);
            Ls *= f;
#pragma unroll
            for (int j = 0; j < kCB; ++j) {
                const float w = expf(mb[j] - Mn);
                oc.x = fmaf(ob[j].x, w, oc.x);
                oc.y = fmaf(ob[j].y, w, oc.y);
                oc.z = fmaf(ob[j].z, w, oc.z);
                oc.w = fmaf(ob[j].w, w, oc.w);
                Ls = fmaf(lb[j], w, Ls);
            }
            Mx = Mn;
        }
    }
    if constexpr (NGc > 1) {
        float4 *gs = reinterpret_cast<float4 *>(ring);   // [NGc][NO][2] float4: (M, L, -, -), o
        gs[2 * (grp * NO + o)] = make_float4(Mx, Ls, 0.f, 0.f);
        gs[2 * (grp * NO + o) + 1] = oc;
        __syncthreads();
        if (grp == 0 && h < rep) {
#pragma unroll
            for (int g = 1; g < NGc; ++g) {
                const float4 ml = gs[2 * (g * NO + o)], og = gs[2 * (g * NO + o) + 1];
                const float Mn = fmaxf(Mx, ml.x);
                const float fa = expf(Mx - Mn), fg = expf(ml.x - Mn);
                oc = make_float4(oc.x * fa + og.x * fg, oc.y * fa + og.y * fg, oc.z * fa + og.z * fg,
                                  oc.w * fa + og.w * fg);
                Ls = Ls * fa + ml.y * fg;
                Mx = Mn;
            }
        }
    }
    if (grp == 0 && h < rep) {
        const float il = Ls > 0.f ? 1.0f / Ls : 0.f;
        reinterpret_cast<float4 *>(a.out + (kh * rep + h) * kHD)[q4] =
            make_float4(oc.x * il, oc.y * il, oc.z * il, oc.w * il);
    }
    ATT_STAMP(7);
    if (tid == 0) a.count[kh] = 0u;   // ready for the next layer / token
}


#if TB_ATTN_STAMPS
// Instrumented builds: every attention launch gets its own slot of 16 stamps per
// CTA (a captured graph keeps the slot of its capture), read back by tb_attn_stamps.
static unsigned long long *g_attn_stamps = nullptr;
static unsigned g_attn_n = 0;
static constexpr unsigned kAttnSlots = 1024, kAttnSlotCtas = 160;
static unsigned long long *attn_stamp_slot()
{
    return g_attn_stamps ? g_attn_stamps + size_t(g_attn_n++ % kAttnSlots) * kAttnSlotCtas * 16 : nullptr;
}
}  // namespace tb
extern "C" int tb_attn_stamps_init()
{
    using namespace tb;
    const size_t n = size_t(kAttnSlots) * kAttnSlotCtas * 16;
    if (!g_attn_stamps && cudaMalloc(&g_attn_stamps, n * 8) != cudaSuccess) return 0;
    g_attn_n = 0;
    return cudaMemset(g_attn_stamps, 0, n * 8) == cudaSuccess;
}
extern "C" int tb_attn_stamps(unsigned long long *host, int max_launches)
{
    using namespace tb;
    if (!g_attn_stamps) return -1;
    const unsigned n = g_attn_n < unsigned(max_launches) ? g_attn_n : unsigned(max_launches);
    cudaDeviceSynchronize();
    cudaMemcpy(host, g_attn_stamps, size_t(n < kAttnSlots ? n : kAttnSlots) * kAttnSlotCtas * 128, cudaMemcpyDeviceToHost);
    return static_cast<int>(g_attn_n);
}
namespace tb {
#endif

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

// Tensor-parallel exchange of the ranks' best (value, vocabulary index)
// pairs; world 1 leaves it unused.
struct ArgTP {
    int rank, world, base;                  // base: this rank's first vocabulary index
    unsigned long long *am[kMaxRanks];      // every rank's pair slots ([world])
    unsigned long long *ctr[kMaxRanks];     // every rank's argmax arrival counter
    const unsigned long long *own_am, *own_ctr;
    int *epoch;                             // steps completed
    uint32_t wait_limit;
    int *err;
};

__device__ __forceinline__ unsigned long long pack_best(ArgBest b)
{
    return (static_cast<unsigned long long>(static_cast<uint32_t>(b.i)) << 32) | __float_as_uint(b.v);
}
__device__ __forceinline__ ArgBest unpack_best(unsigned long long u)
{
    return ArgBest{__uint_as_float(static_cast<uint32_t>(u)), static_cast<int>(u >> 32)};
}

__global__ void __launch_bounds__(kArgThreads) k_argmax_step(const float *logits, int n, float *pv, int *pi,
                                                              unsigned *count, int *token, int *pos, const ArgTP tp)
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
    if (tp.world > 1) {
        // this rank's best to every rank, then the best of all ranks (the
        // first index of the largest value, as on one device)
        const ArgBest mine{b.v, b.i == 0x7FFFFFFF ? 0x7FFFFFFF : tp.base + b.i};
        if (lane < tp.world) tp.am[lane][tp.rank] = pack_best(mine);
        __threadfence_system();
        __syncwarp();
        if (lane < tp.world) atomicAdd_system(tp.ctr[lane], 1ull);
        bool ok = true;
        if (lane == 0 && *reinterpret_cast<volatile int *>(tp.err) == 0)
            ok = wait_counter(tp.own_ctr, static_cast<unsigned long long>(*tp.epoch + 1) * tp.world, tp.wait_limit);
        ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
        if (!ok && lane == 0) atomicExch(tp.err, ERR_WAIT_TIMEOUT);
        b = ArgBest{-FLT_MAX, 0x7FFFFFFF};
        if (lane < tp.world) b = unpack_best(__ldcg(tp.own_am + lane));
        b = warp_best(b);
    }
    if (lane == 0) {
        *token = b.i == 0x7FFFFFFF ? 0 : b.i;
        *pos = *pos + 1;
        if (tp.epoch) *tp.epoch = *tp.epoch + 1;
        *count = 0u;
    }
}

// ---------------------------------------------------------------------------
// Mixture-of-experts routing and combine (layer4/tb_infer.c:351-374, 753-850)
// ---------------------------------------------------------------------------
static constexpr int kMoeThreads = 256;   // experts per router at most (tb_infer.c:254 caps at 256)

// Router: p = softmax(logits) over the E experts (max-shifted, the sum taken
// in expert order as the reference's loop does), the top k experts, and
// their weights renormalised to sum 1 (tb_infer.c:351-374).  Written to
// ids[0..k) / wts[0..k) in rank order: largest probability first, equal
// probabilities by lower expert index.  (The reference's replace-the-minimum
// scan selects the same set except among exactly equal probabilities, and
// lists it in scan order; only the rounding of the weighted sum depends on
// that order.)  A non-finite logit sets the error word and selects nothing.
// Expert parallelism (ep_n > 0): this rank holds experts [ep_lo, ep_lo +
// ep_n); the selected ones among them are also listed, in rank order, as local
// indices lids[0..*nloc) with their weights lw.
__global__ void __launch_bounds__(kMoeThreads) k_moe_topk(const float *logits, int E, int k, int *ids, float *wts,
                                                           int *err, int ep_lo, int ep_n, int *lids, float *lw,
                                                           int *nloc)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ float p[kMoeThreads];
    __shared__ float sel[kMoeThreads];
    __shared__ float red[kMoeThreads / 32];
    __shared__ float s_sum;
    const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
    const float v = e < E ? logits[e] : -FLT_MAX;
    float m = v;
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < kMoeThreads / 32; ++w) m = fmaxf(m, red[w]);
    bool fin = isfinite(m);
    if (e < E) {
        fin = fin && isfinite(v);
        p[e] = expf(v - m);
    }
    const bool all_fin = __syncthreads_and(fin ? 1 : 0) != 0;
    if (!all_fin) {
        if (e == 0) atomicExch(err, ERR_RUNTIME);
        return;
    }
    if (e == 0) {
        float s = 0.f;
        for (int j = 0; j < E; ++j) s += p[j];
        s_sum = s;
    }
    __syncthreads();
    const float q = e < E ? p[e] / s_sum : 0.f;
    __syncthreads();
    if (e < E) p[e] = q;
    __syncthreads();
    if (e < E) {
        int rank = 0;
        for (int j = 0; j < E; ++j) rank += (p[j] > q || (p[j] == q && j < e)) ? 1 : 0;
        if (rank < k) {
            ids[rank] = e;
            sel[rank] = q;
        }
    }
    __syncthreads();
    if (e == 0) {
        float ws = 0.f;
        for (int i = 0; i < k; ++i) ws += sel[i];
        s_sum = ws;
    }
    __syncthreads();
    const float wk = s_sum > 0.f ? sel[e < k ? e : 0] / s_sum : sel[e < k ? e : 0];
    if (e < k) wts[e] = wk;
    if (ep_n > 0) {
        // the local experts in rank order: a ballot over the k ranks (k <= 32 lanes of warp 0)
        if (warp == 0) {
            const int id = e < k ? ids[e] : -1;
            const bool mine = e < k && id >= ep_lo && id < ep_lo + ep_n;
            const unsigned bal = __ballot_sync(0xFFFFFFFFu, mine);
            if (mine) {
                const int j = __popc(bal & ((1u << lane) - 1u));
                lids[j] = id - ep_lo;
                lw[j] = wk;
            }
            if (e == 0) *nloc = __popc(bal);
        }
    }
}

// x[i] = x2[i] + sum_r wts[r] * t[r][i], r in rank order (tb_infer.c:845-848,
// 876: the experts' weighted outputs accumulated, then the residual).
__global__ void __launch_bounds__(kMoeThreads) k_moe_combine(const float *x2, const float *t, const float *wts, int k,
                                                              int H, float *x)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int i = blockIdx.x * kMoeThreads + threadIdx.x;
    if (i >= H) return;
    float acc = 0.f;
    for (int r = 0; r < k; ++r) acc = fmaf(wts[r], t[static_cast<size_t>(r) * H + i], acc);
    x[i] = x2[i] + acc;
}

// The end of an exchange launch: this CTA's stores are fenced at system
// scope before its ticket, and the CTA whose ticket completes the launch
// counts this rank once on each of the world counters.
__device__ __forceinline__ void exchange_arrive(unsigned long long *tk, unsigned long long *const *ctr, int world)
{
    __threadfence_system();
    __syncthreads();
    __shared__ unsigned long long s_t;
    if (threadIdx.x == 0) s_t = atomicAdd(tk, 1ull);
    __syncthreads();
    if ((s_t + 1) % gridDim.x == 0) {
        __threadfence_system();
        if (threadIdx.x < static_cast<unsigned>(world)) atomicAdd_system(ctr[threadIdx.x], 1ull);
    }
}

// Tensor-parallel sampling: this rank's slice of the logits (n values, its
// vocabulary rows [base, base + n)) into every rank's whole-vocabulary buffer
// over NVLink, then each CTA counts itself on every rank's counter; the
// sampler waits for world x gridDim.x arrivals per step.
struct GatherTP {
    float *full[kMaxRanks];
    unsigned long long *ctr[kMaxRanks];
    unsigned long long *tk;
    int world, base;
};
__global__ void __launch_bounds__(256) k_logits_gather(const float *lg, int n, const GatherTP g)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int G = gridDim.x;
    const int i0 = static_cast<int>((static_cast<long long>(n) * blockIdx.x) / G);
    const int i1 = static_cast<int>((static_cast<long long>(n) * (blockIdx.x + 1)) / G);
    for (int i = i0 + static_cast<int>(threadIdx.x); i < i1; i += 256) {
        const float v = lg[i];
        for (int p = 0; p < g.world; ++p) g.full[p][g.base + i] = v;
    }
    exchange_arrive(g.tk, g.ctr, g.world);
}

// Expert-parallel combine: this rank's share sum_{j < *nloc} lw[j] * t[j][i]
// of the routed FFN's output, stored tagged into row `rank` of every rank's
// exchange slots over NVLink (ys[p] + rank * H; one 64-bit word per value, as
// the tensor-parallel matvecs store theirs): the next layer's q/k/v matvec
// waits for the tags and adds the world rows, in rank order, onto x2.
struct CombineEP {
    unsigned long long *ys[kMaxRanks];   // every rank's tagged slot row of this rank
    const int *epoch;                    // tag = epoch * mul + add (mod 2^32)
    unsigned long long mul, add;
    int world;
};

__global__ void __launch_bounds__(kMoeThreads) k_moe_combine_ep(const float *t, const float *lw, const int *nloc,
                                                                 int k, int H, const CombineEP ex)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int n = min(max(*nloc, 0), k);
    const int G = gridDim.x;
    const int i0 = static_cast<int>((static_cast<long long>(H) * blockIdx.x) / G);
    const int i1 = static_cast<int>((static_cast<long long>(H) * (blockIdx.x + 1)) / G);
    const uint32_t tag = static_cast<uint32_t>(static_cast<unsigned long long>(*ex.epoch) * ex.mul + ex.add);
    for (int i = i0 + static_cast<int>(threadIdx.x); i < i1; i += kMoeThreads) {
        float acc = 0.f;
        for (int j = 0; j < n; ++j) acc = fmaf(lw[j], t[static_cast<size_t>(j) * H + i], acc);
        const unsigned long long wv = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(acc);
        for (int p = 0; p < ex.world; ++p)
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(ex.ys[p] + i), "l"(wv) : "memory");
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
    // mixture of experts: router [E][H]; per expert e the (gate, up) row pairs
    // [E][2F][H] (interleaved like wgu) and down [E][H][F]
    const void *wr = nullptr, *wgu_e = nullptr, *wd_e = nullptr;
    int r_qt = -1, gue_qt = -1, de_qt = -1;
};

struct Decoder {
    DecConfig cfg{};
    int dev = 0, sms = 0, nchunk = 1;
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
    // tensor parallelism: cfg holds this rank's shape (heads, FFN rows and
    // vocabulary divided by world); vocab_full is the embedding table's rows.
    int rank = 0, world = 1, vocab_full = 0;
    int krot = 1;   // rotations of each new K row (the whole model's n_heads / n_kv_heads in the reference order)
    // exchange region (own memory, mapped by the peers through CUDA IPC):
    // [o partials world x H][down partials world x H] (tagged 64-bit words)
    // [argmax pairs world]
    // [arrival counters: o, down, argmax, logits][whole-vocabulary logits (sampling)]
    uint8_t *xch = nullptr;
    size_t off_xd = 0, off_am = 0, off_ctr = 0, off_full = 0, xch_bytes = 0;
    uint8_t *peer[kMaxRanks] = {};   // every rank's region, this rank's own included
    bool peer_opened[kMaxRanks] = {};
    int *epoch = nullptr;            // steps completed (device)
    unsigned long long *tk = nullptr;   // ticket counters (device): [2] the logits gather
    // mixture of experts (n_exp > 0): every layer's FFN is routed to top_k of
    // n_exp experts of cfg.ffn_dim rows each
    int n_exp = 0, top_k = 0;
    float *rlog = nullptr, *wts = nullptr, *hbuf = nullptr, *tbuf = nullptr;
    int *ids = nullptr;
    // expert parallelism (routed, world > 1): this rank holds experts
    // [rank * n_loc_exp, (rank + 1) * n_loc_exp); the selected local ones as
    // local indices lids[0..*nloc) with weights lw (rank order)
    int n_loc_exp = 0;
    int *lids = nullptr, *nloc = nullptr;
    float *lw = nullptr;
    // sampling (tb_infer.c:1031-1038): greedy while smp_temp < 0.01, else
    // top-k when smp_k > 0, else the nucleus of smp_p; step i of a run draws
    // the caller's variate u_buf[i] (u_idx counts the steps on the device)
    float smp_temp = 0.f, smp_p = 0.f;
    int smp_k = 0;
    float *u_buf = nullptr;
    SmpScratch smp_scr;   // two-stage top-k candidates (allocated with the variates)
    int *u_idx = nullptr;
    // batched prefill buffers (allocated on the first tb_cuda_dec_prefill)
    PfBufs pf{};
    int *pf_tok = nullptr;
    bool sampling() const { return smp_temp >= 0.01f; }

    unsigned long long *slot_o(int p) const { return reinterpret_cast<unsigned long long *>(peer[p]); }
    float *full_logits(int p) const { return reinterpret_cast<float *>(peer[p] + off_full); }
    unsigned long long *slot_d(int p) const { return reinterpret_cast<unsigned long long *>(peer[p] + off_xd); }
    unsigned long long *am(int p) const { return reinterpret_cast<unsigned long long *>(peer[p] + off_am); }
    unsigned long long *ctr(int p, int k) const { return reinterpret_cast<unsigned long long *>(peer[p] + off_ctr) + k; }
    bool connected() const
    {
        for (int p = 0; p < world; ++p)
            if (!peer[p]) return false;
        return true;
    }

    size_t kv_layer_floats() const
    {
        return static_cast<size_t>(cfg.n_kv_heads) * cfg.max_ctx * cfg.head_dim;
    }
    bool ready() const
    {
        if (!emb || !lm || !out_norm) return false;
        for (int l = 0; l < cfg.n_layers; ++l) {
            const DecLayer &w = layers[l];
            if (!w.wqkv || !w.wo || !w.attn_norm || !w.ffn_norm) return false;
            if (n_exp ? (!w.wr || !w.wgu_e || !w.wd_e) : (!w.wgu || !w.wd)) return false;
        }
        return true;
    }
    bool enqueue(cudaStream_t s);
    bool enqueue_tp(cudaStream_t s);
    bool enqueue_moe(cudaStream_t s, const DecLayer &w);
    bool enqueue_moe_ep(cudaStream_t s, const DecLayer &w, int l, unsigned long long per_x,
                        unsigned long long per_step);
};

// The routed FFN of one layer (tb_infer.c:753-850): router logits of
// rmsnorm(x2), top-k and weights, the k experts' SwiGLU FFNs as two
// expert-group matvecs (each expert on its own CTAs, its weights found from
// the id on the device), then x = x2 + the weighted sum of their outputs.
bool Decoder::enqueue_moe(cudaStream_t s, const DecLayer &w)
{
    const DecConfig &c = cfg;
    const int H = c.hidden, F = c.ffn_dim;
    const uint32_t lim = 1u << 22;
    MvFuse f;
    f.xmode = MV_X_RMSNORM;
    f.nw = w.ffn_norm;
    f.eps = c.norm_eps;
    f.w_early = true;
    if (!mv_launch(w.wr, w.r_qt, n_exp, H, x2, rlog, s, err, sms, lim, &f)) return false;
    if (!launch_pdl(k_moe_topk, dim3(1), dim3(kMoeThreads), 0, s, static_cast<const float *>(rlog), n_exp, top_k,
                    ids, wts, err, 0, 0, static_cast<int *>(nullptr), static_cast<float *>(nullptr),
                    static_cast<int *>(nullptr)))
        return false;
    const Geom gg = geom_of(w.gue_qt), gd = geom_of(w.de_qt);
    f = MvFuse{};
    f.xmode = MV_X_RMSNORM;
    f.nw = w.ffn_norm;
    f.eps = c.norm_eps;
    f.ymode = MV_Y_SWIGLU_PAIRS;
    f.ng = static_cast<uint32_t>(top_k);
    f.n_experts = static_cast<uint32_t>(n_exp);
    f.ids = ids;
    f.w_stride = 2ull * F * (H / gg.block_weights) * gg.block_bytes;
    f.y_stride = static_cast<uint32_t>(F);
    if (!mv_launch(w.wgu_e, w.gue_qt, 2 * F, H, x2, hbuf, s, err, sms, lim, &f)) return false;
    f = MvFuse{};
    f.ng = static_cast<uint32_t>(top_k);
    f.n_experts = static_cast<uint32_t>(n_exp);
    f.ids = ids;
    f.w_stride = static_cast<unsigned long long>(H) * (F / gd.block_weights) * gd.block_bytes;
    f.x_stride = static_cast<uint32_t>(F);
    f.y_stride = static_cast<uint32_t>(H);
    if (!mv_launch(w.wd_e, w.de_qt, H, F, hbuf, tbuf, s, err, sms, lim, &f)) return false;
    return launch_pdl(k_moe_combine, dim3((H + kMoeThreads - 1) / kMoeThreads), dim3(kMoeThreads), 0, s,
                      static_cast<const float *>(x2), static_cast<const float *>(tbuf),
                      static_cast<const float *>(wts), top_k, H, x);
}

// The routed FFN of one layer under expert parallelism (world > 1): the
// router (replicated, all n_exp experts) on rmsnorm(x2), x2 = x + the o
// partials (gathered here, its CTA 0 writing x2); the top k; this rank's
// selected experts' gate/up and down as expert groups whose count is read on
// the device (the whole grid shared among them); then this rank's weighted
// share of the FFN output to every rank (k_moe_combine_ep), which the next
// q/k/v matvec gathers like the down partials of the dense step.
bool Decoder::enqueue_moe_ep(cudaStream_t s, const DecLayer &w, int l, unsigned long long per_x,
                             unsigned long long per_step)
{
    const DecConfig &c = cfg;
    const int H = c.hidden, F = c.ffn_dim;
    const uint32_t lim = 1u << 22;
    MvFuse f;
    f.xmode = MV_X_RMSNORM;
    f.nw = w.ffn_norm;
    f.eps = c.norm_eps;
    f.w_early = true;
    f.xs = slot_o(rank);
    f.nsl = static_cast<uint32_t>(world);
    f.xs_epoch = epoch;
    f.xs_mul = per_step;
    f.xs_add = static_cast<unsigned long long>(l + 1) * per_x;
    f.xout = x2;
    if (!mv_launch(w.wr, w.r_qt, n_exp, H, x, rlog, s, err, sms, lim, &f)) return false;
    if (!launch_pdl(k_moe_topk, dim3(1), dim3(kMoeThreads), 0, s, static_cast<const float *>(rlog), n_exp, top_k,
                    ids, wts, err, rank * n_loc_exp, n_loc_exp, lids, lw, nloc))
        return false;
    const Geom gg = geom_of(w.gue_qt), gd = geom_of(w.de_qt);
    f = MvFuse{};
    f.xmode = MV_X_RMSNORM;
    f.nw = w.ffn_norm;
    f.eps = c.norm_eps;
    f.ymode = MV_Y_SWIGLU_PAIRS;
    f.ng = static_cast<uint32_t>(top_k);
    f.ng_dev = nloc;
    f.n_experts = static_cast<uint32_t>(n_loc_exp);
    f.ids = lids;
    f.w_stride = 2ull * F * (H / gg.block_weights) * gg.block_bytes;
    f.y_stride = static_cast<uint32_t>(F);
    if (!mv_launch(w.wgu_e, w.gue_qt, 2 * F, H, x2, hbuf, s, err, sms, lim, &f)) return false;
    f = MvFuse{};
    f.ng = static_cast<uint32_t>(top_k);
    f.ng_dev = nloc;
    f.n_experts = static_cast<uint32_t>(n_loc_exp);
    f.ids = lids;
    f.w_stride = static_cast<unsigned long long>(H) * (F / gd.block_weights) * gd.block_bytes;
    f.x_stride = static_cast<uint32_t>(F);
    f.y_stride = static_cast<uint32_t>(H);
    if (!mv_launch(w.wd_e, w.de_qt, H, F, hbuf, tbuf, s, err, sms, lim, &f)) return false;
    CombineEP ex{};
    ex.world = world;
    ex.epoch = epoch;
    ex.mul = per_step;
    ex.add = static_cast<unsigned long long>(l + 1) * per_x;   // the next layer's q/k/v (or the output) reads it
    for (int p = 0; p < world; ++p) ex.ys[p] = slot_d(p) + static_cast<size_t>(rank) * H;
    const int G = H < sms ? H : sms;
    return launch_pdl(k_moe_combine_ep, dim3(G), dim3(kMoeThreads), 0, s, static_cast<const float *>(tbuf),
                      static_cast<const float *>(lw), static_cast<const int *>(nloc), top_k, H, ex);
}

bool Decoder::enqueue(cudaStream_t s)
{
    if (world > 1) return enqueue_tp(s);
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
        a.wait_limit = lim;
        a.quirks = c.quirks;
        a.krot = krot;
        a.eps = c.norm_eps;
        a.rope_base = c.rope_base;
        a.scale = 1.0f / sqrtf(static_cast<float>(HD));
        const size_t smem = attn_smem_bytes(NH / NK, (c.max_ctx + nchunk - 1) / nchunk);
#if TB_ATTN_STAMPS
        a.stamp = attn_stamp_slot();
#endif
        if (!launch_pdl(attn_kernel(NH / NK), dim3(NK, nchunk), dim3(kAttnThreads), smem, s, a)) return false;
        // x2 = x + Wo @ att
        f = MvFuse{};
        f.res = x;
        f.w_early = true;
        if (!mv_launch(w.wo, w.o_qt, H, NH * HD, att, x2, s, err, sms, lim, &f)) return false;
        if (n_exp) {
            if (!enqueue_moe(s, w)) return false;
            continue;
        }
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
    if (sampling())
        return sample_launch(logits, c.vocab, smp_k, smp_p, smp_temp, 0.f, tok, err, s, u_buf, u_idx, pos, nullptr,
                             &smp_scr) != 0;
    const int G = sms;
    ArgTP tp{};
    tp.world = 1;
    return launch_pdl(k_argmax_step, dim3(G), dim3(kArgThreads), 0, s, static_cast<const float *>(logits),
                      c.vocab, argv, argi, counts + NK, tok, pos, tp);
}

// Tensor-parallel step (world > 1).  q/k/v and gate/up hold this rank's heads
// and FFN row pairs, attention is local; o and down hold this rank's K slice
// and write their partial y into every rank's slots over NVLink.  The next
// matvec sums the world partials (rank order, so every rank gets the same
// bits) onto the residual, each slot word waited for until it carries this
// exchange's tag, and its CTA 0 writes the new residual.  Residual stream: x
// (after the down exchange) and x2 (after the o exchange), alternating.  Tags
// follow the device-side step count: the o and down exchanges of layer l in
// step e carry (e L + l + 1) world (mod 2^32), each kind in its own slots, so
// a word left from an earlier exchange never matches.
bool Decoder::enqueue_tp(cudaStream_t s)
{
    const DecConfig &c = cfg;
    const int H = c.hidden, NH = c.n_heads, NK = c.n_kv_heads, HD = c.head_dim, F = c.ffn_dim, L = c.n_layers;
    const int QKV = (NH + 2 * NK) * HD;
    const uint32_t lim = 1u << 22;
    const unsigned long long per_x = static_cast<unsigned long long>(world);   // tag step of a layer
    const unsigned long long per_step = static_cast<unsigned long long>(L) * per_x;
    auto gather_in = [&](MvFuse &f, int kind, unsigned long long add, float *xout) {
        f.xs = kind == 0 ? slot_o(rank) : slot_d(rank);
        f.nsl = static_cast<uint32_t>(world);
        f.xs_epoch = epoch;
        f.xs_mul = per_step;
        f.xs_add = add;
        f.xout = xout;
    };
    auto scatter_out = [&](MvFuse &f, int kind, unsigned long long add) {
        f.ny = static_cast<uint32_t>(world);
        for (int p = 0; p < world; ++p) f.ys[p] = (kind == 0 ? slot_o(p) : slot_d(p)) + static_cast<size_t>(rank) * H;
        f.y_epoch = epoch;
        f.y_mul = per_step;
        f.y_add = add;
    };
    if (!dq_embed_launch(emb, emb_qt, vocab_full, H, tok, x, s)) return false;
    for (int l = 0; l < L; ++l) {
        const DecLayer &w = layers[l];
        MvFuse f;
        // q | k | v of this rank's heads = Wqkv @ rmsnorm(x), x = x2 + the down partials
        f = MvFuse{};
        f.xmode = MV_X_RMSNORM;
        f.nw = w.attn_norm;
        f.eps = c.norm_eps;
        f.w_early = true;
        if (l > 0) gather_in(f, 1, static_cast<unsigned long long>(l) * per_x, x);
        if (!mv_launch(w.wqkv, w.qkv_qt, QKV, H, l > 0 ? x2 : x, qkv, s, err, sms, lim, &f)) return false;
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
        a.wait_limit = lim;
        a.quirks = c.quirks;
        a.krot = krot;
        a.eps = c.norm_eps;
        a.rope_base = c.rope_base;
        a.scale = 1.0f / sqrtf(static_cast<float>(HD));
        const size_t smem = attn_smem_bytes(NH / NK, (c.max_ctx + nchunk - 1) / nchunk);
#if TB_ATTN_STAMPS
        a.stamp = attn_stamp_slot();
#endif
        if (!launch_pdl(attn_kernel(NH / NK), dim3(NK, nchunk), dim3(kAttnThreads), smem, s, a)) return false;
        // this rank's share of Wo @ att to every rank
        f = MvFuse{};
        f.w_early = true;
        scatter_out(f, 0, static_cast<unsigned long long>(l + 1) * per_x);
        if (!mv_launch(w.wo, w.o_qt, H, NH * HD, att, x2, s, err, sms, lim, &f)) return false;
        if (n_exp) {
            if (!enqueue_moe_ep(s, w, l, per_x, per_step)) return false;
            continue;
        }
        // act = swiglu(gate, up) of this rank's rows, of rmsnorm(x2), x2 = x + the o partials
        f = MvFuse{};
        f.xmode = MV_X_RMSNORM;
        f.nw = w.ffn_norm;
        f.eps = c.norm_eps;
        f.ymode = MV_Y_SWIGLU_PAIRS;
        f.w_early = true;
        gather_in(f, 0, static_cast<unsigned long long>(l + 1) * per_x, x2);
        if (!mv_launch(w.wgu, w.gu_qt, 2 * F, H, x, gu, s, err, sms, lim, &f)) return false;
        // this rank's share of Wd @ act to every rank
        f = MvFuse{};
        f.w_early = true;
        scatter_out(f, 1, static_cast<unsigned long long>(l + 1) * per_x);
        if (!mv_launch(w.wd, w.d_qt, H, F, gu, x, s, err, sms, lim, &f)) return false;
    }
    MvFuse f;
    f.xmode = MV_X_RMSNORM;
    f.nw = out_norm;
    f.eps = c.norm_eps;
    f.w_early = true;
    gather_in(f, 1, static_cast<unsigned long long>(L) * per_x, nullptr);
    if (!mv_launch(lm, lm_qt, c.vocab, H, x2, logits, s, err, sms, lim, &f)) return false;
    if (sampling()) {
        // every rank gathers the whole vocabulary's logits and samples them with
        // the same variate, so all ranks take the same token
        GatherTP g{};
        g.world = world;
        g.base = rank * c.vocab;
        g.tk = tk + 2;
        for (int p = 0; p < world; ++p) {
            g.full[p] = full_logits(p);
            g.ctr[p] = ctr(p, 3);
        }
        const int G = sms;
        if (!launch_pdl(k_logits_gather, dim3(G), dim3(256), 0, s, static_cast<const float *>(logits), c.vocab, g))
            return false;
        SmpTP tp{};
        tp.ctr = ctr(rank, 3);
        tp.epoch = epoch;
        tp.per_step = static_cast<unsigned long long>(world);
        tp.wait_limit = lim;
        return sample_launch(full_logits(rank), vocab_full, smp_k, smp_p, smp_temp, 0.f, tok, err, s, u_buf, u_idx,
                             pos, &tp, &smp_scr) != 0;
    }
    ArgTP tp{};
    tp.rank = rank;
    tp.world = world;
    tp.base = rank * c.vocab;
    for (int p = 0; p < world; ++p) {
        tp.am[p] = am(p);
        tp.ctr[p] = ctr(p, 2);
    }
    tp.own_am = am(rank);
    tp.own_ctr = ctr(rank, 2);
    tp.epoch = epoch;
    tp.wait_limit = lim;
    tp.err = err;
    const int G = sms;
    return launch_pdl(k_argmax_step, dim3(G), dim3(kArgThreads), 0, s, static_cast<const float *>(logits), c.vocab,
                      argv, argi, counts + NK, tok, pos, tp);
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
    void *bufs[] = {d->x,    d->x2,  d->qkv, d->att, d->gu,     d->logits, d->kc,   d->vc,   d->part,
                    d->argv, d->argi, d->tok, d->pos, d->counts, d->err,    d->rlog, d->wts, d->hbuf,
                    d->tbuf, d->ids, d->u_buf, d->u_idx, d->lids, d->lw, d->nloc,
                    d->smp_scr.cv, d->smp_scr.ci, d->smp_scr.nonfin};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (d->hostio) cudaFreeHost(d->hostio);
    for (int p = 0; p < kMaxRanks; ++p)
        if (d->peer_opened[p]) cudaIpcCloseMemHandle(d->peer[p]);
    if (d->xch) cudaFree(d->xch);
    if (d->epoch) cudaFree(d->epoch);
    if (d->tk) cudaFree(d->tk);
    for (void *b : {static_cast<void *>(d->pf.X), static_cast<void *>(d->pf.QKV), static_cast<void *>(d->pf.Y),
                    static_cast<void *>(d->pf.GU), d->pf.A, d->pf.AO, d->pf.ACT, static_cast<void *>(d->pf_tok)})
        if (b) cudaFree(b);
    delete[] d->layers;
    delete d;
}

// full: the whole model's shape; rank / world: this process's share
// (world 1 = the whole model on one device).
Decoder *dec_create(const DecConfig &full, int rank, int world, int n_exp = 0, int top_k = 0)
{
    if (n_exp < 0 || n_exp > kMoeThreads ||
        (n_exp && (top_k < 1 || top_k > n_exp || top_k > 32 || n_exp % world))) {
        fprintf(stderr, "[tb_cuda] decoder: unsupported experts (%d, top %d; at most %d experts and top 32, "
                        "a whole number per rank)\n", n_exp, top_k, kMoeThreads);
        return nullptr;
    }
    // kv heads: split over the ranks, or (world a multiple of n_kv_heads) each
    // held by world / n_kv_heads ranks, every rank computing its q heads' share
    const bool kv_split = full.n_kv_heads > 0 && full.n_kv_heads % world == 0;
    const bool kv_repl = full.n_kv_heads > 0 && world % full.n_kv_heads == 0;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || full.n_heads % world ||
        !(kv_split || kv_repl) || (!n_exp && full.ffn_dim % world) || full.vocab % world) {
        fprintf(stderr, "[tb_cuda] decoder: rank %d of %d does not divide the heads, FFN rows and vocabulary\n",
                rank, world);
        return nullptr;
    }
    DecConfig c = full;
    c.n_heads /= world;
    c.n_kv_heads = kv_split ? full.n_kv_heads / world : 1;
    if (!n_exp) c.ffn_dim /= world;   // routed: whole experts per rank, each of ffn_dim rows
    c.vocab /= world;
    if (c.n_layers <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim != kHD ||
        c.n_heads % c.n_kv_heads || c.n_heads / c.n_kv_heads > 8 || c.ffn_dim <= 0 || c.vocab <= 0 ||
        c.max_ctx <= 0) {
        fprintf(stderr, "[tb_cuda] decoder: unsupported configuration (head_dim must be %d, n_heads/n_kv_heads <= 8)\n", kHD);
        return nullptr;
    }
    Decoder *d = new Decoder;
    d->cfg = c;
    d->krot = c.quirks ? full.n_heads / full.n_kv_heads : 1;
    d->rank = rank;
    d->world = world;
    d->vocab_full = full.vocab;
    d->layers = new DecLayer[c.n_layers];
    cudaGetDevice(&d->dev);
    cudaDeviceGetAttribute(&d->sms, cudaDevAttrMultiProcessorCount, d->dev);
    // context chunks: one wave of one attention CTA per SM over all KV heads,
    // more if a chunk's scores would not fit the shared memory left by the ring
    d->nchunk = d->sms / c.n_kv_heads;
    if (d->nchunk < 1) d->nchunk = 1;
    {
        const int rep = c.n_heads / c.n_kv_heads;
        const long long room = static_cast<long long>(kSmemCap) - static_cast<long long>(attn_smem_bytes(rep, 0));
        const int lcap = static_cast<int>(room / (static_cast<long long>(sizeof(float)) * attn_r2(rep))) & ~3;
        if (lcap < 4) {
            fprintf(stderr, "[tb_cuda] decoder: attention does not fit shared memory\n");
            dec_free(d);
            return nullptr;
        }
        const int need = (c.max_ctx + lcap - 1) / lcap;
        if (d->nchunk < need) d->nchunk = need;
    }
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
    if (ok && n_exp) {
        d->n_exp = n_exp;
        d->top_k = top_k;
        ok = dec_ok(cudaMalloc(&d->rlog, sizeof(float) * n_exp), "router logits") &&
             dec_ok(cudaMalloc(&d->wts, sizeof(float) * top_k), "expert weights") &&
             dec_ok(cudaMalloc(&d->ids, sizeof(int) * top_k), "expert ids") &&
             dec_ok(cudaMalloc(&d->hbuf, sizeof(float) * static_cast<size_t>(top_k) * c.ffn_dim), "expert act") &&
             dec_ok(cudaMalloc(&d->tbuf, sizeof(float) * static_cast<size_t>(top_k) * c.hidden), "expert out");
        if (ok && world > 1) {
            d->n_loc_exp = n_exp / world;
            ok = dec_ok(cudaMalloc(&d->lids, sizeof(int) * top_k), "local expert ids") &&
                 dec_ok(cudaMalloc(&d->lw, sizeof(float) * top_k), "local expert weights") &&
                 dec_ok(cudaMalloc(&d->nloc, sizeof(int)), "local expert count") &&
                 dec_ok(cudaMemset(d->nloc, 0, sizeof(int)), "memset");
        }
    }
    if (ok && world > 1) {
        // the exchange region, 256-byte aligned parts; CUDA IPC maps whole allocations
        auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
        const size_t slots = up(sizeof(unsigned long long) * static_cast<size_t>(world) * c.hidden);   // tagged words
        d->off_xd = slots;
        d->off_am = 2 * slots;
        d->off_ctr = d->off_am + up(sizeof(unsigned long long) * world);
        d->off_full = d->off_ctr + up(4 * sizeof(unsigned long long));
        d->xch_bytes = d->off_full + up(sizeof(float) * static_cast<size_t>(full.vocab));
        ok = dec_ok(cudaMalloc(&d->xch, d->xch_bytes), "exchange region") &&
             dec_ok(cudaMemset(d->xch, 0, d->xch_bytes), "memset") &&
             dec_ok(cudaMalloc(&d->epoch, sizeof(int)), "epoch") &&
             dec_ok(cudaMemset(d->epoch, 0, sizeof(int)), "memset") &&
             dec_ok(cudaMalloc(&d->tk, 4 * sizeof(unsigned long long)), "tickets") &&
             dec_ok(cudaMemset(d->tk, 0, 4 * sizeof(unsigned long long)), "memset");
        d->peer[rank] = d->xch;
    }
    if (ok) {
        ok = dec_ok(cudaMemset(d->counts, 0, sizeof(unsigned) * (NK + 1)), "memset") &&
             dec_ok(cudaMemset(d->err, 0, sizeof(int)), "memset") &&
             dec_ok(cudaMemset(d->kc, 0, sizeof(float) * kvf), "memset") &&
             dec_ok(cudaMemset(d->vc, 0, sizeof(float) * kvf), "memset");
        const size_t smem = attn_smem_bytes(NH / NK, (c.max_ctx + d->nchunk - 1) / d->nchunk);
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
    const NvtxRange nvtx("tb.decode.capture");
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

// Runs n tokens back to back from (token, pos): token_i+1 = the token step i
// picks (greedy, or sampled with the variate u[i] when sampling is set).
// tokens[i] receives each generated token when not null; ms receives the device
// time of the n replays (CUDA events on the decoder's stream).
int dec_run(Decoder *d, int token, int pos, int n, int *tokens, float *logits_host, float *ms,
            const float *u = nullptr)
{
    const NvtxRange nvtx("tb.decode.steps");
    if (!d || n <= 0 || token < 0 || token >= d->vocab_full || pos < 0 || pos + n > d->cfg.max_ctx) return 0;
    if (d->sampling()) {
        if (!u) {
            fprintf(stderr, "[tb_cuda] decoder: sampling is set: pass the variates (tb_cuda_dec_generate_u)\n");
            return 0;
        }
        for (int i = 0; i < n; ++i)
            if (!(u[i] >= 0.f && u[i] < 1.f)) {
                fprintf(stderr, "[tb_cuda] decoder: variate %d outside [0, 1)\n", i);
                return 0;
            }
        if (!dec_ok(cudaMemcpyAsync(d->u_buf, u, sizeof(float) * n, cudaMemcpyHostToDevice, d->st), "variates") ||
            !dec_ok(cudaMemsetAsync(d->u_idx, 0, sizeof(int), d->st), "variates"))
            return 0;
    }
    if (d->world > 1 && !d->connected()) {
        fprintf(stderr, "[tb_cuda] decoder: tensor-parallel ranks not connected (tb_cuda_dec_tp_connect)\n");
        return 0;
    }
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
    return tb::dec_create(k, 0, 1);
}

void *tb_cuda_dec_create_tp(const tb_dec_config *c, int rank, int world)
{
    if (!c) return nullptr;
    tb::DecConfig k{c->n_layers, c->hidden, c->n_heads, c->n_kv_heads, c->head_dim, c->ffn_dim,
                    c->vocab, c->max_ctx, c->rope_base, c->norm_eps, c->quirks};
    return tb::dec_create(k, rank, world);
}

void *tb_cuda_dec_create_moe(const tb_dec_config *c, int n_experts, int top_k)
{
    if (!c || n_experts < 1) return nullptr;
    tb::DecConfig k{c->n_layers, c->hidden, c->n_heads, c->n_kv_heads, c->head_dim, c->ffn_dim,
                    c->vocab, c->max_ctx, c->rope_base, c->norm_eps, c->quirks};
    return tb::dec_create(k, 0, 1, n_experts, top_k);
}

void *tb_cuda_dec_create_moe_tp(const tb_dec_config *c, int n_experts, int top_k, int rank, int world)
{
    if (!c || n_experts < 1 || world < 2) return nullptr;
    tb::DecConfig k{c->n_layers, c->hidden, c->n_heads, c->n_kv_heads, c->head_dim, c->ffn_dim,
                    c->vocab, c->max_ctx, c->rope_base, c->norm_eps, c->quirks};
    return tb::dec_create(k, rank, world, n_experts, top_k);
}

int tb_cuda_dec_set_moe_layer(void *dec, int layer, const void *w_router, int router_qtype,
                              const void *w_gate_up_exps, int gate_up_qtype, const void *w_down_exps,
                              int down_qtype)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !d->n_exp || layer < 0 || layer >= d->cfg.n_layers || !w_router || !w_gate_up_exps || !w_down_exps)
        return 0;
    for (int qt : {router_qtype, gate_up_qtype, down_qtype})
        if (!tb::geom_of(qt).block_weights) return 0;
    if (d->cfg.hidden % tb::geom_of(router_qtype).block_weights || d->cfg.hidden % tb::geom_of(gate_up_qtype).block_weights ||
        d->cfg.ffn_dim % tb::geom_of(down_qtype).block_weights)
        return 0;
    tb::DecLayer &l = d->layers[layer];
    l.wr = w_router;
    l.r_qt = router_qtype;
    l.wgu_e = w_gate_up_exps;
    l.gue_qt = gate_up_qtype;
    l.wd_e = w_down_exps;
    l.de_qt = down_qtype;
    if (d->gexec) {
        cudaGraphExecDestroy(d->gexec);
        d->gexec = nullptr;
    }
    return 1;
}

int tb_cuda_dec_tp_handle(void *dec, void *handle_out)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !handle_out || d->world < 2 || !d->xch) return 0;
    cudaIpcMemHandle_t h;
    if (!tb::dec_ok(cudaIpcGetMemHandle(&h, d->xch), "ipc handle")) return 0;
    memcpy(handle_out, &h, sizeof(h));
    return 1;
}

int tb_cuda_dec_tp_connect(void *dec, const void *handles)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !handles || d->world < 2) return 0;
    const uint8_t *hb = static_cast<const uint8_t *>(handles);
    for (int p = 0; p < d->world; ++p) {
        if (p == d->rank || d->peer_opened[p]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + static_cast<size_t>(p) * sizeof(h), sizeof(h));
        void *ptr = nullptr;
        if (!tb::dec_ok(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc open")) return 0;
        d->peer[p] = static_cast<uint8_t *>(ptr);
        d->peer_opened[p] = true;
    }
    if (d->gexec) {   // peers changed: capture again on the next step
        cudaGraphExecDestroy(d->gexec);
        d->gexec = nullptr;
    }
    return 1;
}

int tb_cuda_dec_set_layer(void *dec, int layer, const tb_dec_layer *w)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !w || layer < 0 || layer >= d->cfg.n_layers) return 0;
    for (int qt : {w->qkv_qtype, w->o_qtype})
        if (!tb::geom_of(qt).block_weights) return 0;
    if (!d->n_exp)   // a routed decoder takes its FFN from tb_cuda_dec_set_moe_layer
        for (int qt : {w->gate_up_qtype, w->down_qtype})
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

int tb_cuda_dec_generate_u(void *dec, int token, int pos, int n, const float *u, int *tokens_out,
                           float *logits_host, float *device_ms)
{
    return tb::dec_run(static_cast<tb::Decoder *>(dec), token, pos, n, tokens_out, logits_host, device_ms, u);
}

int tb_cuda_dec_set_sampling(void *dec, float temperature, int top_k, float top_p)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !(temperature == temperature) || top_k < 0) return 0;
    const bool smp = temperature >= 0.01f;
    if (smp) {
        if ((top_k > 0 && top_k < d->vocab_full && top_k > 2048) || (top_k == 0 && !(top_p > 0.f && top_p <= 1.f)))
            return 0;
        if (!d->u_buf &&
            !(tb::dec_ok(cudaMalloc(&d->u_buf, sizeof(float) * d->cfg.max_ctx), "variates") &&
              tb::dec_ok(cudaMalloc(&d->u_idx, sizeof(int)), "variates")))
            return 0;
        if (!d->smp_scr.cv &&   // without it top-k runs in one CTA
            !(tb::dec_ok(cudaMalloc(&d->smp_scr.cv, sizeof(float) * tb::kSmpPreCap), "top-k candidates") &&
              tb::dec_ok(cudaMalloc(&d->smp_scr.ci, sizeof(int) * tb::kSmpPreCap), "top-k candidates") &&
              tb::dec_ok(cudaMalloc(&d->smp_scr.nonfin, sizeof(int)), "top-k candidates") &&
              tb::dec_ok(cudaMemset(d->smp_scr.nonfin, 0, sizeof(int)), "top-k candidates")))
            d->smp_scr.cv = nullptr;
    }
    if (d->sampling() != smp || (smp && (d->smp_temp != temperature || d->smp_k != top_k || d->smp_p != top_p))) {
        if (d->gexec) {   // the last kernel changes: capture again on the next step
            cudaGraphExecDestroy(d->gexec);
            d->gexec = nullptr;
        }
    }
    d->smp_temp = smp ? temperature : 0.f;
    d->smp_k = top_k;
    d->smp_p = top_p;
    return 1;
}

int tb_cuda_dec_prefill(void *dec, const int *tokens, int n, int pos0, int *next_token, float *logits_host)
{
    tb::Decoder *d = static_cast<tb::Decoder *>(dec);
    if (!d || !tokens || n < 1 || pos0 < 0 || pos0 + n > d->cfg.max_ctx) return 0;
    const tb::DecConfig &c = d->cfg;
    if (d->world != 1 || d->n_exp || !d->ready()) {
        fprintf(stderr, "[tb_cuda] decoder: prefill needs a dense single-device decoder with its tensors set\n");
        return 0;
    }
    const int H = c.hidden, NH = c.n_heads, NK = c.n_kv_heads, F = c.ffn_dim;
    for (int l = 0; l < c.n_layers; ++l) {
        const tb::DecLayer &w = d->layers[l];
        if (!tb::pf_supported(w.qkv_qt, (NH + 2 * NK) * 128, H) || !tb::pf_supported(w.o_qt, H, NH * 128) ||
            !tb::pf_supported(w.gu_qt, 2 * F, H) || !tb::pf_supported(w.d_qt, H, F)) {
            fprintf(stderr, "[tb_cuda] decoder: prefill needs Q4_K / Q6_K projections the tensor-core GEMM takes "
                            "(rows a multiple of 128, K of 256, row bytes of 16)\n");
            return 0;
        }
    }
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= d->vocab_full) return 0;
    constexpr int kT = 512;   // tokens per chunk (the GEMM's largest T)
    tb::PfBufs &b = d->pf;
    if (!b.X) {
        const size_t r = kT;
        const bool ok = tb::dec_ok(cudaMalloc(&b.X, sizeof(float) * r * H), "prefill") &&
                        tb::dec_ok(cudaMalloc(&b.QKV, sizeof(float) * r * (NH + 2 * NK) * 128), "prefill") &&
                        tb::dec_ok(cudaMalloc(&b.Y, sizeof(float) * r * H), "prefill") &&
                        tb::dec_ok(cudaMalloc(&b.GU, sizeof(float) * r * 2 * F), "prefill") &&
                        tb::dec_ok(cudaMalloc(&b.A, 2 * r * H), "prefill") &&
                        tb::dec_ok(cudaMalloc(&b.AO, 2 * r * NH * 128), "prefill") &&
                        tb::dec_ok(cudaMalloc(&b.ACT, 2 * r * F), "prefill") &&
                        tb::dec_ok(cudaMalloc(&d->pf_tok, sizeof(int) * r), "prefill");
        if (!ok) return 0;
    }
    const tb::NvtxRange nvtx("tb.decode.prefill");
    tb::PfShape ps{H, NH, NK, F, c.max_ctx, c.quirks, c.norm_eps, c.rope_base};
    cudaStream_t s = d->st;
    int last = 0;
    for (int c0 = 0; c0 < n; c0 += kT) {
        const int T = n - c0 < kT ? n - c0 : kT, Tp = (T + 15) & ~15;
        if (!tb::dec_ok(cudaMemcpyAsync(d->pf_tok, tokens + c0, sizeof(int) * T, cudaMemcpyHostToDevice, s),
                        "prefill tokens") ||
            !tb::dq_embed_launch(d->emb, d->emb_qt, d->vocab_full, H, d->pf_tok, b.X, s, T))
            return 0;
        for (int l = 0; l < c.n_layers; ++l) {
            const tb::DecLayer &w = d->layers[l];
            tb::PfLayer pl{w.wqkv, w.wo, w.wgu, w.wd, w.qkv_qt, w.o_qt, w.gu_qt, w.d_qt, w.attn_norm, w.ffn_norm,
                           w.q_norm, w.k_norm, d->kc + static_cast<size_t>(l) * d->kv_layer_floats(),
                           d->vc + static_cast<size_t>(l) * d->kv_layer_floats()};
            if (!tb::pf_layer(pl, ps, b, pos0 + c0, T, Tp, s, d->err, d->sms)) return 0;
        }
        last = T - 1;
        // the host token buffer is read by the copy above before the next chunk's copy
        if (!tb::dec_ok(cudaStreamSynchronize(s), "prefill")) return 0;
    }
    // the last token's residual is the decode step's x: the final norm, the
    // output matvec and the greedy argmax (which advances pos to pos0 + n)
    d->hostio[1] = pos0 + n - 1;
    if (!tb::dec_ok(cudaMemcpyAsync(d->x, b.X + static_cast<size_t>(last) * H, sizeof(float) * H,
                                    cudaMemcpyDeviceToDevice, s), "prefill x") ||
        !tb::dec_ok(cudaMemcpyAsync(d->pos, &d->hostio[1], sizeof(int), cudaMemcpyHostToDevice, s), "prefill pos"))
        return 0;
    tb::MvFuse f;
    f.xmode = tb::MV_X_RMSNORM;
    f.nw = d->out_norm;
    f.eps = c.norm_eps;
    if (!tb::mv_launch(d->lm, d->lm_qt, c.vocab, H, d->x, d->logits, s, d->err, d->sms, 1u << 22, &f)) return 0;
    tb::ArgTP tp{};
    tp.world = 1;
    if (!tb::launch_pdl(tb::k_argmax_step, dim3(d->sms), dim3(tb::kArgThreads), 0, s,
                        static_cast<const float *>(d->logits), c.vocab, d->argv, d->argi, d->counts + NK, d->tok,
                        d->pos, tp))
        return 0;
    if (logits_host)
        cudaMemcpyAsync(logits_host, d->logits, sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, s);
    cudaMemcpyAsync(&d->hostio[0], d->tok, sizeof(int), cudaMemcpyDeviceToHost, s);
    cudaMemcpyAsync(&d->hostio[2], d->err, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (!tb::dec_ok(cudaStreamSynchronize(s), "prefill")) return 0;
    if (d->hostio[2]) {
        fprintf(stderr, "[tb_cuda] decoder: device error %d in prefill\n", d->hostio[2]);
        cudaMemsetAsync(d->err, 0, sizeof(int), s);
        cudaStreamSynchronize(s);
        return 0;
    }
    if (next_token) *next_token = d->hostio[0];
    return 1;
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
    case 6: src = d->rlog, size = d->n_exp; break;
    case 7: src = d->wts, size = d->top_k; break;
    case 8: src = reinterpret_cast<const float *>(d->ids), size = d->top_k; break;
    case 9: src = d->hbuf, size = static_cast<long long>(d->top_k) * c.ffn_dim; break;
    case 10: src = reinterpret_cast<const float *>(d->nloc), size = d->nloc ? 1 : 0; break;
    case 11: src = reinterpret_cast<const float *>(d->lids), size = d->lids ? d->top_k : 0; break;
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
