// tb_matvec.cu — persistent sm_100a GGUF dequant x fp32 matvec.
//
// Replaces the ten one-CTA-per-row kernels of layer4/tb_gguf_dequant.cu:89-332
// (plus Q2_K, which the reference lacks).  One CTA per SM, 16 warps at most:
// up to 15 consumer warps decode, one producer warp streams and reduces.
//
//   * A row of K weights is ceil(K/32) groups of 32, cut into CS column slots
//     of GPL consecutive groups (GPL per type, tb_decoders.cuh).  Every
//     consumer thread owns one slot for the whole launch and keeps the slot's
//     activations in registers, in the decoder's form; P = floor(consumer
//     threads / CS) rows are decoded side by side ("phases").
//   * Prologue: the CTA turns x into per-slot records in shared memory (for
//     the integer decoders in two passes: every thread loads, transforms and
//     quantizes 8 activations at its slot's scale, then one thread per
//     32-activation group packs its record), and every consumer thread with
//     rows copies its slot's record into registers.
//   * Each CTA owns a contiguous range of rows and streams it in tiles of TR
//     rows (TR*row_bytes contiguous bytes) through a ring of NST shared-memory
//     stages.  The producer warp fills a stage with one 1-D bulk copy
//     (cp.async.bulk, TMA engine, no multicast) widened to 16-byte boundaries,
//     with an L2 evict-first hint; a "full" mbarrier counts the bytes in.
//   * Consumers decode their rows of the tile, add each row's per-slot sums
//     across up to 8 neighbouring lanes with shuffles, store one partial per
//     (row, lane group) and arrive on the stage's "empty" mbarrier.  The
//     producer waits for all consumer warps there, sums every row's partials
//     in a fixed order, writes y and refills the stage with the tile NST
//     ahead.  The summation order never depends on timing, so results are
//     run-to-run deterministic.  Every wait is bounded.
#include <atomic>
#include <type_traits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "tb_common.cuh"
#include "tb_decoders.cuh"
#include "tb_decoders_f32.cuh"
#include "tb_internal.h"

namespace tb {

struct MvArgs {
    const uint8_t *W;
    const float *x;
    float *y;
    int *err;
    uint32_t M, K;        // K: the columns this launch multiplies (a window of the row when k_off > 0 or
    uint32_t k_off;       // K < the row's length); k_off: the window's first column (whole blocks)
    unsigned long long row_bytes;   // bytes of a whole row (the row stride)
    uint32_t block_weights, block_bytes;
    uint32_t cs;       // column slots per row
    uint32_t phases;   // rows decoded side by side
    uint32_t rpl;      // rows per consumer thread per tile
    uint32_t tr;       // rows per tile (= phases * rpl)
    uint32_t rw;       // lanes pre-reduced by shuffles (1, 2, 4 or 8; divides cs)
    uint32_t npart;    // partial sums per row (= cs / rw)
    uint32_t nst;      // stages in the ring
    uint32_t cap;      // bytes per stage
    uint32_t ncw;      // consumer warps; warp ncw is the producer
    uint32_t wait_limit;
    unsigned long long *stamp;   // TB_MV_STAMPS builds only: 16 device-clock stamps per CTA
    // fused input / output transforms (MvFuse): x is x (plain), x*rms*nw
    // (RMSNorm, rms = 1/sqrt(mean(x^2) + eps)) or silu(x)*x2 (SwiGLU); y gets
    // res added when res is not null
    uint32_t xmode, ymode;
    const float *x2, *nw, *res;
    float eps;
    uint32_t w_early;   // W is not written by the previous kernel: prefetch before griddepcontrol.wait
    // tensor-parallel exchange through tagged slots (MvFuse)
    const unsigned long long *xs;
    const int *xs_epoch;
    unsigned long long xs_mul, xs_add;
    float *xout;
    uint32_t nsl, ny;
    unsigned long long *ys[kMaxRanks];
    const int *y_epoch;
    unsigned long long y_mul, y_add;
    // expert groups (MvFuse): ng > 0 splits the grid into ng equal runs of CTAs
    const int *ids;
    const int *ng_dev;   // device count of the groups present (<= ng), or null
    uint32_t ng, n_experts;
    unsigned long long w_stride;
    uint32_t x_stride, y_stride;
};

#ifndef TB_MV_MIN_TILES
#define TB_MV_MIN_TILES 3         // tiles per CTA the planner keeps a single matvec at, when rows allow
#endif
#ifndef TB_MV_GROUP_TILES
#define TB_MV_GROUP_TILES 1
#endif
#ifndef TB_MV_MIN_TILES_EARLY
#define TB_MV_MIN_TILES_EARLY 2   // the same for a launch that prefetches its first tile before the wait
#endif
#ifndef TB_LL_SLEEP_NS
#define TB_LL_SLEEP_NS 64   // back-off between polls of a tagged slot word
#endif
#ifndef TB_LL_QUIET
#define TB_LL_QUIET 0
#endif
#ifndef TB_MV_TP_EARLY
#define TB_MV_TP_EARLY 1
#endif
static constexpr uint32_t kFull = 0xFFFFFFFFu;
static constexpr uint32_t kDrainLimit = 1u << 26;
static constexpr int kMaxThreads = 512;      // 15 consumer warps + 1 producer, <= 128 registers

// Threads of decoder D's CTA: D::kThreads when it declares one (the fp32
// decoders: 256 threads of up to 255 registers), else kMaxThreads.
template <class D, class = void>
struct ThreadsOf : std::integral_constant<int, kMaxThreads> {};
template <class D>
struct ThreadsOf<D, std::void_t<decltype(D::kThreads)>> : std::integral_constant<int, D::kThreads> {};

// Shared-memory layout: [full NST][empty NST] [reduction scratch 64 floats]
// [slot records] [partials NST*TR*NPART] [ring NST*CAP].
struct MvSmem {
    size_t red, table, part, ring, total;
};
__host__ __device__ inline size_t up16(size_t v) { return (v + 15) & ~size_t(15); }
__host__ __device__ inline MvSmem mv_smem(uint32_t nst, uint32_t cs, uint32_t rec, uint32_t tr,
                                          uint32_t npart, uint32_t cap)
{
    MvSmem s;
    s.red = up16(16ull * nst);
    s.table = up16(s.red + 256);
    s.part = up16(s.table + 4ull * cs * rec);
    s.ring = (s.part + 4ull * nst * tr * npart + 127) & ~size_t(127);
    s.total = s.ring + static_cast<size_t>(nst) * cap;
    return s;
}

// Elements [k0, k0 + N) of p (zeros past K): N/4 16-byte loads when the whole
// run is inside K and p is 16-byte aligned.  CG: through L2 (ld.global.cg),
// for slots written by peers over NVLink during the launch chain, which no
// non-coherent cached copy may serve.
template <int N, bool CG = false>
__device__ __forceinline__ void loadn(const float *p, uint32_t k0, uint32_t K, float (&v)[N])
{
    if (k0 + N <= K && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        const float4 *q = reinterpret_cast<const float4 *>(p + k0);
#pragma unroll
        for (int i = 0; i < N / 4; ++i) {
            const float4 t = CG ? __ldcg(q + i) : __ldg(q + i);
            v[4 * i] = t.x;
            v[4 * i + 1] = t.y;
            v[4 * i + 2] = t.z;
            v[4 * i + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = k0 + i < K ? (CG ? __ldcg(p + k0 + i) : __ldg(p + k0 + i)) : 0.f;
    }
}

// Elements [k0, k0 + N) of a row of tagged slot words (zeros past K): all N
// words are read whole at system scope (two per 16-byte load when aligned),
// and read again together until every one carries `tag`, so the wait costs
// one round trip after the last word lands, not one per word.  Still
// incomplete after `limit` rounds, or once this device's error word is set:
// the error word is set by the caller and the words read as what is there
// (returns false).
template <int N>
__device__ __forceinline__ bool load_tagged(const unsigned long long *p, uint32_t k0, uint32_t K, uint32_t tag,
                                            float (&t)[N], int *err, uint32_t limit)
{
    unsigned long long w[N];
    const bool vec = k0 + N <= K && (reinterpret_cast<uintptr_t>(p + k0) & 15u) == 0;
    auto read = [&]() {
        if (vec) {
#pragma unroll
            for (int i = 0; i < N; i += 2)
                asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];"
                             : "=l"(w[i]), "=l"(w[i + 1]) : "l"(p + k0 + i) : "memory");
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i) {
                w[i] = static_cast<unsigned long long>(tag) << 32;   // past K: a ready zero
                if (k0 + i < K) asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[i]) : "l"(p + k0 + i) : "memory");
            }
        }
    };
    read();
    bool ok = true;
    for (uint32_t it = 0;; ++it) {
        bool all = true;
#pragma unroll
        for (int i = 0; i < N; ++i) all = all && static_cast<uint32_t>(w[i] >> 32) == tag;
        if (all) break;
        if (it >= limit || *reinterpret_cast<volatile int *>(err) != 0) {
            ok = false;
            break;
        }
        __nanosleep(TB_LL_SLEEP_NS);
        read();   // words already carrying the tag keep their value: a slot is rewritten only by the next exchange
    }
#pragma unroll
    for (int i = 0; i < N; ++i) t[i] = __uint_as_float(static_cast<uint32_t>(w[i]));
    return ok;
}

// The tag of an exchange: (epoch * mul + add) mod 2^32.
__device__ __forceinline__ uint32_t xch_tag(const int *epoch, unsigned long long mul, unsigned long long add)
{
    return static_cast<uint32_t>(static_cast<unsigned long long>(*epoch) * mul + add);
}

// Activations [k0, k0 + N) (zeros past K) after the fused input transform,
// and ss += the sum of the squares of the raw x.
//   RMSNorm: x * nw; the scalar 1/rms of layer1/tb_tensor.c:194-199 is applied
//            to each slot's scale once the whole sum of squares is known.
//   SwiGLU:  silu(x) * x2, silu(g) = g / (1 + e^-g) (layer4/tb_infer.c:130-135).
template <int N>
__device__ __forceinline__ void load_x_part(const MvArgs &a, uint32_t xoff, uint32_t k0, float (&v)[N], float &ss)
{
    loadn<N>(a.x + xoff, k0, a.K, v);
    if (a.nsl) {   // tensor-parallel input: the residual plus the ranks' partials
        const uint32_t tag = xch_tag(a.xs_epoch, a.xs_mul, a.xs_add);
        bool ok = true;
        for (uint32_t r = 0; r < a.nsl; ++r) {
            float t[N];
            ok = load_tagged<N>(a.xs + static_cast<size_t>(r) * a.K, k0, a.K, tag, t, a.err, a.wait_limit) && ok;
#pragma unroll
            for (int i = 0; i < N; ++i) v[i] += t[i];
        }
        if (!ok) atomicExch(a.err, ERR_WAIT_TIMEOUT);
        if (a.xout && blockIdx.x == 0)
#pragma unroll
            for (int i = 0; i < N; ++i)
                if (k0 + i < a.K) a.xout[k0 + i] = v[i];
    }
    if (a.xmode == MV_X_RMSNORM) {
        float w[N];
        loadn<N>(a.nw, k0, a.K, w);
#pragma unroll
        for (int i = 0; i < N; ++i) {
            ss = fmaf(v[i], v[i], ss);
            v[i] *= w[i];
        }
    } else if (a.xmode == MV_X_SWIGLU) {
        float u[N];
        loadn<N>(a.x2 + xoff, k0, a.K, u);
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = (v[i] / (1.0f + expf(-v[i]))) * u[i];
    }
}

// A lane's activations scaled by f (the RMSNorm factor): the slot scale of the
// integer path, the activation registers of the float path.
template <class LY>
__device__ __forceinline__ void lane_scale(LaneInt<LY> &L, float f)
{
    L.r[LY::SX] = __float_as_uint(__uint_as_float(L.r[LY::SX]) * f);
}
__device__ __forceinline__ void lane_scale(XRegs &L, float f)
{
#pragma unroll
    for (int q = 0; q < 16; ++q) L.a[q] = make_float2(L.a[q].x * f, L.a[q].y * f);
}

// The consumer warps' tile loop.  Per tile: wait for the stage, decode this
// thread's rows (ph, ph + P, ...; a lane past the tile's rows decodes row 0 of
// the tile again and discards it, so the warp never diverges around the
// decode), add each row's slot sums over RW neighbouring lanes, store one
// partial per (row, lane group), arrive on the stage's "empty" barrier.
#if TB_MV_STAMPS
#define MV_STAMP(k)                                                                       \
    do {                                                                                  \
        if (a.stamp) {                                                                    \
            unsigned long long t_;                                                        \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                        \
            a.stamp[blockIdx.x * 16u + (k)] = t_;                                          \
        }                                                                                 \
    } while (0)
#else
#define MV_STAMP(k) \
    do {            \
    } while (0)
#endif

template <class D, int RW>
__device__ __forceinline__ void consume(const MvArgs &a, const typename D::Lane &lx, const Pos &pos, uint64_t *full,
                                        uint64_t *empty, float *part, const uint8_t *ring, uintptr_t w_lo,
                                        uintptr_t tile_bytes, uint32_t r_lo, uint32_t r_hi, uint32_t n_tiles,
                                        uint32_t cs, uint32_t ph, bool useful, bool active, uint32_t row_bytes32)
{
    const uint32_t lane = threadIdx.x & 31u;
    const bool writer = active && (cs % RW) == 0;
    const uint32_t npart = a.npart, phases = a.phases, rpl = a.rpl, tr = a.tr, nst = a.nst, cap = a.cap;
    const uint32_t part_col = cs / RW;
    uint32_t s = 0, par = 0, t0 = r_lo;
    uintptr_t lo = w_lo;
    float *pb = part;
    const uint8_t *stage = ring;
    const uint32_t pstride = tr * npart;
    for (uint32_t it = 0; it < n_tiles; ++it) {
        const bool ok = mbar_wait_bounded(smem_u32(full + s), par, a.err, a.wait_limit);
        if (!__all_sync(kFull, ok)) break;   // no arrival: the producer's wait runs out as well
        if (it == 0 && threadIdx.x == 0) MV_STAMP(4);
        const uint32_t nrows = min(tr, r_hi - t0);
        const uint32_t sbase = shared_after(smem_u32(stage) + static_cast<uint32_t>(lo & 15u));
#pragma unroll 2
        for (uint32_t i = 0; i < rpl; ++i) {
            const uint32_t rt = ph + i * phases;
            const bool live = useful && rt < nrows;
            if (!__any_sync(kFull, live)) break;   // rows ascend with i: none of the warp's later rows is live
            float v = D::row_dot(sbase + (live ? rt : 0u) * row_bytes32, pos, lx);
#pragma unroll
            for (int o = 1; o < RW; o <<= 1) v += __shfl_xor_sync(kFull, v, o);
            if (writer && live) pb[rt * npart + part_col] = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(empty + s));
        t0 += tr;
        lo += tile_bytes;
        if (++s == nst) {
            s = 0;
            par ^= 1u;
            pb = part;
            stage = ring;
        } else {
            pb += pstride;
            stage += cap;
        }
    }
    if (threadIdx.x == 0) MV_STAMP(5);
}

template <class D>
__global__ void __launch_bounds__(ThreadsOf<D>::value, 1) k_matvec(const MvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
    if (tid == 0) MV_STAMP(0);

    uint32_t G = gridDim.x, c = blockIdx.x, grp = 0;
    if (a.ng > 0 && !a.ng_dev) {   // expert groups: ng equal runs of CTAs, each a whole matvec
        const uint32_t cpg = G / a.ng;
        grp = c / cpg;
        c -= grp * cpg;
        G = cpg;
    }
    const uint32_t ua = a.ymode == MV_Y_SWIGLU_PAIRS ? 2u : 1u;   // rows per output unit
    uint32_t r_lo = 0, r_hi = 0, n_tiles = 0;
    auto span = [&]() {   // this CTA's rows of its group's matvec
        r_lo = ua * static_cast<uint32_t>((static_cast<unsigned long long>(a.M / ua) * c) / G);
        r_hi = ua * static_cast<uint32_t>((static_cast<unsigned long long>(a.M / ua) * (c + 1)) / G);
        n_tiles = (r_hi - r_lo + a.tr - 1) / a.tr;
    };
    // with a device-side group count (ng_dev) the partition is known only
    // after the dependency wait
    if (!a.ng_dev) {
        span();
        if (r_lo >= r_hi) return;
    }
    const uint32_t ngp = a.cs * D::GPL;   // groups of all slots (past K: zeros)

    const MvSmem L = mv_smem(a.nst, a.cs, D::REC, a.tr, a.npart, a.cap);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + a.nst;
    uint32_t *table = reinterpret_cast<uint32_t *>(smem + L.table);
    float *part = reinterpret_cast<float *>(smem + L.part);
    uint8_t *ring = smem + L.ring;
    const bool producer = warp == a.ncw;

    const uint64_t pol = l2_evict_first_policy();
    // Tiles advance by TR rows and TR*row_bytes bytes; stage index and barrier
    // phase are carried along, so the loops below need no division.
    uintptr_t w_lo = reinterpret_cast<uintptr_t>(a.W) + static_cast<uintptr_t>(r_lo) * a.row_bytes;
    if (a.ng > 0 && !a.ids) w_lo += static_cast<uintptr_t>(grp) * a.w_stride;
    const uintptr_t tile_bytes = static_cast<uintptr_t>(a.tr) * a.row_bytes;
    auto issue = [&](uint32_t s, uint32_t t0, uintptr_t lo) {   // one thread of the producer warp
        const uint32_t nrows = min(a.tr, r_hi - t0);
        const uintptr_t g0 = lo & ~uintptr_t(15);
        const uintptr_t g1 = (lo + nrows * a.row_bytes + 15) & ~uintptr_t(15);
        const uint32_t bar = smem_u32(full + s);
        mbar_expect_tx(bar, static_cast<uint32_t>(g1 - g0));
        bulk_g2s(smem_u32(ring + static_cast<size_t>(s) * a.cap), reinterpret_cast<const void *>(g0),
                 static_cast<uint32_t>(g1 - g0), bar, pol);
    };

    if (producer && lane == 0) {
        for (uint32_t s = 0; s < a.nst; ++s) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), a.ncw);
        }
        fence_mbar_init();
    }
    // Programmatic dependent launch: nothing below touches global memory other
    // than W before the previous kernel has finished and its writes are
    // visible.  Both instructions are no-ops without the launch attribute.
    // Stage 0 is requested before the prologue and the other stages after it:
    // the prologue's x loads would otherwise queue behind NST stages of weight
    // misses (up to ~200 KB per SM) and the consumers could not start any
    // sooner.  With w_early stage 0 is requested before the wait, so the
    // weight stream overlaps the previous kernel's tail (W is never written by
    // a kernel of the same chain in that case).
    // A consumer's column slot and phase (row offset within a tile): pure
    // functions of the shape, computed while the previous kernel finishes.
    const bool active = !producer && tid < a.phases * a.cs;
    const uint32_t cs = active ? tid % a.cs : 0;
    const uint32_t ph = active ? tid / a.cs : 0;
    bool useful = active && ph < r_hi - r_lo;
    Pos pos;
    {
        const uint32_t g0 = cs * D::GPL;                 // first group of the slot
        const uint32_t ngrp = (a.K + 31) / 32;           // groups per row
        if (a.block_weights == 256) {
            pos.off = ((a.k_off >> 8) + (g0 >> 3)) * a.block_bytes;
            pos.gi0 = g0 & 7u;
        } else if (a.block_weights == 32) {
            pos.off = ((a.k_off >> 5) + g0) * a.block_bytes;
            pos.gi0 = 0;
        } else {
            pos.off = (a.k_off + g0 * 32u) * a.block_bytes;
            pos.gi0 = 0;
        }
        pos.ng = static_cast<int>(min(static_cast<uint32_t>(D::GPL), ngrp - min(ngrp, g0)));
        pos.n = static_cast<int>(min(32u, a.K - min(a.K, 32u * (g0 + pos.ng - 1))));
    }
    // quiet: a matvec that waits for the other ranks' partials requests no
    // weights before they are in (the peers' NVLink stores would queue behind
    // this GPU's own weight stream in its L2)
    const bool quiet = TB_LL_QUIET && a.nsl > 0;
    if (a.w_early && !quiet && producer && lane == 0 && n_tiles) issue(0, r_lo, w_lo);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (tid == 0) MV_STAMP(1);
    // The next kernel may start once every CTA is past the wait: what the
    // kernels before this one wrote is then complete, so the next one may read
    // it ahead of its own wait (the decode step's attention streams its cached
    // rows that way).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (a.ng_dev) {   // the groups present this time (a count the previous kernel wrote): the grid is split among them
        const uint32_t ngd = min(static_cast<uint32_t>(max(*a.ng_dev, 0)), a.ng);
        if (ngd == 0) return;
        const uint32_t cpg = gridDim.x / ngd;
        grp = blockIdx.x / cpg;
        if (grp >= ngd) return;
        c = blockIdx.x - grp * cpg;
        G = cpg;
        span();
        if (r_lo >= r_hi) return;
        w_lo = reinterpret_cast<uintptr_t>(a.W) + static_cast<uintptr_t>(r_lo) * a.row_bytes;
        useful = active && ph < r_hi - r_lo;
    }
    if (a.ng > 0 && a.ids) {   // the group's expert, chosen by the previous kernel (same for the whole CTA)
        const int e = a.ids[grp];
        if (e < 0 || static_cast<uint32_t>(e) >= a.n_experts) {
            if (tid == 0) atomicExch(a.err, ERR_RUNTIME);
            return;
        }
        w_lo += static_cast<uintptr_t>(e) * a.w_stride;
    }
    if (!a.w_early && !quiet && producer && lane == 0 && n_tiles) issue(0, r_lo, w_lo);
    // A matvec whose input waits on the other ranks' partials requests the rest
    // of its ring as well (the fp32 prologue does not use the ring), so its
    // weights stream while the exchange completes.
    const bool ring_early = TB_MV_TP_EARLY && !quiet && IsF32X<D>::value && a.nsl > 0;
    if (ring_early && producer && lane == 0)
        for (uint32_t it = 1; it < min(a.nst, n_tiles); ++it) issue(it, r_lo + it * a.tr, w_lo + it * tile_bytes);

    // ---- prologue: x -> one record per column slot ----
    float ss = 0.f;   // RMSNorm: this thread's share of sum(x^2)
    float *red = reinterpret_cast<float *>(smem + L.red);
    // Integer decoders, when the digits fit ring stages 1.. (stage 0 may be in
    // flight; the others are requested only after the prologue): two passes.
    // Pass 1, all threads, 8 activations each ("quarters" of a group): load,
    // input transform, the slot's largest |x| by a shuffle over its 4*GPL
    // neighbouring lanes, the 16-bit digits X into shared memory, the slot's
    // exponent.  Pass 2, one thread per group: the type's record from its 32 X.
    // Otherwise one pass, one thread per group.
    const uint32_t xq_bytes = ngp * 64u, xe_off = xq_bytes;
    bool split = false;
    if constexpr (D::kInt) split = a.nst >= 2 && (a.nst - 1ull) * a.cap >= xq_bytes + 4ull * a.cs;
    if constexpr (IsF32X<D>::value) {
        // fp32 decoders: the record is the slot's transformed activations
        // themselves plus the magnitude bits of its largest |x| (each consumer
        // thread prescales its copy: writing them prescaled here, in register
        // order, was measured slower, the scattered 4-byte stores costing the
        // prologue more than they saved the consumers).  All threads, 8
        // activations each; the QPS quarters of a slot are neighbouring lanes.
        constexpr uint32_t QPS = 4u * D::GPL;
        const uint32_t nq = 4 * ngp;
        for (uint32_t base = 0; base < nq; base += nthr) {   // same trip count in every thread
            const uint32_t q = base + tid;
            const bool have = q < nq;
            float v[8];
            if (have) {
                load_x_part<8>(a, grp * a.x_stride + a.k_off, 8 * q, v, ss);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = 0.f;
            }
            uint32_t mb = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) mb = max(mb, __float_as_uint(v[i]) & 0x7FFFFFFFu);
#pragma unroll
            for (uint32_t o = 1; o < QPS; o <<= 1) mb = max(mb, __shfl_xor_sync(kFull, mb, o));
            if (have) {
                uint32_t *rec = table + (q / QPS) * D::REC;
                float4 *dst = reinterpret_cast<float4 *>(rec + (q % QPS) * 8);
                dst[0] = make_float4(v[0], v[1], v[2], v[3]);
                dst[1] = make_float4(v[4], v[5], v[6], v[7]);
                if (q % QPS == 0) rec[D::XN] = mb;
            }
        }
    } else if (split) {
        uint8_t *xq = ring + a.cap;                          // [ngp * 4][8] int16, then [cs] int32 exponents
        int *xe = reinterpret_cast<int *>(xq + xe_off);
        constexpr uint32_t QPS = 4u * D::GPL;                // quarters per slot (a power of two <= 32)
        const uint32_t nq = 4 * ngp;
        for (uint32_t base = 0; base < nq; base += nthr) {   // same trip count in every thread
            const uint32_t q = base + tid;
            const bool have = q < nq;
            float v[8];
            if (have) {
                load_x_part<8>(a, grp * a.x_stride + a.k_off, 8 * q, v, ss);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = 0.f;
            }
            // largest |x| as an integer max of the magnitude bits: an inf or NaN
            // gives bits >= 0x7F800000, which marks the slot non-finite
            uint32_t mb = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) mb = max(mb, __float_as_uint(v[i]) & 0x7FFFFFFFu);
#pragma unroll
            for (uint32_t o = 1; o < QPS; o <<= 1) mb = max(mb, __shfl_xor_sync(kFull, mb, o));
            if (have) {
                const bool sfin = mb < 0x7F800000u;
                const int E = slot_exponent(sfin ? __uint_as_float(mb) : 0.f);
                const float up = exp2i(14 - E);
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    int q0, q1;
                    asm("{\n\t.reg .s16 t;\n\tcvt.rni.sat.s16.f32 t, %1;\n\tcvt.s32.s16 %0, t;\n\t}"
                        : "=r"(q0) : "f"(v[2 * i] * up));
                    asm("{\n\t.reg .s16 t;\n\tcvt.rni.sat.s16.f32 t, %1;\n\tcvt.s32.s16 %0, t;\n\t}"
                        : "=r"(q1) : "f"(v[2 * i + 1] * up));
                    w[i] = __byte_perm(static_cast<uint32_t>(q0), static_cast<uint32_t>(q1), 0x5410u);
                }
                reinterpret_cast<uint4 *>(xq)[q] = make_uint4(w[0], w[1], w[2], w[3]);
                if (q % QPS == 0) xe[q / QPS] = sfin ? E : INT32_MIN;
            }
        }
        __syncthreads();
        for (uint32_t g = tid; g < ngp; g += nthr) {
            GroupX gx;
            const uint4 *src = reinterpret_cast<const uint4 *>(xq) + 4 * g;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 t = src[c];
                const uint32_t tw[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    gx.X[8 * c + 2 * i] = static_cast<int>(static_cast<int16_t>(tw[i] & 0xFFFFu));
                    gx.X[8 * c + 2 * i + 1] = static_cast<int>(tw[i]) >> 16;
                }
            }
            const int e = xe[g / D::GPL];
            const bool sfin = e != INT32_MIN;
            if constexpr (D::kInt)
                D::prep(gx, sfin ? e : 0, sfin, static_cast<int>(g % D::GPL), table + (g / D::GPL) * D::REC);
        }
    } else {
        // Thread g handles group g (then g + nthr, ...).  The GPL groups of a
        // slot are neighbouring lanes of one warp, so the slot's largest |x| is
        // a shuffle.
        for (uint32_t base = 0; base < ngp; base += nthr) {   // same trip count in every thread
            const uint32_t g = base + tid;
            const bool have = g < ngp;
            float v[32];
            if (have) {
                load_x_part<32>(a, grp * a.x_stride + a.k_off, 32 * g, v, ss);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0.f;
            }
            uint32_t *rec = table + (g / D::GPL) * D::REC;
            if constexpr (D::kInt) {
                uint32_t mb = 0;
#pragma unroll
                for (int i = 0; i < 32; ++i) mb = max(mb, __float_as_uint(v[i]) & 0x7FFFFFFFu);
#pragma unroll
                for (int o = 1; o < D::GPL; o <<= 1) mb = max(mb, __shfl_xor_sync(kFull, mb, o));
                if (have) {
                    const bool sfin = mb < 0x7F800000u;
                    const int E = slot_exponent(sfin ? __uint_as_float(mb) : 0.f);
                    GroupX gx;
                    quantize_group(v, E, gx);
                    D::prep(gx, E, sfin, static_cast<int>(g % D::GPL), rec);
                }
            } else {
                if (have) prep_float(v, rec);
            }
        }
    }
    if (a.xmode == MV_X_RMSNORM) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
        if (lane == 0) red[warp] = ss;
    }
    __syncthreads();   // records complete; barrier inits visible
    if (tid == 0) MV_STAMP(2);

    if (producer && lane == 0) {
        const uint32_t pre = min(a.nst, n_tiles);
        fence_proxy_async_smem();   // stages 1.. may have held the prologue's digits (generic proxy)
        for (uint32_t it = ring_early ? pre : (quiet ? 0 : 1); it < pre; ++it)
            issue(it, r_lo + it * a.tr, w_lo + it * tile_bytes);
    }
    if (producer) {
        // ---- producer: reduce each finished tile, write y, refill its stage ----
        uint32_t issued = min(a.nst, n_tiles), done = 0;
        bool fail = false;
        uint32_t s = 0, par = 0, t0 = r_lo;
        uintptr_t lo_next = w_lo + static_cast<uintptr_t>(a.nst) * tile_bytes;   // tile it + NST
        const uint32_t rows_ahead = a.nst * a.tr;
        const float *pb = part;
        const uint32_t pstride = a.tr * a.npart;
        float *const yg = a.y + grp * a.y_stride;
        const uint32_t ytag = a.ny ? xch_tag(a.y_epoch, a.y_mul, a.y_add) : 0u;
        for (uint32_t it = 0; it < n_tiles; ++it) {
            const bool ok = mbar_wait_bounded(smem_u32(empty + s), par, a.err, a.wait_limit);
            if (!__all_sync(kFull, ok)) {
                fail = true;
                break;
            }
            done = it + 1;
            const uint32_t nrows = min(a.tr, r_hi - t0);
            if (a.ymode == MV_Y_SWIGLU_PAIRS) {   // tiles hold whole (gate, up) pairs
                for (uint32_t r = 2 * lane; r < nrows; r += 64) {
                    const float *pg = pb + r * a.npart, *pu = pg + a.npart;
                    float gs = 0.f, us = 0.f;
                    for (uint32_t j = 0; j < a.npart; ++j) {
                        gs += pg[j];
                        us += pu[j];
                    }
                    yg[(t0 + r) / 2] = (gs / (1.0f + expf(-gs))) * us;
                }
            } else {
                for (uint32_t r = lane; r < nrows; r += 32) {
                    const float *pr = pb + r * a.npart;
                    float acc = 0.f;
                    for (uint32_t j = 0; j < a.npart; ++j) acc += pr[j];
                    if (a.ny) {   // tensor-parallel output: this rank's partial to every rank, tagged
                        const unsigned long long wv = (static_cast<unsigned long long>(ytag) << 32) | __float_as_uint(acc);
                        for (uint32_t p = 0; p < a.ny; ++p)
                            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a.ys[p] + t0 + r), "l"(wv) : "memory");
                    } else {
                        yg[t0 + r] = a.res ? acc + a.res[t0 + r] : acc;
                    }
                }
            }
            __syncwarp();
            if (it + a.nst < n_tiles) {
                if (lane == 0) {
                    fence_proxy_async_smem();   // the stage was read through the generic proxy
                    issue(s, t0 + rows_ahead, lo_next);
                }
                ++issued;
            }
            __syncwarp();
            t0 += a.tr;
            lo_next += tile_bytes;
            if (++s == a.nst) {
                s = 0;
                par ^= 1u;
                pb = part;
            } else {
                pb += pstride;
            }
        }
        if (lane == 0) MV_STAMP(6);
        if (fail && lane == 0) {
            // A wait ran out: let every copy still in flight land before the CTA
            // exits (fixed, generous bound: they target valid memory and complete).
            for (uint32_t it = done; it < issued; ++it)
                mbar_wait_bounded(smem_u32(full + it % a.nst), (it / a.nst) & 1u, nullptr, kDrainLimit);
        }
        return;
    }

    // ---- consumers ----
    // (slot and phase were set up before the dependency wait; a thread whose
    // phase is past this CTA's rows never decodes, so it loads no record)
    typename D::Lane lx;
    if (useful) {
        D::load(lx, table + cs * D::REC);
        if (a.xmode == MV_X_RMSNORM) {   // 1/sqrt(sum(x^2)/K + eps), summed in warp order
            float t = 0.f;
            for (uint32_t w = 0; w < nthr / 32; ++w) t += red[w];
            lane_scale(lx, 1.0f / sqrtf(t / static_cast<float>(a.K) + a.eps));
        }
    }
    if (tid == 0) MV_STAMP(3);
    const uint32_t row_bytes32 = static_cast<uint32_t>(a.row_bytes);   // a tile's rows fit one stage
    // the reduction width as a template argument: no runtime selects per row
    switch (a.rw) {
    case 8: consume<D, 8>(a, lx, pos, full, empty, part, ring, w_lo, tile_bytes, r_lo, r_hi, n_tiles, cs, ph,
                          useful, active, row_bytes32); break;
    case 4: consume<D, 4>(a, lx, pos, full, empty, part, ring, w_lo, tile_bytes, r_lo, r_hi, n_tiles, cs, ph,
                          useful, active, row_bytes32); break;
    case 2: consume<D, 2>(a, lx, pos, full, empty, part, ring, w_lo, tile_bytes, r_lo, r_hi, n_tiles, cs, ph,
                          useful, active, row_bytes32); break;
    default: consume<D, 1>(a, lx, pos, full, empty, part, ring, w_lo, tile_bytes, r_lo, r_hi, n_tiles, cs, ph,
                           useful, active, row_bytes32); break;
    }
}

// ---------------------------------------------------------------------------
// host side: launch planning (cached per kernel, shape and device)
// ---------------------------------------------------------------------------
static constexpr int kSmemMax = 232448;          // 227 KB opt-in per CTA on sm_100
static constexpr uint32_t kStageMax = 98304;     // bytes of weights per stage at most
static constexpr uint32_t kMaxRpl = 8;           // rows per thread per tile at most
static constexpr uint32_t kMaxStages = 8;

struct Plan {
    const void *kern;
    unsigned long long row_bytes;
    uint32_t M, K, sms, ymode, ng, w_early;
    int dev;
    uint32_t nthr, grid, cs, phases, rpl, tr, rw, npart, nst, cap, ncw;
    size_t smem;
};

// A few recent plans per host thread: a decode step reuses a handful of shapes.
static constexpr int kPlanCache = 64;
static thread_local Plan t_plans[kPlanCache];
static thread_local int t_nplans = 0, t_next = 0;

template <class D>
static bool make_plan(Plan &p, unsigned long long row_bytes)
{
    constexpr uint32_t kMaxConsumerWarps = ThreadsOf<D>::value / 32 - 1;
    const uint32_t ngrp = (p.K + 31) / 32;
    p.cs = (ngrp + D::GPL - 1) / D::GPL;
    if (p.cs > 32 * kMaxConsumerWarps) {
        fprintf(stderr, "[tb_cuda] matvec: K=%u needs %u column slots, more than %u threads\n", p.K, p.cs,
                32 * kMaxConsumerWarps);
        return false;
    }
    // consumer warps: the most threads owning a slot, then the fewest idle ones
    uint32_t best_used = 0;
    p.ncw = 0;
    for (uint32_t w = 1; w <= kMaxConsumerWarps; ++w) {
        const uint32_t used = ((32 * w) / p.cs) * p.cs;
        if (used > best_used) {
            best_used = used;
            p.ncw = w;
        }
    }
    if (!p.ncw) return false;
    p.rw = (p.cs % 8 == 0) ? 8 : (p.cs % 4 == 0) ? 4 : (p.cs % 2 == 0) ? 2 : 1;
    p.npart = p.cs / p.rw;
    // TB_MV_STAGE_KB / TB_MV_RPL_MAX: planner tuning knobs (stage bytes, rows per thread)
    static const uint32_t stage_max = getenv("TB_MV_STAGE_KB") ? 1024u * atoi(getenv("TB_MV_STAGE_KB")) : kStageMax;
    static const uint32_t rpl_max = getenv("TB_MV_RPL_MAX") ? atoi(getenv("TB_MV_RPL_MAX")) : kMaxRpl;
    // Rows per thread per tile: as many as keep a stage within kStageMax and
    // two stages in shared memory (the per-tile cost is paid once per rpl
    // rows) and, for a single matvec, still give each CTA at least three
    // tiles (two when the first is requested before the dependency wait): a
    // CTA with one tile, or one and a sliver, cannot overlap its decoding with
    // its stream (measured 7-10 % faster on 14-28 MB projections, no change on
    // the large ones; in the decode step two measured better than three);
    // then as many stages as fit.  When even one
    // row per thread does not fit (long rows over few column slots: many
    // phases of whole rows), fewer consumer warps make fewer phases.
    // rows of one CTA: a single matvec spreads M rows over min(M, SMs) CTAs;
    // expert groups give each group's M rows (output units of ua rows) to
    // SMs / ng CTAs (TB_MV_GROUP_TILES: the rule for groups too)
    uint32_t rows_cta = 0;
    {
        const uint32_t ua = p.ymode == MV_Y_SWIGLU_PAIRS ? 2u : 1u, units = p.M / ua;
        if (p.ng == 0) {
            const uint32_t g = p.M < p.sms ? p.M : p.sms;
            rows_cta = g ? (p.M + g - 1) / g : 0u;
        } else if (TB_MV_GROUP_TILES && units) {
            uint32_t cpg = p.sms / p.ng;
            cpg = cpg < 1 ? 1 : (cpg > units ? units : cpg);
            rows_cta = ua * ((units + cpg - 1) / cpg);
        }
    }
    // (a launch that requests its first tile before the dependency wait keeps
    // bigger tiles: more of its weights stream while the previous kernel ends)
    const uint32_t min_tiles = p.w_early ? TB_MV_MIN_TILES_EARLY : TB_MV_MIN_TILES;
    p.nst = 0;
    for (const uint32_t min_ncw = (p.cs + 31) / 32; !p.nst && p.ncw >= min_ncw; --p.ncw) {
        p.nthr = 32 * (p.ncw + 1);
        p.phases = (32 * p.ncw) / p.cs;
        for (uint32_t rpl = rpl_max; rpl >= 1 && !p.nst; --rpl) {
            const unsigned long long bytes = static_cast<unsigned long long>(p.phases) * rpl * row_bytes;
            if (rpl > 1 && bytes > stage_max) continue;
            if (p.ymode == MV_Y_SWIGLU_PAIRS && (p.phases * rpl) % 2) continue;   // tiles of whole pairs
            const uint32_t tr = p.phases * rpl;
            if (rpl > 1 && rows_cta && (rows_cta + tr - 1) / tr < min_tiles) continue;   // tiles a CTA
            const uint32_t cap = static_cast<uint32_t>((bytes + 32 + 127) & ~127ull);
            for (uint32_t n = kMaxStages; n >= 2; --n) {
                const MvSmem s = mv_smem(n, p.cs, D::REC, tr, p.npart, cap);
                if (s.total <= static_cast<size_t>(kSmemMax)) {
                    p.rpl = rpl;
                    p.tr = tr;
                    p.cap = cap;
                    p.nst = n;
                    p.smem = s.total;
                    break;
                }
            }
        }
        if (p.nst) break;
    }
    if (!p.nst) {
        fprintf(stderr, "[tb_cuda] matvec: a %u-row tile of %llu-byte rows does not fit shared memory\n", p.phases,
                row_bytes);
        return false;
    }
    if (p.ng > 0) {   // equal runs of CTAs per group, each at most one per output unit
        const uint32_t units = p.ymode == MV_Y_SWIGLU_PAIRS ? p.M / 2 : p.M;
        uint32_t cpg = p.sms / p.ng;
        cpg = cpg < 1 ? 1 : (cpg > units ? units : cpg);
        p.grid = p.ng * cpg;
    } else {
        p.grid = p.M < p.sms ? p.M : p.sms;
    }
    return true;
}

template <class D>
static int launch_dec(MvArgs &a, int num_sms, cudaStream_t st)
{
    auto kern = k_matvec<D>;
    const void *kp = reinterpret_cast<const void *>(kern);
    int dev = 0;
    cudaGetDevice(&dev);
    const Plan *p = nullptr;
    for (int i = 0; i < t_nplans; ++i) {
        const Plan &q = t_plans[i];
        if (q.kern == kp && q.M == a.M && q.K == a.K && q.row_bytes == a.row_bytes && q.dev == dev &&
            q.sms == static_cast<uint32_t>(num_sms) && q.ymode == a.ymode && q.ng == a.ng &&
            q.w_early == a.w_early) {
            p = &q;
            break;
        }
    }
    if (!p) {
        if (!smem_attr_once(kp, kSmemMax)) return 0;
        Plan np{};
        np.kern = kp;
        np.row_bytes = a.row_bytes;
        np.M = a.M;
        np.K = a.K;
        np.dev = dev;
        np.sms = static_cast<uint32_t>(num_sms);
        np.ymode = a.ymode;
        np.ng = a.ng;
        np.w_early = a.w_early;
        if (!make_plan<D>(np, a.row_bytes)) return 0;
        if (getenv("TB_MV_VERBOSE"))
            fprintf(stderr,
                    "[tb_cuda] matvec plan M=%u K=%u: threads %u cs %u phases %u rpl %u tr %u nst %u cap %u "
                    "smem %zu grid %u\n",
                    np.M, np.K, np.nthr, np.cs, np.phases, np.rpl, np.tr, np.nst, np.cap, np.smem, np.grid);
        const int slot = t_nplans < kPlanCache ? t_nplans++ : (t_next++ % kPlanCache);
        t_plans[slot] = np;
        p = &t_plans[slot];
    }
    a.cs = p->cs;
    a.phases = p->phases;
    a.rpl = p->rpl;
    a.tr = p->tr;
    a.rw = p->rw;
    a.npart = p->npart;
    a.nst = p->nst;
    a.cap = p->cap;
    a.ncw = p->ncw;
    // launched with programmatic stream serialization, so back-to-back matvecs
    // overlap one kernel's launch with the previous one's tail
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(p->nthr);
    cfg.dynamicSmemBytes = p->smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

// Activation arithmetic of the quantized types: MV_ARITH_FP32 (default) or the
// opt-in MV_ARITH_INT16.  Read at each launch; a captured graph keeps the
// kernels it was captured with.
static std::atomic<int> g_arith{MV_ARITH_FP32};

int mv_set_arith(int mode)
{
    if (mode != MV_ARITH_FP32 && mode != MV_ARITH_INT16) return -1;
    return g_arith.exchange(mode);
}

int mv_get_arith() { return g_arith.load(); }

static int mv_dispatch(MvArgs &a, int qtype, const void *W, bool fp32, cudaStream_t st, int num_sms);
static int mv_launch_window(MvArgs a, int qtype, uint32_t k_off, uint32_t K, cudaStream_t st, int num_sms);

#if TB_MV_STAMPS
// Instrumented builds: every launch gets its own slot of 16 stamps per CTA (a
// captured graph keeps the slot of its capture), read back by tb_mv_stamps.
static unsigned long long *g_stamp_buf = nullptr;
static unsigned g_stamp_n = 0;
static constexpr unsigned kStampSlots = 4096, kStampCtas = 160;
}  // namespace tb
extern "C" int tb_mv_stamps_init()
{
    using namespace tb;
    const size_t n = size_t(kStampSlots) * kStampCtas * 16;
    if (!g_stamp_buf && cudaMalloc(&g_stamp_buf, n * 8) != cudaSuccess) return 0;
    g_stamp_n = 0;
    return cudaMemset(g_stamp_buf, 0, n * 8) == cudaSuccess;
}
extern "C" int tb_mv_stamps(unsigned long long *host, int max_launches)
{
    using namespace tb;
    if (!g_stamp_buf) return -1;
    const unsigned n = g_stamp_n < unsigned(max_launches) ? g_stamp_n : unsigned(max_launches);
    cudaDeviceSynchronize();
    cudaMemcpy(host, g_stamp_buf, size_t(n < kStampSlots ? n : kStampSlots) * kStampCtas * 128, cudaMemcpyDeviceToHost);
    return static_cast<int>(g_stamp_n);
}
namespace tb {
#endif

int mv_launch(const void *W, int qtype, int M, int K, const float *d_x, float *d_y,
              cudaStream_t st, int *d_err, int num_sms, uint32_t wait_limit, const MvFuse *fuse)
{
    const NvtxRange nvtx("tb.matvec");
    const Geom g = geom_of(qtype);
    if (!g.block_weights || !W || !d_x || !d_y || M <= 0 || K <= 0 || K % g.block_weights) return 0;
    MvArgs a{};
#if TB_MV_STAMPS
    if (g_stamp_buf) a.stamp = g_stamp_buf + size_t(g_stamp_n++ % kStampSlots) * kStampCtas * 16;
#endif
    if (fuse) {
        if (fuse->xmode > MV_X_SWIGLU || (fuse->xmode == MV_X_RMSNORM && !fuse->nw) ||
            (fuse->xmode == MV_X_SWIGLU && !fuse->x2))
            return 0;
        if (fuse->ymode > MV_Y_SWIGLU_PAIRS || (fuse->ymode == MV_Y_SWIGLU_PAIRS && (M % 2 || fuse->res)))
            return 0;
        a.xmode = fuse->xmode;
        a.ymode = fuse->ymode;
        a.x2 = fuse->x2;
        a.nw = fuse->nw;
        a.eps = fuse->eps;
        a.res = fuse->res;
        a.w_early = fuse->w_early ? 1u : 0u;
        if (fuse->nsl > static_cast<uint32_t>(kMaxRanks) || fuse->ny > static_cast<uint32_t>(kMaxRanks) ||
            (fuse->nsl && (!fuse->xs || !fuse->xs_epoch || fuse->xmode == MV_X_SWIGLU)) ||
            (fuse->ny && (fuse->res || fuse->ymode != MV_Y_PLAIN || !fuse->y_epoch)))
            return 0;
        for (uint32_t p = 0; p < fuse->ny; ++p)
            if (!fuse->ys[p]) return 0;
        a.xs = fuse->xs;
        a.xs_epoch = fuse->xs_epoch;
        a.xs_mul = fuse->xs_mul;
        a.xs_add = fuse->xs_add;
        a.xout = fuse->xout;
        a.nsl = fuse->nsl;
        a.ny = fuse->ny;
        for (int p = 0; p < kMaxRanks; ++p) a.ys[p] = fuse->ys[p];
        a.y_epoch = fuse->y_epoch;
        a.y_mul = fuse->y_mul;
        a.y_add = fuse->y_add;
        if (fuse->ng > 0) {
            // groups: no residual, no tensor-parallel exchange; an expert id
            // read on the device cannot be prefetched ahead of the wait
            if (fuse->ng > 1024 || fuse->res || fuse->nsl || fuse->ny || (fuse->ids && fuse->w_early) ||
                (fuse->ids && !fuse->n_experts) || !fuse->w_stride || (fuse->ng_dev && !fuse->ids))
                return 0;
            a.ng = fuse->ng;
            a.ng_dev = fuse->ng_dev;
            a.n_experts = fuse->n_experts;
            a.ids = fuse->ids;
            a.w_stride = fuse->w_stride;
            a.x_stride = fuse->x_stride;
            a.y_stride = fuse->y_stride;
        }
    }
    a.W = static_cast<const uint8_t *>(W);
    a.x = d_x;
    a.y = d_y;
    a.err = d_err;
    a.M = static_cast<uint32_t>(M);
    a.K = static_cast<uint32_t>(K);
    a.block_weights = static_cast<uint32_t>(g.block_weights);
    a.block_bytes = static_cast<uint32_t>(g.block_bytes);
    a.row_bytes = static_cast<unsigned long long>(K / g.block_weights) * g.block_bytes;
    a.wait_limit = wait_limit;

    const bool fp32 = g_arith.load(std::memory_order_relaxed) == MV_ARITH_FP32 && g.block_weights > 1;
    {
        // A row longer than the decoder's column slots cover (one slot per
        // consumer thread: 64 weights for the fp32 decoders, 128 for the int16
        // ones, 32 for F32 / F16 / BF16) runs as launches over column windows of
        // the same rows, in order: the first writes y (+ res), each later one
        // adds its window onto y.  Each streams whole rows, so these shapes move
        // their weights once per window.
        const uint32_t kCols = g.block_weights == 1 ? 32u * (kMaxThreads - 32u)
                             : fp32 ? 64u * XF_NP * (XfGeom<XF_NP>::THREADS - 32u)
                                    : 128u * (kMaxThreads - 32u);
        if (a.K > kCols && a.k_off == 0) {
            const uint32_t bw = static_cast<uint32_t>(g.block_weights);
            const uint32_t nw = (a.K + kCols - 1) / kCols;              // windows
            const uint32_t step = (((a.K + nw - 1) / nw + bw - 1) / bw) * bw;   // columns per window, whole blocks
            const bool plain = a.xmode != MV_X_RMSNORM && a.ymode == MV_Y_PLAIN && !a.nsl && !a.ny && !a.ng;
            if (!plain || step > kCols) {
                fprintf(stderr, "[tb_cuda] matvec: K=%u is longer than one launch covers%s\n", a.K,
                        plain ? "" : " with this fused mode");
                return 0;
            }
            const uint32_t K0 = a.K;
            for (uint32_t k0 = 0; k0 < K0; k0 += step) {
                if (!mv_launch_window(a, qtype, k0, K0 - k0 < step ? K0 - k0 : step, st, num_sms)) return 0;
                a.res = d_y;   // later windows add onto the result so far
            }
            return 1;
        }
    }
    return mv_dispatch(a, qtype, W, fp32, st, num_sms);
}

static int mv_launch_window(MvArgs a, int qtype, uint32_t k_off, uint32_t K, cudaStream_t st, int num_sms)
{
    a.k_off = k_off;
    a.K = K;
    const bool fp32 = g_arith.load(std::memory_order_relaxed) == MV_ARITH_FP32 && a.block_weights > 1;
    return mv_dispatch(a, qtype, a.W, fp32, st, num_sms);
}

static int mv_dispatch(MvArgs &a, int qtype, const void *W, bool fp32, cudaStream_t st, int num_sms)
{
    const uintptr_t wa = reinterpret_cast<uintptr_t>(W);
    const bool a16 = (wa & 15u) == 0 && (a.row_bytes & 15u) == 0 && (a.w_stride & 15u) == 0;
    const bool a4 = (wa & 3u) == 0 && (a.row_bytes & 3u) == 0 && (a.w_stride & 3u) == 0;
    if (fp32) {
        switch (qtype) {
        case QT_Q4_K:
            return a16 ? launch_dec<DecQ4KF<true>>(a, num_sms, st) : launch_dec<DecQ4KF<false>>(a, num_sms, st);
        case QT_Q5_K:
            return a16 ? launch_dec<DecQ5KF<true>>(a, num_sms, st) : launch_dec<DecQ5KF<false>>(a, num_sms, st);
        case QT_Q6_K: return launch_dec<DecQ6KF<>>(a, num_sms, st);
        case QT_Q3_K:
        case QT_IQ3_S: return launch_dec<DecQ3KF<>>(a, num_sms, st);
        case QT_Q2_K:
            return a4 ? launch_dec<DecQ2KF<true>>(a, num_sms, st) : launch_dec<DecQ2KF<false>>(a, num_sms, st);
        case QT_Q8_0: return launch_dec<DecQ80F<>>(a, num_sms, st);
        case QT_Q4_0: return launch_dec<DecQ40F<>>(a, num_sms, st);
        case QT_Q8_K: return launch_dec<DecQ8KF<>>(a, num_sms, st);
        default: break;   // F32 / F16 / BF16: the float decoders below (fp32 already)
        }
    }
    switch (qtype) {
    case QT_Q4_K: return a16 ? launch_dec<DecQ4K<true>>(a, num_sms, st) : launch_dec<DecQ4K<false>>(a, num_sms, st);
    case QT_Q5_K: return a16 ? launch_dec<DecQ5K<true>>(a, num_sms, st) : launch_dec<DecQ5K<false>>(a, num_sms, st);
    case QT_Q6_K: return launch_dec<DecQ6K>(a, num_sms, st);
    case QT_Q3_K:
    case QT_IQ3_S: return launch_dec<DecQ3K>(a, num_sms, st);
    case QT_Q2_K: return a4 ? launch_dec<DecQ2K<true>>(a, num_sms, st) : launch_dec<DecQ2K<false>>(a, num_sms, st);
    case QT_Q8_0: return launch_dec<DecQ80>(a, num_sms, st);
    case QT_Q4_0: return launch_dec<DecQ40>(a, num_sms, st);
    case QT_Q8_K: return launch_dec<DecQ8K>(a, num_sms, st);
    case QT_F32: return launch_dec<DecFloat<QT_F32>>(a, num_sms, st);
    case QT_F16: return launch_dec<DecFloat<QT_F16>>(a, num_sms, st);
    case QT_BF16: return launch_dec<DecFloat<QT_BF16>>(a, num_sms, st);
    default: return 0;
    }
}

}  // namespace tb
