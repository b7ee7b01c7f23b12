// tb_matvec.cu — persistent sm_100a GGUF dequant x fp32 matvec.
//
// Replaces the ten one-CTA-per-row kernels of layer4/tb_gguf_dequant.cu:89-332
// (plus Q2_K, which the reference lacks).  Layout and schedule:
//
//   * A row of K weights is ceil(K/32) groups of 32, cut into CS column slots
//     of GPL consecutive groups (GPL per type, tb_decoders.cuh).  Every thread
//     of a CTA owns one slot for the whole launch: the slot's activations live
//     in its registers in the decoder's form.  P = floor(threads / CS) rows are
//     decoded side by side ("phases").  x is read from global memory once per
//     CTA, coalesced, into shared memory padded by one float per slot (so the
//     threads' slot reads hit 32 different banks), and from there into
//     registers; every weight then costs only its own bytes.
//   * Each CTA owns a contiguous range of rows and streams it in tiles of TR
//     rows (TR*row_bytes contiguous bytes) through a ring of NST shared-memory
//     stages.  A stage is filled by one 1-D bulk copy (cp.async.bulk, TMA
//     engine, no multicast) widened to 16-byte boundaries, with an L2
//     evict-first hint; completion is an mbarrier transaction count.  Every
//     wait is bounded.
//   * There is no CTA-wide barrier per tile.  A row's per-slot partial sums are
//     added across the 8 (or fewer) consecutive threads of one block by
//     shuffles and written to a per-stage partial buffer; each warp then takes
//     a ticket on the stage.  The warp that takes the last ticket sums every
//     row of the tile in a fixed order, writes y, and refills the stage with
//     the tile NST ahead.  The summation order never depends on timing, so
//     results are run-to-run deterministic.
#include <cstdio>
#include <cstdlib>

#include "tb_common.cuh"
#include "tb_decoders.cuh"
#include "tb_internal.h"

namespace tb {

struct MvArgs {
    const uint8_t *W;
    const float *x;
    float *y;
    int *err;
    uint32_t M, K;
    unsigned long long row_bytes;
    uint32_t block_weights, block_bytes;
    uint32_t cs;       // column slots per row
    uint32_t phases;   // rows decoded side by side
    uint32_t rpl;      // rows per thread per tile
    uint32_t tr;       // rows per tile (= phases * rpl)
    uint32_t rw;       // threads pre-reduced by shuffles (1, 2, 4 or 8; divides cs)
    uint32_t npart;    // partial sums per row (= cs / rw)
    uint32_t nst;      // stages in the ring
    uint32_t cap;      // bytes per stage
    uint32_t wait_limit;
};

static constexpr uint32_t kFull = 0xFFFFFFFFu;
static constexpr uint32_t kDrainLimit = 1u << 26;
static constexpr int kMaxThreads = 384;   // up to 168 registers per thread

// shared-memory layout: [bars NST][tickets NST][issued] [part NST*TR*NPART] [x staging] [ring]
__host__ __device__ inline size_t mv_part_offset(uint32_t nst)
{
    return (8ull * nst + 4ull * nst + 4 + 15) & ~15ull;
}
__host__ __device__ inline size_t mv_x_offset(uint32_t nst, uint32_t tr, uint32_t npart)
{
    return (mv_part_offset(nst) + 4ull * nst * tr * npart + 15) & ~15ull;
}
__host__ __device__ inline size_t mv_ring_offset(uint32_t nst, uint32_t tr, uint32_t npart, uint32_t xfloats)
{
    return (mv_x_offset(nst, tr, npart) + 4ull * xfloats + 127) & ~127ull;
}
// floats of the padded x copy: CS slots of 32*GPL activations, one pad float each
__host__ __device__ inline uint32_t mv_x_floats(uint32_t cs, uint32_t gpl)
{
    return cs * (32 * gpl + 1);
}

template <class D>
__global__ void __launch_bounds__(kMaxThreads, 1) k_matvec(const MvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31;
    const uint32_t nwarps = nthr / 32;

    const uint32_t G = gridDim.x, c = blockIdx.x;
    const uint32_t r_lo = static_cast<uint32_t>((static_cast<unsigned long long>(a.M) * c) / G);
    const uint32_t r_hi = static_cast<uint32_t>((static_cast<unsigned long long>(a.M) * (c + 1)) / G);
    if (r_lo >= r_hi) return;
    const uint32_t n_tiles = (r_hi - r_lo + a.tr - 1) / a.tr;
    constexpr uint32_t SW = 32u * D::GPL;   // activations per slot

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    int *tickets = reinterpret_cast<int *>(smem + 8ull * a.nst);
    int *issued = tickets + a.nst;
    float *part = reinterpret_cast<float *>(smem + mv_part_offset(a.nst));
    float *xst = reinterpret_cast<float *>(smem + mv_x_offset(a.nst, a.tr, a.npart));
    uint8_t *ring = smem + mv_ring_offset(a.nst, a.tr, a.npart, mv_x_floats(a.cs, D::GPL));

    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](uint32_t it) {   // one thread
        const uint32_t t0 = r_lo + it * a.tr;
        const uint32_t nrows = min(a.tr, r_hi - t0);
        const uintptr_t lo = reinterpret_cast<uintptr_t>(a.W) + t0 * a.row_bytes;
        const uintptr_t g0 = lo & ~uintptr_t(15);
        const uintptr_t g1 = (lo + nrows * a.row_bytes + 15) & ~uintptr_t(15);
        const uint32_t s = it % a.nst;
        const uint32_t bar = smem_u32(bars + s);
        mbar_expect_tx(bar, static_cast<uint32_t>(g1 - g0));
        bulk_g2s(smem_u32(ring + static_cast<size_t>(s) * a.cap), reinterpret_cast<const void *>(g0),
                 static_cast<uint32_t>(g1 - g0), bar, pol);
    };

    if (tid == 0) {
        for (uint32_t s = 0; s < a.nst; ++s) {
            mbar_init(smem_u32(bars + s), 1);
            tickets[s] = 0;
        }
        fence_mbar_init();
        const uint32_t pre = min(a.nst, n_tiles);
        for (uint32_t it = 0; it < pre; ++it) issue(it);
        *issued = static_cast<int>(pre);
    }

    // ---- x: coalesced global read into the padded shared copy ----
    // eight independent loads per thread in flight before any store
    for (uint32_t base = 0; base < a.K; base += 8 * nthr) {
        float v[8];
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u) {
            const uint32_t k = base + u * nthr + tid;
            v[u] = k < a.K ? __ldg(a.x + k) : 0.f;
        }
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u) {
            const uint32_t k = base + u * nthr + tid;
            if (k < a.K) xst[k + k / SW] = v[u];
        }
    }
    __syncthreads();   // x staged; barrier inits and tickets visible

    // ---- this thread's column slot and its activations ----
    const bool active = tid < a.phases * a.cs;
    const uint32_t cs = active ? tid % a.cs : 0;
    const uint32_t ph = active ? tid / a.cs : 0;
    const uint32_t g0 = cs * D::GPL;                 // first group of the slot
    const uint32_t ngrp = (a.K + 31) / 32;           // groups per row
    Pos pos;
    if (a.block_weights == 256) {
        pos.off = (g0 >> 3) * a.block_bytes;
        pos.gi0 = g0 & 7u;
    } else if (a.block_weights == 32) {
        pos.off = g0 * a.block_bytes;
        pos.gi0 = 0;
    } else {
        pos.off = g0 * 32u * a.block_bytes;
        pos.gi0 = 0;
    }
    pos.ng = static_cast<int>(min(static_cast<uint32_t>(D::GPL), ngrp - min(ngrp, g0)));
    pos.n = static_cast<int>(min(32u, a.K - min(a.K, 32u * (g0 + pos.ng - 1))));
    typename D::Lane lane_x;
    {
        const int nv = active ? static_cast<int>(min(SW, a.K - min(a.K, 32u * g0))) : 0;
        D::load(lane_x, xst + cs * (SW + 1), nv);
    }
    const uint32_t row_bytes32 = static_cast<uint32_t>(a.row_bytes);   // a tile's rows fit one stage
    const bool writer = active && (cs % a.rw) == 0;
    const uint32_t part_col = cs / a.rw;

    uint32_t consumed = 0;
    bool fail = false;
    for (uint32_t it = 0; it < n_tiles; ++it) {
        const uint32_t s = it % a.nst;
        bool got = mbar_wait_bounded(smem_u32(bars + s), (it / a.nst) & 1u, a.err, a.wait_limit);
        if (!__all_sync(kFull, got)) {
            fail = true;
            break;
        }
        consumed = it + 1;
        const uint32_t t0 = r_lo + it * a.tr;
        const uint32_t nrows = min(a.tr, r_hi - t0);
        float *pb = part + static_cast<size_t>(s) * a.tr * a.npart;
        const uintptr_t lo = reinterpret_cast<uintptr_t>(a.W) + t0 * a.row_bytes;
        const uint8_t *sbase = ring + static_cast<size_t>(s) * a.cap + (lo & 15u);
#pragma unroll 2
        for (uint32_t i = 0; i < a.rpl; ++i) {
            const uint32_t rt = ph + i * a.phases;
            const bool live = active && rt < nrows;
            float v = 0.f;
            if (live) v = D::row_dot(sbase + rt * row_bytes32, pos, lane_x);
#pragma unroll
            for (uint32_t o = 1; o < 8; o <<= 1)
                if (o < a.rw) v += __shfl_xor_sync(kFull, v, o);
            if (writer && rt < nrows) pb[rt * a.npart + part_col] = v;
        }
        // ticket: the last warp through this tile reduces it and refills the stage
        __syncwarp();
        int t = 0;
        if (lane == 0) {
            __threadfence_block();
            t = atomicAdd(tickets + s, 1);
        }
        t = __shfl_sync(kFull, t, 0);
        if (t == static_cast<int>(nwarps) - 1) {
            __threadfence_block();
            for (uint32_t r = lane; r < nrows; r += 32) {
                const float *pr = pb + r * a.npart;
                float acc = 0.f;
                for (uint32_t j = 0; j < a.npart; ++j) acc += pr[j];
                a.y[t0 + r] = acc;
            }
            __syncwarp();
            if (lane == 0) {
                tickets[s] = 0;
                if (it + a.nst < n_tiles) {
                    fence_proxy_async_smem();   // the stage was read through the generic proxy
                    issue(it + a.nst);
                    atomicMax(issued, static_cast<int>(it + a.nst + 1));
                }
            }
            __syncwarp();
        }
    }

    __syncthreads();
    if (fail && tid == 0) {
        // A wait ran out: let every copy still in flight land before the CTA exits
        // (fixed, generous bound: they target valid memory and always complete).
        const uint32_t n_issued = static_cast<uint32_t>(*issued);
        for (uint32_t it = consumed; it < n_issued; ++it)
            mbar_wait_bounded(smem_u32(bars + it % a.nst), (it / a.nst) & 1u, nullptr, kDrainLimit);
    }
}

// ---------------------------------------------------------------------------
// host side: launch planning
// ---------------------------------------------------------------------------
static constexpr int kSmemMax = 232448;          // 227 KB opt-in per CTA on sm_100
static constexpr uint32_t kStageTarget = 32768;  // bytes of weights per stage

template <class D>
static int launch_dec(MvArgs &a, int num_sms, cudaStream_t st)
{
    auto kern = k_matvec<D>;
    const uint32_t groups = (a.K + 31) / 32;
    a.cs = (groups + D::GPL - 1) / D::GPL;
    if (!smem_attr_once(reinterpret_cast<const void *>(kern), kSmemMax)) return 0;
    static thread_local cudaFuncAttributes fa{};
    static thread_local const void *fa_for = nullptr;
    if (fa_for != reinterpret_cast<const void *>(kern)) {
        if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return 0;
        fa_for = reinterpret_cast<const void *>(kern);
    }
    const uint32_t max_warps = static_cast<uint32_t>(fa.maxThreadsPerBlock) / 32;
    if (a.cs > 32 * max_warps) {
        fprintf(stderr, "[tb_cuda] matvec: K=%u needs %u column slots, more than %u threads\n", a.K,
                a.cs, 32 * max_warps);
        return 0;
    }
    // warps per CTA: best fraction of threads owning a slot, preferring 8..12 warps
    uint32_t best_w = 0;
    double best = -1.0;
    for (uint32_t w = 4; w <= max_warps; ++w) {
        const uint32_t P = (32 * w) / a.cs;
        if (!P) continue;
        double util = static_cast<double>(P * a.cs) / (32.0 * w);
        if (w < 8) util -= 0.02 * (8 - w);
        if (util > best + 1e-9) {
            best = util;
            best_w = w;
        }
    }
    if (!best_w) return 0;
    const uint32_t nthr = 32 * best_w;
    a.phases = nthr / a.cs;
    const unsigned long long tile_target = kStageTarget / (a.phases * a.row_bytes);
    a.rpl = static_cast<uint32_t>(tile_target < 1 ? 1 : (tile_target > 8 ? 8 : tile_target));
    a.tr = a.phases * a.rpl;
    a.rw = (a.cs % 8 == 0) ? 8 : (a.cs % 4 == 0) ? 4 : (a.cs % 2 == 0) ? 2 : 1;
    a.npart = a.cs / a.rw;
    a.cap = static_cast<uint32_t>((a.tr * a.row_bytes + 32 + 127) & ~127ull);
    const uint32_t xf = mv_x_floats(a.cs, D::GPL);
    // ring depth: most weight bytes in flight per SM (CTAs per SM x stages ahead)
    size_t bytes = 0;
    int occ = 0;
    unsigned long long best_inflight = 0;
    a.nst = 0;
    for (uint32_t n = 2; n <= 6; ++n) {
        const size_t b = mv_ring_offset(n, a.tr, a.npart, xf) + static_cast<size_t>(n) * a.cap + 16;
        if (b > static_cast<size_t>(kSmemMax)) break;
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, static_cast<int>(nthr), b) != cudaSuccess)
            o = 0;
        if (o < 1) continue;
        const unsigned long long inflight = static_cast<unsigned long long>(o) * (n - 1) * a.cap;
        if (inflight > best_inflight) {
            best_inflight = inflight;
            a.nst = n;
            bytes = b;
            occ = o;
        }
    }
    if (!a.nst) {
        fprintf(stderr, "[tb_cuda] matvec: a %u-row tile of %llu-byte rows does not fit shared memory\n",
                a.tr, a.row_bytes);
        return 0;
    }
    if (getenv("TB_MV_VERBOSE"))
        fprintf(stderr, "[tb_cuda] matvec plan M=%u K=%u: threads %u cs %u phases %u rpl %u tr %u nst %u cap %u smem %zu occ %d\n",
                a.M, a.K, nthr, a.cs, a.phases, a.rpl, a.tr, a.nst, a.cap, bytes, occ);
    const unsigned long long want = static_cast<unsigned long long>(num_sms) * occ;
    const uint32_t grid = static_cast<uint32_t>(want < a.M ? want : a.M);
    kern<<<grid, nthr, bytes, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

int mv_launch(const void *W, int qtype, int M, int K, const float *d_x, float *d_y,
              cudaStream_t st, int *d_err, int num_sms, uint32_t wait_limit)
{
    const Geom g = geom_of(qtype);
    if (!g.block_weights || !W || !d_x || !d_y || M <= 0 || K <= 0 || K % g.block_weights) return 0;
    MvArgs a{};
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

    const bool a16 = (reinterpret_cast<uintptr_t>(W) & 15u) == 0 && (a.row_bytes & 15u) == 0;
    switch (qtype) {
    case QT_Q4_K: return a16 ? launch_dec<DecQ4K<true>>(a, num_sms, st) : launch_dec<DecQ4K<false>>(a, num_sms, st);
    case QT_Q5_K: return a16 ? launch_dec<DecQ5K<true>>(a, num_sms, st) : launch_dec<DecQ5K<false>>(a, num_sms, st);
    case QT_Q6_K: return launch_dec<DecQ6K>(a, num_sms, st);
    case QT_Q3_K:
    case QT_IQ3_S: return launch_dec<DecQ3K>(a, num_sms, st);
    case QT_Q2_K: return launch_dec<DecQ2K>(a, num_sms, st);
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
