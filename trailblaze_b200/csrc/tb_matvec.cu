// tb_matvec.cu — persistent sm_100a GGUF dequant x fp32 matvec.
//
// Replaces the ten one-CTA-per-row kernels of layer4/tb_gguf_dequant.cu:89-332
// (plus Q2_K, which the reference lacks).  Layout and schedule:
//
//   * W is read as one flat stream of "units" (256 weights of one row; rows are
//     contiguous, so the stream is W's memory order).  Each CTA owns a
//     contiguous range of rows; its units are split evenly over its warps.
//   * Each warp runs its own ring of NST shared-memory stages.  Lane 0 fills a
//     stage with one 1-D bulk copy (cp.async.bulk, TMA engine, no multicast) of
//     the next 32 units, widened to 16-byte boundaries, with an L2 evict-first
//     hint; completion is an mbarrier transaction count.  Every wait is bounded.
//   * x is staged once per CTA, prescaled for the decoder's bit-field positions
//     (see tb_decoders.cuh), with 16-element partial sums for the min/offset
//     terms.
//   * Lane l decodes unit (it*32 + l); a segmented shuffle reduction by row
//     combines the lanes, a register carry joins a row across iterations, and
//     rows that straddle two warps are combined in warp order at the end, so the
//     summation order is fixed and results are run-to-run deterministic.
#include <cstdio>

#include "tb_common.cuh"
#include "tb_decoders.cuh"
#include "tb_internal.h"

namespace tb {

struct MvArgs {
    const uint8_t *W;
    const float *x;
    float *y;
    int *err;
    uint32_t M, K, upr;           // rows, columns, units per row
    uint32_t unit_bytes;          // bytes of a full unit
    uint32_t last_unit_bytes;     // bytes of a row's last unit
    uint32_t unit_n, last_unit_n; // blocks (Q4_0/Q8_0) or elements (F*) in full / last unit
    unsigned long long row_bytes;
    FastDiv fd_upr;
    uint32_t nst, cap;            // stages per warp, bytes per stage
    uint32_t wait_limit;
};

static constexpr uint32_t kFull = 0xFFFFFFFFu;
static constexpr uint32_t kDrainLimit = 1u << 26;

template <class D, int NW>
__global__ void __launch_bounds__(NW * 32, 1) k_matvec(const MvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const uint32_t G = gridDim.x, c = blockIdx.x;
    const uint32_t r_lo = static_cast<uint32_t>((static_cast<unsigned long long>(a.M) * c) / G);
    const uint32_t r_hi = static_cast<uint32_t>((static_cast<unsigned long long>(a.M) * (c + 1)) / G);
    if (r_lo >= r_hi) return;
    const uint32_t U_lo = r_lo * a.upr, U = (r_hi - r_lo) * a.upr;
    const uint32_t u0 = U_lo + static_cast<uint32_t>((static_cast<unsigned long long>(U) * warp) / NW);
    const uint32_t u1 = U_lo + static_cast<uint32_t>((static_cast<unsigned long long>(U) * (warp + 1)) / NW);
    const uint32_t n_it = (u1 - u0 + 31) / 32;

    // ---- shared memory carve-up (mirrors mv_smem_bytes on the host) ----
    float *xs = reinterpret_cast<float *>(smem);
    const uint32_t xstride = a.upr * XSTRIDE;
    float *xs16 = xs + D::NXA * xstride;
    uintptr_t p = reinterpret_cast<uintptr_t>(xs16 + a.upr * 16);
    p = (p + 15) & ~uintptr_t(15);
    uint64_t *bars = reinterpret_cast<uint64_t *>(p);
    p += sizeof(uint64_t) * NW * a.nst;
    int2 *bnd = reinterpret_cast<int2 *>(p);
    p += sizeof(int2) * NW * 2;
    p = (p + 127) & ~uintptr_t(127);
    uint8_t *ring = reinterpret_cast<uint8_t *>(p) + static_cast<size_t>(warp) * a.nst * a.cap;
    uint64_t *mybar = bars + warp * a.nst;

    auto unit_addr = [&](uint32_t u, uint32_t &row, uint32_t &j) -> uintptr_t {
        row = fdiv(u, a.fd_upr);
        j = u - row * a.upr;
        return reinterpret_cast<uintptr_t>(a.W) + row * a.row_bytes +
               static_cast<unsigned long long>(j) * a.unit_bytes;
    };

    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](uint32_t it) {   // lane 0 only
        uint32_t r, j;
        const uint32_t ua = u0 + 32 * it, ub = min(ua + 32, u1) - 1;
        const uintptr_t g0 = unit_addr(ua, r, j) & ~uintptr_t(15);
        const uintptr_t gb = unit_addr(ub, r, j);
        const uintptr_t g1 = (gb + (j == a.upr - 1 ? a.last_unit_bytes : a.unit_bytes) + 15) & ~uintptr_t(15);
        const uint32_t s = it % a.nst;
        const uint32_t bar = smem_u32(mybar + s);
        mbar_expect_tx(bar, static_cast<uint32_t>(g1 - g0));
        bulk_g2s(smem_u32(ring + s * a.cap), reinterpret_cast<const void *>(g0),
                 static_cast<uint32_t>(g1 - g0), bar, pol);
    };

    if (lane == 0) {
        for (uint32_t s = 0; s < a.nst; ++s) mbar_init(smem_u32(mybar + s), 1);
        fence_mbar_init();
        const uint32_t pre = min(a.nst, n_it);
        for (uint32_t it = 0; it < pre; ++it) issue(it);
    }
    if (lane < 2) bnd[warp * 2 + lane] = make_int2(-1, 0);
    __syncwarp();

    // ---- stage x: prescaled arrays + 16-element sums, zero beyond K ----
    const uint32_t kpad = a.upr * 256;
    for (uint32_t k = tid; k < kpad; k += NW * 32) {
        const float v = k < a.K ? __ldg(a.x + k) : 0.f;
        const uint32_t jj = k >> 8, i = k & 255;
#pragma unroll
        for (int arr = 0; arr < D::NXA; ++arr)
            xs[arr * xstride + jj * XSTRIDE + i] = v * D::xmul(arr, static_cast<int>(i));
        float s = v;
        s += __shfl_xor_sync(kFull, s, 8);
        s += __shfl_xor_sync(kFull, s, 4);
        s += __shfl_xor_sync(kFull, s, 2);
        s += __shfl_xor_sync(kFull, s, 1);
        if ((lane & 15) == 0) xs16[k >> 4] = s;
    }
    __syncthreads();

    // ---- main loop ----
    uint32_t carry_row = kFull;
    float carry = 0.f;
    uint32_t consumed = 0;
    bool ok = true;
    for (uint32_t it = 0; it < n_it; ++it) {
        const uint32_t s = it % a.nst, ph = (it / a.nst) & 1u;
        const bool got = mbar_wait_bounded(smem_u32(mybar + s), ph, a.err, a.wait_limit);
        if (!__all_sync(kFull, got)) { ok = false; break; }
        consumed = it + 1;

        const uint32_t ua = u0 + 32 * it;
        uint32_t r0, j0;
        const uintptr_t g0 = unit_addr(ua, r0, j0) & ~uintptr_t(15);
        const uint32_t u = ua + lane;
        const bool valid = u < u1;
        uint32_t row = kFull, j = 0;
        float v = 0.f;
        if (valid) {
            const uintptr_t gu = unit_addr(u, row, j);
            const uint8_t *su = ring + s * a.cap + (gu - g0);
            const int n = static_cast<int>(j == a.upr - 1 ? a.last_unit_n : a.unit_n);
            v = D::dot(su, n, xs + j * XSTRIDE, xs + xstride + j * XSTRIDE, xs16 + j * 16);
        }
        __syncwarp();
        if (lane == 0 && it + a.nst < n_it) {
            fence_proxy_async_smem();   // order this warp's reads of stage s before the refill
            issue(it + a.nst);
        }

        // segmented suffix sum over lanes with equal row (rows are non-decreasing)
        const uint32_t last_lane = min(31u, u1 - 1 - ua);
        const uint32_t row_last = __shfl_sync(kFull, row, last_lane);
        const uint32_t j_last = __shfl_sync(kFull, j, last_lane);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float t = __shfl_down_sync(kFull, v, o);
            const uint32_t rr = __shfl_down_sync(kFull, row, o);
            if (lane + o < 32 && rr == row) v += t;
        }
        const uint32_t row_prev = __shfl_up_sync(kFull, row, 1);
        const bool head = valid && (lane == 0 || row_prev != row);
        if (lane == 0 && row == carry_row) v += carry;
        const bool continues = (row == row_last) && (j_last < a.upr - 1);
        const bool carry_next = (j_last < a.upr - 1) && (ua + last_lane + 1 < u1);
        const uint32_t heads = __ballot_sync(kFull, head);
        const int last_head = 31 - __clz(heads);
        const float last_v = __shfl_sync(kFull, v, last_head);
        if (head) {
            const bool started_before = row * a.upr < u0;
            if (continues && carry_next) {
                // joins the next iteration through the carry
            } else if (started_before) {
                bnd[warp * 2 + 0] = make_int2(static_cast<int>(row), __float_as_int(v));
            } else if (continues) {
                bnd[warp * 2 + 1] = make_int2(static_cast<int>(row), __float_as_int(v));
            } else {
                a.y[row] = v;
            }
        }
        if (carry_next) {
            carry_row = row_last;
            carry = last_v;
        } else {
            carry_row = kFull;
        }
    }

    if (!ok && lane == 0) {
        // A wait ran out: let this warp's copies still in flight land before the
        // CTA exits (bounded again), leaving the error word set.
        // The drain limit is fixed and generous (not the caller's wait_limit): the copies were
        // issued to valid addresses and always land; the CTA must not exit before they do.
        const uint32_t issued = min(n_it, consumed + a.nst);
        for (uint32_t it = consumed; it < issued; ++it)
            mbar_wait_bounded(smem_u32(mybar + it % a.nst), (it / a.nst) & 1u, nullptr, kDrainLimit);
    }
    __syncthreads();

    // rows split between warps: combine the partials in warp order
    if (tid == 0 && ok) {
        int cur = -1;
        float acc = 0.f;
        for (int w = 0; w < NW; ++w) {
#pragma unroll
            for (int sl = 0; sl < 2; ++sl) {
                const int2 e = bnd[w * 2 + sl];
                if (e.x < 0) continue;
                if (e.x == cur) {
                    acc += __int_as_float(e.y);
                } else {
                    if (cur >= 0) a.y[cur] = acc;
                    cur = e.x;
                    acc = __int_as_float(e.y);
                }
            }
        }
        if (cur >= 0) a.y[cur] = acc;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static constexpr int kSmemMax = 232448;   // 227 KB opt-in per CTA on sm_100

static size_t mv_smem_bytes(int nxa, uint32_t upr, int nw, uint32_t nst, uint32_t cap)
{
    size_t b = static_cast<size_t>(nxa) * upr * XSTRIDE * 4 + static_cast<size_t>(upr) * 16 * 4;
    b = (b + 15) & ~size_t(15);
    b += 8ull * nw * nst + 8ull * nw * 2;
    b = (b + 127) & ~size_t(127);
    b += static_cast<size_t>(nw) * nst * cap;
    return b + 16;   // tail pad: funnel reads of a stage's last unit may touch 8 bytes past it
}

template <class D, int NW>
static int launch_one(MvArgs &a, int num_sms, cudaStream_t st)
{
    auto kern = k_matvec<D, NW>;
    if (!smem_attr_once(reinterpret_cast<const void *>(kern), kSmemMax)) return 0;
    size_t bytes = 0;
    uint32_t nst = 0;
    for (uint32_t cand = 4; cand >= 2; --cand) {
        bytes = mv_smem_bytes(D::NXA, a.upr, NW, cand, a.cap);
        if (bytes <= static_cast<size_t>(kSmemMax)) { nst = cand; break; }
    }
    if (!nst) return -1;   // does not fit: caller tries fewer warps
    a.nst = nst;
    const uint32_t grid = a.M < static_cast<uint32_t>(num_sms) ? a.M : static_cast<uint32_t>(num_sms);
    kern<<<grid, NW * 32, bytes, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

template <class D>
static int launch_dec(MvArgs &a, int num_sms, cudaStream_t st)
{
    int r = launch_one<D, 8>(a, num_sms, st);
    if (r < 0) r = launch_one<D, 4>(a, num_sms, st);
    if (r < 0) {
        fprintf(stderr, "[tb_cuda] matvec: K=%u too large for the shared-memory x stage\n", a.K);
        return 0;
    }
    return r;
}

int mv_launch(const void *W, int qtype, int M, int K, const float *d_x, float *d_y,
              cudaStream_t st, int *d_err, int num_sms, uint32_t wait_limit)
{
    const Geom g = geom_of(qtype);
    if (!g.block_weights || !W || !d_x || !d_y || M <= 0 || K <= 0 || K % g.block_weights)
        return 0;
    const uint32_t nb = static_cast<uint32_t>(K / g.block_weights);   // blocks per row
    const uint32_t upr = (nb + g.unit_blocks - 1) / g.unit_blocks;
    if (static_cast<unsigned long long>(upr) * static_cast<unsigned long long>(M) >= (1ull << 31))
        return 0;
    MvArgs a{};
    a.W = static_cast<const uint8_t *>(W);
    a.x = d_x;
    a.y = d_y;
    a.err = d_err;
    a.M = static_cast<uint32_t>(M);
    a.K = static_cast<uint32_t>(K);
    a.upr = upr;
    a.unit_bytes = static_cast<uint32_t>(g.unit_blocks * g.block_bytes);
    const uint32_t last_blocks = nb - (upr - 1) * g.unit_blocks;
    a.last_unit_bytes = last_blocks * g.block_bytes;
    const bool per_elem = g.block_weights == 1;
    a.unit_n = per_elem ? 256u : static_cast<uint32_t>(g.unit_blocks);
    a.last_unit_n = last_blocks;
    a.row_bytes = static_cast<unsigned long long>(nb) * g.block_bytes;
    a.fd_upr = make_fastdiv(upr);
    a.cap = (32u * a.unit_bytes + 32u + 127u) & ~127u;
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
