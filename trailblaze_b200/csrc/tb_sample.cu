// tb_sample.cu — top-k and nucleus (top-p) sampling of one logits vector on
// the device (layer1/tb_tensor.c:411-540, tb_sample_top_p / tb_sample_top_k).
//
// One CTA of kSmpThreads threads; warp w owns a contiguous segment of the
// vocabulary, read coalesced kChunk elements at a time (warp order = index
// order; within a warp, ballots keep index order).  The caller supplies the uniform variate u
// in [0, 1) that the reference draws with rand() / (RAND_MAX + 1.0f); the
// kernel writes the chosen token index.
//
// Inside the decode graph the variate comes from device memory instead
// (u_dev[*u_idx], the step's entry of a caller-filled array) and the kernel
// also advances the step: pos <- pos + 1, u_idx <- u_idx + 1.
//
// top-p (tb_tensor.c:423-504): softmax of logits / t (t = temperature when
//   > 0.01, else 1) over the whole vocabulary; candidates = the tokens whose
//   probability is >= 1e-4 of the largest, in index order, at most 2047 of
//   them; sorted by probability, largest first (equal probabilities keep
//   index order, as the reference's insertion sort does); cut after the first
//   prefix whose sum reaches p; r = u * (sum of the kept), the first kept
//   token whose running sum reaches r.
// top-k (tb_tensor.c:506-540): k >= vocab falls back to top-p with p = 0.95;
//   else the k largest logits (found here by a radix select on their bits,
//   equal values by lower index), softmax of (l - l_max) / t (t = temperature
//   when > 0, else 1), r = u * sum, the first whose running sum reaches r.
//
// Sums over the vocabulary are tree sums here and sequential in the
// reference (a rounding-level difference); the running sums over the kept
// candidates are sequential, in the reference's order.
#include <cfloat>
#include <cstdint>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

static constexpr int kSmpThreads = 1024;
static constexpr int kNucleusMax = 2048;   // candidate slots (the reference keeps at most 2047)
static constexpr int kSmpWarps = kSmpThreads / 32;
static constexpr int kPer = 8;                   // coalesced loads in flight per lane
static constexpr int kChunk = 32 * kPer;         // elements a warp reads per iteration

struct SmpArgs {
    const float *logits;
    int *token;
    int *err;
    int vocab, k;
    float p, temp, u;
    const float *u_dev;   // not null: u = u_dev[*u_idx], and the step advances
    int *u_idx, *pos;
    SmpTP tp;             // tensor parallelism: wait for the ranks' logits, count the step
    // two-stage top-k: logits are the candidates of k_topk_pre, cmap their
    // vocabulary indices; *nonfin (read and reset here) reports a non-finite
    // logit anywhere in the vocabulary
    const int *cmap;
    int *nonfin;
};

// Thread 0: the chosen token, and the decode step's advance when the variate
// came from device memory.
__device__ __forceinline__ void finish(const SmpArgs &a, int token)
{
    *a.token = token;
    if (a.u_dev) {
        *a.pos = *a.pos + 1;
        *a.u_idx = *a.u_idx + 1;
    }
    if (a.tp.epoch) *a.tp.epoch = *a.tp.epoch + 1;
}

__device__ __forceinline__ float variate(const SmpArgs &a)
{
    return a.u_dev ? a.u_dev[*a.u_idx] : a.u;
}

// fp32 bits mapped to unsigned integers of the same order (NaN excluded).
__device__ __forceinline__ uint32_t ord_key(float f)
{
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float block_max(float v, float *red)
{
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < kSmpThreads / 32; ++w) m = fmaxf(m, red[w]);
    return m;
}

__device__ __forceinline__ float block_sum(float v, float *red)
{
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
    for (int w = 0; w < kSmpThreads / 32; ++w) s += red[w];
    return s;
}

// Exclusive prefix of one count per thread, in thread order; returns the total.
__device__ __forceinline__ int block_scan(int c, int &excl, int *red)
{
    int incl = c;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += t;
    }
    __syncthreads();
    if (lane == 31) red[warp] = incl;
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < kSmpThreads / 32; ++w) {
        if (w < warp) before += red[w];
        total += red[w];
    }
    excl = before + incl - c;
    return total;
}

// Sorts n <= kNucleusMax (value, index) pairs: value descending, index
// ascending among equal values (bitonic network over the next power of two).
__device__ void sort_desc(float *val, int *idx, int n)
{
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    for (int i = n + threadIdx.x; i < n2; i += kSmpThreads) {   // pads sort last
        val[i] = -FLT_MAX;
        idx[i] = 0x7FFFFFFF;
    }
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n2; i += kSmpThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    // "a before b": larger value, or equal value and lower index
                    const bool ib = val[i] > val[j] || (val[i] == val[j] && idx[i] < idx[j]);
                    const bool up = (i & size) == 0;   // this half sorted in the final order
                    if (ib != up) {
                        const float tv = val[i];
                        val[i] = val[j];
                        val[j] = tv;
                        const int ti = idx[i];
                        idx[i] = idx[j];
                        idx[j] = ti;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ int warp_sum(int v)
{
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Running sum of v[0..n) in index order: the first index whose running sum
// reaches target, or n - 1 when none does; cum receives the running sum at
// that index.  Loads run 8 ahead of the dependent additions.
__device__ __forceinline__ int first_reaching(const float *v, int n, float target, float &cum)
{
    float acc = 0.f;
    for (int i0 = 0; i0 < n; i0 += 8) {
        float w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = i0 + j < n ? v[i0 + j] : 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (i0 + j < n) {
                acc += w[j];
                if (acc >= target) {
                    cum = acc;
                    return i0 + j;
                }
            }
        }
    }
    cum = acc;
    return n - 1;
}

// One radix step's bin, by warp 0: the largest b in 255 .. 1 whose bins b ..
// 255 hold at least `need` keys (else 0), and need minus the keys in the bins
// above it: what a scan from bin 255 downwards finds, with lane l adding bins
// 255 - 8l down to 248 - 8l and a shuffle prefix over the lanes.
__device__ __forceinline__ void select_bin(const int *hist, int need, int *sel, int *rem)
{
    const int lane = threadIdx.x & 31, hi = 255 - 8 * lane;
    int t = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += hist[hi - j];
    int incl = t;
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += u;
    }
    const int excl = incl - t;   // keys in the bins above this lane's
    const unsigned reach = __ballot_sync(0xFFFFFFFFu, incl >= need);
    const int L = reach ? __ffs(reach) - 1 : 31;
    if (lane == L) {
        // lane L's lowest bin is taken untested: its bins reach need (lanes
        // before it did not), or it is bin 0, which the downward scan takes
        // untested as well
        int acc = excl, b = hi;
        for (; b > hi - 7; --b) {
            if (acc + hist[b] >= need) break;
            acc += hist[b];
        }
        *sel = b;
        *rem = need - acc;
    }
}

// Visits the warp's segment [lo, hi) of the logits: each iteration loads
// kChunk consecutive elements, kPer per lane (element b + 32 j + lane), and
// calls f(index, value, in_range) in ascending index order, j-major; every
// lane of the warp calls f the same number of times, so f may vote.
template <class F>
__device__ __forceinline__ void for_seg(const float *lg, int lo, int hi, int lane, F &&f)
{
    for (int b = lo; b < hi; b += kChunk) {
        float v[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = b + j * 32 + lane;
            v[j] = i < hi ? __ldcg(lg + i) : 0.f;   // through L2: peers may have written them (tensor parallel)
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) f(b + j * 32 + lane, v[j], b + j * 32 + lane < hi);
    }
}

__global__ void __launch_bounds__(kSmpThreads, 1) k_sample(const SmpArgs a)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ float cval[kNucleusMax];
    __shared__ int cidx[kNucleusMax];
    __shared__ float red[kSmpWarps];
    __shared__ int ired[kSmpWarps];
    __shared__ int hist[256];
    __shared__ int s_n, s_sel;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, V = a.vocab;
    if (a.tp.ctr) {
        // tensor parallelism: every rank's logits slice has arrived (a bounded
        // wait; once a wait of this device ran out the step only finishes)
        if (tid == 0 && *reinterpret_cast<volatile int *>(a.err) == 0 &&
            !wait_counter(a.tp.ctr, static_cast<unsigned long long>(*a.tp.epoch + 1) * a.tp.per_step, a.tp.wait_limit))
            atomicExch(a.err, ERR_WAIT_TIMEOUT);
        __syncthreads();
    }
    if (a.nonfin) {   // two-stage top-k: a slice held a non-finite logit
        if (tid == 0) {
            s_sel = *a.nonfin;
            *a.nonfin = 0;
        }
        __syncthreads();
        if (s_sel) {
            if (tid == 0) {
                atomicExch(a.err, ERR_RUNTIME);
                finish(a, 0);
            }
            return;
        }
        __syncthreads();
    }
    const float *lg = a.logits;
    const unsigned below = (1u << lane) - 1u;   // the lanes before this one
    // the warp's contiguous segment of the vocabulary (warp order = index order)
    const int seg = ((V + kSmpWarps - 1) / kSmpWarps + kChunk - 1) / kChunk * kChunk;
    const int wlo = min(V, warp * seg), whi = min(V, wlo + seg);

    int n = 0;   // candidates, sorted into cval / cidx by value descending
    const bool topk = a.k > 0 && a.k < V;
    bool fin = true;   // every logit finite (else the error word and token 0)
    if (!topk) {
        float m = -FLT_MAX;
        for_seg(lg, wlo, whi, lane, [&](int, float v, bool ok) {
            if (ok) {
                fin = fin && isfinite(v);
                m = fmaxf(m, v);
            }
        });
        if (!__syncthreads_and(fin ? 1 : 0)) {
            if (tid == 0) {
                atomicExch(a.err, ERR_RUNTIME);
                finish(a, 0);
            }
            return;
        }
        m = block_max(m, red);
        // ---- nucleus candidates: probabilities >= 1e-4 of the peak ----
        const float p = a.k > 0 ? 0.95f : a.p;   // tb_sample_top_k's fallback for k >= vocab
        const float t = a.temp > 0.01f ? a.temp : 1.0f;
        float s = 0.f;
        for_seg(lg, wlo, whi, lane, [&](int, float v, bool ok) { s += ok ? expf((v - m) / t) : 0.f; });
        const float sum = block_sum(s, red);
        const float inv = sum > 0.f ? 1.0f / sum : 1.0f;
        // the peak probability is that of the largest logit: expf(0) * inv
        const float thr = inv * 1e-4f;
        // a logit more than 9.5 t below the peak has a probability below
        // e^-9.49 < 7.6e-5 of the peak, far from the 1e-4 test: no expf needed
        const float lcut = m - 9.5f * t;
        int c = 0;
        for_seg(lg, wlo, whi, lane, [&](int, float v, bool ok) {
            c += ok && v >= lcut && expf((v - m) / t) * inv >= thr ? 1 : 0;
        });
        c = warp_sum(c);
        int base;
        const int total = block_scan(lane == 0 ? c : 0, base, ired);
        base = __shfl_sync(0xFFFFFFFFu, base, 0);   // candidates in the warps before this one
        n = min(total, kNucleusMax - 1);
        for_seg(lg, wlo, whi, lane, [&](int i, float v, bool ok) {
            float q = 0.f;
            bool take = false;
            if (ok && v >= lcut) {
                q = expf((v - m) / t) * inv;
                take = q >= thr;
            }
            const unsigned vote = __ballot_sync(0xFFFFFFFFu, take);
            const int at = base + __popc(vote & below);
            if (take && at < n) {
                cval[at] = q;
                cidx[at] = i;
            }
            base += __popc(vote);
        });
        __syncthreads();
        sort_desc(cval, cidx, n);
        if (tid == 0) {
            // cut after the first prefix reaching p; its running sum is the
            // sum of the kept candidates, added in the same order
            float cum, acc;
            const int cut = first_reaching(cval, n, p, cum);
            const float r = variate(a) * cum;
            // the first kept candidate reaching r (the last kept when none does)
            finish(a, cidx[first_reaching(cval, cut + 1, r, acc)]);
        }
        return;
    }

    // ---- top-k: radix select of the k-th largest key, 8 bits at a time ----
    uint32_t prefix = 0, pmask = 0;
    int need = a.k;   // how many of the keys with this prefix are still to be taken
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += kSmpThreads) hist[b] = 0;
        __syncthreads();
        // the lanes that fall into one bin add their count with one shared
        // atomic (the upper bytes of nearby logits agree, so bins are crowded)
        for_seg(lg, wlo, whi, lane, [&](int, float v, bool ok) {
            uint32_t bin = 256u;
            if (ok) {
                fin = fin && isfinite(v);
                const uint32_t key = ord_key(v);
                if ((key & pmask) == prefix) bin = (key >> shift) & 255u;
            }
            if (__any_sync(0xFFFFFFFFu, bin < 256u)) {   // later passes: most warps match nothing
                const uint32_t same = __match_any_sync(0xFFFFFFFFu, bin);
                if (bin < 256u && lane == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
            }
        });
        if (shift == 24) {   // the first pass read every logit
            if (!__syncthreads_and(fin ? 1 : 0)) {
                if (tid == 0) {
                    atomicExch(a.err, ERR_RUNTIME);
                    finish(a, 0);
                }
                return;
            }
        } else {
            __syncthreads();
        }
        if (warp == 0) select_bin(hist, need, &s_sel, &s_n);
        __syncthreads();
        prefix |= static_cast<uint32_t>(s_sel) << shift;
        pmask |= 255u << shift;
        need = s_n;
        __syncthreads();
    }
    // prefix is the k-th largest key: every key above it, and the first `need`
    // keys equal to it in index order
    int cg = 0, ce = 0;
    for_seg(lg, wlo, whi, lane, [&](int, float v, bool ok) {
        const uint32_t key = ord_key(v);
        cg += ok && key > prefix ? 1 : 0;
        ce += ok && key == prefix ? 1 : 0;
    });
    cg = warp_sum(cg);
    ce = warp_sum(ce);
    int bg, be;
    const int ng = block_scan(lane == 0 ? cg : 0, bg, ired);
    block_scan(lane == 0 ? ce : 0, be, ired);
    bg = __shfl_sync(0xFFFFFFFFu, bg, 0);
    be = __shfl_sync(0xFFFFFFFFu, be, 0);
    for_seg(lg, wlo, whi, lane, [&](int i, float v, bool ok) {
        const uint32_t key = ord_key(v);
        const bool gt = ok && key > prefix, eq = ok && key == prefix;
        const unsigned vg = __ballot_sync(0xFFFFFFFFu, gt), ve = __ballot_sync(0xFFFFFFFFu, eq);
        if (gt) {
            const int at = bg + __popc(vg & below);
            cval[at] = v;
            cidx[at] = a.cmap ? a.cmap[i] : i;
        } else if (eq) {
            const int rank = be + __popc(ve & below);
            if (rank < need) {
                cval[ng + rank] = v;
                cidx[ng + rank] = a.cmap ? a.cmap[i] : i;
            }
        }
        bg += __popc(vg);
        be += __popc(ve);
    });
    n = a.k;
    __syncthreads();
    sort_desc(cval, cidx, n);
    // softmax numerators from the top logit on every thread; thread 0 then
    // adds them in rank order, as the reference's loop does
    const float t = a.temp > 0.f ? a.temp : 1.0f;
    const float mv = cval[0];
    __syncthreads();
    for (int i = tid; i < n; i += kSmpThreads) cval[i] = expf((cval[i] - mv) / t);
    __syncthreads();
    if (tid == 0) {
        float sum = 0.f;
        for (int i = 0; i < n; ++i) sum += cval[i];
        const float r = variate(a) * sum;
        float acc;
        const int j = first_reaching(cval, n, r, acc);
        finish(a, acc >= r ? cidx[j] : cidx[0]);   // the top candidate when no running sum reaches r
    }
}

// ---- two-stage top-k, stage 1 ----
// CTA c takes the vocabulary slice [c V / G, (c+1) V / G) (at least k and at
// most kSliceMax logits), selects its k largest by the same order as k_sample
// (value descending, lower index first among equal values: a radix select of
// the k-th largest key over the slice in shared memory) and writes them, in
// vocabulary order, to cv / ci [c k, (c+1) k).  The k largest of the whole
// vocabulary are among the G k candidates, in the same relative order, so
// k_sample's top-k over the candidates (cmap = ci) selects the same tokens.
// A non-finite logit sets *nonfin instead (k_sample reports it).
static constexpr int kPreThreads = 512;
static constexpr int kSliceMax = 4096;

struct PreArgs {
    const float *logits;
    int vocab, k;
    float *cv;
    int *ci, *nonfin, *err;
    SmpTP tp;
};

__device__ __forceinline__ float key_val(uint32_t key)
{
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

__global__ void __launch_bounds__(kPreThreads) k_topk_pre(const PreArgs p)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ uint32_t keys[kSliceMax];
    __shared__ int hist[256];
    __shared__ int wsum[kPreThreads / 32], wsum2[kPreThreads / 32];
    __shared__ int s_sel, s_n;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kPreThreads / 32;
    if (p.tp.ctr) {   // tensor parallelism: every rank's logits slice has arrived
        if (tid == 0 && *reinterpret_cast<volatile int *>(p.err) == 0 &&
            !wait_counter(p.tp.ctr, static_cast<unsigned long long>(*p.tp.epoch + 1) * p.tp.per_step, p.tp.wait_limit))
            atomicExch(p.err, ERR_WAIT_TIMEOUT);
        __syncthreads();
    }
    const int G = gridDim.x, c = blockIdx.x;
    const int lo = static_cast<int>((static_cast<long long>(p.vocab) * c) / G);
    const int n = static_cast<int>((static_cast<long long>(p.vocab) * (c + 1)) / G) - lo;
    bool fin = true;
    for (int i = tid; i < n; i += kPreThreads) {
        const float v = __ldcg(p.logits + lo + i);
        fin = fin && isfinite(v);
        keys[i] = ord_key(v);
    }
    if (!__syncthreads_and(fin ? 1 : 0)) {
        if (tid == 0) atomicOr(p.nonfin, 1);
        return;
    }
    // the k-th largest key of the slice, 8 bits at a time
    uint32_t prefix = 0, pmask = 0;
    int need = p.k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += kPreThreads) hist[b] = 0;
        __syncthreads();
        for (int i = tid; i < n; i += kPreThreads) {
            const uint32_t key = keys[i];
            if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
        }
        __syncthreads();
        if (warp == 0) select_bin(hist, need, &s_sel, &s_n);
        __syncthreads();
        prefix |= static_cast<uint32_t>(s_sel) << shift;
        pmask |= 255u << shift;
        need = s_n;
        __syncthreads();
    }
    // the keys above prefix and the first `need` equal to it, in slice order:
    // per pass of kPreThreads elements, block-wide ordered ranks of the equal
    // keys and of the taken ones
    const unsigned below = (1u << lane) - 1u;
    int eq_done = 0, out = 0;
    for (int base = 0; base < n; base += kPreThreads) {
        const int i = base + tid;
        const uint32_t key = i < n ? keys[i] : 0u;
        const bool gt = i < n && key > prefix, eq = i < n && key == prefix;
        const unsigned ve = __ballot_sync(0xFFFFFFFFu, eq);
        if (lane == 0) wsum[warp] = __popc(ve);
        __syncthreads();
        int ebefore = 0, etot = 0;
        for (int w = 0; w < NW; ++w) {
            ebefore += w < warp ? wsum[w] : 0;
            etot += wsum[w];
        }
        const bool take = gt || (eq && eq_done + ebefore + __popc(ve & below) < need);
        const unsigned vt = __ballot_sync(0xFFFFFFFFu, take);
        if (lane == 0) wsum2[warp] = __popc(vt);
        __syncthreads();
        int tbefore = 0, ttot = 0;
        for (int w = 0; w < NW; ++w) {
            tbefore += w < warp ? wsum2[w] : 0;
            ttot += wsum2[w];
        }
        if (take) {
            const int at = c * p.k + out + tbefore + __popc(vt & below);
            p.cv[at] = key_val(key);
            p.ci[at] = lo + i;
        }
        eq_done += etot;
        out += ttot;
        __syncthreads();
    }
}

int sample_launch(const float *d_logits, int vocab, int top_k, float top_p, float temperature, float u,
                  int *d_token, int *d_err, cudaStream_t st, const float *d_u, int *d_u_idx, int *d_pos,
                  const SmpTP *tp, const SmpScratch *scr)
{
    const NvtxRange nvtx("tb.sample");
    if (!d_logits || !d_token || vocab <= 0 || top_k < 0 || (top_k > 0 && top_k < vocab && top_k > kNucleusMax) ||
        (top_k == 0 && !(top_p > 0.f && top_p <= 1.f)))
        return 0;
    if (d_u ? (!d_u_idx || !d_pos) : !(u >= 0.f && u < 1.f)) return 0;
    SmpArgs a{d_logits, d_token, d_err, vocab, top_k, top_p, temperature, u, d_u, d_u_idx, d_pos, SmpTP{},
              nullptr, nullptr};
    if (tp) a.tp = *tp;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    // Two stages when the top k is a small share of the vocabulary: G slices of
    // at least 4k (and at most kSliceMax) logits, G between 8 and the SM count.
    int dev = 0, sms = 0;
    if (scr && scr->cv && top_k > 0 && top_k < vocab && cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
        int G = vocab / (4 * top_k);
        if (G > sms) G = sms;
        if (G * top_k > kSmpPreCap) G = kSmpPreCap / top_k;
        if (G >= 8 && (vocab + G - 1) / G <= kSliceMax) {
            PreArgs pa{d_logits, vocab, top_k, scr->cv, scr->ci, scr->nonfin, d_err, a.tp};
            cudaLaunchConfig_t pc{};
            pc.gridDim = dim3(G);
            pc.blockDim = dim3(kPreThreads);
            pc.stream = st;
            pc.attrs = attr;
            pc.numAttrs = 1;
            if (cudaLaunchKernelEx(&pc, k_topk_pre, pa) != cudaSuccess) {
                cudaGetLastError();
                return 0;
            }
            a.logits = scr->cv;
            a.vocab = G * top_k;
            a.cmap = scr->ci;
            a.nonfin = scr->nonfin;
            a.tp.ctr = nullptr;   // the first stage waited; the step is still counted (epoch)
        }
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kSmpThreads);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_sample, a) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return 1;
}

}  // namespace tb
