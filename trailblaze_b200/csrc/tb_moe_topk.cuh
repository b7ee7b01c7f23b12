// tb_moe_topk.cuh — the routed layer's expert selection for one thread block.
//
// Softmax of the E router logits, the top k ranked by probability (then lower
// index), their weights renormalised to sum to 1 (layer4/tb_infer.c:351-374),
// and with ep_n > 0 the selected experts that live on this rank (ids in
// [ep_lo, ep_lo + ep_n)) as local indices lids[0 .. *nloc) with weights lw, in
// rank order.  Called by every thread of a block of at least E threads
// (E <= kTopkMax); sh is 2 * kTopkMax + 34 floats of shared memory.  The
// logits are read through L2, so they may come from other CTAs of the same
// launch (after the caller's fence and ticket).
#pragma once

#include <cfloat>
#include <cstdint>

namespace tb {

static constexpr int kTopkMax = 256;   // experts per router at most (tb_infer.c:254 caps at 256)

__device__ __forceinline__ void moe_topk_block(const float *logits, int E, int k, int *ids, float *wts, int *err,
                                               int ep_lo, int ep_n, int *lids, float *lw, int *nloc, float *sh,
                                               int err_code)
{
    float *p = sh, *sel = sh + kTopkMax, *red = sh + 2 * kTopkMax, *s_sum = red + 32;
    const int e = static_cast<int>(threadIdx.x), lane = e & 31, warp = e >> 5;
    const int nw = static_cast<int>(blockDim.x) / 32;
    const float v = e < E ? __ldcg(logits + e) : -FLT_MAX;
    float m = v;
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < nw; ++w) m = fmaxf(m, red[w]);
    bool fin = isfinite(m);
    if (e < E) {
        fin = fin && isfinite(v);
        p[e] = expf(v - m);
    }
    const bool all_fin = __syncthreads_and(fin ? 1 : 0) != 0;
    if (!all_fin) {
        if (e == 0) atomicExch(err, err_code);
        return;
    }
    if (e == 0) {
        float s = 0.f;
        for (int j = 0; j < E; ++j) s += p[j];
        *s_sum = s;
    }
    __syncthreads();
    const float q = e < E ? p[e] / *s_sum : 0.f;
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
        *s_sum = ws;
    }
    __syncthreads();
    const float wk = *s_sum > 0.f ? sel[e < k ? e : 0] / *s_sum : sel[e < k ? e : 0];
    if (e < k) wts[e] = wk;
    if (ep_n > 0 && warp == 0) {
        // the local experts in rank order: a ballot over the k ranks (k <= 32 lanes of warp 0)
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

}  // namespace tb
