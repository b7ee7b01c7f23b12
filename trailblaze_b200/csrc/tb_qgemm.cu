// tb_qgemm.cu — batched-prefill quantized GEMM on the 5th-generation tensor
// cores (tcgen05, sm_100a).
//
//   C[t][n] = sum_k A[t][k] * dequant(W)[n][k]      t < T tokens, n < N, k < K
//
// W is GGUF Q4_K or Q6_K (rows = output features, exactly as the file stores
// them), A is bf16 [T][K], C is fp32 [T][N].  It is the batched form of the
// reference's prefill, which runs one matvec per token
// (layer4/tb_infer.c:1071-1074 feeding tb_gguf_tensor_matvec): row t of C is
// the matvec of W with token t's activations.
//
// One CTA owns 128 rows of W (the MMA's M) and all T tokens (the MMA's N, at
// most 256 per instruction; T = 512 takes two), accumulating in TMEM (T fp32
// columns).  Per stage of 64 K:
//   warp 0     one thread: the TMA load of A's [T][64] bf16 tile (128-byte
//              swizzle) and, once both tiles are in, four tcgen05.mma of K 16
//              (kind::f16, bf16 x bf16 -> f32), then tcgen05.commit to the
//              stage's "empty" barrier;
//   warps 1-8  dequantise W's [128][64] tile into bf16 in shared memory, in
//              the same 128-byte-swizzled K-major layout, with the arithmetic
//              of the bit-exact dequant (tb_dequant.cu deq1) before the bf16
//              rounding.
// After the last stage warps 1-4 read the accumulators back (tcgen05.ld, one
// TMEM lane quarter each) and store C.  With split K (few 128-row tiles) the
// CTAs of one tile add their partial sums into C (C is zeroed first).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdio>
#include <cstring>

#include "tb_common.cuh"
#include "tb_internal.h"

namespace tb {

static constexpr int kGM = 128;                    // W rows per CTA (MMA M)
static constexpr int kGK = 64;                     // K per stage (one 128-byte bf16 row)
static constexpr int kGThreads = 288;              // warp 0 + 8 dequant warps
static constexpr int kGDeqThreads = 256;
static constexpr uint32_t kGTileW = kGM * kGK * 2; // 16 KB of bf16 W per stage

struct QgArgs {
    const uint8_t *W;
    float *C;
    int *err;
    uint32_t N, K, T, ksplit, k_per_split, row_bytes, nst, tcols;
    uint32_t wait_limit;
};

// ---- tcgen05 / TMA primitives (PTX ISA 8.7, sm_100a) ----
__device__ __forceinline__ void tmem_alloc(uint32_t smem_slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_slot), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, one thread
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on bar once every tcgen05.mma issued so far by this thread has completed
__device__ __forceinline__ void umma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// 16 fp32 columns [col, col + 16) of the warp's TMEM lane quarter
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                   "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 2-D tiled TMA load (no multicast): box at (x = inner element, y = row)
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major bf16 tile with the 128-byte
// swizzle: rows of 128 bytes, 8-row atoms of 1 KB one after another (stride
// byte offset 1024), version 1 (sm_100), layout type 2 (128-byte swizzle).
// The tile starts on a 1 KB boundary; the start address may be advanced by 32
// bytes per K 16 inside the atom.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);          // start address
    d |= static_cast<uint64_t>(1u) << 16;                        // leading byte offset (unused, 16 B)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;                 // stride byte offset
    d |= static_cast<uint64_t>(1u) << 46;                         // version
    d |= static_cast<uint64_t>(2u) << 61;                         // 128-byte swizzle
    return d;
}

// Instruction descriptor, kind::f16: D f32, A and B bf16, both K-major,
// M = 128, N = n (a multiple of 16, at most 256).
__host__ __device__ constexpr uint32_t umma_idesc(uint32_t n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

// Byte offset of element (r, k) (k < 64) in a [rows][64] bf16 tile with the
// 128-byte swizzle: 16-byte chunk k / 8 of row r sits at chunk (k / 8) ^ (r % 8).
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t chunk)
{
    return r * 128u + ((chunk ^ (r & 7u)) << 4);
}

// ---- the 32 weights of group g (0..7) of one super-block, fp32, with the
// operations of tb_dequant.cu deq1 (so bit-identical before the bf16 rounding)
__device__ __forceinline__ uint32_t ld8(const uint8_t *p, int i) { return __ldg(p + i); }
__device__ __forceinline__ uint32_t ld16(const uint8_t *p, int i) { return ld8(p, i) | (ld8(p, i + 1) << 8); }

// Q4_K (tb_gguf_dequant.cu:98-116): w = d*s[g]*q - dmin*m[g]; byte 16 + 16 g + t
// holds weights 32 g + 2 t (low nibble) and 32 g + 2 t + 1 (high nibble).
__device__ __forceinline__ void group_q4k(const uint8_t *b, int g, float (&w)[32])
{
    const float d = h2f_ref(ld16(b, 0)), dmin = h2f_ref(ld16(b, 2));
    uint32_t s, m;
    if (g < 4) {
        s = ld8(b, 4 + g) & 63u;
        m = ld8(b, 8 + g) & 63u;
    } else {
        const int k = g - 4;
        s = (ld8(b, 4 + k) >> 6) | ((ld8(b, 12 + k) & 15u) << 2);
        m = (ld8(b, 8 + k) >> 6) | ((ld8(b, 12 + k) >> 4) << 2);
    }
    const float S = __fmul_rn(d, static_cast<float>(s));
    const float Mn = __fmul_rn(dmin, static_cast<float>(m));
    const uint4 q4 = __ldg(reinterpret_cast<const uint4 *>(b + 16 + 16 * g));   // 16-byte aligned
    const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
    for (int t = 0; t < 16; ++t) {
        const uint32_t byte = (qw[t >> 2] >> ((t & 3) * 8)) & 0xFFu;
        w[2 * t] = __fsub_rn(__fmul_rn(S, static_cast<float>(byte & 15u)), Mn);
        w[2 * t + 1] = __fsub_rn(__fmul_rn(S, static_cast<float>(byte >> 4)), Mn);
    }
}

// Q6_K (tb_gguf_dequant.cu:196-217): w = (d * sc[i/16]) * (q - 32), q = the
// nibble of ql[i/2] | 2 bits of qh[128 + i/4] << 4.  Blocks are 210 bytes, so
// only 2-byte alignment is assumed.
__device__ __forceinline__ void group_q6k(const uint8_t *b, int g, float (&w)[32])
{
    const float d = h2f_ref(ld16(b, 208));
    const float S0 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(ld8(b, 192 + 2 * g))));
    const float S1 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(ld8(b, 192 + 2 * g + 1))));
    uint32_t ql[4], qh[2];
#pragma unroll
    for (int j = 0; j < 4; ++j) ql[j] = ld16(b, 16 * g + 4 * j) | (ld16(b, 16 * g + 4 * j + 2) << 16);
#pragma unroll
    for (int j = 0; j < 2; ++j) qh[j] = ld16(b, 128 + 8 * g + 4 * j) | (ld16(b, 128 + 8 * g + 4 * j + 2) << 16);
#pragma unroll
    for (int e = 0; e < 32; ++e) {
        const uint32_t lo = (ql[e >> 3] >> (((e >> 1) & 3) * 8 + (e & 1) * 4)) & 15u;
        const uint32_t hi = (qh[e >> 4] >> (((e >> 2) & 3) * 8 + (e & 3) * 2)) & 3u;
        w[e] = __fmul_rn(e < 16 ? S0 : S1, static_cast<float>(static_cast<int>(lo | (hi << 4)) - 32));
    }
}

// Shared memory: [nst][W tile 16 KB | A tile T*128 B] (1 KB aligned), then the
// barriers fullA[nst], fullW[nst], empty[nst], done, and the TMEM base slot.
__host__ __device__ inline size_t qg_stage_bytes(uint32_t T)
{
    return static_cast<size_t>(kGTileW) + static_cast<size_t>(T) * 128u;
}
__host__ __device__ inline size_t qg_smem_bytes(uint32_t T, uint32_t nst)
{
    return 1024 + static_cast<size_t>(nst) * qg_stage_bytes(T) + 8 * (3 * nst + 1) + 16;
}

template <int QT>
__global__ void __launch_bounds__(kGThreads, 1) k_qgemm(const __grid_constant__ CUtensorMap amap, const QgArgs a)
{
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t nst = a.nst, T = a.T;
    const size_t sb = qg_stage_bytes(T);
    uint64_t *fullA = reinterpret_cast<uint64_t *>(sm + nst * sb);
    uint64_t *fullW = fullA + nst;
    uint64_t *empty = fullW + nst;
    uint64_t *done = empty + nst;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(done + 1);
    __shared__ int s_fail;

    const uint32_t n0 = blockIdx.x * kGM;                      // first W row
    const uint32_t split = blockIdx.y;
    const uint32_t k_lo = split * a.k_per_split;
    const uint32_t nk = a.k_per_split / kGK;                   // stages of this CTA
    constexpr Geom geo = geom_of(QT);

    if (tid == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
            mbar_init(smem_u32(fullA + s), 1);
            mbar_init(smem_u32(fullW + s), kGDeqThreads / 32);
            mbar_init(smem_u32(empty + s), 1);
        }
        mbar_init(smem_u32(done), 1);
        fence_mbar_init();
        s_fail = 0;
    }
    if (warp == 0) {   // TMEM: one fp32 column per token
        tmem_alloc(smem_u32(tslot), a.tcols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- A loads and the MMAs, one thread ----
            const uint32_t nA = T > 256 ? 256 : T;              // tokens per MMA (and per TMA box)
            const uint32_t idesc = umma_idesc(nA);
            uint32_t issued = 0, mma_done = 0;
            auto load_a = [&](uint32_t it) {
                const uint32_t s = it % nst;
                uint8_t *st = sm + s * sb;
                mbar_expect_tx(smem_u32(fullA + s), T * 128u);
                for (uint32_t t0 = 0; t0 < T; t0 += nA)
                    tma_load_2d(smem_u32(st + kGTileW + t0 * 128u), &amap, static_cast<int>(k_lo + it * kGK),
                                static_cast<int>(t0), smem_u32(fullA + s));
            };
            for (; issued < nst && issued < nk; ++issued) load_a(issued);
            bool fail = false;
            for (uint32_t it = 0; it < nk; ++it) {
                const uint32_t s = it % nst, par = (it / nst) & 1u;
                if (!mbar_wait_bounded(smem_u32(fullA + s), par, a.err, a.wait_limit) ||
                    !mbar_wait_bounded(smem_u32(fullW + s), par, a.err, a.wait_limit)) {
                    fail = true;
                    break;
                }
                tc_fence_after();
                const uint32_t wbase = smem_u32(sm + s * sb), abase = wbase + kGTileW;
#pragma unroll
                for (uint32_t j = 0; j < kGK / 16; ++j)
                    for (uint32_t t0 = 0; t0 < T; t0 += nA)
                        umma_f16(tbase + t0, sw128_desc(wbase + 32u * j), sw128_desc(abase + t0 * 128u + 32u * j),
                                 idesc, (it | j) != 0 ? 1u : 0u);
                umma_commit(smem_u32(empty + s));   // the stage is free once these MMAs are done
                mma_done = it + 1;
                // refill the previous iteration's stage (its MMAs were committed one
                // iteration ago; this iteration's are queued behind them meanwhile)
                if (it >= 1 && issued < nk) {
                    const uint32_t sp = (it - 1) % nst, pp = ((it - 1) / nst) & 1u;
                    if (!mbar_wait_bounded(smem_u32(empty + sp), pp, a.err, a.wait_limit)) {
                        fail = true;
                        break;
                    }
                    load_a(issued);   // issued == it - 1 + nst, stage sp
                    ++issued;
                }
            }
            if (fail) atomicExch(&s_fail, 1);
            // every MMA issued so far (possibly none) completes before the epilogue reads TMEM
            umma_commit(smem_u32(done));
            (void)mma_done;
        }
        __syncwarp();
    } else {
        // ---- W dequant, 256 threads: thread = (row r, half h): 32 weights ----
        const uint32_t dt = tid - 32, r = dt >> 1, h = dt & 1;
        const uint8_t *wrow = a.W + static_cast<size_t>(n0 + r) * a.row_bytes;
        for (uint32_t it = 0; it < nk; ++it) {
            const uint32_t s = it % nst, par = (it / nst) & 1u;
            if (it >= nst) {   // the MMAs that read this stage's previous tile are done
                if (!mbar_wait_bounded(smem_u32(empty + s), par ^ 1u, a.err, a.wait_limit)) {
                    atomicExch(&s_fail, 1);
                    break;
                }
            }
            if (*reinterpret_cast<volatile int *>(&s_fail)) break;
            const uint32_t k = k_lo + it * kGK + h * 32;       // first weight of the group
            const uint8_t *blk = wrow + static_cast<size_t>(k / geo.block_weights) * geo.block_bytes;
            const int g = static_cast<int>((k % geo.block_weights) >> 5);
            float w[32];
            if constexpr (QT == QT_Q4_K) group_q4k(blk, g, w);
            else group_q6k(blk, g, w);
            uint8_t *wt = sm + s * sb;
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) {   // 16-byte chunks h*4 + c of row r
                __nv_bfloat162 p[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) p[e] = __floats2bfloat162_rn(w[8 * c + 2 * e], w[8 * c + 2 * e + 1]);
                *reinterpret_cast<uint4 *>(wt + sw128_off(r, h * 4 + c)) = *reinterpret_cast<uint4 *>(p);
            }
            fence_proxy_async_smem();   // generic stores -> visible to the tensor core's async proxy
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(fullW + s));
        }
    }

    // ---- epilogue: warps 1-4 read their TMEM lane quarter, C[t][n0 + lane row] ----
    if (warp >= 1 && warp <= 4) {
        const bool ok = mbar_wait_bounded(smem_u32(done), 0, a.err, a.wait_limit);
        tc_fence_after();
        const uint32_t q = warp & 3u;                 // TMEM lanes 32q .. 32q + 31 (warp id mod 4)
        const uint32_t n = n0 + 32 * q + lane;
        if (ok && !*reinterpret_cast<volatile int *>(&s_fail)) {
            for (uint32_t c0 = 0; c0 < T; c0 += 16) {
                float v[16];
                tmem_ld16(tbase + ((32u * q) << 16) + c0, v);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float *dst = a.C + static_cast<size_t>(c0 + i) * a.N + n;
                    if (a.ksplit > 1) atomicAdd(dst, v[i]);
                    else *dst = v[i];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, a.tcols);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_tiled()
{
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

static constexpr size_t kGSmemCap = 232448;   // 227 KB opt-in per CTA

int qg_launch(const void *W, int qtype, int N, int K, const void *A, int T, float *C, cudaStream_t st, int *d_err,
              int num_sms, uint32_t wait_limit)
{
    if (qtype != QT_Q4_K && qtype != QT_Q6_K) return 0;
    if (!W || !A || !C || N <= 0 || K <= 0 || N % kGM || K % 256 || T < 16 || T > 512 || T % 16) return 0;
    const uintptr_t wa = reinterpret_cast<uintptr_t>(W), aa = reinterpret_cast<uintptr_t>(A);
    if ((aa & 15u) || (qtype == QT_Q4_K && (wa & 15u)) || (wa & 1u)) return 0;
    const Geom g = geom_of(qtype);
    EncodeTiled enc = encode_tiled();
    if (!enc) {
        fprintf(stderr, "[tb_cuda] qgemm: cuTensorMapEncodeTiled not available\n");
        return 0;
    }
    const uint32_t nA = T > 256 ? 256u : static_cast<uint32_t>(T);
    CUtensorMap map;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(T)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2u};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kGK), nA};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(A), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        fprintf(stderr, "[tb_cuda] qgemm: tensor map encode failed\n");
        return 0;
    }
    QgArgs a{};
    a.W = static_cast<const uint8_t *>(W);
    a.C = C;
    a.err = d_err;
    a.N = static_cast<uint32_t>(N);
    a.K = static_cast<uint32_t>(K);
    a.T = static_cast<uint32_t>(T);
    a.row_bytes = static_cast<uint32_t>((K / g.block_weights) * g.block_bytes);
    a.wait_limit = wait_limit;
    // split K until the grid is about one wave (each part a multiple of 256)
    const uint32_t tiles = static_cast<uint32_t>(N / kGM);
    uint32_t ks = 1;
    while (tiles * ks * 2 <= static_cast<uint32_t>(num_sms) && (K / (ks * 2)) % 256 == 0 && K / (ks * 2) >= 512)
        ks *= 2;
    a.ksplit = ks;
    a.k_per_split = static_cast<uint32_t>(K) / ks;
    uint32_t tc = 32;
    while (tc < a.T) tc <<= 1;
    a.tcols = tc;
    uint32_t nst = 8;
    while (nst > 2 && qg_smem_bytes(a.T, nst) > kGSmemCap) --nst;
    if (qg_smem_bytes(a.T, nst) > kGSmemCap) return 0;
    a.nst = nst;
    const size_t smem = qg_smem_bytes(a.T, nst);
    void (*kern)(const CUtensorMap, const QgArgs) = qtype == QT_Q4_K ? k_qgemm<QT_Q4_K> : k_qgemm<QT_Q6_K>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (ks > 1 && cudaMemsetAsync(C, 0, sizeof(float) * static_cast<size_t>(T) * N, st) != cudaSuccess) return 0;
    kern<<<dim3(tiles, ks), kGThreads, smem, st>>>(map, a);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

}  // namespace tb
