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
// columns per accumulator; MMAs into one accumulator wait for each other, so
// for T <= 256 consecutive K-16 steps rotate over 2 or 4 accumulators that the
// epilogue adds in a fixed order).  Per stage of 64 K:
//   warp 9     one thread: the TMA load of A's [T][64] bf16 tile (128-byte
//              swizzle), nst stages ahead;
//   warps 1-8  dequantise W's [128][64] tile into bf16 in shared memory, in
//              the same 128-byte-swizzled K-major layout, with the arithmetic
//              of the bit-exact dequant (tb_dequant.cu deq1) before the bf16
//              rounding; the raw blocks arrive by bulk copies a few
//              super-blocks ahead;
//   warp 0     one thread: once both tiles are in, four tcgen05.mma of K 16
//              (kind::f16, bf16 x bf16 -> f32), then tcgen05.commit to the
//              stage's "empty" barrier.  It never waits for an MMA to finish.
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
static constexpr int kGThreads = 352;              // warp 0 (MMA), 8 dequant warps, warp 9 (A), warp 10 (W)
static constexpr int kGDeqThreads = 256;
static constexpr uint32_t kGTileW = kGM * kGK * 2; // 16 KB of bf16 W per stage

struct QgArgs {
    const uint8_t *W;
    float *C;
    int *err;
    uint32_t N, K, T, ksplit, row_bytes, nst, nraw, tcols, bw;
    uint32_t nacc;   // independent accumulators (consecutive K-16 steps rotate over them)
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

// One lane of a converged warp (elect.sync): the tensor-core and TMA issue
// below runs with the whole warp in step and one lane elected per instruction.
__device__ __forceinline__ bool elect_one()
{
    uint32_t p = 0;
    asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.u32 %0, 1, 0, P;\n\t}" : "=r"(p));
    return p != 0;
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
// (the block bytes sit in shared memory, staged by bulk copies)
__device__ __forceinline__ uint32_t ld8(const uint8_t *p, int i) { return p[i]; }
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
    const uint4 q4 = *reinterpret_cast<const uint4 *>(b + 16 + 16 * g);   // 16-byte aligned
    const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
    // S * q - Mn per weight, two weights per paired op; q as an exact float by
    // the 2^23 + q bit pattern minus 2^23 (no integer conversion); a - b is
    // a + (-b) with the same rounding
    const float2 S2 = make_float2(S, S), M2 = make_float2(-Mn, -Mn), B2 = make_float2(-8388608.f, -8388608.f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t lo = qw[c] & 0x0F0F0F0Fu, hi = (qw[c] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 q = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650u | k)),
                                                    __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650u | k))),
                                        B2);
            const float2 v = __fadd2_rn(__fmul2_rn(S2, q), M2);
            w[8 * c + 2 * k] = v.x;
            w[8 * c + 2 * k + 1] = v.y;
        }
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
    // (q - 32) as an exact float: the 2^23 + q bit pattern minus 2^23 + 32; two
    // weights per paired multiply
    const float2 B2 = make_float2(-8388640.f, -8388640.f);
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        const uint32_t lo0 = (ql[e >> 3] >> (((e >> 1) & 3) * 8)) & 15u;
        const uint32_t lo1 = (ql[e >> 3] >> (((e >> 1) & 3) * 8 + 4)) & 15u;
        const uint32_t hi0 = (qh[e >> 4] >> (((e >> 2) & 3) * 8 + (e & 3) * 2)) & 3u;
        const uint32_t hi1 = (qh[e >> 4] >> (((e >> 2) & 3) * 8 + ((e + 1) & 3) * 2)) & 3u;
        const float2 q = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | lo0 | (hi0 << 4)),
                                                __uint_as_float(0x4B000000u | lo1 | (hi1 << 4))),
                                    B2);
        const float S = e < 16 ? S0 : S1;
        const float2 v = __fmul2_rn(make_float2(S, S), q);
        w[e] = v.x;
        w[e + 1] = v.y;
    }
}

// Raw weight bytes are staged one super-block (256 K) of the CTA's 128 rows at
// a time, by one 2-D TMA load of W viewed as [N rows][row_bytes / 2] uint16: a
// box of 128 rows x kGEnv / 2 elements starting at the block rounded down to 16
// bytes (a Q6_K block of 210 bytes then sits 0-14 bytes into its 224-byte box
// row; past the row's end TMA fills zeros).
static constexpr uint32_t kGEnv = 224;
static constexpr uint32_t kGRawStage = kGM * kGEnv;

// Shared memory: [nst][W tile 16 KB | A tile T*128 B] (1 KB aligned), the raw
// ring [nraw][128][kGEnv], then the barriers fullA[nst], fullW[nst],
// empty[nst], rawfull[nraw], rawempty[nraw], done, and the TMEM base slot.
__host__ __device__ inline size_t qg_stage_bytes(uint32_t T)
{
    return static_cast<size_t>(kGTileW) + static_cast<size_t>(T) * 128u;
}
__host__ __device__ inline size_t qg_smem_bytes(uint32_t T, uint32_t nst, uint32_t nraw)
{
    return 1024 + static_cast<size_t>(nst) * qg_stage_bytes(T) + static_cast<size_t>(nraw) * kGRawStage +
           8 * (3 * nst + 2 * nraw + 1) + 16;
}

template <int QT>
__global__ void __launch_bounds__(kGThreads, 2) k_qgemm(const __grid_constant__ CUtensorMap amap,
                                                        const __grid_constant__ CUtensorMap wmap, const QgArgs a)
{
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t nst = a.nst, T = a.T;
    const size_t sb = qg_stage_bytes(T);
    uint8_t *raw = sm + nst * sb;
    const uint32_t nraw = a.nraw;
    uint64_t *fullA = reinterpret_cast<uint64_t *>(raw + nraw * kGRawStage);
    uint64_t *fullW = fullA + nst;
    uint64_t *empty = fullW + nst;
    uint64_t *rawfull = empty + nst;
    uint64_t *rawempty = rawfull + nraw;
    uint64_t *done = rawempty + nraw;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(done + 1);
    __shared__ int s_fail;

    const uint32_t n0 = blockIdx.x * kGM;                      // first W row
    const uint32_t split = blockIdx.y;
    // this CTA's super-blocks: an even share of the K / 256, the ksplit parts
    // differing by at most one super-block
    const uint32_t nsb_all = a.K / 256;
    const uint32_t kb0 = (split * nsb_all) / a.ksplit, kb1 = ((split + 1) * nsb_all) / a.ksplit;
    const uint32_t k_lo = kb0 * 256;
    const uint32_t nk = (kb1 - kb0) * (256 / kGK);               // stages of this CTA
    constexpr Geom geo = geom_of(QT);

    if (tid == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
            mbar_init(smem_u32(fullA + s), 1);
            mbar_init(smem_u32(fullW + s), kGDeqThreads / 32);
            mbar_init(smem_u32(empty + s), 1);
        }
        for (uint32_t s = 0; s < nraw; ++s) {
            mbar_init(smem_u32(rawfull + s), 1);
            mbar_init(smem_u32(rawempty + s), kGDeqThreads / 32);
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

    const uint32_t nsb = kb1 - kb0;                             // super-blocks of this CTA
    if (warp == 10) {
        // ---- W's raw super-blocks by TMA, nraw ahead; a slot is refilled once
        // the dequant warps are done with it (whole warp, one lane issues) ----
        for (uint32_t j = 0; j < nsb; ++j) {
            const uint32_t slot = j % nraw;
            bool ok = j < nraw ||
                      mbar_wait_bounded(smem_u32(rawempty + slot), ((j / nraw) - 1u) & 1u, a.err, a.wait_limit);
            ok = __all_sync(0xFFFFFFFFu, ok) && !*reinterpret_cast<volatile int *>(&s_fail);
            if (!ok) {
                if (lane == 0) atomicExch(&s_fail, 1);
                break;
            }
            if (elect_one()) {
                const uint32_t x = ((kb0 + j) * geo.block_bytes / 2u) & ~7u;   // 16-byte aligned start
                mbar_expect_tx(smem_u32(rawfull + slot), kGM * a.bw * 2u);
                tma_load_2d(smem_u32(raw + slot * kGRawStage), &wmap, static_cast<int>(x), static_cast<int>(n0),
                            smem_u32(rawfull + slot));
            }
            __syncwarp();
        }
    } else if (warp == 9) {
        // ---- A tiles by TMA, nst ahead; a stage is refilled once its MMAs are done ----
        const uint32_t nA = T > 256 ? 256 : T;
        for (uint32_t it = 0; it < nk; ++it) {
            const uint32_t s = it % nst;
            bool ok = it < nst ||
                      mbar_wait_bounded(smem_u32(empty + s), ((it / nst) - 1u) & 1u, a.err, a.wait_limit);
            ok = __all_sync(0xFFFFFFFFu, ok) && !*reinterpret_cast<volatile int *>(&s_fail);
            if (!ok) {
                if (lane == 0) atomicExch(&s_fail, 1);
                break;
            }
            if (elect_one()) {
                uint8_t *st = sm + s * sb;
                mbar_expect_tx(smem_u32(fullA + s), T * 128u);
                for (uint32_t t0 = 0; t0 < T; t0 += nA)
                    tma_load_2d(smem_u32(st + kGTileW + t0 * 128u), &amap, static_cast<int>(k_lo + it * kGK),
                                static_cast<int>(t0), smem_u32(fullA + s));
            }
            __syncwarp();
        }
    } else if (warp == 0) {
        // ---- the MMAs: the whole warp waits, one elected lane issues four K-16
        // steps per stage and the commit ----
        const uint32_t nA = T > 256 ? 256 : T;              // tokens per MMA
        const uint32_t idesc = umma_idesc(nA);
        bool fail = false;
        for (uint32_t it = 0; it < nk; ++it) {
            const uint32_t s = it % nst, par = (it / nst) & 1u;
            bool ok = mbar_wait_bounded(smem_u32(fullA + s), par, a.err, a.wait_limit) &&
                      mbar_wait_bounded(smem_u32(fullW + s), par, a.err, a.wait_limit);
            if (!__all_sync(0xFFFFFFFFu, ok)) {
                fail = true;
                break;
            }
            tc_fence_after();
            const uint32_t wbase = smem_u32(sm + s * sb), abase = wbase + kGTileW;
            if (elect_one()) {
                // MMAs into one accumulator wait for each other; consecutive K-16
                // steps therefore rotate over nacc accumulators (columns acc * T)
#pragma unroll
                for (uint32_t j = 0; j < kGK / 16; ++j) {
                    const uint32_t step = it * (kGK / 16) + j;
                    const uint32_t acc = step % a.nacc;
                    for (uint32_t t0 = 0; t0 < T; t0 += nA)
                        umma_f16(tbase + acc * T + t0, sw128_desc(wbase + 32u * j),
                                 sw128_desc(abase + t0 * 128u + 32u * j), idesc, step >= a.nacc ? 1u : 0u);
                }
                umma_commit(smem_u32(empty + s));   // the stage is free once these MMAs are done
            }
            __syncwarp();
        }
        if (fail && lane == 0) atomicExch(&s_fail, 1);
        // every MMA issued so far (possibly none) completes before the epilogue reads TMEM
        if (elect_one()) umma_commit(smem_u32(done));
        __syncwarp();
    } else {
        // ---- W dequant, 256 threads: thread = (row r, half h): 32 weights ----
        // Row r's super-block j sits in raw slot j % nraw; each 64-K stage
        // decodes its groups 2 sub + h.
        const uint32_t dt = tid - 32, r = dt >> 1, h = dt & 1;
        bool failed = false;
        for (uint32_t it = 0; it < nk; ++it) {
            const uint32_t s = it % nst, par = (it / nst) & 1u;
            const uint32_t j = it >> 2, sub = it & 3u;          // super-block, 64-K part of it
            failed = failed || *reinterpret_cast<volatile int *>(&s_fail) != 0;
            if (!failed && it >= nst)   // the MMAs that read this stage's previous tile are done
                failed = !mbar_wait_bounded(smem_u32(empty + s), par ^ 1u, a.err, a.wait_limit);
            if (!failed)
                failed = !mbar_wait_bounded(smem_u32(rawfull + j % nraw), (j / nraw) & 1u, a.err, a.wait_limit);
            if (failed) {
                atomicExch(&s_fail, 1);
                break;
            }
            const uint32_t boff = (kb0 + j) * geo.block_bytes;
            const uint8_t *blk = raw + (j % nraw) * kGRawStage + r * (a.bw * 2u) + (boff & 15u);
            float w[32];
            if constexpr (QT == QT_Q4_K) group_q4k(blk, static_cast<int>(2 * sub + h), w);
            else group_q6k(blk, static_cast<int>(2 * sub + h), w);
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
            if (lane == 0) {
                mbar_arrive(smem_u32(fullW + s));
                if (sub == 3) mbar_arrive(smem_u32(rawempty + j % nraw));   // done with super-block j
            }
        }
    }

    // ---- epilogue: warps 1-4 read their TMEM lane quarter, C[t][n0 + lane row] ----
    if (warp >= 1 && warp <= 4) {
        const bool ok = mbar_wait_bounded(smem_u32(done), 0, a.err, a.wait_limit);
        tc_fence_after();
        const uint32_t q = warp & 3u;                 // TMEM lanes 32q .. 32q + 31 (warp id mod 4)
        const uint32_t n = n0 + 32 * q + lane;
        if (ok && !*reinterpret_cast<volatile int *>(&s_fail)) {
            const uint32_t used = nk * (kGK / 16) < a.nacc ? nk * (kGK / 16) : a.nacc;   // accumulators written
            for (uint32_t c0 = 0; c0 < T; c0 += 16) {
                float v[16];
                tmem_ld16(tbase + ((32u * q) << 16) + c0, v);
                for (uint32_t u = 1; u < used; ++u) {   // fixed order: accumulator 0 + 1 + ...
                    float t[16];
                    tmem_ld16(tbase + ((32u * q) << 16) + u * T + c0, t);
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] += t[i];
                }
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
    const NvtxRange nvtx("tb.qgemm");
    if (qtype != QT_Q4_K && qtype != QT_Q6_K) return 0;
    if (!W || !A || !C || N <= 0 || K <= 0 || N % kGM || K % 256 || T < 16 || T > 512 || T % 16) return 0;
    const uintptr_t wa = reinterpret_cast<uintptr_t>(W), aa = reinterpret_cast<uintptr_t>(A);
    const Geom g = geom_of(qtype);
    const unsigned long long rb = static_cast<unsigned long long>(K / g.block_weights) * g.block_bytes;
    if ((aa & 15u) || (wa & 15u) || (rb & 15u)) return 0;   // TMA: 16-byte base and row stride
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
    // W as [N rows][row_bytes / 2] uint16, boxes of 128 rows x one block rounded out to 16 bytes
    const uint32_t bw = qtype == QT_Q4_K ? 72u : 112u;
    CUtensorMap wmap;
    const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(rb / 2), static_cast<cuuint64_t>(N)};
    const cuuint64_t wstrides[1] = {static_cast<cuuint64_t>(rb)};
    const cuuint32_t wbox[2] = {bw, static_cast<cuuint32_t>(kGM)};
    if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(W), wdims, wstrides, wbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        fprintf(stderr, "[tb_cuda] qgemm: weight tensor map encode failed\n");
        return 0;
    }
    QgArgs a{};
    a.bw = bw;
    a.W = static_cast<const uint8_t *>(W);
    a.C = C;
    a.err = d_err;
    a.N = static_cast<uint32_t>(N);
    a.K = static_cast<uint32_t>(K);
    a.T = static_cast<uint32_t>(T);
    a.row_bytes = static_cast<uint32_t>(rb);
    a.wait_limit = wait_limit;
    // Two CTAs per SM when their shared memory fits (two MMA issuers per SM),
    // else one; split K until the grid is about one wave (each part a multiple
    // of 256); a raw ring of 2-3 super-blocks, then as many MMA stages as fit.
    uint32_t per_sm = 2, nraw = 2, nst = 8;
    size_t cap = (kGSmemCap - 2048) / 2;
    while (nst > 3 && qg_smem_bytes(a.T, nst, nraw) > cap) --nst;
    if (qg_smem_bytes(a.T, nst, nraw) > cap) {
        per_sm = 1;
        cap = kGSmemCap;
        nraw = 3;
        nst = 8;
        while (nst > 2 && qg_smem_bytes(a.T, nst, nraw) > cap) --nst;
        if (qg_smem_bytes(a.T, nst, nraw) > cap) nraw = 2;
        if (qg_smem_bytes(a.T, nst, nraw) > cap) return 0;
    }
    const uint32_t tiles = static_cast<uint32_t>(N / kGM);
    // K parts per row tile.  Few tokens (T <= 32, a weight stream): as many
    // parts as keep the grid within one wave of CTA slots, each at least two
    // super-blocks (parts may differ by one super-block).  More tokens: the
    // partial sums' atomic adds grow with T, so parts only double while the
    // grid stays within one wave (measured: the finer split was no faster at
    // T = 128 and 12288 x 4096 T = 16 went from 55.5 to 43.6 us).
    const uint32_t slots = static_cast<uint32_t>(num_sms) * per_sm;
    const uint32_t nsb_all = static_cast<uint32_t>(K) / 256;
    uint32_t ks = 1;
    if (a.T <= 32) {
        ks = slots / tiles;
        if (ks > nsb_all / 2) ks = nsb_all / 2;
        if (ks < 1) ks = 1;
    } else {
        while (tiles * ks * 2 <= slots && (K / (ks * 2)) % 256 == 0 && K / (ks * 2) >= 512) ks *= 2;
    }
    a.ksplit = ks;
    a.nst = nst;
    a.nraw = nraw;
    // accumulators: nacc * T TMEM columns, at most 512 per SM (256 per CTA when two share it)
    const uint32_t tmem_cap = per_sm == 2 ? 256u : 512u;
    a.nacc = 4;
    while (a.nacc > 1 && a.nacc * a.T > tmem_cap) a.nacc >>= 1;
    uint32_t tc = 32;
    while (tc < a.T * a.nacc) tc <<= 1;
    a.tcols = tc;
    const size_t smem = qg_smem_bytes(a.T, nst, nraw);
    void (*kern)(const CUtensorMap, const CUtensorMap, const QgArgs) =
        qtype == QT_Q4_K ? k_qgemm<QT_Q4_K> : k_qgemm<QT_Q6_K>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (ks > 1 && cudaMemsetAsync(C, 0, sizeof(float) * static_cast<size_t>(T) * N, st) != cudaSuccess) return 0;
    kern<<<dim3(tiles, ks), kGThreads, smem, st>>>(map, wmap, a);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

}  // namespace tb
