// tb_common.cuh — shared definitions for the sm_100a GGUF dequant/matvec library.
//
// Block geometry follows the reference (layer4/tb_gguf_dequant.cu:37-47,
// layer4/tb_gguf.c:380-393).  A "unit" is the piece of a row that one lane of
// the matvec kernel decodes: one 256-weight super-block for the K-quants, eight
// 32-weight blocks for Q4_0/Q8_0, and 64 elements for F32/F16/BF16 (so a stage
// of 32 units stays a few KB for every type).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tb {

enum QType : int {
    QT_F32 = 0, QT_F16 = 1, QT_Q4_0 = 2, QT_Q8_0 = 8, QT_Q2_K = 10, QT_Q3_K = 11,
    QT_Q4_K = 12, QT_Q5_K = 13, QT_Q6_K = 14, QT_Q8_K = 15, QT_IQ3_S = 21, QT_BF16 = 30
};

enum DevErr : int { ERR_NONE = 0, ERR_WAIT_TIMEOUT = 1, ERR_RUNTIME = 2 };

struct Geom {
    int block_weights;   // weights per block
    int block_bytes;     // bytes per block
    int unit_blocks;     // blocks per matvec unit (256 weights; 64 for F32/F16/BF16)
};

__host__ __device__ constexpr Geom geom_of(int qt)
{
    return qt == QT_F32   ? Geom{1, 4, 64}
         : qt == QT_F16   ? Geom{1, 2, 64}
         : qt == QT_BF16  ? Geom{1, 2, 64}
         : qt == QT_Q4_0  ? Geom{32, 18, 8}
         : qt == QT_Q8_0  ? Geom{32, 34, 8}
         : qt == QT_Q2_K  ? Geom{256, 84, 1}
         : qt == QT_Q3_K  ? Geom{256, 110, 1}
         : qt == QT_IQ3_S ? Geom{256, 110, 1}
         : qt == QT_Q4_K  ? Geom{256, 144, 1}
         : qt == QT_Q5_K  ? Geom{256, 176, 1}
         : qt == QT_Q6_K  ? Geom{256, 210, 1}
         : qt == QT_Q8_K  ? Geom{256, 292, 1}
                          : Geom{0, 0, 0};
}

// ── reference fp16 / bf16 converters ─────────────────────────────────────────
// tb_gguf_dequant.cu:54-63: exponent 0 maps to sign | mantissa<<13 (a float
// denormal), exponent 31 to inf/nan, otherwise the exponent is rebased by 112.
// Written branch-free: the 15 magnitude bits shifted into place, plus a rebias
// that depends only on the exponent class.
__device__ __forceinline__ float h2f_ref(uint32_t h)
{
    uint32_t mag = (h & 0x7FFFu) << 13;
    uint32_t e = h & 0x7C00u;
    uint32_t bias = (e == 0x7C00u) ? (224u << 23) : (e == 0u ? 0u : (112u << 23));
    return __uint_as_float(((h & 0x8000u) << 16) | (mag + bias));
}

__device__ __forceinline__ float bf2f(uint32_t b) { return __uint_as_float(b << 16); }

// The two fp16 halves of w through the same reference converter, for the matvec
// path: the hardware conversion, then the exponent-0 rule (m*2^-136 where IEEE
// gives m*2^-24, i.e. a factor 2^-112, exact as an fp32 subnormal).  Finite
// values and infinities are bit-identical to h2f_ref; a NaN stays a NaN (its
// payload can differ, which no product with it can show).
__device__ __forceinline__ float2 h2f2_ref(uint32_t w)
{
    float2 f = __half22float2(__halves2half2(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)),
                                             __ushort_as_half(static_cast<unsigned short>(w >> 16))));
    f.x *= (w & 0x00007C00u) ? 1.0f : 0x1p-112f;
    f.y *= (w & 0x7C000000u) ? 1.0f : 0x1p-112f;
    return f;
}

// ── 32-bit fast division by a runtime-constant divisor (Granlund–Montgomery,
//    "round-up" form).  Exact for every 32-bit numerator.                   ──
struct FastDiv {
    uint32_t d, m, s;
};

inline FastDiv make_fastdiv(uint32_t d)
{
    FastDiv f{d, 0, 0};
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    // m = floor(2^32 * (2^l - d) / d) + 1
    f.m = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    f.s = l;
    return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f)
{
    if (f.d == 1) return n;
    uint32_t t = __umulhi(n, f.m);
    return (t + ((n - t) >> 1)) >> (f.s - 1);
}

// ── shared-memory byte-stream reader ─────────────────────────────────────────
// The matvec decoders read staged weight rows by 32-bit shared-window address
// (ld.shared, 32-bit address arithmetic).  These loads are plain (not volatile)
// asm so the compiler may merge the repeated word loads of neighbouring
// unaligned reads; they cannot run ahead of the mbarrier wait that publishes a
// stage because every address derives from shared_after(), a volatile move
// issued after that wait.
__device__ __forceinline__ uint32_t lds_u32(uint32_t a)
{
    uint32_t v;
    asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds_u128(uint32_t a)
{
    uint4 v;
    asm("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// An opaque copy of a shared address, ordered after the preceding volatile asm
// (the mbarrier wait): loads whose address derives from it stay after the wait.
__device__ __forceinline__ uint32_t shared_after(uint32_t a)
{
    uint32_t v;
    asm volatile("mov.b32 %0, %1;" : "=r"(v) : "r"(a));
    return v;
}

// Units of 210-, 110-, 84-, 34- or 18-byte blocks start at arbitrary byte
// offsets in the staged copy, so their 32-bit words are read as a funnel shift
// of two aligned words.  `sh` is 8*(offset & 3); a shift of 0 returns `lo`.
struct UnitBytes {
    uint32_t base;   // 4-byte aligned shared address at or below the unit start
    uint32_t sh;     // funnel shift in bits (0, 8, 16, 24)

    __device__ __forceinline__ UnitBytes(uint32_t unit) : base(unit & ~3u), sh((unit & 3u) * 8u) {}
    // 32-bit little-endian word at byte offset 4*i + 0 of the unit
    __device__ __forceinline__ uint32_t w(int i) const
    {
        return __funnelshift_r(lds_u32(base + 4 * i), lds_u32(base + 4 * i + 4), sh);
    }
    // 32-bit word at an arbitrary byte offset `off` of the unit
    __device__ __forceinline__ uint32_t at(int off) const
    {
        const uint32_t p = base + (off & ~3);
        uint32_t s = sh + 8u * (off & 3);
        uint32_t lo = lds_u32(p), hi = lds_u32(p + 4), hi2 = lds_u32(p + 8);
        return s >= 32 ? __funnelshift_r(hi, hi2, s - 32) : __funnelshift_r(lo, hi, s);
    }
};

// ── mbarrier / bulk-copy (TMA) primitives, inline PTX for sm_100a ─────────────
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> shared, completion signalled on `bar` (complete_tx).
// Both addresses 16-byte aligned, size a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Plain arrival (release semantics at CTA scope) on a pipeline barrier.
__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// ── 4-way byte dot products (dp4a), one form per operand signedness ──────────
// a holds the weight fields, b the activation digits; c + sum_k a_k * b_k.
__device__ __forceinline__ int dp_us(uint32_t a, uint32_t b, int c)   // a unsigned, b signed
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp_uu(uint32_t a, uint32_t b, int c)   // both unsigned
{
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp_ss(uint32_t a, uint32_t b, int c)   // both signed
{
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp_su(uint32_t a, uint32_t b, int c)   // a signed, b unsigned
{
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Byte k of w, zero- or sign-extended to 32 bits (one byte permute each).
__device__ __forceinline__ int ubyte(uint32_t w, int k)
{
    return static_cast<int>(__byte_perm(w, 0u, 0x4440u | static_cast<uint32_t>(k)));
}
__device__ __forceinline__ int sbyte(uint32_t w, int k)
{
    // prmt selector nibble 8|k replicates the sign bit of byte k
    const uint32_t s = 0x8u | static_cast<uint32_t>(k);
    const uint32_t sel = (s << 12) | (s << 8) | (s << 4) | static_cast<uint32_t>(k);
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0u), "r"(sel));
    return static_cast<int>(r);
}

// Bounded wait: gives up after `limit` polls, records ERR_WAIT_TIMEOUT and
// returns false.  Every wait in this library goes through here.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int *err,
                                                  uint32_t limit)
{
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
    return false;
}

// Bounded wait until *ctr >= target (system-scope acquire load); the counter
// is raised by peers over NVLink.  False when the limit runs out.
__device__ __forceinline__ bool wait_counter(const unsigned long long *ctr, unsigned long long target, uint32_t limit)
{
    for (uint32_t i = 0; i < limit; ++i) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ctr) : "memory");
        if (v >= target) return true;
        __nanosleep(32);
    }
    return false;
}

}  // namespace tb
