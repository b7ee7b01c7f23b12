// tb_decoders_f32.cuh — fp32-activation row decoders of the sm_100a matvec
// (the default arithmetic for every quantized type).
//
// The reference multiplies each dequantised weight by an fp32 activation and
// accumulates in fp32 (layer4/tb_gguf_dequant.cu:113-114:
// acc += fmaf(S*q, x, -Mn*x)).  These decoders do the same arithmetic with the
// sub-block scales factored out of the inner sum:
//
//   y = sum_g S_g * sum_{i in g} q_i * x_i  -  sum_g Mn_g * sum_{i in g} x_i
//
// where every product q_i * x_i and every sum is an fp32 operation on the
// unrounded fp32 activation (no rounding of x to a narrower type anywhere).
//
// * Exact field conversion.  A quant field of value q masked in place at bit
//   position P (its top bit at most bit 23) of a 32-bit word is, read as an
//   fp32 bit pattern, exactly q * 2^(P-149): a subnormal, or for a field that
//   reaches bit 23 the smallest normal binade, which has the same spacing.  So
//   one AND turns a field into an fp32 operand, and one paired FMA
//   (__ffma2_rn, sm_100) multiplies two such fields by two activations.
// * Prescaled activations.  Each lane keeps its column slot's 64 activations
//   in registers as x'_i = x_i * 2^(107 - E - P_i), E the exponent of the
//   slot's largest |x| (clamped to [-20, 126]) and P_i the bit position the
//   decoder masks weight i's field at.  Multiplying by a power of two is exact
//   (no overflow or underflow in that range), so x'_i carries x_i's full fp32
//   mantissa, and every product is exactly q_i * x_i * 2^(-42-E), rounded once
//   to fp32 like the reference's product; the sums run in fp32.  The sums of
//   x used by the mins and offsets carry the same factor, and the result is
//   scaled back by 2^42 (folded into the fp16 scale conversion) and 2^E.
// * Pairs.  Both halves of a paired FMA take the same field position from two
//   sub-blocks (or groups, or blocks) of the slot, so one accumulator pair
//   holds two sub-block sums and the scales are applied with paired ops too.
//
// Slot = GPL = 2 NP groups (64 NP weights; NP = 1 by default): a quarter of a
// K-quant super-block or two Q8_0 / Q4_0 blocks, processed as one or two pair
// units of two groups or sub-blocks.  The 64 prescaled activations take 64
// registers, so these kernels run 16 warps of up to 128 registers (NP = 2: 128
// activations at 8 warps of up to 255); the per-row header decode (scales,
// mins, d) is paid once per slot.  Decode semantics are those of
// layer4/tb_gguf_dequant.cu:89-284 (Q2_K: layer4/tb_gguf.c:210-225), the same
// field layouts as the integer-path decoders in tb_decoders.cuh.
#pragma once

#include <type_traits>

#include "tb_decoders.cuh"

namespace tb {

// IsF32X<D>: D is an fp32-activation decoder (declares kF32X = true).
template <class D, class = void>
struct IsF32X : std::false_type {};
template <class D>
struct IsF32X<D, std::void_t<decltype(D::kF32X)>> : std::integral_constant<bool, D::kF32X> {};

// NP pair units (64 activations each) per column slot; the default NP = 1
// keeps 64 prescaled activations in registers at 16 warps per CTA, NP = 2
// keeps 128 at 8 warps of up to 255 registers.
#ifndef TB_XF_THREADS
#define TB_XF_THREADS 512   // threads per CTA of the one-unit (NP = 1) decoders
#endif
template <int NP>
struct XfGeom {
    static constexpr int N = 64 * NP;                    // activations per slot
    static constexpr int THREADS = NP == 1 ? TB_XF_THREADS : 256;  // threads per CTA
    static constexpr int REC = rec_stride(N + 1);        // record: N floats, the max word, padding
};
#ifndef TB_XF_NP
#define TB_XF_NP 1
#endif
constexpr int XF_NP = TB_XF_NP;
constexpr float kTwo23 = 8388608.0f;

// Common part of every fp32-path lane: the slot's output scale 2^E (times the
// RMSNorm factor when the input is normalised).
struct LaneXF {
    float sx;
};

__device__ __forceinline__ void lane_scale(LaneXF &L, float f) { L.sx *= f; }

// The slot exponent from the magnitude bits of its largest |x|: 0 and
// subnormal maxima give -20 (the products then sit lower in the normal range),
// inf / nan give 126 (they propagate as in the reference).
__device__ __forceinline__ int xf_exponent(uint32_t mb)
{
    const int e = static_cast<int>(mb >> 23) - 127;
    return e < -20 ? -20 : (e > 126 ? 126 : e);
}

// The record's N activations and the slot exponent (N / 4 + 1 shared loads).
template <int N>
__device__ __forceinline__ int xf_raw(const uint32_t *rec, float (&r)[N])
{
    const uint32_t a = shared_after(static_cast<uint32_t>(__cvta_generic_to_shared(rec)));
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
        const uint4 v = lds_u128(a + 16 * i);
        r[4 * i] = __uint_as_float(v.x);
        r[4 * i + 1] = __uint_as_float(v.y);
        r[4 * i + 2] = __uint_as_float(v.z);
        r[4 * i + 3] = __uint_as_float(v.w);
    }
    return xf_exponent(lds_u32(a + 4 * N));
}

// Sum of r[i0 .. i0+n) scaled like the products: (sum * 2^-E) * 2^-42.
template <int N, int R>
__device__ __forceinline__ float xf_sum(const float (&r)[R], int i0, int E)
{
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) s += r[i0 + i];
    return (s * exp2i(-E)) * 0x1p-42f;
}

// Both fp16 halves of w through the reference converter, times 2^42 (exact).
__device__ __forceinline__ float2 h2f2_x42(uint32_t w)
{
    float2 f = __half22float2(__halves2half2(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)),
                                             __ushort_as_half(static_cast<unsigned short>(w >> 16))));
    f.x *= (w & 0x00007C00u) ? 0x1p42f : 0x1p-70f;
    f.y *= (w & 0x7C000000u) ? 0x1p42f : 0x1p-70f;
    return f;
}

// Unsigned byte k (0..3, may be a runtime value) of w as 2^23 + byte, and the
// signed-byte form 2^23 + 128 + (int8)byte; subtract the bias to get the value.
__device__ __forceinline__ float u8_biased(uint32_t w, uint32_t k)
{
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | k));
}
__device__ __forceinline__ float s8_biased(uint32_t w, uint32_t k)
{
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | k) ^ 0x80u);
}
__device__ __forceinline__ float2 u8pair(uint32_t w, uint32_t k0, uint32_t k1)
{
    return __fadd2_rn(f2(u8_biased(w, k0), u8_biased(w, k1)), f2(-kTwo23, -kTwo23));
}
__device__ __forceinline__ float2 s8pair(uint32_t w, uint32_t k0, uint32_t k1)
{
    return __fadd2_rn(f2(s8_biased(w, k0), s8_biased(w, k1)), f2(-(kTwo23 + 128.f), -(kTwo23 + 128.f)));
}

// One paired FMA of two fields masked in place from words a and b.
__device__ __forceinline__ float2 fma_m(uint32_t a, uint32_t b, uint32_t mask, float2 x, float2 acc)
{
    return __ffma2_rn(f2(fbits(a & mask), fbits(b & mask)), x, acc);
}

// Bit position of byte lane b's field after the decoders' extraction: lanes
// 0..2 are masked in place, lane 3 is shifted down by 24 first.
__host__ __device__ constexpr int lane_pos(int b) { return b < 3 ? 8 * b : 0; }

// The four byte-lane fields (width MASK) of words a and b against pairs x[0..3],
// alternating between two accumulators.  Lane 3 is read as word >> 24, so a
// field there must fill the top byte's low bits only (top bits zero).
template <uint32_t MASK>
__device__ __forceinline__ void lanes4(uint32_t a, uint32_t b, const float2 *x, float2 &c0, float2 &c1)
{
    c0 = fma_m(a, b, MASK, x[0], c0);
    c1 = fma_m(a, b, MASK << 8, x[1], c1);
    c0 = fma_m(a, b, MASK << 16, x[2], c0);
    c1 = __ffma2_rn(f2(fbits(a >> 24), fbits(b >> 24)), x[3], c1);
}

// Conventions of the decoders below.  A "pair unit" is two groups or
// sub-blocks of the slot decoded side by side; pair p of unit u holds the
// prescaled activations of the same field position in both (x[u][p]), and
// xs[u] their two x sums.  A slot is NP units of 64 weights (GPL = 2 NP
// groups of 32).
#define TB_XF_TRAITS                                                  \
    static constexpr int GPL = 2 * NP;                                \
    static constexpr bool kInt = false, kF32X = true;                 \
    static constexpr int REC = XfGeom<NP>::REC;                       \
    static constexpr int kThreads = XfGeom<NP>::THREADS;              \
    static constexpr int XN = XfGeom<NP>::N;

// ---- Q4_K — 144 B: d,dmin @0, scales @4, qs @16 (tb_gguf_dequant.cu:89-118) ----
// Slot = groups gi0 .. gi0 + 2 NP - 1, units (gi0, gi0+1), (gi0+2, gi0+3).  qs word t of a group: nibble n = weight 8t + n,
// at bit 4n; nibbles 6, 7 are read from the word shifted right by 8 (bits 16,
// 20).  Pair 8t + n of unit u = weight 8t + n of its two groups.
template <bool A16, int NP = XF_NP>
struct DecQ4KF {
    TB_XF_TRAITS
    struct Lane : LaneXF {
        float2 x[NP][32];
        float2 xs[NP];
    };
    __host__ __device__ static constexpr int pos(int n) { return n < 6 ? 4 * n : 4 * n - 8; }
    __device__ static void load(Lane &L, const uint32_t *rec)
    {
        float r[XN];
        const int E = xf_raw(rec, r);
#pragma unroll
        for (int u = 0; u < NP; ++u) {
#pragma unroll
            for (int w = 0; w < 32; ++w) {
                const float f = exp2i(107 - E - pos(w & 7));
                L.x[u][w] = f2(r[64 * u + w] * f, r[64 * u + 32 + w] * f);
            }
            L.xs[u] = f2(xf_sum<32>(r, 64 * u, E), xf_sum<32>(r, 64 * u + 32, E));
        }
        L.sx = exp2i(E);
    }
    __device__ static float2 unit(const Words<A16> &W, uint32_t gi, const float2 (&x)[32])
    {
        const uint4 qa = W.q4(16 + 16 * gi), qb = W.q4(32 + 16 * gi);
        const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, wb[4] = {qb.x, qb.y, qb.z, qb.w};
        float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t a = wa[t], b = wb[t], a8 = a >> 8, b8 = b >> 8;
            const float2 *xx = x + 8 * t;
            c0 = fma_m(a, b, 0xFu, xx[0], c0);
            c1 = fma_m(a, b, 0xF0u, xx[1], c1);
            c0 = fma_m(a, b, 0xF00u, xx[2], c0);
            c1 = fma_m(a, b, 0xF000u, xx[3], c1);
            c0 = fma_m(a, b, 0xF0000u, xx[4], c0);
            c1 = fma_m(a, b, 0xF00000u, xx[5], c1);
            c0 = fma_m(a8, b8, 0xF0000u, xx[6], c0);
            c1 = fma_m(a8, b8, 0xF00000u, xx[7], c1);
        }
        return __fadd2_rn(c0, c1);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<A16> W(row + p.off);
        const uint4 h = W.q4(0);
        const uint32_t upper = p.gi0 >> 2;
        const uint32_t sw = sm_half(h.y, h.w, upper, false), mw = sm_half(h.z, h.w, upper, true);
        const uint32_t k0 = p.gi0 & 3u;   // byte of group gi0 in the half's scale words
        float2 r2 = f2(0.f, 0.f), m2 = f2(0.f, 0.f);
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            const uint32_t k = k0 + 2 * u;
            r2 = __ffma2_rn(u8pair(sw, k, k + 1), unit(W, p.gi0 + 2 * u, x.x[u]), r2);
            m2 = __ffma2_rn(u8pair(mw, k, k + 1), x.xs[u], m2);
        }
        const float2 dd = h2f2_x42(h.x);
        return x.sx * fmaf(dd.x, r2.x + r2.y, -dd.y * (m2.x + m2.y));
    }
};

// ---- Q5_K — 176 B: d,dmin @0, scales @4, qh @16, qs @48 (tb_gguf_dequant.cu:158-191) ----
// Group words are transposed as in the integer decoder (six byte permutes:
// byte b of c_k = qs byte 4b + k, i.e. weights 8b + 2k, 8b + 2k + 1), then
// field word j (0..7) holds weight 8b + j in byte lane b with its qh bit at
// bit 4.  Units (gi0, gi0+1), (gi0+2, gi0+3); pair 4j + b = weight 8b + j.
template <bool A16, int NP = XF_NP>
struct DecQ5KF {
    TB_XF_TRAITS
    struct Lane : LaneXF {
        float2 x[NP][32];
        float2 xs[NP];
    };
    __device__ static void load(Lane &L, const uint32_t *rec)
    {
        float r[XN];
        const int E = xf_raw(rec, r);
#pragma unroll
        for (int u = 0; u < NP; ++u) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float f = exp2i(107 - E - lane_pos(b));
                    L.x[u][4 * j + b] = f2(r[64 * u + 8 * b + j] * f, r[64 * u + 32 + 8 * b + j] * f);
                }
            L.xs[u] = f2(xf_sum<32>(r, 64 * u, E), xf_sum<32>(r, 64 * u + 32, E));
        }
        L.sx = exp2i(E);
    }
    // the eight field words of one group
    __device__ static void fields(const Words<A16> &W, uint32_t gi, uint32_t (&F)[8])
    {
        constexpr uint32_t N = 0x0F0F0F0Fu, B = 0x10101010u;
        const uint4 q = W.q4(48 + 16 * gi);
        const uint32_t hb = W(4 + gi);
        const uint32_t t0 = __byte_perm(q.x, q.y, 0x5140u), t1 = __byte_perm(q.z, q.w, 0x5140u);
        const uint32_t t2 = __byte_perm(q.x, q.y, 0x7362u), t3 = __byte_perm(q.z, q.w, 0x7362u);
        const uint32_t c0 = __byte_perm(t0, t1, 0x5410u), c1 = __byte_perm(t0, t1, 0x7632u);
        const uint32_t c2 = __byte_perm(t2, t3, 0x5410u), c3 = __byte_perm(t2, t3, 0x7632u);
        F[0] = (c0 & N) | ((hb << 4) & B);
        F[1] = ((c0 >> 4) & N) | ((hb << 3) & B);
        F[2] = (c1 & N) | ((hb << 2) & B);
        F[3] = ((c1 >> 4) & N) | ((hb << 1) & B);
        F[4] = (c2 & N) | (hb & B);
        F[5] = ((c2 >> 4) & N) | ((hb >> 1) & B);
        F[6] = (c3 & N) | ((hb >> 2) & B);
        F[7] = ((c3 >> 4) & N) | ((hb >> 3) & B);
    }
    __device__ static float2 unit(const Words<A16> &W, uint32_t gi, const float2 (&x)[32])
    {
        uint32_t Fa[8], Fb[8];
        fields(W, gi, Fa);
        fields(W, gi + 1, Fb);
        float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) lanes4<0x1Fu>(Fa[j], Fb[j], x + 4 * j, c0, c1);
        return __fadd2_rn(c0, c1);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<A16> W(row + p.off);
        const uint4 h = W.q4(0);
        const uint32_t upper = p.gi0 >> 2;
        const uint32_t sw = sm_half(h.y, h.w, upper, false), mw = sm_half(h.z, h.w, upper, true);
        const uint32_t k0 = p.gi0 & 3u;   // byte of group gi0 in the half's scale words
        float2 r2 = f2(0.f, 0.f), m2 = f2(0.f, 0.f);
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            const uint32_t k = k0 + 2 * u;
            r2 = __ffma2_rn(u8pair(sw, k, k + 1), unit(W, p.gi0 + 2 * u, x.x[u]), r2);
            m2 = __ffma2_rn(u8pair(mw, k, k + 1), x.xs[u], m2);
        }
        const float2 dd = h2f2_x42(h.x);
        return x.sx * fmaf(dd.x, r2.x + r2.y, -dd.y * (m2.x + m2.y));
    }
};

// ---- Q6_K — 210 B: ql @0, qh @128, int8 scales @192, d @208 (tb_gguf_dequant.cu:196-217) ----
// Slot = sub-blocks u = 2*gi0 + s, s = 0 .. 4 NP - 1 (16 weights each),
// units (0,1), (2,3), ...  A sub-block's field words (two byte
// permutes of its ql words, then the qh bits or-ed in, as in the integer
// decoder): word j holds weight 4b + j of the sub-block in byte lane b (6
// bits).  The -32 is applied per sub-block as -32 * (sum of its x).  Pair
// 4j + b of a unit = weight 4b + j of its two sub-blocks.
template <int NP = XF_NP>
struct DecQ6KF {
    TB_XF_TRAITS
    struct Lane : LaneXF {
        float2 x[2 * NP][16];
        float2 xs[2 * NP];
    };
    __device__ static void load(Lane &L, const uint32_t *rec)
    {
        float r[XN];
        const int E = xf_raw(rec, r);
#pragma unroll
        for (int sp = 0; sp < 2 * NP; ++sp) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float f = exp2i(107 - E - lane_pos(b));
                    const int i = 32 * sp + 4 * b + j;
                    L.x[sp][4 * j + b] = f2(r[i] * f, r[i + 16] * f);
                }
            L.xs[sp] = f2(xf_sum<16>(r, 32 * sp, E), xf_sum<16>(r, 32 * sp + 16, E));
        }
        L.sx = exp2i(E);
    }
    __device__ static void fields(uint32_t A, uint32_t B, uint32_t h, uint32_t (&F)[4])
    {
        constexpr uint32_t N = 0x0F0F0F0Fu, M = 0x30303030u;
        const uint32_t e = __byte_perm(A, B, 0x6420u);   // ql bytes 0,2,4,6: weights 4b (lo), 4b+1 (hi)
        const uint32_t o = __byte_perm(A, B, 0x7531u);   // ql bytes 1,3,5,7: weights 4b+2, 4b+3
        F[0] = (e & N) | ((h << 4) & M);
        F[1] = ((e >> 4) & N) | ((h << 2) & M);
        F[2] = (o & N) | (h & M);
        F[3] = ((o >> 4) & N) | ((h >> 2) & M);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<false> W(row + p.off);
        const float d = h2f2_x42(W(52)).x;
        uint32_t sc[NP];   // the slot's int8 scales, four per word
#pragma unroll
        for (int i = 0; i < NP; ++i) sc[i] = W(48 + (p.gi0 >> 1) + i);
        float2 r2 = f2(0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < 2 * NP; ++sp) {
            const uint32_t u = 2 * p.gi0 + 2 * sp;
            uint32_t F0[4], F1[4];
            fields(W(2 * u), W(2 * u + 1), W(32 + u), F0);
            fields(W(2 * u + 2), W(2 * u + 3), W(33 + u), F1);
            float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 4; ++j) lanes4<0x3Fu>(F0[j], F1[j], x.x[sp] + 4 * j, c0, c1);
            const float2 v = __ffma2_rn(f2(-32.f, -32.f), x.xs[sp], __fadd2_rn(c0, c1));
            r2 = __ffma2_rn(s8pair(sc[sp >> 1], 2 * (sp & 1), 2 * (sp & 1) + 1), v, r2);
        }
        return x.sx * (d * (r2.x + r2.y));
    }
};

// ---- Q3_K — 110 B: hmask @0, qs @32, scales @96, d @108 (tb_gguf_dequant.cu:124-151) ----
// Slot = groups gi0 .. gi0 + 2 NP - 1; unit g pairs the two sub-blocks s = 0,
// 1 of group gi0 + g (scale index is = (2 gi + s) mod 8: the signed bytes g of the
// even / odd scale words).  Field word k of a sub-block holds weight 4b + k in
// byte lane b as l | h << 2 (three bits), as in the integer decoder; the -4 is
// applied per sub-block as -4 * (sum of its x).  Pair 4k + b = weight 4b + k.
template <int NP = XF_NP>
struct DecQ3KF {
    TB_XF_TRAITS
    struct Lane : LaneXF {
        float2 x[2 * NP][16];
        float2 xs[2 * NP];
    };
    __device__ static void load(Lane &L, const uint32_t *rec)
    {
        float r[XN];
        const int E = xf_raw(rec, r);
#pragma unroll
        for (int g = 0; g < 2 * NP; ++g) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float f = exp2i(107 - E - lane_pos(b));
                    const int i = 32 * g + 4 * b + k;
                    L.x[g][4 * k + b] = f2(r[i] * f, r[i + 16] * f);
                }
            L.xs[g] = f2(xf_sum<16>(r, 32 * g, E), xf_sum<16>(r, 32 * g + 16, E));
        }
        L.sx = exp2i(E);
    }
    __device__ static void fields(uint32_t q, uint32_t h, uint32_t (&F)[4])
    {
        F[0] = (q & 0x03030303u) | ((h << 2) & 0x04040404u);
        F[1] = ((q >> 2) & 0x03030303u) | ((h << 1) & 0x04040404u);
        F[2] = ((q >> 4) & 0x03030303u) | (h & 0x04040404u);
        F[3] = ((q >> 6) & 0x03030303u) | ((h >> 1) & 0x04040404u);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<false> W(row + p.off);
        const float d = h2f2_x42(W(27)).x;
        uint32_t ev, od;
        DecQ3K::scales(W(24), W(26), ev, od);   // signed (scale - 32) bytes, even / odd index
        ev ^= 0x80808080u;                      // offset by 128 for the biased conversion
        od ^= 0x80808080u;
        float2 r2 = f2(0.f, 0.f);
#pragma unroll
        for (int g = 0; g < 2 * NP; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint32_t hm = W(gi);
            uint32_t F0[4], F1[4];
            fields(W(8 + 2 * gi), DecQ3K::spread(hm, 0x1100u), F0);
            fields(W(9 + 2 * gi), DecQ3K::spread(hm, 0x3322u), F1);
            float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 4; ++k) lanes4<0x07u>(F0[k], F1[k], x.x[g] + 4 * k, c0, c1);
            const float2 v = __ffma2_rn(f2(-4.f, -4.f), x.xs[g], __fadd2_rn(c0, c1));
            const uint32_t m = gi & 3u;   // the byte of scale index (2 gi + s) mod 8, halved
            const float2 sc = __fadd2_rn(f2(u8_biased(ev, m), u8_biased(od, m)),
                                         f2(-(kTwo23 + 128.f), -(kTwo23 + 128.f)));
            r2 = __ffma2_rn(sc, v, r2);
        }
        return x.sx * (d * (r2.x + r2.y));
    }
};

// ---- Q2_K — 84 B: scales @0 (lo4 scale, hi4 min), qs @16, d @80, dmin @82 ----
// (tb_gguf.c:210-225) Slot = sub-blocks u = 2*gi0 + s, s = 0 .. 4 NP - 1,
// units (0,1), (2,3), ...  A sub-block's qs word holds weight 4b + k at bit
// 8b + 2k; lanes 0..2 are masked in place, lane 3 from the word shifted right
// by 24.  Pair 4b + k of a unit = weight 4b + k of its two sub-blocks.
template <bool A4, int NP = XF_NP>
struct DecQ2KF {
    TB_XF_TRAITS
    struct Lane : LaneXF {
        float2 x[2 * NP][16];
        float2 xs[2 * NP];
    };
    __device__ static void load(Lane &L, const uint32_t *rec)
    {
        float r[XN];
        const int E = xf_raw(rec, r);
#pragma unroll
        for (int sp = 0; sp < 2 * NP; ++sp) {
#pragma unroll
            for (int b = 0; b < 4; ++b)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float f = exp2i(107 - E - lane_pos(b) - 2 * k);
                    const int i = 32 * sp + 4 * b + k;
                    L.x[sp][4 * b + k] = f2(r[i] * f, r[i + 16] * f);
                }
            L.xs[sp] = f2(xf_sum<16>(r, 32 * sp, E), xf_sum<16>(r, 32 * sp + 16, E));
        }
        L.sx = exp2i(E);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<A4> W(row + p.off);
        const float2 dd = h2f2_x42(W(20));
        uint32_t scl[NP], mnl[NP];   // the slot's scale / min bytes, four per word
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            const uint32_t w = W((p.gi0 >> 1) + i);
            scl[i] = w & 0x0F0F0F0Fu;
            mnl[i] = (w >> 4) & 0x0F0F0F0Fu;
        }
        float2 r2 = f2(0.f, 0.f), m2 = f2(0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < 2 * NP; ++sp) {
            const uint32_t a = W(4 + 2 * p.gi0 + 2 * sp), b = W(5 + 2 * p.gi0 + 2 * sp);
            const uint32_t a24 = a >> 24, b24 = b >> 24;
            const float2 *xx = x.x[sp];
            float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
            for (int bb = 0; bb < 3; ++bb) {
                c0 = fma_m(a, b, 0x3u << (8 * bb), xx[4 * bb + 0], c0);
                c1 = fma_m(a, b, 0xCu << (8 * bb), xx[4 * bb + 1], c1);
                c0 = fma_m(a, b, 0x30u << (8 * bb), xx[4 * bb + 2], c0);
                c1 = fma_m(a, b, 0xC0u << (8 * bb), xx[4 * bb + 3], c1);
            }
            c0 = fma_m(a24, b24, 0x3u, xx[12], c0);
            c1 = fma_m(a24, b24, 0xCu, xx[13], c1);
            c0 = fma_m(a24, b24, 0x30u, xx[14], c0);
            c1 = fma_m(a24, b24, 0xC0u, xx[15], c1);
            const uint32_t k = 2 * (sp & 1);
            r2 = __ffma2_rn(u8pair(scl[sp >> 1], k, k + 1), __fadd2_rn(c0, c1), r2);
            m2 = __ffma2_rn(u8pair(mnl[sp >> 1], k, k + 1), x.xs[sp], m2);
        }
        return x.sx * fmaf(dd.x, r2.x + r2.y, -dd.y * (m2.x + m2.y));
    }
};

// ---- Q8_0 — 34 B / 32 weights: d @0, int8 qs @2 (tb_gguf_dequant.cu:246-262) ----
// Slot = blocks 0 .. 2 NP - 1 (fewer at a row's end: p.ng), units (0,1), (2,3).
// Signed bytes are read offset by 128 (xor 0x80) and the offset taken back as
// -128 * (sum of the block's x).  Pair 4t + lane = weight 4t + lane.
template <int NP = XF_NP>
struct DecQ80F {
    TB_XF_TRAITS
    struct Lane : LaneXF {
        float2 x[NP][32];
        float2 xs[NP];
    };
    __device__ static void load(Lane &L, const uint32_t *rec)
    {
        float r[XN];
        const int E = xf_raw(rec, r);
#pragma unroll
        for (int u = 0; u < NP; ++u) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float f = exp2i(107 - E - lane_pos(i & 3));
                L.x[u][i] = f2(r[64 * u + i] * f, r[64 * u + 32 + i] * f);
            }
            L.xs[u] = f2(xf_sum<32>(r, 64 * u, E), xf_sum<32>(r, 64 * u + 32, E));
        }
        L.sx = exp2i(E);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        float tot = 0.f;
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            // a block past the row's end (p.ng) re-reads block 0 (in bounds); its values are discarded
            const bool ha = 2 * u < p.ng, hb = 2 * u + 1 < p.ng;
            const uint32_t ra = row + p.off + (ha ? 68u * u : 0u), rb = row + p.off + (hb ? 68u * u + 34u : 0u);
            const UnitBytes Ha(ra), Hb(rb), qa(ra + 2), qb(rb + 2);
            const float da = ha ? h2f2_x42(Ha.w(0)).x : 0.f;
            const float db = hb ? h2f2_x42(Hb.w(0)).x : 0.f;
            float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 8; ++t)
                lanes4<0xFFu>(qa.w(t) ^ 0x80808080u, qb.w(t) ^ 0x80808080u, x.x[u] + 4 * t, c0, c1);
            const float2 v = __ffma2_rn(f2(-128.f, -128.f), x.xs[u], __fadd2_rn(c0, c1));
            tot = fmaf(da, v.x, fmaf(db, v.y, tot));
        }
        return x.sx * tot;
    }
};

// ---- Q4_0 — 18 B / 32 weights: d @0, qs @2 (tb_gguf_dequant.cu:222-241) ----
// w[2t] = d*(lo-8), w[2t+1] = d*(hi-8); the -8 as -8 * (sum of the block's x).
// Nibble n of qs word t = weight 8t + n, read as in Q4_K.  Units (0,1), ...
template <int NP = XF_NP>
struct DecQ40F {
    TB_XF_TRAITS
    struct Lane : LaneXF {
        float2 x[NP][32];
        float2 xs[NP];
    };
    __device__ static void load(Lane &L, const uint32_t *rec)
    {
        float r[XN];
        const int E = xf_raw(rec, r);
#pragma unroll
        for (int u = 0; u < NP; ++u) {
#pragma unroll
            for (int w = 0; w < 32; ++w) {
                const float f = exp2i(107 - E - DecQ4KF<false, NP>::pos(w & 7));
                L.x[u][w] = f2(r[64 * u + w] * f, r[64 * u + 32 + w] * f);
            }
            L.xs[u] = f2(xf_sum<32>(r, 64 * u, E), xf_sum<32>(r, 64 * u + 32, E));
        }
        L.sx = exp2i(E);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        float tot = 0.f;
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            const bool ha = 2 * u < p.ng, hb = 2 * u + 1 < p.ng;
            const uint32_t ra = row + p.off + (ha ? 36u * u : 0u), rb = row + p.off + (hb ? 36u * u + 18u : 0u);
            const UnitBytes Ha(ra), Hb(rb), qa(ra + 2), qb(rb + 2);
            const float da = ha ? h2f2_x42(Ha.w(0)).x : 0.f;
            const float db = hb ? h2f2_x42(Hb.w(0)).x : 0.f;
            float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t a = qa.w(t), b = qb.w(t), a8 = a >> 8, b8 = b >> 8;
                const float2 *xx = x.x[u] + 8 * t;
                c0 = fma_m(a, b, 0xFu, xx[0], c0);
                c1 = fma_m(a, b, 0xF0u, xx[1], c1);
                c0 = fma_m(a, b, 0xF00u, xx[2], c0);
                c1 = fma_m(a, b, 0xF000u, xx[3], c1);
                c0 = fma_m(a, b, 0xF0000u, xx[4], c0);
                c1 = fma_m(a, b, 0xF00000u, xx[5], c1);
                c0 = fma_m(a8, b8, 0xF0000u, xx[6], c0);
                c1 = fma_m(a8, b8, 0xF00000u, xx[7], c1);
            }
            const float2 v = __ffma2_rn(f2(-8.f, -8.f), x.xs[u], __fadd2_rn(c0, c1));
            tot = fmaf(da, v.x, fmaf(db, v.y, tot));
        }
        return x.sx * tot;
    }
};

// ---- Q8_K — 292 B: f32 d @0, int8 qs @4, bsums ignored (tb_gguf_dequant.cu:268-284) ----
// Slot = 64 NP consecutive weights of a block (its first at qs word 8 * gi0);
// unit u pairs weights 64u + i and 64u + 32 + i, signed bytes offset by 128
// as in Q8_0.
template <int NP = XF_NP>
struct DecQ8KF {
    TB_XF_TRAITS
    using Lane = typename DecQ80F<NP>::Lane;   // same register layout and load as Q8_0
    __device__ static void load(Lane &L, const uint32_t *rec) { DecQ80F<NP>::load(L, rec); }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<false> W(row + p.off);
        const float d = __uint_as_float(W(0)) * 0x1p42f;
        const int b0 = 1 + 8 * static_cast<int>(p.gi0);
        float tot = 0.f;
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            float2 c0 = f2(0.f, 0.f), c1 = f2(0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 8; ++t)
                lanes4<0xFFu>(W(b0 + 16 * u + t) ^ 0x80808080u, W(b0 + 16 * u + 8 + t) ^ 0x80808080u,
                              x.x[u] + 4 * t, c0, c1);
            const float2 v = __ffma2_rn(f2(-128.f, -128.f), x.xs[u], __fadd2_rn(c0, c1));
            tot += v.x + v.y;
        }
        return x.sx * (d * tot);
    }
};

#undef TB_XF_TRAITS

}  // namespace tb
