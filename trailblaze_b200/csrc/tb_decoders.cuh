// tb_decoders.cuh — per-type unit decoders of the sm_100a matvec.
//
// Each decoder returns sum_i w_i * x_i over one unit (256 weights) whose raw
// bytes sit in shared memory, for the reference decode semantics of
// layer4/tb_gguf_dequant.cu:89-332 (Q2_K: layer4/tb_gguf.c:210-225).
//
// Integer fields become floats without any int->float conversion.  A field of
// value q masked in place at bit position P (P + width <= 24) of a 32-bit word
// is, read as an fp32 bit pattern, exactly q * 2^(P-149): a subnormal, or for
// P + width = 24 the first normal binade, which has the same spacing.  The
// activation is stored prescaled by 2^(149-P-C) for the P at which its weight's
// field is extracted, so every product is q*x*2^-C exactly as fp32 rounds q*x,
// and one power-of-two factor 2^C per group undoes the scale.  Per weight that
// is one LOP3 plus half of an FFMA2 (the sm_100 paired fp32 FMA).  The kernels
// are built without -ftz, so subnormal operands keep their value.
//
// Position patterns (field index m inside its 32-bit word; fields at bits 24+
// are first moved down by 8 with one shift per word):
//   P4(m) = m<6 ? 4m : 4m-8    nibbles  (8 per word)
//   P2(m) = m<12 ? 2m : 2m-8   2-bit    (16 per word)
//   P1(m) = m<24 ? m : m-8     1-bit    (32 per word)
//   P8(m) = m<3 ? 8m : 16      bytes    (4 per word)
#pragma once

#include "tb_common.cuh"

namespace tb {

constexpr int XC = 100;                   // common product scale exponent
constexpr int XSTRIDE = 260;              // floats per unit in a staged x array (256 + bank skew)

__host__ __device__ constexpr int P4(int m) { return m < 6 ? 4 * m : 4 * m - 8; }
__host__ __device__ constexpr int P2(int m) { return m < 12 ? 2 * m : 2 * m - 8; }
__host__ __device__ constexpr int P1(int m) { return m < 24 ? m : m - 8; }
__host__ __device__ constexpr int P8(int m) { return m < 3 ? 8 * m : 16; }

// 2^e as an fp32 bit pattern, e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(uint32_t(127 + e) << 23); }

__device__ __forceinline__ float fbits(uint32_t v) { return __uint_as_float(v); }

// small unsigned integer (< 2^23) to float, exact, without I2F
__device__ __forceinline__ float u2f_small(uint32_t v)
{
    return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// ---- field extraction + paired FMA over one word ---------------------------
// 8 nibbles of w against x[0..7] (prescaled with P4); two accumulators.
__device__ __forceinline__ void acc_nib8(uint32_t w, const float *x, float2 &a0, float2 &a1)
{
    const float4 xl = *reinterpret_cast<const float4 *>(x);
    const float4 xh = *reinterpret_cast<const float4 *>(x + 4);
    const uint32_t w8 = w >> 8;
    a0 = ffma2(f2(fbits(w & 0xFu), fbits(w & 0xF0u)), f2(xl.x, xl.y), a0);
    a1 = ffma2(f2(fbits(w & 0xF00u), fbits(w & 0xF000u)), f2(xl.z, xl.w), a1);
    a0 = ffma2(f2(fbits(w & 0xF0000u), fbits(w & 0xF00000u)), f2(xh.x, xh.y), a0);
    a1 = ffma2(f2(fbits(w8 & 0xF0000u), fbits(w8 & 0xF00000u)), f2(xh.z, xh.w), a1);
}

// 16 two-bit fields of w against x[0..15] (prescaled with P2).
__device__ __forceinline__ void acc_2b16(uint32_t w, const float *x, float2 &a0, float2 &a1)
{
    const float4 x0 = *reinterpret_cast<const float4 *>(x);
    const float4 x1 = *reinterpret_cast<const float4 *>(x + 4);
    const float4 x2 = *reinterpret_cast<const float4 *>(x + 8);
    const float4 x3 = *reinterpret_cast<const float4 *>(x + 12);
    const uint32_t w8 = w >> 8;
    a0 = ffma2(f2(fbits(w & 0x3u), fbits(w & 0xCu)), f2(x0.x, x0.y), a0);
    a1 = ffma2(f2(fbits(w & 0x30u), fbits(w & 0xC0u)), f2(x0.z, x0.w), a1);
    a0 = ffma2(f2(fbits(w & 0x300u), fbits(w & 0xC00u)), f2(x1.x, x1.y), a0);
    a1 = ffma2(f2(fbits(w & 0x3000u), fbits(w & 0xC000u)), f2(x1.z, x1.w), a1);
    a0 = ffma2(f2(fbits(w & 0x30000u), fbits(w & 0xC0000u)), f2(x2.x, x2.y), a0);
    a1 = ffma2(f2(fbits(w & 0x300000u), fbits(w & 0xC00000u)), f2(x2.z, x2.w), a1);
    a0 = ffma2(f2(fbits(w8 & 0x30000u), fbits(w8 & 0xC0000u)), f2(x3.x, x3.y), a0);
    a1 = ffma2(f2(fbits(w8 & 0x300000u), fbits(w8 & 0xC00000u)), f2(x3.z, x3.w), a1);
}

// 16 one-bit fields of w starting at bit `base` (0 or 16) against x[0..15]
// (prescaled with P1 of the bit index within the word).
template <int BASE>
__device__ __forceinline__ void acc_1b16(uint32_t w, const float *x, float2 &a0, float2 &a1)
{
    const float4 x0 = *reinterpret_cast<const float4 *>(x);
    const float4 x1 = *reinterpret_cast<const float4 *>(x + 4);
    const float4 x2 = *reinterpret_cast<const float4 *>(x + 8);
    const float4 x3 = *reinterpret_cast<const float4 *>(x + 12);
    if (BASE == 0) {
        a0 = ffma2(f2(fbits(w & 0x1u), fbits(w & 0x2u)), f2(x0.x, x0.y), a0);
        a1 = ffma2(f2(fbits(w & 0x4u), fbits(w & 0x8u)), f2(x0.z, x0.w), a1);
        a0 = ffma2(f2(fbits(w & 0x10u), fbits(w & 0x20u)), f2(x1.x, x1.y), a0);
        a1 = ffma2(f2(fbits(w & 0x40u), fbits(w & 0x80u)), f2(x1.z, x1.w), a1);
        a0 = ffma2(f2(fbits(w & 0x100u), fbits(w & 0x200u)), f2(x2.x, x2.y), a0);
        a1 = ffma2(f2(fbits(w & 0x400u), fbits(w & 0x800u)), f2(x2.z, x2.w), a1);
        a0 = ffma2(f2(fbits(w & 0x1000u), fbits(w & 0x2000u)), f2(x3.x, x3.y), a0);
        a1 = ffma2(f2(fbits(w & 0x4000u), fbits(w & 0x8000u)), f2(x3.z, x3.w), a1);
    } else {
        const uint32_t w8 = w >> 8;   // bits 24..31 -> 16..23
        a0 = ffma2(f2(fbits(w & 0x10000u), fbits(w & 0x20000u)), f2(x0.x, x0.y), a0);
        a1 = ffma2(f2(fbits(w & 0x40000u), fbits(w & 0x80000u)), f2(x0.z, x0.w), a1);
        a0 = ffma2(f2(fbits(w & 0x100000u), fbits(w & 0x200000u)), f2(x1.x, x1.y), a0);
        a1 = ffma2(f2(fbits(w & 0x400000u), fbits(w & 0x800000u)), f2(x1.z, x1.w), a1);
        a0 = ffma2(f2(fbits(w8 & 0x10000u), fbits(w8 & 0x20000u)), f2(x2.x, x2.y), a0);
        a1 = ffma2(f2(fbits(w8 & 0x40000u), fbits(w8 & 0x80000u)), f2(x2.z, x2.w), a1);
        a0 = ffma2(f2(fbits(w8 & 0x100000u), fbits(w8 & 0x200000u)), f2(x3.x, x3.y), a0);
        a1 = ffma2(f2(fbits(w8 & 0x400000u), fbits(w8 & 0x800000u)), f2(x3.z, x3.w), a1);
    }
}

// 4 bytes of w (already biased to unsigned) against x[0..3] (prescaled with P8).
__device__ __forceinline__ void acc_b4(uint32_t w, const float *x, float2 &a0, float2 &a1)
{
    const float4 xv = *reinterpret_cast<const float4 *>(x);
    a0 = ffma2(f2(fbits(w & 0xFFu), fbits(w & 0xFF00u)), f2(xv.x, xv.y), a0);
    a1 = ffma2(f2(fbits(w & 0xFF0000u), fbits((w >> 8) & 0xFF0000u)), f2(xv.z, xv.w), a1);
}

__device__ __forceinline__ float hsum(float2 a0, float2 a1) { return (a0.x + a0.y) + (a1.x + a1.y); }

// 8 six-bit (Q4_K/Q5_K) scales and mins, unpacked four per word.
// tb_gguf_dequant.cu:103-108: s[j]=sc[j]&63, m[j]=sc[j+4]&63,
// s[j+4]=(sc[j]>>6)|((sc[j+8]&15)<<2), m[j+4]=(sc[j+4]>>6)|((sc[j+8]>>4)<<2).
__device__ __forceinline__ void unpack_sm(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t &sl,
                                          uint32_t &sh, uint32_t &ml, uint32_t &mh)
{
    sl = s0 & 0x3F3F3F3Fu;
    ml = s1 & 0x3F3F3F3Fu;
    sh = ((s0 >> 6) & 0x03030303u) | ((s2 << 2) & 0x3C3C3C3Cu);
    mh = ((s1 >> 6) & 0x03030303u) | ((s2 >> 2) & 0x3C3C3C3Cu);
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return (w >> (8 * j)) & 0xFFu; }

// ============================================================================
// Q4_K — 144 B: d,dmin @0, scales @4, qs @16 (tb_gguf_dequant.cu:89-118).
// ============================================================================
template <bool A16>
struct DecQ4K {
    static constexpr int NXA = 1;
    __device__ static float xmul(int, int i) { return exp2i(149 - P4(i & 7) - XC); }

    __device__ static float dot(const uint8_t *u, int, const float *xa, const float *,
                                const float *xs16)
    {
        uint32_t h0, s0, s1, s2;
        UnitBytes ub(u);
        if (A16) {
            const uint4 h = *reinterpret_cast<const uint4 *>(u);
            h0 = h.x; s0 = h.y; s1 = h.z; s2 = h.w;
        } else {
            h0 = ub.w(0); s0 = ub.w(1); s1 = ub.w(2); s2 = ub.w(3);
        }
        const float d = h2f_ref(h0 & 0xFFFFu), dmin = h2f_ref(h0 >> 16);
        uint32_t sl, sh, ml, mh;
        unpack_sm(s0, s1, s2, sl, sh, ml, mh);
        const float dC = d * exp2i(XC);
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            uint32_t q[4];
            if (A16) {
                const uint4 v = *reinterpret_cast<const uint4 *>(u + 16 + 16 * g);
                q[0] = v.x; q[1] = v.y; q[2] = v.z; q[3] = v.w;
            } else {
#pragma unroll
                for (int t = 0; t < 4; ++t) q[t] = ub.w(4 + 4 * g + t);
            }
            float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 4; ++t) acc_nib8(q[t], xa + 32 * g + 8 * t, a0, a1);
            const uint32_t sw = g < 4 ? sl : sh, mw = g < 4 ? ml : mh;
            const float S = dC * u2f_small(byte_of(sw, g & 3));
            const float Mn = dmin * u2f_small(byte_of(mw, g & 3));
            const float X = xs16[2 * g] + xs16[2 * g + 1];
            tot = fmaf(S, hsum(a0, a1), tot);
            tot = fmaf(-Mn, X, tot);
        }
        return tot;
    }
};

// ============================================================================
// Q5_K — 176 B: d,dmin @0, scales @4, qh @16, qs @48 (tb_gguf_dequant.cu:158-191).
// q = nibble | qh_bit<<4; the high bit is accumulated against x*16.
// ============================================================================
template <bool A16>
struct DecQ5K {
    static constexpr int NXA = 2;
    __device__ static float xmul(int a, int i)
    {
        return a == 0 ? exp2i(149 - P4(i & 7) - XC) : exp2i(149 + 4 - P1(i & 31) - XC);
    }

    __device__ static float dot(const uint8_t *u, int, const float *xa, const float *xb,
                                const float *xs16)
    {
        uint32_t h0, s0, s1, s2;
        UnitBytes ub(u);
        if (A16) {
            const uint4 h = *reinterpret_cast<const uint4 *>(u);
            h0 = h.x; s0 = h.y; s1 = h.z; s2 = h.w;
        } else {
            h0 = ub.w(0); s0 = ub.w(1); s1 = ub.w(2); s2 = ub.w(3);
        }
        const float d = h2f_ref(h0 & 0xFFFFu), dmin = h2f_ref(h0 >> 16);
        uint32_t sl, sh, ml, mh;
        unpack_sm(s0, s1, s2, sl, sh, ml, mh);
        const float dC = d * exp2i(XC);
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            uint32_t q[4], hb;
            if (A16) {
                const uint4 v = *reinterpret_cast<const uint4 *>(u + 48 + 16 * g);
                q[0] = v.x; q[1] = v.y; q[2] = v.z; q[3] = v.w;
                hb = *reinterpret_cast<const uint32_t *>(u + 16 + 4 * g);
            } else {
#pragma unroll
                for (int t = 0; t < 4; ++t) q[t] = ub.w(12 + 4 * g + t);
                hb = ub.w(4 + g);
            }
            float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 4; ++t) acc_nib8(q[t], xa + 32 * g + 8 * t, a0, a1);
            acc_1b16<0>(hb, xb + 32 * g, a0, a1);
            acc_1b16<16>(hb, xb + 32 * g + 16, a0, a1);
            const uint32_t sw = g < 4 ? sl : sh, mw = g < 4 ? ml : mh;
            const float S = dC * u2f_small(byte_of(sw, g & 3));
            const float Mn = dmin * u2f_small(byte_of(mw, g & 3));
            const float X = xs16[2 * g] + xs16[2 * g + 1];
            tot = fmaf(S, hsum(a0, a1), tot);
            tot = fmaf(-Mn, X, tot);
        }
        return tot;
    }
};

// ============================================================================
// Q6_K — 210 B: ql @0, qh @128, int8 scales @192, d @208 (tb_gguf_dequant.cu:196-217).
// w = d*sc[i>>4]*(q-32), q = ql nibble | qh 2 bits<<4.
// ============================================================================
struct DecQ6K {
    static constexpr int NXA = 2;
    __device__ static float xmul(int a, int i)
    {
        return a == 0 ? exp2i(149 - P4(i & 7) - XC) : exp2i(149 + 4 - P2(i & 15) - XC);
    }

    __device__ static float dot(const uint8_t *u, int, const float *xa, const float *xb,
                                const float *xs16)
    {
        UnitBytes ub(u);
        const float d = h2f_ref(ub.w(52) & 0xFFFFu);
        const uint32_t sc4[4] = {ub.w(48), ub.w(49), ub.w(50), ub.w(51)};
        const float C = exp2i(XC);
        float tot = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t l0 = ub.w(2 * j), l1 = ub.w(2 * j + 1), hq = ub.w(32 + j);
            float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
            acc_nib8(l0, xa + 16 * j, a0, a1);
            acc_nib8(l1, xa + 16 * j + 8, a0, a1);
            acc_2b16(hq, xb + 16 * j, a0, a1);
            const int sc = static_cast<int8_t>(byte_of(sc4[j >> 2], j & 3));
            const float ds = d * static_cast<float>(sc);
            tot = fmaf(ds, fmaf(hsum(a0, a1), C, -32.f * xs16[j]), tot);
        }
        return tot;
    }
};

// ============================================================================
// Q3_K — 110 B: hmask @0, qs @32, scales @96, d @108 (tb_gguf_dequant.cu:124-151).
// S[j] = d*((lo4|hi2<<4)-32) with is=(j<8?j:j-8); w = S[i>>4]*(low2|hbit<<2 - 4).
// ============================================================================
struct DecQ3K {
    static constexpr int NXA = 2;
    __device__ static float xmul(int a, int i)
    {
        return a == 0 ? exp2i(149 - P2(i & 15) - XC) : exp2i(149 + 2 - P1(i & 31) - XC);
    }

    __device__ static float dot(const uint8_t *u, int, const float *xa, const float *xb,
                                const float *xs16)
    {
        UnitBytes ub(u);
        // scale bytes 96..107; sub-scales read sr[0..3] and sr[8..9] only
        const uint32_t r0 = ub.w(24), r2 = ub.w(26);
        const float d = h2f_ref(ub.w(27) & 0xFFFFu);
        const float C = exp2i(XC);
        float S[8];
#pragma unroll
        for (int is = 0; is < 8; ++is) {
            const uint32_t lo_byte = byte_of(r0, is >> 1);
            const uint32_t lo4 = (lo_byte >> ((is & 1) * 4)) & 15u;
            const uint32_t hi2 = (byte_of(r2, is >> 2) >> ((is & 3) * 2)) & 3u;
            S[is] = d * static_cast<float>(static_cast<int>(lo4 | (hi2 << 4)) - 32);
        }
        float tot = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t lq = ub.w(8 + j), hm = ub.w(j >> 1);
            float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
            acc_2b16(lq, xa + 16 * j, a0, a1);
            if (j & 1) acc_1b16<16>(hm, xb + 16 * j, a0, a1);
            else       acc_1b16<0>(hm, xb + 16 * j, a0, a1);
            tot = fmaf(S[j & 7], fmaf(hsum(a0, a1), C, -4.f * xs16[j]), tot);
        }
        return tot;
    }
};

// ============================================================================
// Q2_K — 84 B: scales @0 (lo4 scale, hi4 min), qs @16, d @80, dmin @82
// (tb_gguf.c:210-225).  w = d*(sc&15)*q - dmin*(sc>>4) per 16 weights.
// ============================================================================
struct DecQ2K {
    static constexpr int NXA = 1;
    __device__ static float xmul(int, int i) { return exp2i(149 - P2(i & 15) - XC); }

    __device__ static float dot(const uint8_t *u, int, const float *xa, const float *,
                                const float *xs16)
    {
        UnitBytes ub(u);
        const uint32_t sc4[4] = {ub.w(0), ub.w(1), ub.w(2), ub.w(3)};
        const uint32_t dd = ub.w(20);
        const float d = h2f_ref(dd & 0xFFFFu), dmin = h2f_ref(dd >> 16);
        const float dC = d * exp2i(XC);
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < 16; ++g) {
            float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
            acc_2b16(ub.w(4 + g), xa + 16 * g, a0, a1);
            const uint32_t sb = byte_of(sc4[g >> 2], g & 3);
            const float sc = dC * u2f_small(sb & 15u);
            const float mn = dmin * u2f_small(sb >> 4);
            tot = fmaf(sc, hsum(a0, a1), tot);
            tot = fmaf(-mn, xs16[g], tot);
        }
        return tot;
    }
};

// ============================================================================
// Q8_0 — 34 B / 32 weights, 8 blocks per unit: d @0, int8 qs @2
// (tb_gguf_dequant.cu:246-262).  Bytes biased by 128 (xor 0x80), bias removed
// with the block's x sum.
// ============================================================================
struct DecQ80 {
    static constexpr int NXA = 1;
    __device__ static float xmul(int, int i) { return exp2i(149 - P8(i & 3) - XC); }

    __device__ static float dot(const uint8_t *u, int nblk, const float *xa, const float *,
                                const float *xs16)
    {
        const float C = exp2i(XC);
        float tot = 0.f;
        for (int b = 0; b < nblk; ++b) {
            const uint8_t *blk = u + 34 * b;
            UnitBytes hb(blk);
            UnitBytes qb(blk + 2);
            const float d = h2f_ref(hb.w(0) & 0xFFFFu);
            float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 8; ++t) acc_b4(qb.w(t) ^ 0x80808080u, xa + 32 * b + 4 * t, a0, a1);
            const float X = xs16[2 * b] + xs16[2 * b + 1];
            tot = fmaf(d, fmaf(hsum(a0, a1), C, -128.f * X), tot);
        }
        return tot;
    }
};

// ============================================================================
// Q4_0 — 18 B / 32 weights, 8 blocks per unit: d @0, qs @2
// (tb_gguf_dequant.cu:222-241).  w[2t]=d*(lo-8), w[2t+1]=d*(hi-8).
// ============================================================================
struct DecQ40 {
    static constexpr int NXA = 1;
    __device__ static float xmul(int, int i) { return exp2i(149 - P4(i & 7) - XC); }

    __device__ static float dot(const uint8_t *u, int nblk, const float *xa, const float *,
                                const float *xs16)
    {
        const float C = exp2i(XC);
        float tot = 0.f;
        for (int b = 0; b < nblk; ++b) {
            const uint8_t *blk = u + 18 * b;
            UnitBytes hb(blk);
            UnitBytes qb(blk + 2);
            const float d = h2f_ref(hb.w(0) & 0xFFFFu);
            float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 4; ++t) acc_nib8(qb.w(t), xa + 32 * b + 8 * t, a0, a1);
            const float X = xs16[2 * b] + xs16[2 * b + 1];
            tot = fmaf(d, fmaf(hsum(a0, a1), C, -8.f * X), tot);
        }
        return tot;
    }
};

// ============================================================================
// Q8_K — 292 B: f32 d @0, int8 qs @4, bsums ignored (tb_gguf_dequant.cu:268-284).
// ============================================================================
struct DecQ8K {
    static constexpr int NXA = 1;
    __device__ static float xmul(int, int i) { return exp2i(149 - P8(i & 3) - XC); }

    __device__ static float dot(const uint8_t *u, int, const float *xa, const float *,
                                const float *xs16)
    {
        UnitBytes ub(u);
        const float d = __uint_as_float(ub.w(0));
        float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
#pragma unroll 16
        for (int t = 0; t < 64; ++t) acc_b4(ub.w(1 + t) ^ 0x80808080u, xa + 4 * t, a0, a1);
        float X = 0.f;
#pragma unroll
        for (int g = 0; g < 16; ++g) X += xs16[g];
        return d * fmaf(hsum(a0, a1), exp2i(XC), -128.f * X);
    }
};

// ============================================================================
// F32 / F16 / BF16 — 256 elements per unit, `n` valid (the last unit of a row
// may be partial).  F16 uses the reference converter (tb_gguf_dequant.cu:54-63).
// ============================================================================
template <int QT>
struct DecFloat {
    static constexpr int NXA = 1;
    __device__ static float xmul(int, int) { return 1.f; }

    __device__ static float dot(const uint8_t *u, int n, const float *xa, const float *,
                                const float *)
    {
        UnitBytes ub(u);
        float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
        if (QT == QT_F32) {
            int i = 0;
            for (; i + 2 <= n; i += 2)
                a0 = ffma2(f2(__uint_as_float(ub.w(i)), __uint_as_float(ub.w(i + 1))),
                           f2(xa[i], xa[i + 1]), a0);
            if (i < n) a1.x = fmaf(__uint_as_float(ub.w(i)), xa[i], a1.x);
        } else {
            int t = 0;
            for (; 2 * t + 2 <= n; ++t) {
                const uint32_t w = ub.w(t);
                const float lo = QT == QT_F16 ? h2f_ref(w & 0xFFFFu) : __uint_as_float(w << 16);
                const float hi = QT == QT_F16 ? h2f_ref(w >> 16) : __uint_as_float(w & 0xFFFF0000u);
                a0 = ffma2(f2(lo, hi), f2(xa[2 * t], xa[2 * t + 1]), a0);
            }
            if (2 * t < n) {
                const uint32_t w = ub.w(t);
                const float lo = QT == QT_F16 ? h2f_ref(w & 0xFFFFu) : __uint_as_float(w << 16);
                a1.x = fmaf(lo, xa[2 * t], a1.x);
            }
        }
        return hsum(a0, a1);
    }
};

}  // namespace tb
