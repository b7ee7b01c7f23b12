// tb_decoders.cuh — per-type row decoders of the sm_100a matvec.
//
// The matvec kernel gives every thread ("lane") a fixed run of GPL consecutive
// 32-weight groups of a row (a column slot) for the whole launch.  The lane's
// activations for that slot live in registers (struct Lane, filled once by
// load()), and row_dot() returns sum_i w_i * x_i over the slot for one row whose
// raw GGUF bytes are staged in shared memory.  Decode semantics are those of
// layer4/tb_gguf_dequant.cu:89-332 (Q2_K: layer4/tb_gguf.c:210-225).
//
// Two arithmetic paths:
//
// * Integer path (Q4_K, Q5_K, Q6_K, Q2_K, Q8_0, Q4_0, Q8_K).  Each group's 32
//   activations are written exactly as X_i * 2^(E-20), E the exponent of the
//   group's largest |x|, X_i = round(x_i * 2^(20-E)) a 22-bit integer, and X_i
//   is split into three int8 digits X = H*2^14 + M*2^7 + L (H in [-128,127],
//   M, L in [0,127]).  The quant fields are masked four at a time into the
//   bytes of a word and multiplied against packed digits with dp4a (4 int8
//   MACs per instruction, exact int32 sums); one group's sums are combined in
//   fp32 and scaled by the block scales.  The only approximation is the
//   rounding of x to 2^-21 of its group's largest magnitude, below fp32's own
//   accumulation error for 32-term sums; products and sums are exact.
//   Digits are packed in the byte order in which a type's fields come out of
//   their words (see pk_index), so no field is ever moved after masking.
//
// * Float path (Q3_K, F32, F16, BF16), one group per lane.  A field of value q
//   masked in place at bit position P (P + width <= 24) of a 32-bit word is,
//   read as an fp32 bit pattern, exactly q * 2^(P-149) (a subnormal, or the
//   first normal binade, which has the same spacing).  Activations are stored
//   prescaled by 2^(149-P-C) for the position of their field, so every product
//   is q*x*2^-C with fp32 rounding; one power of two per group undoes the scale.
//   The library is built without -ftz, so subnormal operands keep their value.
#pragma once

#include "tb_common.cuh"

namespace tb {

constexpr int XC = 100;   // product scale exponent of the float path

__host__ __device__ constexpr int P2(int m) { return m < 12 ? 2 * m : 2 * m - 8; }

// 2^e as an fp32 bit pattern, e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(uint32_t(127 + e) << 23); }
__device__ __forceinline__ float fbits(uint32_t v) { return __uint_as_float(v); }
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float hsum(float2 a0, float2 a1) { return (a0.x + a0.y) + (a1.x + a1.y); }

// byte b of w placed in the low byte of 0x4B000000 (= 2^23 + byte) minus 2^23:
// an exact small-integer-to-float conversion with one PRMT and one FADD.
__device__ __forceinline__ float byte_to_float(uint32_t w, uint32_t b)
{
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + b)) - 8388608.0f;
}
__device__ __forceinline__ float sbyte_to_float(uint32_t w, uint32_t b)
{
    return static_cast<float>(static_cast<int8_t>((w >> (8 * b)) & 0xFFu));
}

// Where, inside a row, a lane's slot starts.
struct Pos {
    uint32_t off;   // byte offset of the block holding the slot's first group
    uint32_t gi0;   // index of that group inside its block (0..7 for 256-weight blocks)
    int ng;         // groups of the slot present in the row (GPL, fewer at the row's end)
    int n;          // weights of the slot's last group present (32, fewer only for floats)
};

// 32-bit words of a block whose staged copy may start at any byte.
// A16 = the caller guarantees 16-byte alignment (plain vector loads).
template <bool A16>
struct Words {
    const uint8_t *p;
    UnitBytes ub;
    __device__ __forceinline__ explicit Words(const uint8_t *blk) : p(blk), ub(blk) {}
    __device__ __forceinline__ uint32_t operator()(int i) const
    {
        return A16 ? reinterpret_cast<const uint32_t *>(p)[i] : ub.w(i);
    }
    __device__ __forceinline__ uint4 q4(int byte_off) const
    {
        if (A16) return *reinterpret_cast<const uint4 *>(p + byte_off);
        const int i = byte_off >> 2;
        return make_uint4(ub.w(i), ub.w(i + 1), ub.w(i + 2), ub.w(i + 3));
    }
};

// Reads the 32 activations of the slot's group `g` from the slot's staged copy
// `xs` (shared memory); `nv` = activations of the slot that exist (zeros after).
__device__ __forceinline__ void load_group(const float *xs, int nv, int g, float (&v)[32])
{
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (32 * g + i < nv) ? xs[32 * g + i] : 0.f;
}

// ============================================================================
// Integer path
// ============================================================================

// Digit packings: the activation index (0..31 in the group) that lands in byte
// b of packed word w, matching how each field layout is masked:
//   PK_NIB   nibbles of four 4-byte words: word t<4 low nibbles (w & 0x0F0F0F0F)
//            = weights 8t+2b, word 4+t high nibbles = weights 8t+2b+1
//   PK_TWO16 2-bit fields of two 16-weight words: (w >> 2j) & 0x03030303 of
//            word h = weights 16h + 4b + j, packed at 4h + j
//   PK_ONE32 bits of one 32-weight word: (w >> j) & 0x01010101 = weights j + 8b
//   PK_BYTE  bytes in order: weights 4w + b
enum { PK_NIB = 0, PK_TWO16 = 1, PK_ONE32 = 2, PK_BYTE = 3 };

__host__ __device__ constexpr int pk_index(int pk, int w, int b)
{
    return pk == PK_NIB ? 8 * (w & 3) + 2 * b + (w >> 2)
         : pk == PK_TWO16 ? 16 * (w >> 2) + 4 * b + (w & 3)
         : pk == PK_ONE32 ? w + 8 * b
                          : 4 * w + b;
}

// A lane's activations for GPL groups: NPK digit packings x 3 digits x 8 words.
template <int GPL, int NPK>
struct LaneI8 {
    int dg[GPL][NPK][3][8];
    float sx[GPL];      // 2^(E-20) per group
    float X[GPL][2];    // plain fp32 sums of x over each group's two 16-halves
};

template <int GPL, int PK0, int PK1>
__device__ __forceinline__ void load_i8(LaneI8<GPL, (PK1 < 0 ? 1 : 2)> &L, const float *xs, int nv)
{
#pragma unroll
    for (int g = 0; g < GPL; ++g) {
        float v[32];
        load_group(xs, nv, g, v);
        float s0 = 0.f, s1 = 0.f, mx = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            s0 += v[i];
            s1 += v[16 + i];
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
        L.X[g][0] = s0;
        L.X[g][1] = s1;
        int E = mx > 0.f ? static_cast<int>((__float_as_uint(mx) >> 23) & 255u) - 127 : 0;
        E = E < -100 ? -100 : E;
        const float up = exp2i(20 - E);
        L.sx[g] = exp2i(E - 20);
        int H[32], Mi[32], Lo[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            int q = __float2int_rn(v[i] * up);   // |q| <= 2^21
            q = q > 2097151 ? 2097151 : (q < -2097152 ? -2097152 : q);
            H[i] = q >> 14;
            Mi[i] = (q >> 7) & 127;
            Lo[i] = q & 127;
        }
#pragma unroll
        for (int pk = 0; pk < (PK1 < 0 ? 1 : 2); ++pk) {
            const int P = pk == 0 ? PK0 : PK1;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                uint32_t a = 0, b = 0, c = 0;
#pragma unroll
                for (int byte = 0; byte < 4; ++byte) {
                    const int i = pk_index(P, w, byte);
                    a |= (static_cast<uint32_t>(H[i]) & 0xFFu) << (8 * byte);
                    b |= (static_cast<uint32_t>(Mi[i]) & 0xFFu) << (8 * byte);
                    c |= (static_cast<uint32_t>(Lo[i]) & 0xFFu) << (8 * byte);
                }
                L.dg[g][pk][0][w] = static_cast<int>(a);
                L.dg[g][pk][1][w] = static_cast<int>(b);
                L.dg[g][pk][2][w] = static_cast<int>(c);
            }
        }
    }
}

// Three-digit accumulator: I[d] += fields . digits[d], kept as two independent
// chains (even / odd adds) so consecutive dp4a do not wait on each other.
struct Acc3 {
    int h0 = 0, m0 = 0, l0 = 0, h1 = 0, m1 = 0, l1 = 0;
    bool odd = false;
    __device__ __forceinline__ void add(uint32_t f, const int (&d)[3][8], int w)
    {
        if (!odd) {
            h0 = __dp4a(static_cast<int>(f), d[0][w], h0);
            m0 = __dp4a(static_cast<int>(f), d[1][w], m0);
            l0 = __dp4a(static_cast<int>(f), d[2][w], l0);
        } else {
            h1 = __dp4a(static_cast<int>(f), d[0][w], h1);
            m1 = __dp4a(static_cast<int>(f), d[1][w], m1);
            l1 = __dp4a(static_cast<int>(f), d[2][w], l1);
        }
        odd = !odd;
    }
    // sum_i f_i X_i = H*2^14 + M*2^7 + L as fp32 (exact up to the final rounding)
    __device__ __forceinline__ float value() const
    {
        return fmaf(static_cast<float>(h0 + h1), 16384.f, static_cast<float>((m0 + m1) * 128 + l0 + l1));
    }
    // same, combined in int32: valid while |sum f_i H_i| * 2^14 stays below 2^31
    // (fields below 32 on 32 weights, or below 64 on 16 weights)
    __device__ __forceinline__ float value_i32() const
    {
        return static_cast<float>((h0 + h1) * 16384 + (m0 + m1) * 128 + l0 + l1);
    }
};

// Low / high nibbles of a 4-byte word against PK_NIB words t and 4+t.
__device__ __forceinline__ void nib_word(Acc3 &a, uint32_t w, const int (&d)[3][8], int t)
{
    a.add(w & 0x0F0F0F0Fu, d, t);
    a.add((w >> 4) & 0x0F0F0F0Fu, d, 4 + t);
}

// The eight 6-bit Q4_K/Q5_K scales (or mins) of one half of a block as 4 bytes.
// tb_gguf_dequant.cu:103-108: for j<4 s[j] = sc[j]&63; s[j+4] =
// (sc[j]>>6) | ((sc[j+8]&15)<<2); mins likewise from sc[j+4] and sc[j+8]>>4.
// Written as one mux so a lane's half needs no branch: with upper = 0 the shift
// is 0 and the mask keeps all six bits of w_lo; with upper = 1 it keeps the top
// two bits of w_lo (moved down) and takes four bits of the third word.
__device__ __forceinline__ uint32_t sm_half(uint32_t w_lo, uint32_t w_hi8, uint32_t upper, bool mins)
{
    const uint32_t x = w_lo >> (6u * upper);
    const uint32_t y = mins ? (w_hi8 >> 2) : (w_hi8 << 2);
    const uint32_t k = upper ? 0x03030303u : 0x3F3F3F3Fu;
    return ((x & k) | (y & ~k)) & 0x3F3F3F3Fu;
}

// ---- Q4_K — 144 B: d,dmin @0, scales @4, qs @16 (tb_gguf_dequant.cu:89-118) ----
// w = d*s_g*q - dmin*m_g: group sum = d*s_g*sum(q x) - dmin*m_g*sum(x).
template <bool A16>
struct DecQ4K {
    static constexpr int GPL = 4;
    using Lane = LaneI8<GPL, 1>;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_i8<GPL, PK_NIB, -1>(L, xs, nv);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &L)
    {
        const Words<A16> W(row + p.off);
        const uint4 h = W.q4(0);
        const uint32_t upper = p.gi0 >> 2;
        const uint32_t sw = sm_half(h.y, h.w, upper, false), mw = sm_half(h.z, h.w, upper, true);
        const float2 dd = h2f2_ref(h.x);
        const float d = dd.x, dmin = dd.y;
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint4 q = W.q4(16 + 16 * (p.gi0 + g));
            Acc3 a;
            nib_word(a, q.x, L.dg[g][0], 0);
            nib_word(a, q.y, L.dg[g][0], 1);
            nib_word(a, q.z, L.dg[g][0], 2);
            nib_word(a, q.w, L.dg[g][0], 3);
            const uint32_t sb = (p.gi0 & 3u) + g;
            const float S = d * byte_to_float(sw, sb), Mn = dmin * byte_to_float(mw, sb);
            tot = fmaf(S * L.sx[g], a.value_i32(), tot);
            tot = fmaf(-Mn, L.X[g][0] + L.X[g][1], tot);
        }
        return tot;
    }
};

// ---- Q5_K — 176 B: d,dmin @0, scales @4, qh @16, qs @48 (tb_gguf_dequant.cu:158-191) ----
// q = nibble | qh_bit<<4; the high bit is masked as 0x10 per byte (already x16).
template <bool A16>
struct DecQ5K {
    static constexpr int GPL = 2;
    using Lane = LaneI8<GPL, 2>;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_i8<GPL, PK_NIB, PK_ONE32>(L, xs, nv);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &L)
    {
        const Words<A16> W(row + p.off);
        const uint4 h = W.q4(0);
        const uint32_t upper = p.gi0 >> 2;
        const uint32_t sw = sm_half(h.y, h.w, upper, false), mw = sm_half(h.z, h.w, upper, true);
        const float2 dd = h2f2_ref(h.x);
        const float d = dd.x, dmin = dd.y;
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint4 q = W.q4(48 + 16 * gi);
            const uint32_t hb = W(4 + gi);
            Acc3 a;
            nib_word(a, q.x, L.dg[g][0], 0);
            nib_word(a, q.y, L.dg[g][0], 1);
            nib_word(a, q.z, L.dg[g][0], 2);
            nib_word(a, q.w, L.dg[g][0], 3);
            a.add((hb << 4) & 0x10101010u, L.dg[g][1], 0);
            a.add((hb << 3) & 0x10101010u, L.dg[g][1], 1);
            a.add((hb << 2) & 0x10101010u, L.dg[g][1], 2);
            a.add((hb << 1) & 0x10101010u, L.dg[g][1], 3);
            a.add(hb & 0x10101010u, L.dg[g][1], 4);
            a.add((hb >> 1) & 0x10101010u, L.dg[g][1], 5);
            a.add((hb >> 2) & 0x10101010u, L.dg[g][1], 6);
            a.add((hb >> 3) & 0x10101010u, L.dg[g][1], 7);
            const uint32_t sb = (p.gi0 & 3u) + g;
            const float S = d * byte_to_float(sw, sb), Mn = dmin * byte_to_float(mw, sb);
            tot = fmaf(S * L.sx[g], a.value_i32(), tot);
            tot = fmaf(-Mn, L.X[g][0] + L.X[g][1], tot);
        }
        return tot;
    }
};

// ---- Q6_K — 210 B: ql @0, qh @128, int8 scales @192, d @208 (tb_gguf_dequant.cu:196-217) ----
// w = d*sc[i>>4]*(q-32), q = ql nibble | (qh 2 bits)<<4; the high bits are
// masked as 0x30 per byte (already x16); each 16-weight half has its own scale.
struct DecQ6K {
    static constexpr int GPL = 2;
    using Lane = LaneI8<GPL, 2>;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_i8<GPL, PK_NIB, PK_TWO16>(L, xs, nv);
    }
    __device__ static void hi16(Acc3 &a, uint32_t hq, const int (&d)[3][8], int base)
    {
        a.add((hq << 4) & 0x30303030u, d, base + 0);
        a.add((hq << 2) & 0x30303030u, d, base + 1);
        a.add(hq & 0x30303030u, d, base + 2);
        a.add((hq >> 2) & 0x30303030u, d, base + 3);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &L)
    {
        const Words<false> W(row + p.off);
        const float d = h2f2_ref(W(52)).x;
        const uint32_t scw = W.ub.at(192 + 2 * p.gi0);   // the slot's 2*GPL int8 scales
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint4 l = W.q4(16 * gi);
            const uint32_t h0 = W(32 + 2 * gi), h1 = W(33 + 2 * gi);
            Acc3 a, b;
            nib_word(a, l.x, L.dg[g][0], 0);
            nib_word(a, l.y, L.dg[g][0], 1);
            hi16(a, h0, L.dg[g][1], 0);
            nib_word(b, l.z, L.dg[g][0], 2);
            nib_word(b, l.w, L.dg[g][0], 3);
            hi16(b, h1, L.dg[g][1], 4);
            const float s0 = sbyte_to_float(scw, 2 * g), s1 = sbyte_to_float(scw, 2 * g + 1);
            const float t0 = fmaf(a.value_i32(), L.sx[g], -32.f * L.X[g][0]);
            const float t1 = fmaf(b.value_i32(), L.sx[g], -32.f * L.X[g][1]);
            tot = fmaf(d * s0, t0, tot);
            tot = fmaf(d * s1, t1, tot);
        }
        return tot;
    }
};

// ---- Q2_K — 84 B: scales @0 (lo4 scale, hi4 min), qs @16, d @80, dmin @82 ----
// (tb_gguf.c:210-225) w = d*(sc&15)*q - dmin*(sc>>4) per 16-weight scale block.
struct DecQ2K {
    static constexpr int GPL = 2;   // the slot's 2*GPL scale bytes are read as one word
    using Lane = LaneI8<GPL, 1>;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_i8<GPL, PK_TWO16, -1>(L, xs, nv);
    }
    __device__ static void two16(Acc3 &a, uint32_t q, const int (&d)[3][8], int base)
    {
        a.add(q & 0x03030303u, d, base + 0);
        a.add((q >> 2) & 0x03030303u, d, base + 1);
        a.add((q >> 4) & 0x03030303u, d, base + 2);
        a.add((q >> 6) & 0x03030303u, d, base + 3);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &L)
    {
        const Words<false> W(row + p.off);
        const uint32_t dd = W(20);
        const float2 df = h2f2_ref(dd);
        const float d = df.x, dmin = df.y;
        const uint32_t s01 = W(p.gi0 >> 1);   // the 2*GPL scale bytes of the slot
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint32_t q0 = W(4 + 2 * gi), q1 = W(5 + 2 * gi);
            Acc3 a, b;
            two16(a, q0, L.dg[g][0], 0);
            two16(b, q1, L.dg[g][0], 4);
            const uint32_t c0 = (s01 >> (16 * g)) & 0xFFu, c1 = (s01 >> (16 * g + 8)) & 0xFFu;
            const float sc0 = d * byte_to_float(c0 & 15u, 0), mn0 = dmin * byte_to_float(c0 >> 4, 0);
            const float sc1 = d * byte_to_float(c1 & 15u, 0), mn1 = dmin * byte_to_float(c1 >> 4, 0);
            tot = fmaf(sc0 * L.sx[g], a.value_i32(), tot);
            tot = fmaf(sc1 * L.sx[g], b.value_i32(), tot);
            tot = fmaf(-mn0, L.X[g][0], tot);
            tot = fmaf(-mn1, L.X[g][1], tot);
        }
        return tot;
    }
};

// ---- Q8_0 — 34 B / 32 weights: d @0, int8 qs @2 (tb_gguf_dequant.cu:246-262) ----
struct DecQ80 {
    static constexpr int GPL = 4;
    using Lane = LaneI8<GPL, 1>;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_i8<GPL, PK_BYTE, -1>(L, xs, nv);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &L)
    {
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            if (g >= p.ng) break;
            const uint8_t *blk = row + p.off + 34 * g;
            const UnitBytes hb(blk), qb(blk + 2);
            const float d = h2f2_ref(hb.w(0)).x;
            Acc3 a;
#pragma unroll
            for (int t = 0; t < 8; ++t) a.add(qb.w(t), L.dg[g][0], t);
            tot = fmaf(d * L.sx[g], a.value(), tot);
        }
        return tot;
    }
};

// ---- Q4_0 — 18 B / 32 weights: d @0, qs @2 (tb_gguf_dequant.cu:222-241) ----
// w[2t] = d*(lo-8), w[2t+1] = d*(hi-8).
struct DecQ40 {
    static constexpr int GPL = 4;
    using Lane = LaneI8<GPL, 1>;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_i8<GPL, PK_NIB, -1>(L, xs, nv);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &L)
    {
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            if (g >= p.ng) break;
            const uint8_t *blk = row + p.off + 18 * g;
            const UnitBytes hb(blk), qb(blk + 2);
            const float d = h2f2_ref(hb.w(0)).x;
            Acc3 a;
            nib_word(a, qb.w(0), L.dg[g][0], 0);
            nib_word(a, qb.w(1), L.dg[g][0], 1);
            nib_word(a, qb.w(2), L.dg[g][0], 2);
            nib_word(a, qb.w(3), L.dg[g][0], 3);
            tot = fmaf(d, fmaf(a.value_i32(), L.sx[g], -8.f * (L.X[g][0] + L.X[g][1])), tot);
        }
        return tot;
    }
};

// ---- Q8_K — 292 B: f32 d @0, int8 qs @4, bsums ignored (tb_gguf_dequant.cu:268-284) ----
struct DecQ8K {
    static constexpr int GPL = 4;
    using Lane = LaneI8<GPL, 1>;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_i8<GPL, PK_BYTE, -1>(L, xs, nv);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &L)
    {
        const Words<false> W(row + p.off);
        const float d = __uint_as_float(W(0));
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const int b = 1 + 8 * static_cast<int>(p.gi0 + g);
            Acc3 a;
#pragma unroll
            for (int t = 0; t < 8; ++t) a.add(W(b + t), L.dg[g][0], t);
            tot = fmaf(L.sx[g], a.value(), tot);
        }
        return d * tot;
    }
};

// ============================================================================
// Float path
// ============================================================================

// The lane's 32 activations as 16 register pairs (two prescaled arrays) plus
// the plain fp32 sums of each 16-half.
struct XRegs {
    float2 a[16];
    float2 b[16];
    float X0, X1;
};

template <class MulA, class MulB>
__device__ __forceinline__ void load_f32(XRegs &L, const float *xs, int nv, MulA ma, MulB mb)
{
    float v[32];
    load_group(xs, nv, 0, v);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        s0 += v[i];
        s1 += v[16 + i];
    }
    L.X0 = s0;
    L.X1 = s1;
#pragma unroll
    for (int p = 0; p < 16; ++p) {
        L.a[p] = f2(v[2 * p] * ma(2 * p), v[2 * p + 1] * ma(2 * p + 1));
        L.b[p] = f2(v[2 * p] * mb(2 * p), v[2 * p + 1] * mb(2 * p + 1));
    }
}

// 16 two-bit fields at P2 positions against x pairs O..O+7.
template <int O>
__device__ __forceinline__ void two16f(uint32_t w, const float2 (&x)[16], float2 &a0, float2 &a1)
{
    const uint32_t w8 = w >> 8;
    a0 = ffma2(f2(fbits(w & 0x3u), fbits(w & 0xCu)), x[O + 0], a0);
    a1 = ffma2(f2(fbits(w & 0x30u), fbits(w & 0xC0u)), x[O + 1], a1);
    a0 = ffma2(f2(fbits(w & 0x300u), fbits(w & 0xC00u)), x[O + 2], a0);
    a1 = ffma2(f2(fbits(w & 0x3000u), fbits(w & 0xC000u)), x[O + 3], a1);
    a0 = ffma2(f2(fbits(w & 0x30000u), fbits(w & 0xC0000u)), x[O + 4], a0);
    a1 = ffma2(f2(fbits(w & 0x300000u), fbits(w & 0xC00000u)), x[O + 5], a1);
    a0 = ffma2(f2(fbits(w8 & 0x30000u), fbits(w8 & 0xC0000u)), x[O + 6], a0);
    a1 = ffma2(f2(fbits(w8 & 0x300000u), fbits(w8 & 0xC00000u)), x[O + 7], a1);
}

// 8 one-bit fields at bits m (m < 8) against x pairs O..O+3.
template <int O>
__device__ __forceinline__ void bit8f(uint32_t w, const float2 (&x)[16], float2 &a0, float2 &a1)
{
    a0 = ffma2(f2(fbits(w & 0x1u), fbits(w & 0x2u)), x[O + 0], a0);
    a1 = ffma2(f2(fbits(w & 0x4u), fbits(w & 0x8u)), x[O + 1], a1);
    a0 = ffma2(f2(fbits(w & 0x10u), fbits(w & 0x20u)), x[O + 2], a0);
    a1 = ffma2(f2(fbits(w & 0x40u), fbits(w & 0x80u)), x[O + 3], a1);
}

// ---- Q3_K — 110 B: hmask @0, qs @32, scales @96, d @108 (tb_gguf_dequant.cu:124-151) ----
// Scale block j uses is = (j<8 ? j : j-8): lo4 = (sc[is>>1] >> 4(is&1)) & 15 =
// (word24 >> 4is) & 15, hi2 = (sc[8+(is>>2)] >> 2(is&3)) & 3 = (word26 >> 2is) & 3;
// w = d*((lo4|hi2<<4)-32) * (low2 | hbit<<2 - 4).  The high bit accumulates
// against x*4 (second array), read 8 bits at a time at positions 0..7.
struct DecQ3K {
    static constexpr int GPL = 1;
    using Lane = XRegs;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_f32(L, xs, nv, [](int i) { return exp2i(149 - P2(i & 15) - XC); },
                 [](int i) { return exp2i(149 + 2 - (i & 7) - XC); });
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &x)
    {
        const Words<false> W(row + p.off);
        const uint32_t hm = W(p.gi0);
        const uint32_t q0 = W(8 + 2 * p.gi0), q1 = W(9 + 2 * p.gi0);
        const uint32_t r0 = W(24), r2 = W(26), dw = W(27);
        float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f), b0 = f2(0.f, 0.f), b1 = f2(0.f, 0.f);
        two16f<0>(q0, x.a, a0, a1);
        bit8f<0>(hm, x.b, a0, a1);
        bit8f<4>(hm >> 8, x.b, a0, a1);
        two16f<8>(q1, x.a, b0, b1);
        bit8f<8>(hm >> 16, x.b, b0, b1);
        bit8f<12>(hm >> 24, x.b, b0, b1);
        const float d = h2f2_ref(dw).x;
        const uint32_t j0 = 2 * p.gi0, is0 = j0 < 8 ? j0 : j0 - 8, is1 = is0 + 1;
        const int v0 = static_cast<int>(((r0 >> (4 * is0)) & 15u) | (((r2 >> (2 * is0)) & 3u) << 4)) - 32;
        const int v1 = static_cast<int>(((r0 >> (4 * is1)) & 15u) | (((r2 >> (2 * is1)) & 3u) << 4)) - 32;
        const float S0 = d * static_cast<float>(v0), S1 = d * static_cast<float>(v1);
        const float C = exp2i(XC);
        const float t0 = fmaf(hsum(a0, a1), C, -4.f * x.X0);
        const float t1 = fmaf(hsum(b0, b1), C, -4.f * x.X1);
        return fmaf(S0, t0, S1 * t1);
    }
};

// ---- F32 / F16 / BF16 — `n` valid elements in the slot's group ----
// F16 uses the reference converter (tb_gguf_dequant.cu:54-63).
template <int QT>
struct DecFloat {
    static constexpr int GPL = 1;
    using Lane = XRegs;
    __device__ static void load(Lane &L, const float *xs, int nv)
    {
        load_f32(L, xs, nv, [](int) { return 1.f; }, [](int) { return 0.f; });
    }
    __device__ static float elem(const UnitBytes &ub, int i)
    {
        if (QT == QT_F32) return __uint_as_float(ub.w(i));
        const uint32_t w = ub.w(i >> 1);
        const uint32_t h = (i & 1) ? (w >> 16) : (w & 0xFFFFu);
        return QT == QT_F16 ? h2f_ref(h) : __uint_as_float(h << 16);
    }
    __device__ static float row_dot(const uint8_t *row, const Pos &p, const Lane &x)
    {
        const UnitBytes ub(row + p.off);
        float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
        if (p.n == 32) {
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                float2 w;
                if (QT == QT_F32) {
                    w = f2(__uint_as_float(ub.w(2 * q)), __uint_as_float(ub.w(2 * q + 1)));
                } else {
                    const uint32_t v = ub.w(q);
                    w = QT == QT_F16 ? f2(h2f_ref(v & 0xFFFFu), h2f_ref(v >> 16))
                                     : f2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
                }
                if (q & 1) a1 = ffma2(w, x.a[q], a1);
                else       a0 = ffma2(w, x.a[q], a0);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                if (2 * q < p.n) a0.x = fmaf(elem(ub, 2 * q), x.a[q].x, a0.x);
                if (2 * q + 1 < p.n) a0.y = fmaf(elem(ub, 2 * q + 1), x.a[q].y, a0.y);
            }
        }
        return hsum(a0, a1);
    }
};

}  // namespace tb
