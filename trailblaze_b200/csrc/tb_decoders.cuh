// tb_decoders.cuh — per-type row decoders of the sm_100a matvec.
//
// The matvec kernel gives every thread ("lane") a fixed run of GPL consecutive
// 32-weight groups of a row (a column slot) for the whole launch.  The lane's
// activations for that slot live in registers (struct Lane), loaded once from
// a per-slot record that the CTA prepares cooperatively in shared memory
// (prep(): one thread per 32-activation group).  row_dot() then returns
// sum_i w_i * x_i over the slot for one row whose raw GGUF bytes are staged in
// shared memory.  Decode semantics are those of layer4/tb_gguf_dequant.cu:89-332
// (Q2_K: layer4/tb_gguf.c:210-225).
//
// Two arithmetic paths:
//
// * Integer path (every quantized type).  The slot's activations are written
//   exactly as X_i * 2^(E-14), E the exponent of the slot's largest |x|,
//   X_i = round(x_i * 2^(14-E)) a 16-bit integer, split into two byte digits
//   X = 256*H + L (H signed, L unsigned).  Quant fields are masked four at a
//   time into the bytes of a word and multiplied against packed digits with
//   dp4a: 4 exact byte MACs per instruction.  The sub-block scales are
//   integers, so they are applied with one integer multiply-add per digit and
//   the whole slot is summed exactly in int32; one float conversion per slot
//   remains.  The only approximation is the rounding of x to 2^-15 of the
//   slot's largest magnitude (a relative error of a few 1e-5 in y for Gaussian
//   x, against the 1e-3 bar); every product and sum is exact.  Digits are
//   packed in the byte order in which a type's fields come out of their words
//   (see pk_index), so no field is moved after masking.
//
// * Float path (F32, F16, BF16), one group per lane: paired fp32 FMAs
//   (__ffma2_rn) of the converted weights against the lane's 32 activations.
#pragma once

#include "tb_common.cuh"

namespace tb {

// 2^e as an fp32 bit pattern, e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(uint32_t(127 + e) << 23); }
__device__ __forceinline__ float fbits(uint32_t v) { return __uint_as_float(v); }
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float hsum(float2 a0, float2 a1) { return (a0.x + a0.y) + (a1.x + a1.y); }

// Where, inside a row, a lane's slot starts.
struct Pos {
    uint32_t off;   // byte offset of the block holding the slot's first group
    uint32_t gi0;   // index of that group inside its block (0..7 for 256-weight blocks)
    int ng;         // groups of the slot present in the row (GPL, fewer at the row's end)
    int n;          // weights of the slot's last group present (32, fewer only for floats)
};

// 32-bit words of a block whose staged copy (a shared-window address) may start
// at any byte.  A16 = the caller guarantees 16-byte alignment (vector loads).
template <bool A16>
struct Words {
    uint32_t p;
    UnitBytes ub;
    __device__ __forceinline__ explicit Words(uint32_t blk) : p(blk), ub(blk) {}
    __device__ __forceinline__ uint32_t operator()(int i) const { return A16 ? lds_u32(p + 4 * i) : ub.w(i); }
    __device__ __forceinline__ uint4 q4(int byte_off) const
    {
        if (A16) return lds_u128(p + byte_off);
        const int i = byte_off >> 2;
        return make_uint4(ub.w(i), ub.w(i + 1), ub.w(i + 2), ub.w(i + 3));
    }
};

// ============================================================================
// Slot records: what prep() writes to shared memory and load() reads back.
// ============================================================================

// Record stride in 32-bit words for `words` of content: a multiple of 4 (16-byte
// records) with an odd number of 16-byte chunks, so the 128-bit loads of eight
// consecutive lanes (consecutive slots) fall on eight different bank quads.
__host__ __device__ constexpr int rec_stride(int words)
{
    return ((words + 3) / 4) % 2 ? ((words + 3) / 4) * 4 : ((words + 3) / 4 + 1) * 4;
}

// Copies a record of W words (W a multiple of 4) into registers, 16 bytes at a
// time, by ld.shared (called once per launch, after the barrier that completes
// the records; the laundered address keeps the loads after it).
template <int W>
__device__ __forceinline__ void load_rec(uint32_t (&r)[W], const uint32_t *rec)
{
    static_assert(W % 4 == 0, "records are whole 16-byte chunks");
    const uint32_t a = shared_after(static_cast<uint32_t>(__cvta_generic_to_shared(rec)));
#pragma unroll
    for (int i = 0; i < W / 4; ++i) {
        const uint4 v = lds_u128(a + 16 * i);
        r[4 * i] = v.x;
        r[4 * i + 1] = v.y;
        r[4 * i + 2] = v.z;
        r[4 * i + 3] = v.w;
    }
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

// Layout of an integer-path record (and of the lane registers, which hold a
// copy of it): digit words dg[g][p][d][w] (group g < GPL, packing slot p < NPK,
// digit d: 0 = H (signed bytes), 1 = L (unsigned bytes), word w < 8), then NC
// type constants (int32), then sx = 2^(E-14) (fp32 bits).
template <int GPL_, int NPK_, int NC_>
struct IntLayout {
    static constexpr int GPL = GPL_, NPK = NPK_, NC = NC_;
    static constexpr int DG = GPL * NPK * 16;
    static constexpr int CST = DG;
    static constexpr int SX = DG + NC;
    static constexpr int WORDS = (DG + NC + 1 + 3) / 4 * 4;
    static constexpr int STRIDE = rec_stride(DG + NC + 1);
    __host__ __device__ static constexpr int dg(int g, int p, int d, int w)
    {
        return ((g * NPK + p) * 2 + d) * 8 + w;
    }
};

// A group's 32 activations as 16-bit integers at the slot's scale (held
// sign-extended in 32-bit registers: byte 0 is the L digit, byte 1 the H digit).
struct GroupX {
    int X[32];
};

// Slot exponent from the slot's largest |x| (0 for an all-zero slot; bounded
// below so that 2^(E-14) and 2^(14-E) stay normal floats).
__device__ __forceinline__ int slot_exponent(float mx)
{
    int E = mx > 0.f ? static_cast<int>((__float_as_uint(mx) >> 23) & 255u) - 127 : 0;
    return E < -100 ? -100 : E;
}

// X_i = round(x_i * 2^(14-E)), saturated to the int16 range by the conversion.
__device__ __forceinline__ void quantize_group(const float (&v)[32], int E, GroupX &g)
{
    const float up = exp2i(14 - E);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        int q;
        asm("{\n\t.reg .s16 t;\n\tcvt.rni.sat.s16.f32 t, %1;\n\tcvt.s32.s16 %0, t;\n\t}" : "=r"(q) : "f"(v[i] * up));
        g.X[i] = q;
    }
}

// One packing of a group: the H and L digit words.
struct PackedX {
    uint32_t h[8], l[8];
};

// Packs the digits of packing P: word w, byte b holds activation pk_index(P, w, b).
// Four byte permutes give both digit words of four activations.
template <int P>
__device__ __forceinline__ void pack_digits(const GroupX &g, PackedX &pk)
{
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t x0 = static_cast<uint32_t>(g.X[pk_index(P, w, 0)]);
        const uint32_t x1 = static_cast<uint32_t>(g.X[pk_index(P, w, 1)]);
        const uint32_t x2 = static_cast<uint32_t>(g.X[pk_index(P, w, 2)]);
        const uint32_t x3 = static_cast<uint32_t>(g.X[pk_index(P, w, 3)]);
        const uint32_t p01 = __byte_perm(x0, x1, 0x5140u);   // [L0, L1, H0, H1]
        const uint32_t p23 = __byte_perm(x2, x3, 0x5140u);   // [L2, L3, H2, H3]
        pk.l[w] = __byte_perm(p01, p23, 0x5410u);
        pk.h[w] = __byte_perm(p01, p23, 0x7632u);
    }
}

// Writes group j's digit words of one packing into packing slot p of the record
// (each 8-word run is 32-byte aligned: four 128-bit stores).
template <class LAYOUT>
__device__ __forceinline__ void store_packed(const PackedX &pk, int j, int p, uint32_t *rec)
{
    uint4 *h = reinterpret_cast<uint4 *>(rec + LAYOUT::dg(j, p, 0, 0));
    uint4 *l = reinterpret_cast<uint4 *>(rec + LAYOUT::dg(j, p, 1, 0));
    h[0] = make_uint4(pk.h[0], pk.h[1], pk.h[2], pk.h[3]);
    h[1] = make_uint4(pk.h[4], pk.h[5], pk.h[6], pk.h[7]);
    l[0] = make_uint4(pk.l[0], pk.l[1], pk.l[2], pk.l[3]);
    l[1] = make_uint4(pk.l[4], pk.l[5], pk.l[6], pk.l[7]);
}

// Sums of the H and of the L digits over the activations of words [W0, W0 + N).
template <int W0, int N>
__device__ __forceinline__ void psums(const PackedX &pk, int &sh, int &sl)
{
    sh = 0;
    sl = 0;
#pragma unroll
    for (int w = W0; w < W0 + N; ++w) {
        sh = dp_ss(pk.h[w], 0x01010101u, sh);
        sl = dp_uu(pk.l[w], 0x01010101u, sl);
    }
}

// Byte k of the three byte planes (words c[0..2]) of a signed sum |v| < 2^23,
// for dp4a against four packed unsigned byte multipliers: planes 0 and 1 are
// read unsigned, plane 2 signed.
__device__ __forceinline__ void put_planes(int v, int k, uint32_t *c)
{
    uint8_t *b = reinterpret_cast<uint8_t *>(c);
    b[k] = static_cast<uint8_t>(v & 0xFF);
    b[4 + k] = static_cast<uint8_t>((v >> 8) & 0xFF);
    b[8 + k] = static_cast<uint8_t>((v >> 16) & 0xFF);
}

// sum_k m_k * v_k: four unsigned byte multipliers m against the planes of four
// signed sums v.
__device__ __forceinline__ int dot_planes(uint32_t m, uint32_t p0, uint32_t p1, uint32_t p2)
{
    return dp_uu(m, p0, 0) + (dp_uu(m, p1, 0) << 8) + (dp_us(m, p2, 0) << 16);
}

// The same for four signed byte multipliers.
__device__ __forceinline__ int dot_planes_s(uint32_t m, uint32_t p0, uint32_t p1, uint32_t p2)
{
    return dp_su(m, p0, 0) + (dp_su(m, p1, 0) << 8) + (dp_ss(m, p2, 0) << 16);
}

// One field word against digit word w of packing slot pk of group g: the H sum
// into ah, the L sum into al.  mac_u: unsigned byte fields; mac_s: signed.
template <class LAYOUT, int W>
__device__ __forceinline__ void mac_u(int &ah, int &al, uint32_t f, const uint32_t (&r)[W], int g, int pk, int w)
{
    ah = dp_us(f, r[LAYOUT::dg(g, pk, 0, w)], ah);
    al = dp_uu(f, r[LAYOUT::dg(g, pk, 1, w)], al);
}
template <class LAYOUT, int W>
__device__ __forceinline__ void mac_s(int &ah, int &al, uint32_t f, const uint32_t (&r)[W], int g, int pk, int w)
{
    ah = dp_ss(f, r[LAYOUT::dg(g, pk, 0, w)], ah);
    al = dp_su(f, r[LAYOUT::dg(g, pk, 1, w)], al);
}

// 256*H + L as a float (one rounding).
__device__ __forceinline__ float hl_value(int th, int tl)
{
    return fmaf(static_cast<float>(th), 256.f, static_cast<float>(tl));
}

// Common lane type of the integer decoders: a register copy of the record.
template <class LAYOUT>
struct LaneInt {
    uint32_t r[LAYOUT::WORDS];
    __device__ __forceinline__ int cst(int i) const { return static_cast<int>(r[LAYOUT::CST + i]); }
    __device__ __forceinline__ uint32_t cstu(int i) const { return r[LAYOUT::CST + i]; }
    __device__ __forceinline__ float sx() const { return __uint_as_float(r[LAYOUT::SX]); }
};

// Shared part of every integer decoder's prep(): digits of group j for the
// packings P0 (and P1 if >= 0), returned in p0 / p1 for the type's constants,
// and sx from the group that is first in its slot.
template <class LAYOUT, int P0, int P1>
__device__ __forceinline__ void prep_digits(const GroupX &g, int E, bool finite, int j, uint32_t *rec,
                                            PackedX &p0, PackedX &p1)
{
    pack_digits<P0>(g, p0);
    store_packed<LAYOUT>(p0, j, 0, rec);
    if constexpr (P1 >= 0) {
        pack_digits<P1>(g, p1);
        store_packed<LAYOUT>(p1, j, 1, rec);
    }
    if (j == 0) rec[LAYOUT::SX] = finite ? __float_as_uint(exp2i(E - 14)) : 0x7FC00000u;
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

// Byte planes of the per-group (or per-sub-block) x sums used by the mins:
// slot j of 4 gets v; the group that is first in its slot also zeroes the
// bytes no group of the slot writes (slots of fewer than 4 entries).
template <int USED>
__device__ __forceinline__ void put_planes_slot(int v, int k, uint32_t *c)
{
    put_planes(v, k, c);
    if (k == 0)
#pragma unroll
        for (int u = USED; u < 4; ++u) put_planes(0, u, c);
}

// The 8 nibble fields of four ql/qs words (PK_NIB words t and 4+t).
template <class LAYOUT, int W>
__device__ __forceinline__ void nib4(int &ah, int &al, uint4 q, const uint32_t (&r)[W], int g)
{
    mac_u<LAYOUT>(ah, al, q.x & 0x0F0F0F0Fu, r, g, 0, 0);
    mac_u<LAYOUT>(ah, al, (q.x >> 4) & 0x0F0F0F0Fu, r, g, 0, 4);
    mac_u<LAYOUT>(ah, al, q.y & 0x0F0F0F0Fu, r, g, 0, 1);
    mac_u<LAYOUT>(ah, al, (q.y >> 4) & 0x0F0F0F0Fu, r, g, 0, 5);
    mac_u<LAYOUT>(ah, al, q.z & 0x0F0F0F0Fu, r, g, 0, 2);
    mac_u<LAYOUT>(ah, al, (q.z >> 4) & 0x0F0F0F0Fu, r, g, 0, 6);
    mac_u<LAYOUT>(ah, al, q.w & 0x0F0F0F0Fu, r, g, 0, 3);
    mac_u<LAYOUT>(ah, al, (q.w >> 4) & 0x0F0F0F0Fu, r, g, 0, 7);
}

// ---- Q4_K — 144 B: d,dmin @0, scales @4, qs @16 (tb_gguf_dequant.cu:89-118) ----
// w = d*s_g*q - dmin*m_g.  Slot = half a block (4 groups):
// sum = d * sum_g s_g * sum_i q_i X_i - dmin * sum_g m_g * sum_i X_i, all integer.
template <bool A16>
struct DecQ4K {
    using LY = IntLayout<4, 1, 3>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_NIB, -1>(g, E, fin, j, rec, a, b);
        int sh, sl;
        psums<0, 8>(a, sh, sl);
        put_planes_slot<4>(256 * sh + sl, j, rec + LY::CST);
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<A16> W(row + p.off);
        const uint4 h = W.q4(0);
        const uint32_t upper = p.gi0 >> 2;
        const uint32_t sw = sm_half(h.y, h.w, upper, false), mw = sm_half(h.z, h.w, upper, true);
        int th = 0, tl = 0;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint4 q = W.q4(16 + 16 * (p.gi0 + g));
            int ah = 0, al = 0;
            nib4<LY>(ah, al, q, x.r, g);
            const int sc = ubyte(sw, g);
            th = sc * ah + th;
            tl = sc * al + tl;
        }
        const int mn = dot_planes(mw, x.cstu(0), x.cstu(1), x.cstu(2));
        const float2 dd = h2f2_ref(h.x);
        return x.sx() * fmaf(dd.x, hl_value(th, tl), -dd.y * static_cast<float>(mn));
    }
};

// ---- Q5_K — 176 B: d,dmin @0, scales @4, qh @16, qs @48 (tb_gguf_dequant.cu:158-191) ----
// q = nibble | qh_bit<<4, weight i's nibble in qs byte i/2 (low nibble for
// even i) and its high bit at qh byte i/8, bit i%8.  Slot = half a block (4
// groups).  Each group is decoded in the qh bits' order (PK_ONE32: byte b of
// word j = weight 8b + j): a 4x4 byte transpose of the group's four qs words
// (six byte permutes) puts qs byte 4b + k into byte b of word k, so the nibble
// and the high bit of one weight share a byte lane and one dp4a pair covers
// four weights.
template <bool A16>
struct DecQ5K {
    using LY = IntLayout<4, 1, 3>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_ONE32, -1>(g, E, fin, j, rec, a, b);
        int sh, sl;
        psums<0, 8>(a, sh, sl);
        put_planes_slot<4>(256 * sh + sl, j, rec + LY::CST);
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<A16> W(row + p.off);
        const uint4 h = W.q4(0);
        const uint32_t upper = p.gi0 >> 2;
        const uint32_t sw = sm_half(h.y, h.w, upper, false), mw = sm_half(h.z, h.w, upper, true);
        constexpr uint32_t N = 0x0F0F0F0Fu, B = 0x10101010u;
        int th = 0, tl = 0;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint4 q = W.q4(48 + 16 * gi);
            const uint32_t hb = W(4 + gi);
            const uint32_t t0 = __byte_perm(q.x, q.y, 0x5140u), t1 = __byte_perm(q.z, q.w, 0x5140u);
            const uint32_t t2 = __byte_perm(q.x, q.y, 0x7362u), t3 = __byte_perm(q.z, q.w, 0x7362u);
            const uint32_t c0 = __byte_perm(t0, t1, 0x5410u), c1 = __byte_perm(t0, t1, 0x7632u);
            const uint32_t c2 = __byte_perm(t2, t3, 0x5410u), c3 = __byte_perm(t2, t3, 0x7632u);
            int ah = 0, al = 0;
            mac_u<LY>(ah, al, (c0 & N) | ((hb << 4) & B), x.r, g, 0, 0);
            mac_u<LY>(ah, al, ((c0 >> 4) & N) | ((hb << 3) & B), x.r, g, 0, 1);
            mac_u<LY>(ah, al, (c1 & N) | ((hb << 2) & B), x.r, g, 0, 2);
            mac_u<LY>(ah, al, ((c1 >> 4) & N) | ((hb << 1) & B), x.r, g, 0, 3);
            mac_u<LY>(ah, al, (c2 & N) | (hb & B), x.r, g, 0, 4);
            mac_u<LY>(ah, al, ((c2 >> 4) & N) | ((hb >> 1) & B), x.r, g, 0, 5);
            mac_u<LY>(ah, al, (c3 & N) | ((hb >> 2) & B), x.r, g, 0, 6);
            mac_u<LY>(ah, al, ((c3 >> 4) & N) | ((hb >> 3) & B), x.r, g, 0, 7);
            const int sc = ubyte(sw, g);
            th = sc * ah + th;
            tl = sc * al + tl;
        }
        const int mn = dot_planes(mw, x.cstu(0), x.cstu(1), x.cstu(2));
        const float2 dd = h2f2_ref(h.x);
        return x.sx() * fmaf(dd.x, hl_value(th, tl), -dd.y * static_cast<float>(mn));
    }
};

// ---- Q6_K — 210 B: ql @0, qh @128, int8 scales @192, d @208 (tb_gguf_dequant.cu:196-217) ----
// w = d*sc[i>>4]*(q-32), q = ql nibble | (qh 2 bits)<<4, weight i's nibble in
// ql byte i/2 (low nibble for even i) and its 2 bits at qh byte i/4, bit 2(i%4).
// Slot = half a block (4 groups, 8 sub-blocks of 16 weights, two scale words).
// Each sub-block (two ql words A, B and one qh word h) is decoded in the qh
// fields' order (PK_TWO16: byte b of word j = weight 4b + j): two byte permutes
// gather ql bytes 2b (weights 4b, 4b+1) and 2b+1 (4b+2, 4b+3), so every byte
// lane holds the whole 6-bit q of one weight and one dp4a pair covers four
// weights.  The -32 is applied once per slot: -32 * sum_s sc_s * X_s, X_s the
// sub-block's activation sum, by dp4a of the scales against X_s's byte planes.
struct DecQ6K {
    using LY = IntLayout<4, 1, 6>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_TWO16, -1>(g, E, fin, j, rec, a, b);
        int sh, sl;
        uint32_t *c = rec + LY::CST + 3 * (j >> 1);   // planes of the scale word holding sub-blocks 2j, 2j+1
        psums<0, 4>(a, sh, sl);   // PK_TWO16 words 0..3 = activations 0..15
        put_planes(256 * sh + sl, (2 * j) & 3, c);
        psums<4, 4>(a, sh, sl);   // activations 16..31
        put_planes(256 * sh + sl, (2 * j + 1) & 3, c);
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    // One sub-block: ql words A (weights 0..7), B (8..15), qh word h; digit
    // words base..base+3 of group g.
    __device__ static void sub16(int &ah, int &al, uint32_t A, uint32_t B, uint32_t h,
                                 const uint32_t (&r)[LY::WORDS], int g, int base)
    {
        const uint32_t e = __byte_perm(A, B, 0x6420u);   // ql bytes 0,2,4,6: weights 4b (lo), 4b+1 (hi)
        const uint32_t o = __byte_perm(A, B, 0x7531u);   // ql bytes 1,3,5,7: weights 4b+2, 4b+3
        mac_u<LY>(ah, al, (e & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u), r, g, 0, base + 0);
        mac_u<LY>(ah, al, ((e >> 4) & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u), r, g, 0, base + 1);
        mac_u<LY>(ah, al, (o & 0x0F0F0F0Fu) | (h & 0x30303030u), r, g, 0, base + 2);
        mac_u<LY>(ah, al, ((o >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u), r, g, 0, base + 3);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<false> W(row + p.off);
        const float d = h2f2_ref(W(52)).x;
        const uint32_t sc0 = W(48 + (p.gi0 >> 1)), sc1 = W(49 + (p.gi0 >> 1));   // 8 int8 scales
        int th = 0, tl = 0;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint4 l = W.q4(16 * gi);
            const uint32_t h0 = W(32 + 2 * gi), h1 = W(33 + 2 * gi);
            const uint32_t scw = g < 2 ? sc0 : sc1;
            int ah = 0, al = 0;
            sub16(ah, al, l.x, l.y, h0, x.r, g, 0);
            int s = sbyte(scw, 2 * (g & 1));
            th = s * ah + th;
            tl = s * al + tl;
            int bh = 0, bl = 0;
            sub16(bh, bl, l.z, l.w, h1, x.r, g, 4);
            s = sbyte(scw, 2 * (g & 1) + 1);
            th = s * bh + th;
            tl = s * bl + tl;
        }
        const int off = dot_planes_s(sc0, x.cstu(0), x.cstu(1), x.cstu(2)) +
                        dot_planes_s(sc1, x.cstu(3), x.cstu(4), x.cstu(5));
        return x.sx() * d * fmaf(-32.f, static_cast<float>(off), hl_value(th, tl));
    }
};

// ---- Q2_K — 84 B: scales @0 (lo4 scale, hi4 min), qs @16, d @80, dmin @82 ----
// (tb_gguf.c:210-225) w = d*(sc&15)*q - dmin*(sc>>4) per 16-weight sub-block.
// Slot = half a block: 4 groups, 8 sub-blocks, two scale words.
template <bool A4>
struct DecQ2K {
    using LY = IntLayout<4, 1, 6>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_TWO16, -1>(g, E, fin, j, rec, a, b);
        int sh, sl;
        uint32_t *c = rec + LY::CST + 3 * (j >> 1);   // planes of scale word j/2
        psums<0, 4>(a, sh, sl);
        put_planes(256 * sh + sl, 2 * (j & 1), c);
        psums<4, 4>(a, sh, sl);
        put_planes(256 * sh + sl, 2 * (j & 1) + 1, c);
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    __device__ static void two16(int &ah, int &al, uint32_t q, const uint32_t (&r)[LY::WORDS], int g, int base)
    {
        mac_u<LY>(ah, al, q & 0x03030303u, r, g, 0, base + 0);
        mac_u<LY>(ah, al, (q >> 2) & 0x03030303u, r, g, 0, base + 1);
        mac_u<LY>(ah, al, (q >> 4) & 0x03030303u, r, g, 0, base + 2);
        mac_u<LY>(ah, al, (q >> 6) & 0x03030303u, r, g, 0, base + 3);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<A4> W(row + p.off);
        const float2 dd = h2f2_ref(W(20));
        const uint32_t s0 = W(p.gi0 >> 1), s1 = W((p.gi0 >> 1) + 1);
        const uint32_t c0 = s0 & 0x0F0F0F0Fu, c1 = s1 & 0x0F0F0F0Fu;
        int th = 0, tl = 0;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint32_t cw = g < 2 ? c0 : c1;
            int ah = 0, al = 0;
            two16(ah, al, W(4 + 2 * gi), x.r, g, 0);
            int sc = ubyte(cw, 2 * (g & 1));
            th = sc * ah + th;
            tl = sc * al + tl;
            int bh = 0, bl = 0;
            two16(bh, bl, W(5 + 2 * gi), x.r, g, 4);
            sc = ubyte(cw, 2 * (g & 1) + 1);
            th = sc * bh + th;
            tl = sc * bl + tl;
        }
        const int mn = dot_planes((s0 >> 4) & 0x0F0F0F0Fu, x.cstu(0), x.cstu(1), x.cstu(2)) +
                       dot_planes((s1 >> 4) & 0x0F0F0F0Fu, x.cstu(3), x.cstu(4), x.cstu(5));
        return x.sx() * fmaf(dd.x, hl_value(th, tl), -dd.y * static_cast<float>(mn));
    }
};

// ---- Q8_0 — 34 B / 32 weights: d @0, int8 qs @2 (tb_gguf_dequant.cu:246-262) ----
// One fp16 d per group, so the group's sum is scaled in fp32.
struct DecQ80 {
    using LY = IntLayout<4, 1, 0>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_BYTE, -1>(g, E, fin, j, rec, a, b);
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            if (g >= p.ng) break;
            const UnitBytes ub(row + p.off + 34 * g);
            const float d = h2f2_ref(ub.w(0)).x;
            const UnitBytes qb(row + p.off + 34 * g + 2);
            int ah = 0, al = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t) mac_s<LY>(ah, al, qb.w(t), x.r, g, 0, t);
            tot = fmaf(d, hl_value(ah, al), tot);
        }
        return x.sx() * tot;
    }
};

// ---- Q4_0 — 18 B / 32 weights: d @0, qs @2 (tb_gguf_dequant.cu:222-241) ----
// w[2t] = d*(lo-8), w[2t+1] = d*(hi-8); the -8 enters as the initial sums.
struct DecQ40 {
    using LY = IntLayout<4, 1, 8>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_NIB, -1>(g, E, fin, j, rec, a, b);
        int sh, sl;
        psums<0, 8>(a, sh, sl);
        rec[LY::CST + 2 * j] = static_cast<uint32_t>(-8 * sh);
        rec[LY::CST + 2 * j + 1] = static_cast<uint32_t>(-8 * sl);
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            if (g >= p.ng) break;
            const UnitBytes ub(row + p.off + 18 * g);
            const float d = h2f2_ref(ub.w(0)).x;
            const UnitBytes qb(row + p.off + 18 * g + 2);
            int ah = x.cst(2 * g), al = x.cst(2 * g + 1);
            nib4<LY>(ah, al, make_uint4(qb.w(0), qb.w(1), qb.w(2), qb.w(3)), x.r, g);
            tot = fmaf(d, hl_value(ah, al), tot);
        }
        return x.sx() * tot;
    }
};

// ---- Q8_K — 292 B: f32 d @0, int8 qs @4, bsums ignored (tb_gguf_dequant.cu:268-284) ----
struct DecQ8K {
    using LY = IntLayout<4, 1, 0>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_BYTE, -1>(g, E, fin, j, rec, a, b);
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<false> W(row + p.off);
        const float d = __uint_as_float(W(0));
        int th = 0, tl = 0;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const int b = 1 + 8 * static_cast<int>(p.gi0 + g);
#pragma unroll
            for (int t = 0; t < 8; ++t) mac_s<LY>(th, tl, W(b + t), x.r, g, 0, t);
        }
        return x.sx() * d * hl_value(th, tl);
    }
};

// ---- Q3_K — 110 B: hmask @0, qs @32, scales @96, d @108 (tb_gguf_dequant.cu:124-151) ----
// w_i = d * (sc_is - 32) * ((l_i | h_i << 2) - 4), l_i = qs bits 2(i&3) of byte
// i>>2, h_i = hmask bit i&7 of byte i>>3, sub-block j = i>>4 using scale
// is = j & 7 (the two halves of a block share the eight scales), scale bits:
// lo4 = (sc[is>>1] >> 4(is&1)) & 15, hi2 = (sc[8+(is>>2)] >> 2(is&3)) & 3.
// Slot = half a block (4 groups, 8 sub-blocks u = 2g + s), so sub-block u uses
// scale is = u.  The 3-bit value l | h<<2 is assembled per byte: the 16 hmask
// bits of a sub-block are spread to one nibble per byte (bit j of byte b =
// weight 4b + j, the PK_TWO16 order of the qs fields) and merged with one LOP3.
// The -4 enters as -4 * sum_u s_u * (sum of x over u), a dp4a of the signed
// scale bytes against byte planes of the sub-block x sums.  Blocks are 110
// bytes, so every other block is only 2-byte aligned: words are funnel-shifted.
struct DecQ3K {
    using LY = IntLayout<4, 1, 6>;
    static constexpr int GPL = 4;
    static constexpr bool kInt = true;
    static constexpr int REC = LY::STRIDE;
    using Lane = LaneInt<LY>;
    __device__ static void prep(const GroupX &g, int E, bool fin, int j, uint32_t *rec)
    {
        PackedX a, b;
        prep_digits<LY, PK_TWO16, -1>(g, E, fin, j, rec, a, b);
        int sh, sl;
        psums<0, 4>(a, sh, sl);
        put_planes(256 * sh + sl, j, rec + LY::CST);       // sub-block s = 0 of group j
        psums<4, 4>(a, sh, sl);
        put_planes(256 * sh + sl, j, rec + LY::CST + 3);   // s = 1
    }
    __device__ static void load(Lane &L, const uint32_t *rec) { load_rec(L.r, rec); }
    // bits 4b..4b+3 of the 16-bit half selected by `sel` to byte b, bits 0..3
    __device__ static uint32_t spread(uint32_t hm, uint32_t sel)
    {
        const uint32_t t = __byte_perm(hm, 0u, sel);   // [c0, c0, c1, c1]
        return (t & 0x000F000Fu) | ((t >> 4) & 0x0F000F00u);
    }
    // the four 3-bit field words of one sub-block: qs word q, spread high bits h
    __device__ static void sub16(int &ah, int &al, uint32_t q, uint32_t h, const uint32_t (&r)[LY::WORDS],
                                 int g, int base)
    {
        mac_u<LY>(ah, al, (q & 0x03030303u) | ((h << 2) & 0x04040404u), r, g, 0, base + 0);
        mac_u<LY>(ah, al, ((q >> 2) & 0x03030303u) | ((h << 1) & 0x04040404u), r, g, 0, base + 1);
        mac_u<LY>(ah, al, ((q >> 4) & 0x03030303u) | (h & 0x04040404u), r, g, 0, base + 2);
        mac_u<LY>(ah, al, ((q >> 6) & 0x03030303u) | ((h >> 1) & 0x04040404u), r, g, 0, base + 3);
    }
    // the eight 6-bit scales as signed bytes (value - 32): even is in `ev`, odd in `od`
    __device__ static void scales(uint32_t r0, uint32_t r2, uint32_t &ev, uint32_t &od)
    {
        const uint32_t t = __byte_perm(r2, 0u, 0x1100u);   // [sc8, sc8, sc9, sc9]
        const uint32_t he = (t & 0x00030003u) | ((t >> 4) & 0x03000300u);
        const uint32_t ho = ((t >> 2) & 0x00030003u) | ((t >> 6) & 0x03000300u);
        const uint32_t ue = ((r0 & 0x0F0F0F0Fu) | (he << 4)) ^ 0x20202020u;
        const uint32_t uo = (((r0 >> 4) & 0x0F0F0F0Fu) | (ho << 4)) ^ 0x20202020u;
        ev = ue | ((ue & 0x20202020u) * 6u);   // sign-extend bit 5 into bits 6..7
        od = uo | ((uo & 0x20202020u) * 6u);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
    {
        const Words<false> W(row + p.off);
        const float d = h2f2_ref(W(27)).x;
        uint32_t ev, od;
        scales(W(24), W(26), ev, od);
        int th = 0, tl = 0;
#pragma unroll
        for (int g = 0; g < GPL; ++g) {
            const uint32_t gi = p.gi0 + g;
            const uint32_t hm = W(gi);
            int ah = 0, al = 0;
            sub16(ah, al, W(8 + 2 * gi), spread(hm, 0x1100u), x.r, g, 0);
            int s = sbyte(ev, g);
            th = s * ah + th;
            tl = s * al + tl;
            int bh = 0, bl = 0;
            sub16(bh, bl, W(9 + 2 * gi), spread(hm, 0x3322u), x.r, g, 4);
            s = sbyte(od, g);
            th = s * bh + th;
            tl = s * bl + tl;
        }
        const int off = dot_planes_s(ev, x.cstu(0), x.cstu(1), x.cstu(2)) +
                        dot_planes_s(od, x.cstu(3), x.cstu(4), x.cstu(5));
        return x.sx() * d * (hl_value(th, tl) - 4.f * static_cast<float>(off));
    }
};

// ============================================================================
// Float path
// ============================================================================

// Record: the group's 32 activations (zeros past K), padded to REC_F words.
constexpr int REC_F = rec_stride(32);

__device__ __forceinline__ void prep_float(const float (&v)[32], uint32_t *rec)
{
    float4 *p = reinterpret_cast<float4 *>(rec);
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// The lane's 32 activations as 16 register pairs.
struct XRegs {
    float2 a[16];
};

__device__ __forceinline__ void load_f32(XRegs &L, const uint32_t *rec)
{
    const uint32_t a = shared_after(static_cast<uint32_t>(__cvta_generic_to_shared(rec)));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 t = lds_u128(a + 16 * i);
        L.a[2 * i] = f2(__uint_as_float(t.x), __uint_as_float(t.y));
        L.a[2 * i + 1] = f2(__uint_as_float(t.z), __uint_as_float(t.w));
    }
}

// ---- F32 / F16 / BF16 — `n` valid elements in the slot's group ----
// F16 uses the reference converter (tb_gguf_dequant.cu:54-63).
template <int QT>
struct DecFloat {
    static constexpr int GPL = 1;
    static constexpr bool kInt = false;
    static constexpr int REC = REC_F;
    using Lane = XRegs;
    __device__ static void load(Lane &L, const uint32_t *rec) { load_f32(L, rec); }
    __device__ static float elem(const UnitBytes &ub, int i)
    {
        if (QT == QT_F32) return __uint_as_float(ub.w(i));
        const uint32_t w = ub.w(i >> 1);
        const uint32_t h = (i & 1) ? (w >> 16) : (w & 0xFFFFu);
        return QT == QT_F16 ? h2f_ref(h) : __uint_as_float(h << 16);
    }
    __device__ static float row_dot(uint32_t row, const Pos &p, const Lane &x)
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
