/*
 * oracle/tb_oracle.c — CPU restatement of Trailblaze's GGUF dequant semantics.
 *
 * TEST INFRASTRUCTURE ONLY (see tb_oracle.h).  Build with ISO C and
 * -ffp-contract=off so every multiply and add rounds separately, exactly as
 * the reference's `-std=c11` build does.
 *
 * Every decoder below restates one reference routine; each product is fp32 and
 * evaluated in the order the reference writes it.  Byte offsets and field
 * widths are the reference's own (its nibble order is interleaved: qs byte t
 * holds weight 2t in the low nibble and 2t+1 in the high nibble).
 */
#include "tb_oracle.h"

#include <stdlib.h>
#include <string.h>

/* ── converters ────────────────────────────────────────────────────────────
 * tb_gguf.c:92-101 and tb_gguf_dequant.cu:54-63: exponent 0 maps to
 * sign | mantissa<<13 (a float denormal m*2^-136, not m*2^-24); exponent 31
 * maps to inf/nan; otherwise the exponent is rebased by 112.               */
float tbo_h2f(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t expo = (uint32_t)(h & 0x7C00u) >> 10;
    uint32_t mant = (uint32_t)(h & 0x03FFu);
    uint32_t bits;
    if (expo == 0u)
        bits = sign | (mant << 13);
    else if (expo == 31u)
        bits = sign | 0x7F800000u | (mant << 13);
    else
        bits = sign | ((expo + 112u) << 23) | (mant << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* tb_gguf.c:104-107, tb_gguf_dequant.cu:65-68 */
float tbo_bf2f(uint16_t b)
{
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* fp16 field, or bf16 for the dispatch-tier variant (tb_analog_dispatch.c:228). */
static float scale16(const uint8_t *p, int sem)
{
    return sem == TBO_SEM_DISPATCH ? tbo_bf2f(rd16(p)) : tbo_h2f(rd16(p));
}

/* ── geometry (tb_gguf.c:380-393, tb_gguf_dequant.cu:37-47) ─────────────── */
int tbo_qtype_geometry(int qtype, int *bw, int *bb)
{
    int w, b;
    switch (qtype) {
    case TBO_F32:   w = 1;   b = 4;   break;
    case TBO_F16:   w = 1;   b = 2;   break;
    case TBO_BF16:  w = 1;   b = 2;   break;
    case TBO_Q4_0:  w = 32;  b = 18;  break;
    case TBO_Q8_0:  w = 32;  b = 34;  break;
    case TBO_Q2_K:  w = 256; b = 84;  break;
    case TBO_Q3_K:  w = 256; b = 110; break;
    case TBO_IQ3_S: w = 256; b = 110; break;   /* aliased to Q3_K (tb_gguf.c:389) */
    case TBO_Q4_K:  w = 256; b = 144; break;
    case TBO_Q5_K:  w = 256; b = 176; break;
    case TBO_Q6_K:  w = 256; b = 210; break;
    case TBO_Q8_K:  w = 256; b = 292; break;
    default: return 0;
    }
    if (bw) *bw = w;
    if (bb) *bb = b;
    return 1;
}

size_t tbo_row_bytes(int qtype, int K)
{
    int bw, bb;
    if (!tbo_qtype_geometry(qtype, &bw, &bb) || K <= 0 || K % bw) return 0;
    return (size_t)(K / bw) * (size_t)bb;
}

/* ── Q4_K / Q5_K 6-bit scale+min unpack ─────────────────────────────────────
 * CUDA (tb_gguf_dequant.cu:103-108 and :175-180), also tb_analog_dispatch.c
 * q4k_unpack_scales :204-220: for j<4 s=sc[j]&63, m=sc[j+4]&63;
 * s[j+4]=(sc[j]>>6)|((sc[j+8]&15)<<2), m[j+4]=(sc[j+4]>>6)|((sc[j+8]>>4)<<2).
 * `tail` is the 4 bytes that follow the 12 scale bytes in the block; only the
 * shipped tb_gguf.c variants read them.                                      */
static void unpack_sm_cuda(const uint8_t *sc, int s[8], int m[8])
{
    for (int j = 0; j < 4; j++) {
        s[j]     = sc[j] & 63;
        m[j]     = sc[j + 4] & 63;
        s[j + 4] = (sc[j] >> 6) | ((sc[j + 8] & 15) << 2);
        m[j + 4] = (sc[j + 4] >> 6) | ((sc[j + 8] >> 4) << 2);
    }
}

/* tb_gguf.c:163-168 (dequant_q4_k_block): s[j]=(j<4?sc[j]:sc[j+4])&63,
 * m[j]=(j<4?sc[j+4]:sc[j+8])&63; sc[12..15] are the first qs bytes.        */
static void unpack_sm_q4k_gguf_c(const uint8_t *sc, int s[8], int m[8])
{
    for (int j = 0; j < 8; j++) {
        s[j] = sc[j < 4 ? j : j + 4] & 63;
        m[j] = sc[j < 4 ? j + 4 : j + 8] & 63;
    }
}

/* tb_gguf.c:130-144 (q4_k_unpack_scales, used by Q5_K): as CUDA except
 * m[j>=4]=(sc[k+4]>>6)|((sc[k+12]&15)<<2), k=j-4, reading past the 12 bytes. */
static void unpack_sm_q5k_gguf_c(const uint8_t *sc, int s[8], int m[8])
{
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            s[j] = sc[j] & 63;
            m[j] = sc[j + 4] & 63;
        } else {
            int k = j - 4;
            s[j] = (sc[k] >> 6) | ((sc[k + 8] & 15) << 2);
            m[j] = (sc[k + 4] >> 6) | ((sc[k + 12] & 15) << 2);
        }
    }
}

/* ── per-type block decoders ───────────────────────────────────────────── */

/* Q4_K, 144 B: d,dmin @0/2, scales @4, qs @16 (tb_gguf_dequant.cu:98-116).
 * w = S[g]*q - Mn[g], S=d*s, Mn=dmin*m, g = weight>>5.                       */
static void dq_q4k(const uint8_t *b, int sem, float *out)
{
    float d = scale16(b, sem), dmin = scale16(b + 2, sem);
    int s[8], m[8];
    if (sem == TBO_SEM_GGUF_C) unpack_sm_q4k_gguf_c(b + 4, s, m);
    else                       unpack_sm_cuda(b + 4, s, m);
    float S[8], Mn[8];
    for (int j = 0; j < 8; j++) { S[j] = d * (float)s[j]; Mn[j] = dmin * (float)m[j]; }
    const uint8_t *qs = b + 16;
    for (int t = 0; t < 128; t++) {
        int g0 = (2 * t) >> 5, g1 = (2 * t + 1) >> 5;
        out[2 * t]     = S[g0] * (float)(qs[t] & 15) - Mn[g0];
        out[2 * t + 1] = S[g1] * (float)(qs[t] >> 4) - Mn[g1];
    }
}

/* Q5_K, 176 B: d,dmin @0/2, scales @4, qh @16, qs @48 (tb_gguf_dequant.cu:158-191,
 * tb_gguf.c:262-279).  q = nibble | qh_bit<<4; w = S[g]*q - Mn[g].           */
static void dq_q5k(const uint8_t *b, int sem, float *out)
{
    float d = scale16(b, sem), dmin = scale16(b + 2, sem);
    int s[8], m[8];
    if (sem == TBO_SEM_GGUF_C) unpack_sm_q5k_gguf_c(b + 4, s, m);
    else                       unpack_sm_cuda(b + 4, s, m);
    float S[8], Mn[8];
    for (int j = 0; j < 8; j++) { S[j] = d * (float)s[j]; Mn[j] = dmin * (float)m[j]; }
    const uint8_t *qh = b + 16, *qs = b + 48;
    for (int i = 0; i < 256; i++) {
        int lo = (qs[i >> 1] >> ((i & 1) << 2)) & 15;
        int hi = (qh[i >> 3] >> (i & 7)) & 1;
        out[i] = S[i >> 5] * (float)(lo | (hi << 4)) - Mn[i >> 5];
    }
}

/* Q6_K, 210 B: ql @0, qh @128, int8 scales @192, d @208
 * (tb_gguf_dequant.cu:196-217 = tb_gguf.c:190-204): w = d*sc[i>>4]*(q-32).   */
static void dq_q6k(const uint8_t *b, float *out)
{
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = tbo_h2f(rd16(b + 208));
    for (int i = 0; i < 256; i++) {
        int lo = (ql[i >> 1] >> ((i & 1) << 2)) & 15;
        int hi = (qh[i >> 2] >> ((i & 3) << 1)) & 3;
        out[i] = d * (float)sc[i >> 4] * (float)((lo | (hi << 4)) - 32);
    }
}

/* Q3_K, 110 B: hmask @0, qs @32, scales @96, d @108 (tb_gguf_dequant.cu:124-151
 * = tb_gguf.c:230-257).  Sub-scale j uses is=(j<8?j:j-8), so S[8..15]
 * repeat S[0..7]; q = low2 | hbit<<2; w = S[i>>4]*(q-4).                     */
static void dq_q3k(const uint8_t *b, int sem, float *out)
{
    const uint8_t *hm = b, *qs = b + 32, *sr = b + 96;
    float d = scale16(b + 108, sem);
    float S[16];
    for (int j = 0; j < 16; j++) {
        int is = j < 8 ? j : j - 8;
        int lo4 = (sr[is >> 1] >> ((is & 1) << 2)) & 15;
        int hi2 = (sr[8 + (is >> 2)] >> ((is & 3) << 1)) & 3;
        S[j] = d * (float)((lo4 | (hi2 << 4)) - 32);
    }
    for (int i = 0; i < 256; i++) {
        int l = (qs[i >> 2] >> ((i & 3) << 1)) & 3;
        int h = (hm[i >> 3] >> (i & 7)) & 1;
        out[i] = S[i >> 4] * (float)((l | (h << 2)) - 4);
    }
}

/* Q2_K, 84 B: scales @0 (lo4 scale, hi4 min), qs @16, d @80, dmin @82
 * (tb_gguf.c:210-225; no CUDA kernel exists).  w = sc*q - mn per 16 weights. */
static void dq_q2k(const uint8_t *b, float *out)
{
    const uint8_t *scales = b, *qs = b + 16;
    float d = tbo_h2f(rd16(b + 80)), dmin = tbo_h2f(rd16(b + 82));
    for (int g = 0; g < 16; g++) {
        float sc = d * (float)(scales[g] & 15);
        float mn = dmin * (float)(scales[g] >> 4);
        for (int i = 0; i < 16; i++) {
            int wi = g * 16 + i;
            int q = (qs[wi >> 2] >> ((wi & 3) << 1)) & 3;
            out[wi] = sc * (float)q - mn;
        }
    }
}

/* Q8_0, 34 B: d @0, int8 qs @2 (tb_gguf_dequant.cu:246-262, tb_gguf.c:183-187). */
static void dq_q80(const uint8_t *b, float *out)
{
    float d = tbo_h2f(rd16(b));
    for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)b[2 + i];
}

/* Q4_0, 18 B: d @0, qs @2; w[2t]=d*(lo-8), w[2t+1]=d*(hi-8)
 * (tb_gguf_dequant.cu:222-241, tb_gguf.c:110-118).                            */
static void dq_q40(const uint8_t *b, float *out)
{
    float d = tbo_h2f(rd16(b));
    for (int t = 0; t < 16; t++) {
        out[2 * t]     = d * (float)((int)(b[2 + t] & 15) - 8);
        out[2 * t + 1] = d * (float)((int)(b[2 + t] >> 4) - 8);
    }
}

/* Q8_K, 292 B: f32 d @0, int8 qs @4, bsums ignored (tb_gguf_dequant.cu:268-284,
 * tb_gguf.c:283-288).                                                          */
static void dq_q8k(const uint8_t *b, float *out)
{
    float d;
    memcpy(&d, b, 4);
    for (int i = 0; i < 256; i++) out[i] = d * (float)(int8_t)b[4 + i];
}

int tbo_dequant_block(int qtype, int sem, const uint8_t *b, float *out)
{
    switch (qtype) {
    case TBO_F32:  memcpy(out, b, 4); return 1;
    case TBO_F16:  out[0] = tbo_h2f(rd16(b)); return 1;
    case TBO_BF16: out[0] = tbo_bf2f(rd16(b)); return 1;
    case TBO_Q4_0: dq_q40(b, out); return 1;
    case TBO_Q8_0: dq_q80(b, out); return 1;
    case TBO_Q2_K: dq_q2k(b, out); return 1;
    case TBO_Q3_K:
    case TBO_IQ3_S: dq_q3k(b, sem, out); return 1;
    case TBO_Q4_K: dq_q4k(b, sem, out); return 1;
    case TBO_Q5_K: dq_q5k(b, sem, out); return 1;
    case TBO_Q6_K: dq_q6k(b, out); return 1;
    case TBO_Q8_K: dq_q8k(b, out); return 1;
    default: return 0;
    }
}

int tbo_dequant_rows(int qtype, int sem, const void *W, int M, int K, float *out)
{
    int bw, bb;
    if (!tbo_qtype_geometry(qtype, &bw, &bb) || M < 0 || K <= 0 || K % bw) return 0;
    const uint8_t *p = (const uint8_t *)W;
    size_t nblk = (size_t)M * (size_t)(K / bw);
    for (size_t i = 0; i < nblk; i++)
        tbo_dequant_block(qtype, sem, p + i * (size_t)bb, out + i * (size_t)bw);
    return 1;
}

int tbo_matvec_f64(int qtype, int sem, const void *W, int M, int K,
                   const float *x, double *y)
{
    size_t rb = tbo_row_bytes(qtype, K);
    if (!rb) return 0;
    float *row = (float *)malloc((size_t)K * sizeof(float));
    if (!row) return 0;
    const uint8_t *p = (const uint8_t *)W;
    for (int m = 0; m < M; m++) {
        tbo_dequant_rows(qtype, sem, p + (size_t)m * rb, 1, K, row);
        double acc = 0.0;
        for (int k = 0; k < K; k++) acc += (double)row[k] * (double)x[k];
        y[m] = acc;
    }
    free(row);
    return 1;
}

int tbo_matvec_f32_seq(int qtype, int sem, const void *W, int M, int K,
                       const float *x, float *y)
{
    size_t rb = tbo_row_bytes(qtype, K);
    if (!rb) return 0;
    float *row = (float *)malloc((size_t)K * sizeof(float));
    if (!row) return 0;
    const uint8_t *p = (const uint8_t *)W;
    for (int m = 0; m < M; m++) {
        tbo_dequant_rows(qtype, sem, p + (size_t)m * rb, 1, K, row);
        float acc = 0.0f;
        for (int k = 0; k < K; k++) {
            float prod = row[k] * x[k];
            acc = acc + prod;
        }
        y[m] = acc;
    }
    free(row);
    return 1;
}
