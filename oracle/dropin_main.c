/*
 * oracle/dropin_main.c — drop-in proof driver (test infrastructure only).
 *
 * Built together with the reference's UNMODIFIED layer4/tb_gguf.c (compiled
 * with -DTB_CUDA, so its GPU branches are live) and linked against
 * libtb_cuda_sm100.so instead of the reference's tb_gguf_dequant.cu.  It then
 * exercises exactly the reference call sites:
 *   tb_cuda_init                         (tb_infer.c:198)
 *   tb_dispatch_context_set -> tb_cuda_set_snap   (tb_gguf.c:428-434)
 *   tb_gguf_cuda_upload_all -> tb_cuda_upload_tensor (tb_gguf.c:469-520)
 *   tb_gguf_tensor_matvec   -> tb_cuda_matvec_device (tb_gguf.c:438-463)
 *   MoE-style row-offset matvec on d_data + byte offset (tb_infer.c:797-827)
 *   tb_cuda_sync_all / tb_cuda_cleanup
 * and checks every GPU result against the oracle (tb_oracle.c) in fp64.
 * Prints one line per tensor and "DROPIN PASS" / "DROPIN FAIL".
 */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tb_gguf.h"
#include "tb_gguf_dequant.h"
#include "tb_oracle.h"

static uint64_t sm_state;
static uint64_t sm_next(void)
{
    uint64_t z = (sm_state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* random fp16 bit pattern with magnitude in [2^-11, 2^-4) (normal), positive */
static uint16_t rand_scale16(void)
{
    uint32_t e = 4 + (uint32_t)(sm_next() % 7);   /* exponent field 4..10 -> 2^-11..2^-5 */
    uint32_t m = (uint32_t)(sm_next() & 0x3FF);
    return (uint16_t)((e << 10) | m);
}

static void fill_blocks(int qtype, uint8_t *p, size_t nblk, int bb)
{
    for (size_t i = 0; i < nblk * (size_t)bb; i++) p[i] = (uint8_t)sm_next();
    for (size_t b = 0; b < nblk; b++) {
        uint8_t *q = p + b * (size_t)bb;
        uint16_t s0 = rand_scale16(), s1 = rand_scale16();
        switch (qtype) {
        case 12: case 13: memcpy(q, &s0, 2); memcpy(q + 2, &s1, 2); break;
        case 14: memcpy(q + 208, &s0, 2); break;
        case 11: case 21: memcpy(q + 108, &s0, 2); break;
        case 10: memcpy(q + 80, &s0, 2); memcpy(q + 82, &s1, 2); break;
        case 8: case 2: memcpy(q, &s0, 2); break;
        case 15: { float d = 0.01f * (float)(1 + (sm_next() % 100)) / 100.f; memcpy(q, &d, 4); } break;
        case 1: for (int k = 0; k < bb; k += 2) { uint16_t h = rand_scale16() | ((sm_next() & 1) << 15); memcpy(q + k, &h, 2); } break;
        default: break;
        }
    }
}

int main(int argc, char **argv)
{
    sm_state = argc > 1 ? strtoull(argv[1], NULL, 0) : 1234;
    const int qtypes[] = {12, 14, 13, 11, 8, 2, 15, 1, 21};
    const int nq = (int)(sizeof(qtypes) / sizeof(qtypes[0]));
    const int M = 96, K = 1024;

    if (!tb_cuda_init()) { printf("tb_cuda_init failed\nDROPIN FAIL\n"); return 1; }
    TBOscSnapshot snap; memset(&snap, 0, sizeof(snap));
    snap.steps = 100; snap.s_u = 0.2; snap.aphase = 3;   /* would shrink the reference grid (B.6) */
    TBCpuCaps caps; memset(&caps, 0, sizeof(caps));
    tb_dispatch_context_set(&snap, &caps);

    /* one synthetic loaded model: nq tensors of M x K, back to back, 32-B aligned */
    TB_GGUFLoaded g; memset(&g, 0, sizeof(g));
    g.n_tensors = nq;
    g.tensors = (TB_GGUFTensorInfo *)calloc((size_t)nq, sizeof(TB_GGUFTensorInfo));
    size_t off = 0, total = 0;
    for (int i = 0; i < nq; i++) {
        total += (tbo_row_bytes(qtypes[i], K) * M + 31) & ~(size_t)31;
    }
    uint8_t *blob = (uint8_t *)aligned_alloc(64, (total + 63) & ~(size_t)63);
    for (int i = 0; i < nq; i++) {
        TB_GGUFTensorInfo *t = &g.tensors[i];
        snprintf(t->name, sizeof(t->name), "blk.0.t%d", i);
        t->n_dims = 2; t->shape[0] = K; t->shape[1] = M; t->qtype = qtypes[i]; t->offset = off;
        int bw, bb; tbo_qtype_geometry(qtypes[i], &bw, &bb);
        size_t nblk = (size_t)M * (size_t)(K / bw);
        fill_blocks(qtypes[i], blob + off, nblk, bb);
        off += (tbo_row_bytes(qtypes[i], K) * M + 31) & ~(size_t)31;
    }
    g.weights_data = blob;

    int up = tb_gguf_cuda_upload_all(&g);
    float *x = (float *)malloc(sizeof(float) * K), *y = (float *)malloc(sizeof(float) * M);
    double *yr = (double *)malloc(sizeof(double) * M);
    for (int k = 0; k < K; k++) x[k] = (float)((double)(sm_next() >> 11) * (1.0 / 9007199254740992.0) * 2.0 - 1.0);

    int fail = 0;
    for (int i = 0; i < nq; i++) {
        TB_GGUFTensorInfo *t = &g.tensors[i];
        if (!t->d_data) { printf("qtype %2d: not uploaded\n", t->qtype); fail = 1; continue; }
        memset(y, 0, sizeof(float) * M);
        tb_gguf_tensor_matvec(&g, t, M, K, x, y);
        tbo_matvec_f64(t->qtype, TBO_SEM_CUDA, blob + t->offset, M, K, x, yr);
        double num = 0, den = 0;
        for (int m = 0; m < M; m++) { double dd = (double)y[m] - yr[m]; num += dd * dd; den += yr[m] * yr[m]; }
        double rel = sqrt(num / (den > 0 ? den : 1));
        printf("qtype %2d: tb_gguf_tensor_matvec rel_l2 %.3e\n", t->qtype, rel);
        if (!(rel <= 1e-3)) fail = 1;
    }

    /* MoE call-site shape: rows [r0, r0+R) of a packed tensor via d_data + byte offset */
    {
        TB_GGUFTensorInfo *t = &g.tensors[0];   /* Q4_K */
        size_t rb = tbo_row_bytes(t->qtype, K);
        int r0 = 37, R = 21;
        const void *wd = (const uint8_t *)t->d_data + (size_t)r0 * rb;
        int ok = tb_cuda_matvec_device(wd, t->qtype, R, K, x, y);
        tbo_matvec_f64(t->qtype, TBO_SEM_CUDA, blob + t->offset + (size_t)r0 * rb, R, K, x, yr);
        double num = 0, den = 0;
        for (int m = 0; m < R; m++) { double dd = (double)y[m] - yr[m]; num += dd * dd; den += yr[m] * yr[m]; }
        double rel = sqrt(num / (den > 0 ? den : 1));
        printf("expert-slice rows %d..%d: ok=%d rel_l2 %.3e\n", r0, r0 + R, ok, rel);
        if (!ok || !(rel <= 1e-3)) fail = 1;
    }
    /* device-resident x: upload once, matvec with x_host == NULL */
    {
        TB_GGUFTensorInfo *t = &g.tensors[1];   /* Q6_K */
        int ok = tb_cuda_upload_x(x, K) && tb_cuda_matvec_device(t->d_data, t->qtype, M, K, NULL, y);
        tbo_matvec_f64(t->qtype, TBO_SEM_CUDA, blob + t->offset, M, K, x, yr);
        double num = 0, den = 0;
        for (int m = 0; m < M; m++) { double dd = (double)y[m] - yr[m]; num += dd * dd; den += yr[m] * yr[m]; }
        double rel = sqrt(num / (den > 0 ? den : 1));
        printf("upload_x + matvec(x_host=NULL): ok=%d rel_l2 %.3e\n", ok, rel);
        if (!ok || !(rel <= 1e-3)) fail = 1;
    }
    tb_cuda_sync_all();
    for (int i = 0; i < nq; i++) tb_cuda_free_tensor(g.tensors[i].d_data);
    tb_cuda_cleanup();
    tb_cuda_cleanup();
    printf("uploaded %d of %d tensors\n", up, nq);
    printf(fail || up != nq ? "DROPIN FAIL\n" : "DROPIN PASS\n");
    free(blob); free(g.tensors); free(x); free(y); free(yr);
    return fail || up != nq ? 1 : 0;
}
