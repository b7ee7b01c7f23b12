/*
 * oracle/ref_mt.c — timing harness around the reference's own CPU matvec.
 *
 * TEST / BASELINE INFRASTRUCTURE ONLY.  Linked with the reference sources
 * (layer4/tb_gguf.c, src/tb_analog_dispatch.c, ...) into oracle/_ref/; never
 * part of the shipped library.
 *
 * Splits rows into contiguous ranges over pthreads; each thread calls the
 * reference routine unchanged on its slice:
 *   path 0: tb_gguf_dequant_matvec   (layer4/tb_gguf.c:376-419)
 *   path 1: tb_dispatch_matvec, AVX-512 tier (src/tb_analog_dispatch.c:593;
 *           forged snapshot steps=100, s_u=1.0, aphase=0 -> tb_dispatch_classify
 *           :111-145 picks AVX512 when the caps allow it)
 *   path 2: tb_dispatch_matvec, AVX2 tier (aphase=1)
 */
#define _POSIX_C_SOURCE 200809L
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#include <time.h>

#include "tb_analog_dispatch.h"

void tb_gguf_dequant_matvec(const void *W, int qtype, int M, int K, const float *x, float *out);

typedef struct {
    int path, qtype, M, K;
    size_t row_bytes;
    const uint8_t *W;
    const float *x;
    float *out;
    int r0, r1;
    TBOscSnapshot snap;
    TBCpuCaps caps;
} Job;

static void *run_job(void *p)
{
    Job *j = (Job *)p;
    int m = j->r1 - j->r0;
    if (m <= 0) return NULL;
    const uint8_t *w = j->W + (size_t)j->r0 * j->row_bytes;
    if (j->path == 0)
        tb_gguf_dequant_matvec(w, j->qtype, m, j->K, j->x, j->out + j->r0);
    else
        tb_dispatch_matvec(w, j->qtype, m, j->K, j->x, j->out + j->r0, &j->snap, &j->caps);
    return NULL;
}

/* Runs the chosen reference path `reps` times over all M rows with `nthreads`
 * threads; returns the best wall time of one pass in seconds (or -1). */
double tbr_time_matvec(int path, const void *W, int qtype, int M, int K, size_t row_bytes,
                       const float *x, float *out, int nthreads, int reps, int have_avx512)
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    Job jobs[256];
    pthread_t th[256];
    double best = -1.0;
    for (int r = 0; r < reps; r++) {
        for (int t = 0; t < nthreads; t++) {
            Job *j = &jobs[t];
            memset(j, 0, sizeof(*j));
            j->path = path; j->qtype = qtype; j->M = M; j->K = K; j->row_bytes = row_bytes;
            j->W = (const uint8_t *)W; j->x = x; j->out = out;
            j->r0 = (int)((long long)M * t / nthreads);
            j->r1 = (int)((long long)M * (t + 1) / nthreads);
            j->snap.steps = 100; j->snap.s_u = 1.0; j->snap.phase_var = 0.6;
            j->snap.aphase = path == 1 ? 0 : 1;
            j->caps.have_avx2 = 1; j->caps.have_fma = 1;
            j->caps.have_avx512f = have_avx512; j->caps.have_avx512vnni = have_avx512;
        }
        struct timespec a, b;
        clock_gettime(CLOCK_MONOTONIC, &a);
        for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, run_job, &jobs[t]);
        run_job(&jobs[0]);
        for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
        clock_gettime(CLOCK_MONOTONIC, &b);
        double dt = (double)(b.tv_sec - a.tv_sec) + 1e-9 * (double)(b.tv_nsec - a.tv_nsec);
        if (best < 0 || dt < best) best = dt;
    }
    return best;
}
