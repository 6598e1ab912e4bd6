/*
 * ref_glue.c -- wrapper that turns the reference's OWN code into a callable
 * checker and CPU baseline.  TEST INFRASTRUCTURE ONLY.
 *
 * oracle/Makefile compiles this file together with the reference's quant.c
 * (unmodified, from where it lies) and with rms_norm / sigmoidf / silu_mul /
 * route / argmax / rand_unit / sample_top_p / softmax and the YaRN RoPE
 * functions extracted verbatim from the reference's infer.m into a temporary
 * file (REF_SNIPPET).  Nothing of the reference is written into this repository;
 * the only output is oracle/_ref/libref_moe.so.
 *
 * infer.m itself cannot be compiled on Linux (Objective-C, Metal, Accelerate),
 * so the two Accelerate calls of its CPU expert path are restated here:
 * cblas_sgemv (infer.m:350-353, 1081-1090, 1103-1113) becomes a plain fp32
 * dot and cblas_saxpy (infer.m:1915-1917) a plain fp32 loop.
 */
#include <math.h>
#include <stdio.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include "quant.h"

#define HIDDEN_DIM 7168
#define MOE_INTERMEDIATE 2048
#define SHARED_INTERMEDIATE 2048
#define NUM_EXPERTS 256
#define N_GROUP 8
#define TOPK_GROUP 4
#define ROUTED_SCALE 2.5f
#define RMS_NORM_EPS 1e-6f
#define MAX_K 16
#define QK_ROPE_HEAD_DIM 64
#define ROPE_THETA 10000.0f
#define ROPE_SCALE 40.0f
#define ROPE_ORIG_CTX 4096.0f

#include REF_SNIPPET

float ref_sigmoidf(float x) { return sigmoidf(x); }
void ref_silu_mul(const float *g, const float *u, float *o, int d) { silu_mul(g, u, o, d); }
void ref_rms_norm(const float *x, const float *w, float *o, int d) { rms_norm(x, w, o, d); }
void ref_route(const float *logits, const float *bias, int K, int *exp_idx, float *exp_w) {
    route(logits, bias, K, exp_idx, exp_w);
}
/* argmax / rand_unit / sample_top_p (infer.m:390-456), the generator state
 * handed in and out */
int ref_argmax(const float *x, int n) { return argmax(x, n); }
/* softmax / yarn_freq / apply_rope_q / apply_rope_k (infer.m:384-388, 586-656) */
void ref_softmax(float *x, int n) { softmax(x, n); }
float ref_yarn_freq(int i) { yarn_init_once(); return yarn_freq(i); }
void ref_yarn_band(int *lo, int *hi) { yarn_init_once(); *lo = g_yarn_low; *hi = g_yarn_high; }
void ref_rope_q(float *x, int n_heads, int pos) { apply_rope_q(x, n_heads, pos); }
void ref_rope_k(float *x, int pos) { apply_rope_k(x, pos); }
int ref_sample_top_p(const float *logits, int n, float temp, float top_p, uint32_t *state) {
    g_rng = *state;
    int t = sample_top_p(logits, n, temp, top_p);
    *state = g_rng;
    return t;
}

/* ------------------------------------------------------------------------ */
/* The reference CPU expert path (infer.m:1069-1114, 1881-1922), one token,  */
/* spread over n_threads host threads.  Per expert it dequantizes the whole  */
/* gate/up/down matrices to fp32 with quant.c (as expert_worker does) and    */
/* then runs the dots.                                                        */
/* ------------------------------------------------------------------------ */
/* fp32 dot with 16 independent partial sums, so that -O3 vectorizes it the
 * way a BLAS sgemv would (no -ffast-math needed). */
static float dot_f32(const float *a, const float *b, int n) {
    float p[16] = {0};
    int k = 0;
    for (; k + 16 <= n; k += 16)
        for (int j = 0; j < 16; j++) p[j] += a[k + j] * b[k + j];
    float s = 0.0f;
    for (int j = 0; j < 16; j++) s += p[j];
    for (; k < n; k++) s += a[k] * b[k];
    return s;
}

typedef struct {
    const uint8_t *blob; int down_is_q6; const float *x; float *gate_mat, *up_mat, *down_mat;
    float *g, *u, *a, *eo;
} ref_expert;

typedef struct { ref_expert *ex; int n_ex; int phase; long n_tasks; long rows_per; } ref_phase;
typedef struct { ref_phase *ph; long lo, hi; } ref_job;

#define Q4_ROW (HIDDEN_DIM / QK_K * Q4K_BLOCK_SIZE)
#define GATE_BYTES ((size_t)MOE_INTERMEDIATE * Q4_ROW)

static void ref_task(ref_phase *ph, long t) {
    const int per_ex = (int)(ph->n_tasks / ph->n_ex);
    ref_expert *e = &ph->ex[t / per_ex];
    long blk = t % per_ex;
    if (ph->phase == 0) {           /* gate + up rows */
        long r0 = blk * ph->rows_per, r1 = r0 + ph->rows_per;
        if (r1 > MOE_INTERMEDIATE) r1 = MOE_INTERMEDIATE;
        for (long r = r0; r < r1; r++) {
            float *gw = e->gate_mat + r * HIDDEN_DIM, *uw = e->up_mat + r * HIDDEN_DIM;
            dequantize_row_q4_K(e->blob + r * Q4_ROW, gw, HIDDEN_DIM);
            dequantize_row_q4_K(e->blob + GATE_BYTES + r * Q4_ROW, uw, HIDDEN_DIM);
            e->g[r] = dot_f32(gw, e->x, HIDDEN_DIM);
            e->u[r] = dot_f32(uw, e->x, HIDDEN_DIM);
        }
    } else {                        /* down rows */
        long r0 = blk * ph->rows_per, r1 = r0 + ph->rows_per;
        if (r1 > HIDDEN_DIM) r1 = HIDDEN_DIM;
        const uint8_t *down = e->blob + 2 * GATE_BYTES;
        const size_t drow = (size_t)(MOE_INTERMEDIATE / QK_K) * (e->down_is_q6 ? Q6K_BLOCK_SIZE : Q4K_BLOCK_SIZE);
        for (long r = r0; r < r1; r++) {
            float *dw = e->down_mat + r * MOE_INTERMEDIATE;
            if (e->down_is_q6) dequantize_row_q6_K(down + r * drow, dw, MOE_INTERMEDIATE);
            else dequantize_row_q4_K(down + r * drow, dw, MOE_INTERMEDIATE);
            e->eo[r] = dot_f32(dw, e->a, MOE_INTERMEDIATE);
        }
    }
}

static void *ref_worker(void *p) {
    ref_job *j = (ref_job *)p;
    for (long t = j->lo; t < j->hi; t++) ref_task(j->ph, t);
    return NULL;
}

static void run_phase(ref_phase *ph, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 512) n_threads = 512;
    pthread_t th[512]; ref_job jobs[512]; int ok[512];
    long per = (ph->n_tasks + n_threads - 1) / n_threads;
    for (int i = 0; i < n_threads; i++) {
        jobs[i] = (ref_job){ph, i * per, (i + 1) * per < ph->n_tasks ? (i + 1) * per : ph->n_tasks};
        ok[i] = 0;
        if (jobs[i].lo >= jobs[i].hi) continue;
        if (pthread_create(&th[i], NULL, ref_worker, &jobs[i]) == 0) ok[i] = 1;
        else ref_worker(&jobs[i]);
    }
    for (int i = 0; i < n_threads; i++) if (ok[i]) pthread_join(th[i], NULL);
}

static float *g_scr = NULL;
static int g_scr_k = 0;

/* experts: NUM_EXPERTS + 1 blobs ([gate][up][down]); entry NUM_EXPERTS is the
 * shared expert.  logit_bias (may be NULL) is added to the router logits (the
 * synthetic load skew).  out = (sum_k w_k eo_k, slot order) + shared. */
int ref_moe_token_cpu(const void *const *experts, int down_is_q6, const float *router_w, const float *logit_bias,
                      const float *bias, const float *h_post, int K, float *out, int *idx_out, float *w_out,
                      int n_threads) {
    if (K < 1 || K > MAX_K) return -1;
    const size_t big = (size_t)MOE_INTERMEDIATE * HIDDEN_DIM;
    const size_t per_ex = 3 * big + 3 * MOE_INTERMEDIATE + HIDDEN_DIM;
    if (g_scr_k < K + 1) {
        free(g_scr);
        g_scr = (float *)malloc(sizeof(float) * per_ex * (size_t)(K + 1));
        if (!g_scr) { g_scr_k = 0; return -2; }
        g_scr_k = K + 1;
    }
    float logits[NUM_EXPERTS];
    for (int e = 0; e < NUM_EXPERTS; e++) {
        logits[e] = dot_f32(router_w + (size_t)e * HIDDEN_DIM, h_post, HIDDEN_DIM) + (logit_bias ? logit_bias[e] : 0.0f);
    }
    int idx[MAX_K]; float wts[MAX_K];
    route(logits, bias, K, idx, wts);
    ref_expert ex[MAX_K + 1];
    for (int k = 0; k <= K; k++) {
        float *s = g_scr + per_ex * (size_t)k;
        ex[k] = (ref_expert){(const uint8_t *)experts[k < K ? idx[k] : NUM_EXPERTS], down_is_q6, h_post,
                             s, s + big, s + 2 * big, s + 3 * big, s + 3 * big + MOE_INTERMEDIATE,
                             s + 3 * big + 2 * MOE_INTERMEDIATE, s + 3 * big + 3 * MOE_INTERMEDIATE};
    }
    ref_phase p0 = {ex, K + 1, 0, 0, 64};
    p0.n_tasks = (long)(K + 1) * (MOE_INTERMEDIATE / 64);
    run_phase(&p0, n_threads);
    for (int k = 0; k <= K; k++) silu_mul(ex[k].g, ex[k].u, ex[k].a, MOE_INTERMEDIATE);
    ref_phase p1 = {ex, K + 1, 1, 0, 128};
    p1.n_tasks = (long)(K + 1) * (HIDDEN_DIM / 128);
    run_phase(&p1, n_threads);
    float moe_out[HIDDEN_DIM];
    memset(moe_out, 0, sizeof(moe_out));
    for (int k = 0; k < K; k++)
        for (int i = 0; i < HIDDEN_DIM; i++) moe_out[i] += wts[k] * ex[k].eo[i];
    for (int i = 0; i < HIDDEN_DIM; i++) out[i] = moe_out[i] + ex[K].eo[i];
    if (idx_out) memcpy(idx_out, idx, sizeof(int) * (size_t)K);
    if (w_out) memcpy(w_out, wts, sizeof(float) * (size_t)K);
    return 0;
}
