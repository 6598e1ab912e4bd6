/*
 * moe_oracle.c -- CPU restatement of the reference MoE block.  TEST
 * INFRASTRUCTURE ONLY: the checker, never the thing measured or shipped.
 * Built with -ffp-contract=off so that the generator and the quantizer give
 * the same bits as the CUDA library's device versions (which use explicit
 * _rn intrinsics).  Each function cites the reference lines it follows.
 */
#include "oracle.h"
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* tiny parallel-for                                                          */
/* ------------------------------------------------------------------------ */
typedef void (*pf_fn)(void *ctx, long lo, long hi);
typedef struct { pf_fn fn; void *ctx; long lo, hi; } pf_job;
static void *pf_thread(void *a) { pf_job *j = (pf_job *)a; j->fn(j->ctx, j->lo, j->hi); return NULL; }
static void parallel_for(long n, int n_threads, pf_fn fn, void *ctx) {
    if (n_threads <= 1 || n < 2) { fn(ctx, 0, n); return; }
    if (n_threads > 256) n_threads = 256;
    if (n_threads > n) n_threads = (int)n;
    pthread_t th[256]; pf_job jobs[256]; int started[256];
    long per = (n + n_threads - 1) / n_threads;
    for (int t = 0; t < n_threads; t++) {
        long lo = t * per, hi = lo + per < n ? lo + per : n;
        started[t] = 0;
        if (lo >= hi) continue;
        jobs[t] = (pf_job){fn, ctx, lo, hi};
        if (pthread_create(&th[t], NULL, pf_thread, &jobs[t]) == 0) started[t] = 1;
        else fn(ctx, lo, hi);
    }
    for (int t = 0; t < n_threads; t++)
        if (started[t]) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* fp16 (quant.c:4-24)                                                        */
/* ------------------------------------------------------------------------ */
static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE half -> float, subnormals normalised, inf/NaN payload kept
 * (follows quant.c:4-24). */
float or_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return bits_f(sign);
        int sh = 0;
        while ((m & 0x400u) == 0) { m <<= 1; sh++; }
        m &= 0x3FFu;
        return bits_f(sign | ((uint32_t)(113 - sh) << 23) | (m << 13));
    }
    if (e == 31) return bits_f(sign | 0x7F800000u | (m << 13));
    return bits_f(sign | ((e + 112) << 23) | (m << 13));
}

/* float -> half, round to nearest even, overflow to inf (quantizer only). */
uint16_t or_fp32_to_fp16(float f) {
    uint32_t x = f_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (ax >= 0x38800000u) {
        uint32_t mant = ax & 0x7FFFFFu;
        uint32_t h = ((((ax >> 23) - 112u)) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    int e = (int)(ax >> 23);
    int shift = 126 - e;
    if (shift > 24) return (uint16_t)sign;
    uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t hm = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) hm++;
    return (uint16_t)(sign | hm);
}

/* ------------------------------------------------------------------------ */
/* dequant (quant.c:26-92)                                                    */
/* ------------------------------------------------------------------------ */
/* 6-bit scale/min unpack (quant.c:26-34): slots 0-3 live in the low 6 bits
 * of bytes 0-3 / 4-7; slots 4-7 are split between the nibbles of bytes 8-11
 * and the top two bits of bytes 0-7. */
static inline void scale_min_k4(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) { *sc = q[j] & 63; *mn = q[j + 4] & 63; }
    else {
        *sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* Q4_K (quant.c:36-61): 144-byte super-block = d f16, dmin f16, 12 scale
 * bytes, 128 nibble bytes; chunk c (64 weights) uses 32 bytes: low nibbles
 * are weights 64c+l with slot 2c, high nibbles weights 64c+32+l, slot 2c+1.
 * w = d*sc*q - dmin*m. */
void or_dequant_q4k(const void *src, float *y, size_t n) {
    const uint8_t *p = (const uint8_t *)src;
    for (size_t b = 0; b < n / OR_QK; b++, p += OR_Q4K_BYTES) {
        uint16_t dh, mh;
        memcpy(&dh, p, 2); memcpy(&mh, p + 2, 2);
        const float d = or_fp16_to_fp32(dh), dmin = or_fp16_to_fp32(mh);
        const uint8_t *sc = p + 4, *qs = p + 16;
        for (int c = 0; c < 4; c++) {
            int s0, m0, s1, m1;
            scale_min_k4(2 * c, sc, &s0, &m0);
            scale_min_k4(2 * c + 1, sc, &s1, &m1);
            const float d1 = d * (float)s0, n1 = dmin * (float)m0;
            const float d2 = d * (float)s1, n2 = dmin * (float)m1;
            for (int l = 0; l < 32; l++) y[64 * c + l] = d1 * (float)(qs[32 * c + l] & 0x0F) - n1;
            for (int l = 0; l < 32; l++) y[64 * c + 32 + l] = d2 * (float)(qs[32 * c + l] >> 4) - n2;
        }
        y += OR_QK;
    }
}

/* Q6_K (quant.c:63-92): 210-byte super-block = ql[128], qh[64], int8 sc[16],
 * d f16.  Half h (128 weights) uses ql[64h..], qh[32h..], sc[8h..]; for l<32
 * the four 6-bit values of weights 128h+l+{0,32,64,96} take the low/high
 * nibbles of ql[l], ql[l+32] and the bit pairs 0/2/4/6 of qh[l];
 * w = d * sc[16-weight slot] * (q - 32). */
void or_dequant_q6k(const void *src, float *y, size_t n) {
    const uint8_t *p = (const uint8_t *)src;
    for (size_t b = 0; b < n / OR_QK; b++, p += OR_Q6K_BYTES) {
        uint16_t dh; memcpy(&dh, p + 208, 2);
        const float d = or_fp16_to_fp32(dh);
        for (int h = 0; h < 2; h++) {
            const uint8_t *ql = p + 64 * h, *qh = p + 128 + 32 * h;
            const int8_t *sc = (const int8_t *)(p + 192 + 8 * h);
            float *yy = y + 128 * h;
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                yy[l] = d * (float)sc[is + 0] * (float)q1;
                yy[l + 32] = d * (float)sc[is + 2] * (float)q2;
                yy[l + 64] = d * (float)sc[is + 4] * (float)q3;
                yy[l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
        }
        y += OR_QK;
    }
}

size_t or_row_bytes(int type, size_t n_cols) {
    return (n_cols / OR_QK) * (type == OR_TYPE_Q6_K ? OR_Q6K_BYTES : OR_Q4K_BYTES);
}

/* ------------------------------------------------------------------------ */
/* quantizer (new).  Plain min/max fitting; every float op is a single IEEE  */
/* op so the CUDA library reproduces the bytes exactly.                      */
/* ------------------------------------------------------------------------ */
static inline int rnd_i(float v) {
    if (v > 1.0e6f) v = 1.0e6f;
    if (v < -1.0e6f) v = -1.0e6f;
    return v >= 0.0f ? (int)(v + 0.5f) : -(int)(-v + 0.5f);
}
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void or_quantize_q4k(const float *x, void *dst, size_t n) {
    uint8_t *p = (uint8_t *)dst;
    for (size_t b = 0; b < n / OR_QK; b++, x += OR_QK, p += OR_Q4K_BYTES) {
        float scale[8], minv[8], max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; j++) {
            float mn = x[32 * j], mx = x[32 * j];
            for (int i = 1; i < 32; i++) {
                float v = x[32 * j + i];
                if (v < mn) mn = v;
                if (v > mx) mx = v;
            }
            if (mn > 0.0f) mn = 0.0f;
            scale[j] = (mx - mn) / 15.0f;
            minv[j] = -mn;
            if (scale[j] > max_scale) max_scale = scale[j];
            if (minv[j] > max_min) max_min = minv[j];
        }
        uint16_t dh = or_fp32_to_fp16(max_scale / 63.0f), mh = or_fp32_to_fp16(max_min / 63.0f);
        float d = or_fp16_to_fp32(dh), dmin = or_fp16_to_fp32(mh);
        int sc[8], mm[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = d > 0.0f ? clampi(rnd_i(scale[j] / d), 0, 63) : 0;
            mm[j] = dmin > 0.0f ? clampi(rnd_i(minv[j] / dmin), 0, 63) : 0;
        }
        memcpy(p, &dh, 2); memcpy(p + 2, &mh, 2);
        uint8_t *s = p + 4;
        for (int j = 0; j < 4; j++) {
            s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            s[j + 4] = (uint8_t)((mm[j] & 63) | ((mm[j + 4] >> 4) << 6));
            s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mm[j + 4] & 0xF) << 4));
        }
        uint8_t q[256];
        for (int j = 0; j < 8; j++) {
            float ds = d * (float)sc[j], dm = dmin * (float)mm[j];
            for (int i = 0; i < 32; i++)
                q[32 * j + i] = (uint8_t)(ds > 0.0f ? clampi(rnd_i((x[32 * j + i] + dm) / ds), 0, 15) : 0);
        }
        uint8_t *qs = p + 16;
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++)
                qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
    }
}

void or_quantize_q6k(const float *x, void *dst, size_t n) {
    uint8_t *p = (uint8_t *)dst;
    for (size_t b = 0; b < n / OR_QK; b++, x += OR_QK, p += OR_Q6K_BYTES) {
        float scale[16], max_scale = 0.0f;
        for (int j = 0; j < 16; j++) {
            float am = 0.0f;
            for (int i = 0; i < 16; i++) {
                float v = x[16 * j + i];
                float a = v < 0.0f ? -v : v;
                if (a > am) am = a;
            }
            scale[j] = am / 31.0f;
            if (scale[j] > max_scale) max_scale = scale[j];
        }
        uint16_t dh = or_fp32_to_fp16(max_scale / 127.0f);
        float d = or_fp16_to_fp32(dh);
        int sc[16];
        uint8_t q6[256];
        for (int j = 0; j < 16; j++) {
            sc[j] = d > 0.0f ? clampi(rnd_i(scale[j] / d), 0, 127) : 0;
            float ds = d * (float)sc[j];
            for (int i = 0; i < 16; i++)
                q6[16 * j + i] = (uint8_t)((ds > 0.0f ? clampi(rnd_i(x[16 * j + i] / ds), -32, 31) : 0) + 32);
        }
        for (int h = 0; h < 2; h++) {
            uint8_t *ql = p + 64 * h, *qh = p + 128 + 32 * h;
            const uint8_t *qq = q6 + 128 * h;
            for (int l = 0; l < 32; l++) {
                int q1 = qq[l], q2 = qq[l + 32], q3 = qq[l + 64], q4 = qq[l + 96];
                ql[l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
                ql[l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
                qh[l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
            }
        }
        for (int j = 0; j < 16; j++) p[192 + j] = (uint8_t)(int8_t)sc[j];
        memcpy(p + 208, &dh, 2);
    }
}

/* ------------------------------------------------------------------------ */
/* counter-based generator (new): splitmix64 (Steele et al. 2014) keyed by   */
/* (seed, stream, element), Marsaglia polar method with a deterministic log. */
/* ------------------------------------------------------------------------ */
uint64_t or_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* stream id of a synthetic tensor: layer, expert (n_experts = shared), kind
 * (0 gate, 1 up, 2 down, 3 router, 4 bias, 5 norm weight, 6 activations). */
uint64_t or_stream(int layer, int expert, int kind) {
    return ((uint64_t)(uint32_t)layer << 32) | ((uint64_t)(uint32_t)expert << 8) | (uint64_t)(uint32_t)kind;
}

/* ln(s) for s in (0, 1] with IEEE +,-,*,/ only: s = m 2^e, m in [sqrt(1/2),
 * sqrt(2)], ln m = 2 atanh(t), t = (m-1)/(m+1), 13-term odd series. */
double or_det_log(double s) {
    uint64_t b; memcpy(&b, &s, 8);
    int e = (int)((b >> 52) & 0x7FF) - 1023;
    uint64_t mb = (b & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull;
    double m; memcpy(&m, &mb, 8);
    if (m > 1.4142135623730951) { m = m * 0.5; e += 1; }
    double t = (m - 1.0) / (m + 1.0);
    double t2 = t * t;
    double acc = 1.0 / 25.0;
    for (int k = 11; k >= 0; k--) acc = acc * t2 + 1.0 / (double)(2 * k + 1);
    return (double)e * 0.6931471805599453 + 2.0 * t * acc;
}

double or_normal(uint64_t seed, uint64_t stream, uint64_t index) {
    uint64_t key = or_splitmix64(seed ^ or_splitmix64(stream + 0x632BE59BD9B4E019ull));
    for (uint64_t a = 0; a < 64; a++) {
        uint64_t r = or_splitmix64(key + (index << 6) + a);
        double u = (double)(int32_t)(uint32_t)(r >> 32) * (1.0 / 2147483648.0);
        double v = (double)(int32_t)(uint32_t)(r & 0xFFFFFFFFu) * (1.0 / 2147483648.0);
        double s = u * u + v * v;
        if (s < 1.0 && s > 0.0) return u * sqrt(-2.0 * or_det_log(s) / s);
    }
    return 0.0;
}

typedef struct { uint64_t seed, stream, first; double sigma; float *dst; } fill_ctx;
static void fill_part(void *c, long lo, long hi) {
    fill_ctx *f = (fill_ctx *)c;
    for (long i = lo; i < hi; i++) f->dst[i] = (float)(or_normal(f->seed, f->stream, f->first + (uint64_t)i) * f->sigma);
}
void or_fill_normal(uint64_t seed, uint64_t stream, uint64_t first, size_t n, double sigma,
                    float *dst, int n_threads) {
    fill_ctx c = {seed, stream, first, sigma, dst};
    parallel_for((long)n, n_threads, fill_part, &c);
}

typedef struct { uint64_t seed, stream; int type, cols; double sigma; uint8_t *dst; size_t rb; } gen_ctx;
static void gen_rows(void *c, long lo, long hi) {
    gen_ctx *g = (gen_ctx *)c;
    float *row = (float *)malloc(sizeof(float) * (size_t)g->cols);
    for (long r = lo; r < hi; r++) {
        for (int k = 0; k < g->cols; k++)
            row[k] = (float)(or_normal(g->seed, g->stream, (uint64_t)r * (uint64_t)g->cols + (uint64_t)k) * g->sigma);
        if (g->type == OR_TYPE_Q6_K) or_quantize_q6k(row, g->dst + (size_t)r * g->rb, (size_t)g->cols);
        else or_quantize_q4k(row, g->dst + (size_t)r * g->rb, (size_t)g->cols);
    }
    free(row);
}
void or_gen_matrix(uint64_t seed, uint64_t stream, int type, int rows, int cols, double sigma,
                   void *dst, int n_threads) {
    gen_ctx c = {seed, stream, type, cols, sigma, (uint8_t *)dst, or_row_bytes(type, (size_t)cols)};
    parallel_for(rows, n_threads, gen_rows, &c);
}

/* ------------------------------------------------------------------------ */
/* routing pieces                                                             */
/* ------------------------------------------------------------------------ */
/* infer.m:376 */
float or_sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }

/* infer.m:378-383: o = g / (1 + exp(-g)) * u */
void or_silu_mul(const float *g, const float *u, float *o, int d) {
    for (int i = 0; i < d; i++) { float v = g[i]; o[i] = (v / (1.0f + expf(-v))) * u[i]; }
}

/* infer.m:369-374: o = x * (1 / sqrt(mean(x^2) + eps)) * w */
void or_rms_norm(const float *x, const float *w, float *o, int d, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < d; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)d + eps);
    for (int i = 0; i < d; i++) o[i] = w ? x[i] * inv * w[i] : x[i] * inv;
}

/* noaux_tc routing, infer.m:920-991.
 *  choice = sigmoid(logit) + bias; group score = top1 + top2 of choice within
 *  each group (strict '>', infer.m:934-940); the topk_group best groups by
 *  repeated argmax with lowest index winning ties (944-954); other experts
 *  masked to -1e30; top-K by scanning experts ascending and replacing the
 *  first minimum slot when strictly greater (970-980), so exp_idx is in SLOT
 *  order; weights are the unbiased sigmoids renormalised to routed_scale. */
void or_route(const float *logits, const float *bias, int n_experts, int n_group, int topk_group,
              int K, float routed_scale, int *exp_idx, float *exp_w) {
    float scores[1024], choice[1024], masked[1024];
    for (int i = 0; i < n_experts; i++) {
        scores[i] = or_sigmoidf(logits[i]);
        choice[i] = scores[i] + (bias ? bias[i] : 0.0f);
    }
    const int per = n_experts / n_group;
    float gs[64];
    for (int g = 0; g < n_group; g++) {
        float t1 = -1e30f, t2 = -1e30f;
        for (int e = 0; e < per; e++) {
            float s = choice[g * per + e];
            if (s > t1) { t2 = t1; t1 = s; }
            else if (s > t2) t2 = s;
        }
        gs[g] = t1 + t2;
    }
    int sel[64];
    for (int k = 0; k < topk_group; k++) {
        int best = -1; float bs = -1e30f;
        for (int g = 0; g < n_group; g++) {
            int seen = 0;
            for (int j = 0; j < k; j++) if (sel[j] == g) seen = 1;
            if (!seen && gs[g] > bs) { bs = gs[g]; best = g; }
        }
        sel[k] = best;
    }
    for (int i = 0; i < n_experts; i++) masked[i] = -1e30f;
    for (int k = 0; k < topk_group; k++) {
        if (sel[k] < 0) continue;
        for (int e = 0; e < per; e++) masked[sel[k] * per + e] = choice[sel[k] * per + e];
    }
    float key[64];
    for (int k = 0; k < K; k++) { key[k] = -1e30f; exp_idx[k] = 0; }
    for (int i = 0; i < n_experts; i++) {
        int mk = 0;
        for (int k = 1; k < K; k++) if (key[k] < key[mk]) mk = k;
        if (masked[i] > key[mk]) { key[mk] = masked[i]; exp_idx[mk] = i; }
    }
    float s = 0.0f;
    for (int k = 0; k < K; k++) { exp_w[k] = scores[exp_idx[k]]; s += exp_w[k]; }
    if (s > 0.0f) {
        float f = routed_scale / s;
        for (int k = 0; k < K; k++) exp_w[k] *= f;
    }
}

/* ------------------------------------------------------------------------ */
/* dense pieces                                                               */
/* ------------------------------------------------------------------------ */
typedef struct { const uint8_t *W; int type, cols; size_t rb; const float *x; float *y; int dbl; } mv_ctx;
static void mv_rows(void *c, long lo, long hi) {
    mv_ctx *m = (mv_ctx *)c;
    float *row = (float *)malloc(sizeof(float) * (size_t)m->cols);
    for (long r = lo; r < hi; r++) {
        if (m->type == OR_TYPE_Q6_K) or_dequant_q6k(m->W + (size_t)r * m->rb, row, (size_t)m->cols);
        else or_dequant_q4k(m->W + (size_t)r * m->rb, row, (size_t)m->cols);
        if (m->dbl) {
            double a = 0.0;
            for (int k = 0; k < m->cols; k++) a += (double)row[k] * (double)m->x[k];
            m->y[r] = (float)a;
        } else {
            float a = 0.0f;
            for (int k = 0; k < m->cols; k++) a += row[k] * m->x[k];
            m->y[r] = a;
        }
    }
    free(row);
}
void or_qmatvec(const void *W, int type, int rows, int cols, const float *x, float *y, int acc_double,
                int n_threads) {
    mv_ctx c = {(const uint8_t *)W, type, cols, or_row_bytes(type, (size_t)cols), x, y, acc_double};
    parallel_for(rows, n_threads, mv_rows, &c);
}

/* infer.m:1881 (cblas_sgemv fp32 over ffn_gate_inp [E x H]) */
void or_router_logits(const float *Wr, const float *x, int n_experts, int H, float *logits, int acc_double) {
    for (int e = 0; e < n_experts; e++) {
        const float *w = Wr + (size_t)e * H;
        if (acc_double) {
            double a = 0.0;
            for (int k = 0; k < H; k++) a += (double)w[k] * (double)x[k];
            logits[e] = (float)a;
        } else {
            float a = 0.0f;
            for (int k = 0; k < H; k++) a += w[k] * x[k];
            logits[e] = a;
        }
    }
}

size_t or_expert_bytes(int H, int I, int down_type) {
    return 2 * or_row_bytes(OR_TYPE_Q4_K, (size_t)H) * (size_t)I + or_row_bytes(down_type, (size_t)I) * (size_t)H;
}

/* infer.m:1069-1091 with cblas_sgemv replaced by a plain dot. */
void or_expert_forward(const void *gate, const void *up, const void *down, int down_type, const float *x,
                       int H, int I, float *eo, int acc_double, int n_threads) {
    float *g = (float *)malloc(sizeof(float) * (size_t)I * 3);
    float *u = g + I, *a = u + I;
    or_qmatvec(gate, OR_TYPE_Q4_K, I, H, x, g, acc_double, n_threads);
    or_qmatvec(up, OR_TYPE_Q4_K, I, H, x, u, acc_double, n_threads);
    or_silu_mul(g, u, a, I);
    or_qmatvec(down, down_type, H, I, a, eo, acc_double, n_threads);
    free(g);
}

/* One MoE layer (infer.m:1878-1922 without the residual): router logits,
 * route(), the K routed experts and the shared expert, combine in slot order
 * (infer.m:1915-1917) and + shared (1922). */
void or_moe_layer(const or_layer_cfg *cfg, const void *const *experts, const float *router_w,
                  const float *bias, const float *x, int B, const int *force_idx, const float *force_w,
                  float *out, int *idx_out, float *w_out, float *logits_out, int acc_double, int n_threads) {
    const int H = cfg->H, I = cfg->I, K = cfg->K, E = cfg->n_experts;
    const size_t gb = or_row_bytes(OR_TYPE_Q4_K, (size_t)H) * (size_t)I;
    float *logits = (float *)malloc(sizeof(float) * (size_t)E);
    float *eo = (float *)malloc(sizeof(float) * (size_t)H);
    float *acc = (float *)malloc(sizeof(float) * (size_t)H);
    for (int b = 0; b < B; b++) {
        const float *xb = x + (size_t)b * H;
        int idx[64]; float w[64];
        or_router_logits(router_w, xb, E, H, logits, acc_double);
        if (logits_out) memcpy(logits_out + (size_t)b * E, logits, sizeof(float) * (size_t)E);
        if (force_idx) {
            memcpy(idx, force_idx + (size_t)b * K, sizeof(int) * (size_t)K);
            memcpy(w, force_w + (size_t)b * K, sizeof(float) * (size_t)K);
        } else {
            or_route(logits, bias, E, cfg->n_group, cfg->topk_group, K, cfg->routed_scale, idx, w);
        }
        if (idx_out) memcpy(idx_out + (size_t)b * K, idx, sizeof(int) * (size_t)K);
        if (w_out) memcpy(w_out + (size_t)b * K, w, sizeof(float) * (size_t)K);
        for (int i = 0; i < H; i++) acc[i] = 0.0f;
        for (int k = 0; k < K; k++) {
            const uint8_t *blob = (const uint8_t *)experts[idx[k]];
            or_expert_forward(blob, blob + gb, blob + 2 * gb, cfg->down_type, xb, H, I, eo, acc_double, n_threads);
            for (int i = 0; i < H; i++) acc[i] += w[k] * eo[i];
        }
        const uint8_t *sh = (const uint8_t *)experts[E];
        or_expert_forward(sh, sh + gb, sh + 2 * gb, cfg->down_type, xb, H, I, eo, acc_double, n_threads);
        for (int i = 0; i < H; i++) out[(size_t)b * H + i] = acc[i] + eo[i];
    }
    free(logits); free(eo); free(acc);
}

/* ------------------------------------------------------------------------ */
/* The same layer for a batch with the routing given, grouped by expert: each */
/* weight row is dequantized once and dotted with every token the routing     */
/* sends to that expert.  The per-row dot (k order, fp64 or fp32), the SwiGLU */
/* and the combine (slot order, then + shared) are those of or_moe_layer, so  */
/* the outputs are identical bit for bit; only the loop nest differs.         */
/* ------------------------------------------------------------------------ */
typedef struct {
    const uint8_t *W; int type, cols; size_t rb;
    const float *const *xs; float *const *ys; int n; int dbl;
} mvn_ctx;
static void mvn_rows(void *c, long lo, long hi) {
    mvn_ctx *m = (mvn_ctx *)c;
    float *row = (float *)malloc(sizeof(float) * (size_t)m->cols);
    for (long r = lo; r < hi; r++) {
        if (m->type == OR_TYPE_Q6_K) or_dequant_q6k(m->W + (size_t)r * m->rb, row, (size_t)m->cols);
        else or_dequant_q4k(m->W + (size_t)r * m->rb, row, (size_t)m->cols);
        for (int j = 0; j < m->n; j++) {
            const float *x = m->xs[j];
            if (m->dbl) {
                double a = 0.0;
                for (int k = 0; k < m->cols; k++) a += (double)row[k] * (double)x[k];
                m->ys[j][r] = (float)a;
            } else {
                float a = 0.0f;
                for (int k = 0; k < m->cols; k++) a += row[k] * x[k];
                m->ys[j][r] = a;
            }
        }
    }
    free(row);
}

void or_moe_layer_given(const or_layer_cfg *cfg, const void *const *experts, const float *x, int B,
                        const int *idx, const float *w, float *out, int acc_double, int n_threads) {
    const int H = cfg->H, I = cfg->I, K = cfg->K, E = cfg->n_experts;
    const size_t gb = or_row_bytes(OR_TYPE_Q4_K, (size_t)H) * (size_t)I;
    const long P = (long)B * (K + 1);  /* pair p = b * (K + 1) + k, k = K: shared */
    float *eo = (float *)malloc(sizeof(float) * (size_t)P * H);
    float *g = (float *)malloc(sizeof(float) * (size_t)B * I * 3);
    float *u = g + (size_t)B * I, *a = u + (size_t)B * I;
    const float **xs = (const float **)malloc(sizeof(float *) * (size_t)B);
    float **gs = (float **)malloc(sizeof(float *) * (size_t)B * 4);
    float **us = gs + B, **as_ = us + B, **es = as_ + B;
    long *pairs = (long *)malloc(sizeof(long) * (size_t)P);
    for (int e = 0; e <= E; e++) {
        int n = 0;
        for (int b = 0; b < B; b++) {
            for (int k = 0; k < K; k++)
                if (e < E && idx[(size_t)b * K + k] == e) pairs[n++] = (long)b * (K + 1) + k;
            if (e == E) pairs[n++] = (long)b * (K + 1) + K;
        }
        if (!n) continue;
        const uint8_t *blob = (const uint8_t *)experts[e];
        for (int j = 0; j < n; j++) {
            xs[j] = x + (size_t)(pairs[j] / (K + 1)) * H;
            gs[j] = g + (size_t)j * I;
            us[j] = u + (size_t)j * I;
            as_[j] = a + (size_t)j * I;
            es[j] = eo + (size_t)pairs[j] * H;
        }
        mvn_ctx cg = {blob, OR_TYPE_Q4_K, H, or_row_bytes(OR_TYPE_Q4_K, (size_t)H), xs, gs, n, acc_double};
        parallel_for(I, n_threads, mvn_rows, &cg);
        mvn_ctx cu = {blob + gb, OR_TYPE_Q4_K, H, or_row_bytes(OR_TYPE_Q4_K, (size_t)H), xs, us, n, acc_double};
        parallel_for(I, n_threads, mvn_rows, &cu);
        for (int j = 0; j < n; j++) or_silu_mul(gs[j], us[j], as_[j], I);
        mvn_ctx cd = {blob + 2 * gb, cfg->down_type, I, or_row_bytes(cfg->down_type, (size_t)I),
                      (const float *const *)as_, es, n, acc_double};
        parallel_for(H, n_threads, mvn_rows, &cd);
    }
    for (int b = 0; b < B; b++) {
        float *o = out + (size_t)b * H;
        for (int i = 0; i < H; i++) o[i] = 0.0f;
        for (int k = 0; k < K; k++) {
            const float *ek = eo + ((size_t)b * (K + 1) + k) * H;
            const float wk = w[(size_t)b * K + k];
            for (int i = 0; i < H; i++) o[i] += wk * ek[i];
        }
        const float *es_ = eo + ((size_t)b * (K + 1) + K) * H;
        for (int i = 0; i < H; i++) o[i] = o[i] + es_[i];
    }
    free(pairs); free(gs); free(xs); free(g); free(eo);
}

/* ------------------------------------------------------------------------ */
/* dense FFN layers 0-2 (infer.m:1786-1793, 1852-1868)                       */
/* ------------------------------------------------------------------------ */
/* dequant_tensor_full (infer.m:314-348) followed by the fp16 rounding of
 * dequant_tensor_f16 / f32_to_f16_alloc (infer.m:519-538). */
int or_to_f16(int type, const void *src, uint16_t *dst, size_t n) {
    const uint16_t *h = (const uint16_t *)src;
    const float *f = (const float *)src;
    if (type == OR_TYPE_F16) {
        for (size_t i = 0; i < n; i++) dst[i] = or_fp32_to_fp16(or_fp16_to_fp32(h[i]));
        return 0;
    }
    if (type == OR_TYPE_F32) {
        for (size_t i = 0; i < n; i++) dst[i] = or_fp32_to_fp16(f[i]);
        return 0;
    }
    if (type == OR_TYPE_BF16) {
        for (size_t i = 0; i < n; i++) dst[i] = or_fp32_to_fp16(bits_f((uint32_t)h[i] << 16));
        return 0;
    }
    if ((type != OR_TYPE_Q4_K && type != OR_TYPE_Q6_K) || n % OR_QK) return -1;
    float *tmp = (float *)malloc(sizeof(float) * OR_QK);
    const size_t bb = type == OR_TYPE_Q6_K ? OR_Q6K_BYTES : OR_Q4K_BYTES;
    for (size_t b = 0; b < n / OR_QK; b++) {
        if (type == OR_TYPE_Q6_K) or_dequant_q6k((const uint8_t *)src + b * bb, tmp, OR_QK);
        else or_dequant_q4k((const uint8_t *)src + b * bb, tmp, OR_QK);
        for (int i = 0; i < OR_QK; i++) dst[b * OR_QK + i] = or_fp32_to_fp16(tmp[i]);
    }
    free(tmp);
    return 0;
}

typedef struct { const uint16_t *A; const float *x; float *y; int n, dbl; } mvh_ctx;
static void mvh_rows(void *c, long lo, long hi) {
    mvh_ctx *m = (mvh_ctx *)c;
    for (long r = lo; r < hi; r++) {
        const uint16_t *row = m->A + (size_t)r * m->n;
        if (m->dbl) {
            double a = 0.0;
            for (int k = 0; k < m->n; k++) a += (double)or_fp16_to_fp32(row[k]) * (double)m->x[k];
            m->y[r] = (float)a;
        } else {
            float a = 0.0f;
            for (int k = 0; k < m->n; k++) a += or_fp16_to_fp32(row[k]) * m->x[k];
            m->y[r] = a;
        }
    }
}
/* infer.m:459-516 (NEON fp16 -> fp32 widening, fp32 FMA; rows split over
 * worker threads) */
void or_mv_f16(const uint16_t *A, const float *x, float *y, int m, int n, int acc_double, int n_threads) {
    mvh_ctx c = {A, x, y, n, acc_double};
    parallel_for(m, n_threads, mvh_rows, &c);
}

/* infer.m:1855-1865 without the residual add of 1864 */
void or_dense_ffn(const uint16_t *gate, const uint16_t *up, const uint16_t *down, int H, int Id,
                  const float *x, int T, float *out, int acc_double, int n_threads) {
    float *g = (float *)malloc(sizeof(float) * (size_t)Id * 3);
    float *u = g + Id, *a = u + Id;
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * H;
        or_mv_f16(gate, xt, g, Id, H, acc_double, n_threads);
        or_mv_f16(up, xt, u, Id, H, acc_double, n_threads);
        or_silu_mul(g, u, a, Id);
        or_mv_f16(down, a, out + (size_t)t * H, H, Id, acc_double, n_threads);
    }
    free(g);
}

/* ------------------------------------------------------------------------ */
/* next-token choice (infer.m:390-394, 405-456)                              */
/* ------------------------------------------------------------------------ */
/* infer.m:390-394: the first index of the largest value */
int or_argmax(const float *x, int n) {
    int b = 0;
    float v = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > v) { v = x[i]; b = i; }
    return b;
}

/* infer.m:412-418 */
float or_rand_unit(uint32_t *state) {
    uint32_t x = *state;
    x ^= x << 13; x ^= x >> 17; x ^= x << 5;
    *state = x;
    return (x & 0xFFFFFFu) * (1.0f / (float)0x1000000);
}

typedef struct { float p; int idx; } or_pi;
/* descending by p; equal p in index order (qsort's order for ties is
 * unspecified in the reference; this is the order a stable sort gives) */
static int or_cmp_pi(const void *a, const void *b) {
    const or_pi *x = (const or_pi *)a, *y = (const or_pi *)b;
    if (x->p != y->p) return x->p < y->p ? 1 : -1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}

/* infer.m:419-456 (sample_top_p), the draw taken from and written back to
 * *state; cum_out / r_out (may be NULL) return the nucleus mass and the draw */
int or_sample_top_p(const float *logits, int n, float temp, float top_p, uint32_t *state, float *cum_out,
                    float *r_out) {
    if (temp <= 0.0f) return or_argmax(logits, n);
    or_pi *buf = (or_pi *)malloc(sizeof(or_pi) * (size_t)n);
    float inv_t = 1.0f / temp;
    float maxv = -1e30f;
    for (int i = 0; i < n; i++) {
        float v = logits[i] * inv_t;
        if (v > maxv) maxv = v;
    }
    float sum = 0;
    for (int i = 0; i < n; i++) {
        float v = logits[i] * inv_t;
        float p = expf(v - maxv);
        buf[i].p = p; buf[i].idx = i; sum += p;
    }
    float inv_s = 1.0f / sum;
    for (int i = 0; i < n; i++) buf[i].p *= inv_s;
    qsort(buf, (size_t)n, sizeof(or_pi), or_cmp_pi);
    float cum = 0;
    int cutoff = n;
    for (int i = 0; i < n; i++) {
        cum += buf[i].p;
        if (cum >= top_p) { cutoff = i + 1; break; }
    }
    float r = or_rand_unit(state) * cum;
    if (cum_out) *cum_out = cum;
    if (r_out) *r_out = r;
    float c = 0;
    int tok = buf[cutoff - 1].idx;
    for (int i = 0; i < cutoff; i++) {
        c += buf[i].p;
        if (r <= c) { tok = buf[i].idx; break; }
    }
    free(buf);
    return tok;
}

/* ------------------------------------------------------------------------ */
/* MLA attention of one decode token (infer.m:545-903)                       */
/* ------------------------------------------------------------------------ */
/* YaRN band (yarn_init_once, infer.m:591-610): the frequency indices between
 * which the rotary frequencies ramp from extrapolated to interpolated. */
void or_yarn_band(const or_mla_cfg *c, int *lo_out, int *hi_out) {
    const int dim = c->qk_rope;
    const float twopi = 2.0f * (float)M_PI;
    float lo_f = ((float)dim * logf(c->rope_orig_ctx / (32.0f * twopi))) / (2.0f * logf(c->rope_theta));
    float hi_f = ((float)dim * logf(c->rope_orig_ctx / (1.0f * twopi))) / (2.0f * logf(c->rope_theta));
    int lo = (int)floorf(lo_f), hi = (int)ceilf(hi_f);
    if (lo < 0) lo = 0;
    if (hi > dim / 2 - 1) hi = dim / 2 - 1;
    if (hi <= lo) hi = lo + 1;
    *lo_out = lo;
    *hi_out = hi;
}

/* yarn_freq (infer.m:612-624): blend of base^(-2i/dim) and the same / scale */
float or_yarn_freq(const or_mla_cfg *c, int i) {
    int lo, hi;
    or_yarn_band(c, &lo, &hi);
    const int dim = c->qk_rope;
    float freq_extra = 1.0f / powf(c->rope_theta, (float)(2 * i) / (float)dim);
    float freq_inter = freq_extra / c->rope_scale;
    float denom = (float)(hi - lo);
    if (denom < 1e-3f) denom = 1e-3f;
    float ramp = ((float)i - (float)lo) / denom;
    if (ramp < 0.0f) ramp = 0.0f;
    if (ramp > 1.0f) ramp = 1.0f;
    float mask = 1.0f - ramp;
    return freq_inter * (1.0f - mask) + freq_extra * mask;
}

/* apply_rope_q / apply_rope_k (infer.m:628-656): interleaved pairs
 * (x[2i], x[2i+1]) of each head rotated by pos * freq(i) */
void or_rope(const or_mla_cfg *c, float *x, int n_heads, int pos) {
    const int half = c->qk_rope / 2;
    for (int h = 0; h < n_heads; h++) {
        float *xh = x + (size_t)h * c->qk_rope;
        for (int i = 0; i < half; i++) {
            float ang = (float)pos * or_yarn_freq(c, i);
            float cs = cosf(ang), sn = sinf(ang);
            float a = xh[2 * i], b = xh[2 * i + 1];
            xh[2 * i] = a * cs - b * sn;
            xh[2 * i + 1] = a * sn + b * cs;
        }
    }
}

/* softmax (infer.m:384-388) */
void or_softmax(float *x, int n) {
    float m = x[0];
    for (int i = 1; i < n; i++) if (x[i] > m) m = x[i];
    float s = 0;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - m); s += x[i]; }
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

static float dot_h(const uint16_t *a, const float *x, int n, int dbl) {
    if (dbl) {
        double s = 0.0;
        for (int k = 0; k < n; k++) s += (double)or_fp16_to_fp32(a[k]) * (double)x[k];
        return (float)s;
    }
    float s = 0.0f;
    for (int k = 0; k < n; k++) s += or_fp16_to_fp32(a[k]) * x[k];
    return s;
}

static float dot_f(const float *a, const float *x, int n, int dbl) {
    if (dbl) {
        double s = 0.0;
        for (int k = 0; k < n; k++) s += (double)a[k] * (double)x[k];
        return (float)s;
    }
    float s = 0.0f;
    for (int k = 0; k < n; k++) s += a[k] * x[k];
    return s;
}

/* mla_forward (infer.m:766-903) for the token at position pos: RMSNorm,
 * q_a -> RMSNorm -> q_b (per head [nope | rope]), kv_a -> RMSNorm on the
 * latent part, RoPE on q_rope and k_rope, append (c_kv, k_rope) to the cache
 * at *len, absorbed attention (Q_abs = k_b q_nope; scores = scale (Q_abs .
 * c_kv + q_rope . k_rope), scale = (0.1 ln(rope_scale) + 1)^2 / sqrt(qk_nope +
 * qk_rope); softmax; wc = sum_s p_s c_kv[s]; out_h = v_b wc), o_proj, and
 * hidden += o. */
void or_mla_decode(const or_mla_cfg *c, const or_mla_weights *w, float *hidden, float *c_kv, float *k_rope_cache,
                   int *len, int pos, int acc_double) {
    const int H = c->H, NH = c->n_heads, QL = c->q_lora, KL = c->kv_lora, NP = c->qk_nope, RP = c->qk_rope,
              VH = c->v_head, QK = NP + RP, dbl = acc_double;
    float *normed = (float *)malloc(sizeof(float) * (size_t)H);
    float *qa = (float *)malloc(sizeof(float) * (size_t)QL), *qan = (float *)malloc(sizeof(float) * (size_t)QL);
    float *qf = (float *)malloc(sizeof(float) * (size_t)NH * QK);
    float *qn = (float *)malloc(sizeof(float) * (size_t)NH * NP), *qr = (float *)malloc(sizeof(float) * (size_t)NH * RP);
    float *kva = (float *)malloc(sizeof(float) * (size_t)(KL + RP));
    or_rms_norm(hidden, w->attn_norm, normed, H, c->eps);
    for (int r = 0; r < QL; r++) qa[r] = dot_h(w->q_a + (size_t)r * H, normed, H, dbl);
    or_rms_norm(qa, w->q_a_norm, qan, QL, c->eps);
    for (int r = 0; r < NH * QK; r++) qf[r] = dot_h(w->q_b + (size_t)r * QL, qan, QL, dbl);
    for (int h = 0; h < NH; h++) {
        memcpy(qn + (size_t)h * NP, qf + (size_t)h * QK, sizeof(float) * (size_t)NP);
        memcpy(qr + (size_t)h * RP, qf + (size_t)h * QK + NP, sizeof(float) * (size_t)RP);
    }
    for (int r = 0; r < KL + RP; r++) kva[r] = dot_h(w->kv_a + (size_t)r * H, normed, H, dbl);
    const int S = *len + 1;
    float *ckv_new = c_kv + (size_t)(*len) * KL, *kr_new = k_rope_cache + (size_t)(*len) * RP;
    or_rms_norm(kva, w->kv_a_norm, ckv_new, KL, c->eps);
    memcpy(kr_new, kva + KL, sizeof(float) * (size_t)RP);
    or_rope(c, qr, NH, pos);
    or_rope(c, kr_new, 1, pos);
    *len = S;
    const float ms = 0.1f * logf(c->rope_scale) + 1.0f;
    const float scale = (ms * ms) / sqrtf((float)QK);
    float *qabs = (float *)malloc(sizeof(float) * (size_t)KL), *sc = (float *)malloc(sizeof(float) * (size_t)S);
    float *wc = (float *)malloc(sizeof(float) * (size_t)KL), *att = (float *)malloc(sizeof(float) * (size_t)NH * VH);
    for (int h = 0; h < NH; h++) {
        const uint16_t *kb = w->k_b + (size_t)h * KL * NP, *vb = w->v_b + (size_t)h * VH * KL;
        for (int j = 0; j < KL; j++) qabs[j] = dot_h(kb + (size_t)j * NP, qn + (size_t)h * NP, NP, dbl);
        for (int s = 0; s < S; s++) {
            const float a = dot_f(qabs, c_kv + (size_t)s * KL, KL, dbl);
            const float b = dot_f(qr + (size_t)h * RP, k_rope_cache + (size_t)s * RP, RP, dbl);
            sc[s] = scale * a + scale * b;
        }
        or_softmax(sc, S);
        for (int j = 0; j < KL; j++) {
            if (dbl) {
                double a = 0.0;
                for (int s = 0; s < S; s++) a += (double)sc[s] * (double)c_kv[(size_t)s * KL + j];
                wc[j] = (float)a;
            } else {
                float a = 0.0f;
                for (int s = 0; s < S; s++) a += sc[s] * c_kv[(size_t)s * KL + j];
                wc[j] = a;
            }
        }
        for (int v = 0; v < VH; v++) att[(size_t)h * VH + v] = dot_h(vb + (size_t)v * KL, wc, KL, dbl);
    }
    for (int r = 0; r < H; r++) hidden[r] += dot_h(w->o_proj + (size_t)r * NH * VH, att, NH * VH, dbl);
    free(normed); free(qa); free(qan); free(qf); free(qn); free(qr); free(kva);
    free(qabs); free(sc); free(wc); free(att);
}
