/*
 * oracle.h -- CPU restatement of the DeepSeek-V3/R1 MoE block of the reference
 * engine (JohnnyNg6/flash_deepseek), used ONLY as test infrastructure: the
 * checker for the CUDA library in tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py.  Nothing in the product links or calls it.
 *
 * Parity pins (how this restatement is itself checked):
 *   - Q4_K/Q6_K/fp16 decode: bit-exact against the reference's own quant.c
 *     (compiled in place into oracle/_ref/ by oracle/Makefile) and against
 *     gguf-py 0.19.0 dequantize() golden vectors in tests/golden/.
 *   - route / sigmoid / silu_mul / rms_norm: against the reference's own
 *     functions extracted from infer.m at build time (oracle/_ref/), and the
 *     golden vectors they produced (tests/golden/route_golden.npz).
 *   - The expert / layer composition (dequant + dot in place of Accelerate's
 *     cblas_sgemv, which does not exist on Linux) is a restatement of
 *     infer.m:1069-1114 and 1915-1922 built from the pinned pieces.
 *   - dense FFN fp16 rounding, sample_top_p / argmax, softmax and the YaRN
 *     RoPE: against the reference's own functions built in place (the MLA
 *     decode step itself, which calls Metal and Accelerate, is restated from
 *     infer.m:766-903 on those pinned pieces).
 *   - The quantizer and the counter-based RNG have no counterpart in the
 *     reference (it ships neither); they define the synthetic inputs.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_QK 256
#define OR_Q4K_BYTES 144
#define OR_Q6K_BYTES 210
#define OR_TYPE_Q4_K 12
#define OR_TYPE_Q6_K 14

/* ---- fp16 codec (quant.c:4-24) and the quantizer's fp32->fp16 (RNE) ---- */
float    or_fp16_to_fp32(uint16_t h);
uint16_t or_fp32_to_fp16(float f);

/* ---- block dequant (quant.c:26-92) ---- */
void or_dequant_q4k(const void *src, float *dst, size_t n);
void or_dequant_q6k(const void *src, float *dst, size_t n);
size_t or_row_bytes(int type, size_t n_cols);

/* ---- quantizer (new; the reference has none) ---- */
void or_quantize_q4k(const float *x, void *dst, size_t n);
void or_quantize_q6k(const float *x, void *dst, size_t n);

/* ---- counter-based N(0, sigma) generator (new) ---- */
uint64_t or_splitmix64(uint64_t x);
uint64_t or_stream(int layer, int expert, int kind);
double   or_det_log(double s);
double   or_normal(uint64_t seed, uint64_t stream, uint64_t index);
void     or_fill_normal(uint64_t seed, uint64_t stream, uint64_t first,
                        size_t n, double sigma, float *dst, int n_threads);
/* Generate + quantize one [rows x cols] matrix of a synthetic tensor. */
void     or_gen_matrix(uint64_t seed, uint64_t stream, int type, int rows,
                       int cols, double sigma, void *dst, int n_threads);

/* ---- routing pieces (infer.m:369-383, 920-991) ---- */
float or_sigmoidf(float x);
void  or_silu_mul(const float *g, const float *u, float *o, int d);
void  or_rms_norm(const float *x, const float *w, float *o, int d, float eps);
void  or_route(const float *logits, const float *bias, int n_experts,
               int n_group, int topk_group, int K, float routed_scale,
               int *exp_idx, float *exp_w);

/* ---- dense pieces ---- */
/* y[r] = sum_k W[r,k] x[k] over quantized rows; acc_double selects fp64
 * accumulation (tight golden) or a left-to-right fp32 loop (order-only). */
void or_qmatvec(const void *W, int type, int rows, int cols, const float *x,
                float *y, int acc_double, int n_threads);
void or_router_logits(const float *Wr, const float *x, int n_experts, int H,
                      float *logits, int acc_double);
/* One SwiGLU expert (infer.m:1069-1091): eo = Wd (silu(Wg x) * (Wu x)). */
void or_expert_forward(const void *gate, const void *up, const void *down,
                       int down_type, const float *x, int H, int I,
                       float *eo, int acc_double, int n_threads);

/* ---- one MoE layer for B tokens (infer.m:1878-1922, attention = identity) --
 * experts: pointer table of (n_experts + 1) expert blobs; entry n_experts is
 * the shared expert.  Each blob is [gate Q4_K][up Q4_K][down Q4_K|Q6_K].
 * force_idx/force_w (may be NULL) replace the oracle's own routing, so the
 * expert math can be compared on the GPU's routing after a near-tie.
 * out[b] = sum_k w_k eo_k (slot order) + shared.  idx/w outputs optional. */
typedef struct {
    int H, I, n_experts, n_group, topk_group, K;
    float routed_scale;
    int down_type;       /* 12 (Q4_K) or 14 (Q6_K) */
} or_layer_cfg;

void or_moe_layer(const or_layer_cfg *cfg, const void *const *experts,
                  const float *router_w, const float *bias, const float *x,
                  int B, const int *force_idx, const float *force_w,
                  float *out, int *idx_out, float *w_out, float *logits_out,
                  int acc_double, int n_threads);

/* The same layer with the routing given (idx / w [B x K]), grouped by
 * expert: every weight row is dequantized once per expert and dotted with all
 * of its tokens.  Same arithmetic as or_moe_layer, bit for bit. */
void or_moe_layer_given(const or_layer_cfg *cfg, const void *const *experts,
                        const float *x, int B, const int *idx, const float *w,
                        float *out, int acc_double, int n_threads);

size_t or_expert_bytes(int H, int I, int down_type);

/* ---- dense FFN layers (infer.m:1786-1793, 1852-1868) ---- */
#define OR_TYPE_F32 0
#define OR_TYPE_F16 1
#define OR_TYPE_BF16 30
/* dequant_tensor_f16 (infer.m:314-348 + 530-538): n values of a GGUF tensor
 * of `type` (F32, F16, BF16, Q4_K, Q6_K) to fp32, then each rounded to fp16
 * (RNE, f32_to_f16_alloc infer.m:519-527).  Returns 0, or -1 on a type it
 * does not decode (n must be a multiple of 256 for Q4_K / Q6_K). */
int  or_to_f16(int type, const void *src, uint16_t *dst, size_t n);
/* mv_f16 (infer.m:459-516): y = A x, A fp16 [m x n] row-major widened to
 * fp32, fp64 (acc_double) or left-to-right fp32 accumulation. */
void or_mv_f16(const uint16_t *A, const float *x, float *y, int m, int n,
               int acc_double, int n_threads);
/* The dense FFN of T tokens without the residual (infer.m:1855-1865):
 * out[t] = Wd (silu(Wg x[t]) * (Wu x[t])); Wg, Wu fp16 [Id x H], Wd fp16
 * [H x Id]. */
void or_dense_ffn(const uint16_t *gate, const uint16_t *up, const uint16_t *down,
                  int H, int Id, const float *x, int T, float *out,
                  int acc_double, int n_threads);

/* ---- next-token choice (infer.m:390-394, 405-456) ---- */
int   or_argmax(const float *x, int n);
float or_rand_unit(uint32_t *state);
int   or_sample_top_p(const float *logits, int n, float temp, float top_p,
                      uint32_t *state, float *cum_out, float *r_out);

/* ---- MLA attention, one decode token (infer.m:545-903) ---- */
typedef struct {
    int H, n_heads, q_lora, kv_lora, qk_nope, qk_rope, v_head;
    float rope_theta, rope_scale, rope_orig_ctx, eps;
} or_mla_cfg;
/* fp16 bits: q_a [q_lora x H], q_b [n_heads * (qk_nope + qk_rope) x q_lora],
 * kv_a [(kv_lora + qk_rope) x H], k_b [n_heads][kv_lora x qk_nope],
 * v_b [n_heads][v_head x kv_lora], o_proj [H x n_heads * v_head];
 * fp32 norms attn_norm [H], q_a_norm [q_lora], kv_a_norm [kv_lora] */
typedef struct {
    const uint16_t *q_a, *q_b, *kv_a, *k_b, *v_b, *o_proj;
    const float *attn_norm, *q_a_norm, *kv_a_norm;
} or_mla_weights;
void  or_yarn_band(const or_mla_cfg *c, int *lo, int *hi);
float or_yarn_freq(const or_mla_cfg *c, int i);
void  or_rope(const or_mla_cfg *c, float *x, int n_heads, int pos);
void  or_softmax(float *x, int n);
/* hidden [H] += attention output; the cache (c_kv [. x kv_lora], k_rope
 * [. x qk_rope]) gains row *len, which then grows by one */
void  or_mla_decode(const or_mla_cfg *c, const or_mla_weights *w, float *hidden,
                    float *c_kv, float *k_rope, int *len, int pos, int acc_double);

#ifdef __cplusplus
}
#endif
#endif
