/*
 * moe_cuda.h -- C ABI of libmoe_cuda.so: the DeepSeek-V3/R1 mixture-of-experts
 * block (sigmoid router, grouped top-k, dispatch, Q4_K/Q6_K SwiGLU experts,
 * shared expert, weighted combine) on NVIDIA B200 (sm_100a).
 *
 * Drop-in boundary.  The reference engine (JohnnyNg6/flash_deepseek) runs this
 * block inside layer_forward (infer.m:1878-1922) through four seams, each of
 * which has an entry point here:
 *
 *   route(logits, bias, K, exp_idx, exp_w)            infer.m:920-991
 *       -> moe_route()
 *   metal_moe_forward(L, h_post, exp_idx, exp_w, K, moe_out)
 *                                                     infer.m:1604-1700
 *       -> moe_experts_forward()
 *   shared_expert_worker(SharedJob *)                 infer.m:1099-1114
 *       -> moe_shared_forward()
 *   the whole MoE half of layer_forward (logits mv + route + shared + routed
 *   experts + combine, infer.m:1878-1922 without the residual)
 *       -> moe_forward()
 *   the codec dequantize_row_q4_K / dequantize_row_q6_K    quant.h:11-12
 *       -> moe_dequantize_row_q4_K() / moe_dequantize_row_q6_K()
 *
 * Weights enter as the raw GGUF block bytes the reference reads with
 * gguf_tensor_pread (gguf.h:192): the stacked blk.L.ffn_{gate,up,down}_exps
 * tensors (repack_experts.c:126-128) with type ids GGML_TYPE_Q4_K = 12 and
 * GGML_TYPE_Q6_K = 14 (gguf.h:59,61), or the reference's packed per-layer
 * expert file (infer.m:1802-1823).
 *
 * Conventions follow gguf.h: plain pointers and sizes, int return 0 = ok,
 * < 0 = error with the message available from moe_last_error().  All calls on
 * one context come from one host thread.  Host-pointer calls are synchronous;
 * the *_device calls are asynchronous on the stream given (NULL = the
 * context's stream).
 */
#ifndef MOE_CUDA_H
#define MOE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_TYPE_F32 0   /* GGML_TYPE_F32 */
#define MOE_TYPE_F16 1   /* GGML_TYPE_F16 */
#define MOE_TYPE_Q4_K 12 /* GGML_TYPE_Q4_K, gguf.h:59 */
#define MOE_TYPE_Q6_K 14 /* GGML_TYPE_Q6_K, gguf.h:61 */
#define MOE_TYPE_BF16 30 /* GGML_TYPE_BF16 */

#define MOE_OK 0
#define MOE_ERR_ARG (-1)      /* bad argument / shape */
#define MOE_ERR_CUDA (-2)     /* CUDA runtime error */
#define MOE_ERR_NCCL (-3)     /* NCCL error or timeout */
#define MOE_ERR_STATE (-4)    /* layer not loaded, wrong call order */
#define MOE_ERR_TIMEOUT (-5)  /* a bounded device wait gave up */

/* Model constants of infer.m:43-80 made run-time parameters. */
typedef struct moe_config {
    int hidden;         /* H: 7168 (HIDDEN_DIM) */
    int intermediate;   /* I: 2048 (MOE_INTERMEDIATE, also the shared expert) */
    int n_experts;      /* E: 256 (NUM_EXPERTS) */
    int n_group;        /* 8 (N_GROUP) */
    int topk_group;     /* 4 (TOPK_GROUP) */
    int top_k;          /* K: 8 (--k, infer.m:2042); at most 16 (MAX_K) */
    float routed_scale; /* 2.5 (ROUTED_SCALE) */
    float rms_eps;      /* 1e-6 (RMS_NORM_EPS), used by moe_forward_stack */
    int n_layers;       /* number of layer slots in this context */
    int max_tokens;     /* largest token batch of one forward call */
} moe_config;

typedef struct moe_ctx moe_ctx;

/* ------------------------------------------------------------------ setup */
/* Fills 128 bytes with a fresh NCCL unique id (rank 0 only, then broadcast
 * to the other ranks by the caller). */
int moe_get_unique_id(void *out_id128);

/* Creates a context on CUDA device `device` (left current on return).
 * world_size == 1 needs no id.  For world_size > 1 (expert parallel, one
 * process per GPU) routed expert e lives on rank e / (n_experts /
 * world_size); router and shared expert are replicated.  Returns NULL on
 * error (message on stderr).  Every later call on the context runs on its
 * device and gives the caller's current device back on return, so several
 * contexts on different GPUs can share a host thread. */
moe_ctx *moe_create(const moe_config *cfg, int device, int rank, int world_size,
                    const void *unique_id128);
void moe_destroy(moe_ctx *ctx);
const char *moe_last_error(const moe_ctx *ctx);
/* cudaStream_t of the context, for callers that time or chain work. */
void *moe_stream(moe_ctx *ctx);
int moe_rank(const moe_ctx *ctx);
int moe_world_size(const moe_ctx *ctx);
/* 1 when the expert-parallel exchanges of this context run over NVLink peer
 * memory (bounded waits), 0 when they run over NCCL send/recv (world_size 1:
 * 0). */
int moe_ep_peer_memory(const moe_ctx *ctx);

/* ---------------------------------------------------------------- weights */
/* Loads one MoE layer from the GGUF tensors of layer L (host pointers):
 *   gate_exps / up_exps : blk.L.ffn_{gate,up}_exps.weight, Q4_K, E experts of
 *                         [I rows x H cols] stacked expert-major;
 *   down_exps           : blk.L.ffn_down_exps.weight, [H x I] per expert,
 *                         down_type MOE_TYPE_Q4_K or MOE_TYPE_Q6_K;
 *   router_w            : blk.L.ffn_gate_inp.weight as fp32 [E x H];
 *   bias                : blk.L.exp_probs_b.bias fp32 [E] (may be NULL);
 *   sh_gate/sh_up/sh_down: blk.L.ffn_{gate,up,down}_shexp.weight.
 * Each rank copies only its own experts.  Q6_K matrices are repacked on the
 * device into an aligned layout (lossless; moe_read_expert returns the GGUF
 * bytes again). */
int moe_load_layer(moe_ctx *ctx, int layer, const void *gate_exps, const void *up_exps,
                   const void *down_exps, int down_type, const float *router_w,
                   const float *bias, const void *sh_gate, const void *sh_up,
                   const void *sh_down, int sh_down_type);

/* Same, with the stacked expert tensors holding only this rank's routed
 * experts (global ids moe_shard_range's offset / per-expert size on, n_experts
 * / world_size of them), so that each rank of an expert-parallel context
 * reads just its slice of blk.L.ffn_{gate,up,down}_exps.weight with
 * gguf_tensor_pread(t, buf, bytes, offset) (gguf.h:192) instead of the whole
 * tensor.  Router, bias and shared expert as for moe_load_layer. */
int moe_load_layer_shard(moe_ctx *ctx, int layer, const void *gate_slice, const void *up_slice,
                         const void *down_slice, int down_type, const float *router_w,
                         const float *bias, const void *sh_gate, const void *sh_up,
                         const void *sh_down, int sh_down_type);
/* Byte range of this rank's experts inside a stacked expert tensor of
 * per_expert_bytes per expert: *offset = first expert * per_expert_bytes,
 * *bytes = experts per rank * per_expert_bytes. */
int moe_shard_range(const moe_ctx *ctx, size_t per_expert_bytes, size_t *offset, size_t *bytes);

/* Same, from the reference's packed expert file layout (packed_experts/
 * layer_XX.bin: expert e at e*expert_size = [gate][up][down],
 * repack_experts.c:157-238, infer.m:1802-1823); the down type is inferred
 * from expert_size as infer.m:1814-1821 does. */
int moe_load_layer_packed(moe_ctx *ctx, int layer, const void *layer_blob, size_t expert_size,
                          const float *router_w, const float *bias, const void *sh_gate,
                          const void *sh_up, const void *sh_down, int sh_down_type);

/* Synthetic layer generated on the device (no host transfer): every weight
 * N(0, w_sigma) from a counter-based generator keyed by (seed, layer, expert,
 * matrix, element), quantized to Q4_K / down_type; router N(0, router_sigma),
 * bias N(0, bias_sigma).  Bit-identical to the host generator of the test
 * oracle. */
int moe_init_layer_synthetic(moe_ctx *ctx, int layer, uint64_t seed, int down_type,
                             double w_sigma, double router_sigma, double bias_sigma);

/* Adds a per-expert term to the selection bias (exp_probs_b) of a loaded
 * layer. */
int moe_add_router_bias(moe_ctx *ctx, int layer, const float *extra_bias);

/* Sets a per-expert term added to the router logits before the sigmoid
 * (logits = W_r h + logit_bias; NULL clears it).  Used to skew expert load,
 * e.g. by a Zipf profile. */
int moe_set_logit_bias(moe_ctx *ctx, int layer, const float *logit_bias);

/* RMSNorm weight (fp32 [H]) applied before layer L in moe_forward_stack. */
int moe_set_norm_weight(moe_ctx *ctx, int layer, const float *w);

/* Copies expert `expert` (n_experts = shared) of layer L back in the GGUF
 * byte layout [gate][up][down]; only experts this rank holds.  dst_size must
 * be at least moe_expert_bytes(). */
int moe_read_expert(moe_ctx *ctx, int layer, int expert, void *dst, size_t dst_size);
size_t moe_expert_bytes(const moe_ctx *ctx, int layer);

/* Writes the routed experts of layer L that this rank holds into the
 * reference's packed per-layer expert file (packed_experts/layer_XX.bin,
 * written by repack_experts.c:157-238 and read by infer.m:1802-1823): expert
 * e's GGUF bytes [gate][up][down] at e * moe_expert_bytes(), no header.  The
 * file is sized for all n_experts experts and opened without truncation, so
 * the ranks of an expert-parallel context can each write their part of one
 * file. */
int moe_write_layer_packed(moe_ctx *ctx, int layer, const char *path);

/* ------------------------------------------------------- dense FFN layers */
/* The dense FFN of the first layers (L < 3 in DeepSeek-V3: FIRST_MOE_LAYER,
 * infer.m:46), which take the place of the MoE block there.  The three
 * matrices (GGUF blk.L.ffn_gate / ffn_up [intermediate x H], ffn_down
 * [H x intermediate]; DENSE_INTERMEDIATE 18432, infer.m:59) are given as
 * host bytes of GGUF type F32, F16, BF16, Q4_K or Q6_K and kept on the GPU as
 * fp16, rounded as the reference's dequant_tensor_f16 does (infer.m:530-538,
 * loaded at infer.m:1786-1793).  Needs hidden % 256 == 0 and
 * intermediate % 256 == 0.  A layer slot holds either a MoE block or a dense
 * FFN; loading one frees the other. */
int moe_load_dense_layer(moe_ctx *ctx, int layer, int intermediate,
                         const void *gate, int gate_type, const void *up, int up_type,
                         const void *down, int down_type);
/* Synthetic dense layer: fp16 of N(0, w_sigma) values from the generator of
 * moe_init_layer_synthetic (gate / up / down streams of expert id
 * n_experts + 1), reproducible by the oracle. */
int moe_init_dense_synthetic(moe_ctx *ctx, int layer, int intermediate, uint64_t seed, double w_sigma);
/* Copies matrix `which` (0 gate, 1 up, 2 down) of a dense layer back as fp16
 * bits; dst_size >= intermediate * H * 2 bytes. */
int moe_read_dense_weight(moe_ctx *ctx, int layer, int which, void *dst, size_t dst_size);
/* The dense FFN of n_tokens tokens without the residual (infer.m:1855-1865,
 * mv_f16 + silu_mul): out[t] = Wd (silu(Wg h[t]) * (Wu h[t])), fp32
 * [n_tokens x H].  Every rank of an expert-parallel context holds the whole
 * layer and runs its own tokens (no exchange). */
int moe_dense_forward(moe_ctx *ctx, int layer, const float *h_post, int n_tokens, float *out);
/* Same on device buffers (16-byte aligned), asynchronous on `stream`. */
int moe_dense_forward_device(moe_ctx *ctx, int layer, const float *d_h_post, int n_tokens,
                             float *d_out, void *stream);

/* ------------------------------------------------- output head, sampling */
/* The output projection (lm_head, infer.m:1937-1941; GGUF output.weight
 * [vocab x H], VOCAB_SIZE 129280) kept as fp16 like the dense layers (any
 * GGUF type above), and its logits for n_tokens rows of final hidden states
 * (after the output RMSNorm): logits[t] = W h[t], fp32 [n_tokens x vocab]. */
int moe_load_lm_head(moe_ctx *ctx, int vocab, const void *w, int type);
/* Synthetic head: fp16 of N(0, w_sigma) from the generator's stream of
 * (layer 0, expert id n_experts + 2, gate kind). */
int moe_init_lm_head_synthetic(moe_ctx *ctx, int vocab, uint64_t seed, double w_sigma);
/* The kept fp16 weights back (dst_size >= vocab * H * 2). */
int moe_read_lm_head(moe_ctx *ctx, void *dst, size_t dst_size);
int moe_lm_head(moe_ctx *ctx, const float *h, int n_tokens, float *logits);
int moe_lm_head_device(moe_ctx *ctx, const float *d_h, int n_tokens, float *d_logits, void *stream);

/* The next token of each of n_tokens rows of `vocab` logits, as the
 * reference's sample_top_p (infer.m:419-456): argmax (first index of the
 * largest logit) when temp <= 0; otherwise softmax(logits / temp), the
 * smallest prefix of the descending order whose mass reaches top_p, one
 * xorshift32 draw r = rand_unit() * (that mass), and the first token of the
 * prefix at which the running mass reaches r.  Probabilities that are equal
 * are taken in index order.  Row t uses the (t + 1)-th xorshift32 state after
 * *rng_state; the host entry advances *rng_state by n_tokens when temp > 0
 * (the reference's generator starts at 0xa1b2c3d4, infer.m:411).  The
 * cumulative sums are exact (fixed point, 2^-40) where the reference adds in
 * fp32, so a draw within fp32 rounding of a boundary may pick a neighbour.
 * Scratch for max_tokens rows of `vocab` values is allocated by
 * moe_load_lm_head / moe_init_lm_head_synthetic, or by the first call with a
 * larger vocabulary; make that call before any stream capture. */
int moe_sample(moe_ctx *ctx, const float *logits, int n_tokens, int vocab, float temp, float top_p,
               uint32_t *rng_state, int *tokens);
int moe_sample_device(moe_ctx *ctx, const float *d_logits, int n_tokens, int vocab, float temp,
                      float top_p, uint32_t rng_state, int *d_tokens, void *stream);
/* The xorshift32 state after n draws (rand_unit, infer.m:412-418). */
uint32_t moe_rng_advance(uint32_t state, int n);

/* ---------------------------------------------------------------- forward */
/* The full MoE block for n_tokens tokens held by this rank (host buffers):
 * out[t] = sum_k w_k E_{idx_k}(h[t]) + shared(h[t]), fp32 [n_tokens x H].
 * idx_out / w_out (optional, [n_tokens x K]) return the routing in the
 * reference's slot order. */
int moe_forward(moe_ctx *ctx, int layer, const float *h_post, int n_tokens, float *out,
                int *idx_out, float *w_out);
/* Same on device buffers, asynchronous on `stream` (NULL = context stream).
 * Errors that the kernels detect (a bounded wait that gave up, a routing
 * index out of range) are not known when this returns: moe_check_error()
 * reports them. */
int moe_forward_device(moe_ctx *ctx, int layer, const float *d_h_post, int n_tokens,
                       float *d_out, int *d_idx_out, float *d_w_out, void *stream);

/* Waits for the context stream and reports the first error the kernels
 * recorded since the last host-pointer call or check: MOE_ERR_TIMEOUT when a
 * bounded device wait gave up (expert pipeline, prefill pipeline, or a peer
 * exchange -- after which the context refuses further expert-parallel
 * calls), MOE_ERR_ARG for a routing index out of range.  The error word is
 * cleared.  Host-pointer calls (moe_forward, ...) do this themselves; callers
 * of the *_device entry points call it after a batch of steps.  With the
 * NCCL exchange the wait polls and aborts the communicator after
 * MOE_EP_TIMEOUT_S seconds (default 120). */
int moe_check_error(moe_ctx *ctx);

/* Routed experts only, with the routing given (metal_moe_forward,
 * infer.m:1604): moe_out[t] = sum_k exp_w[t,k] E_{exp_idx[t,k]}(h[t]). */
int moe_experts_forward(moe_ctx *ctx, int layer, const float *h_post, int n_tokens,
                        const int *exp_idx, const float *exp_w, int K, float *moe_out);
int moe_experts_forward_device(moe_ctx *ctx, int layer, const float *d_h_post, int n_tokens,
                               const int *d_exp_idx, const float *d_exp_w, int K,
                               float *d_moe_out, void *stream);

/* Shared expert only (shared_expert_worker, infer.m:1099): sd = shared(h). */
int moe_shared_forward(moe_ctx *ctx, int layer, const float *h_post, int n_tokens, float *sd);

/* Routing only (route, infer.m:920-991) for n_tokens rows of logits, with the
 * context's group/top-k constants. */
int moe_route(moe_ctx *ctx, const float *logits, const float *bias, int n_tokens, int *exp_idx,
              float *exp_w);

/* Stack of layers [first, first + n_layers): per layer
 *   h_post = RMSNorm(hidden) * norm_w;  hidden = hidden + FFN(h_post)
 * (infer.m:1850, 1864 / 1922 with attention as identity), FFN the dense FFN
 * of a slot loaded by moe_load_dense_layer, else the MoE block.  hidden is updated in
 * place, device buffer [n_tokens x H]. */
int moe_forward_stack_device(moe_ctx *ctx, int first_layer, int n_layers, float *d_hidden,
                             int n_tokens, void *stream);
int moe_forward_stack(moe_ctx *ctx, int first_layer, int n_layers, float *hidden, int n_tokens);

/* The MoE block for a long batch of tokens (prompt prefill):
 * out[t] = sum_k w_k E_{idx_k}(h[t]) + shared(h[t]) like moe_forward, for any
 * n_tokens >= 1 (not bounded by max_tokens).  The router and the expert
 * products run as tensor-core GEMMs (tcgen05): the router on fp16 hi/lo
 * splits to fp32 accuracy, the experts over fp16 copies of the dequantized
 * weights and of the activations with fp32 accumulation, so results agree
 * with moe_forward to about 1e-3 relative, not bit for bit.  Shapes: hidden
 * a multiple of 512, intermediate a multiple of 256 (MOE_ERR_ARG otherwise).
 * With expert
 * parallelism (world_size > 1) every rank calls with its own tokens (0
 * allowed); the token rows go to the ranks that own their experts and the
 * partial sums come back (NCCL), as in moe_forward.  The first call (and any
 * call with more tokens than before) allocates the prefill workspace (about
 * 0.5 MB per token, more with expert parallelism).  idx_out / w_out are
 * optional.  The reference prefills one token at a time through
 * layer_forward (infer.m:2215-2229); this entry point has no counterpart
 * there. */
int moe_prefill_device(moe_ctx *ctx, int layer, const float *d_h_post, int n_tokens, float *d_out,
                       int *d_idx, float *d_w, void *stream);
int moe_prefill(moe_ctx *ctx, int layer, const float *h_post, int n_tokens, float *out, int *idx_out,
                float *w_out);

/* Routing from hidden states with no allocation: router logits
 * (d_h x d_router_w^T, fp32) then the grouped top-k of moe_route(), writing
 * d_idx / d_w [n_tokens x top_k] -- the routing of moe_forward(): the same
 * kernels and arithmetic up to 4 tokens; for more, moe_forward's logits come
 * from the tensor-core router (fp32 accuracy, another summation order), so
 * the two agree except where two experts' choice scores are within ~1e-6 of
 * each other.  For callers that cannot call cudaMalloc (a
 * fixed memory pool, or a latency-critical decode loop where an allocation
 * may synchronize the device): all scratch lives in a fixed array inside the
 * library (2 MiB per GPU, held until exit).  Limits: n_tokens <= 64,
 * (hidden/256) * n_tokens * n_experts <= 458752 (DeepSeek-V3 at 64 tokens),
 * n_tokens * n_experts <= 65536.  All pointers are device pointers; the call is asynchronous on
 * `stream` (NULL = default stream).  The first call on a device looks up the
 * array's device address; make it before any stream capture.  Every call
 * shares the one array, so calls that overlap on the GPU (other streams,
 * other threads) race.  No counterpart in the reference. */
int moe_route_hidden_noalloc(const moe_config *cfg, const float *d_router_w, const float *d_bias,
                             const float *d_h, int n_tokens, int *d_idx, float *d_w, void *stream);

/* ------------------------------------------------------------------ codec */
/* Device twins of quant.h:11-12 (host buffers in and out). */
int moe_dequantize_row_q4_K(const void *src, float *dst, size_t n);
int moe_dequantize_row_q6_K(const void *src, float *dst, size_t n);

/* ------------------------------------------------------------- statistics */
/* Per-phase device timing of the last forward call (the B200 counterpart of
 * the reference's moe_prof_t phase records, infer.m:177-261): when enabled,
 * CUDA events are recorded on the context stream between the phases below and
 * moe_get_timing() returns their durations in milliseconds. */
#define MOE_PHASE_ROUTER 0     /* router logits GEMV */
#define MOE_PHASE_ROUTE 1      /* sigmoid + grouped top-k + plan + operand */
#define MOE_PHASE_DISPATCH 2   /* expert-parallel dispatch (0 on one GPU) */
#define MOE_PHASE_GATEUP_TC 3  /* busy experts' gate/up on tcgen05 (+ their operand gather) */
#define MOE_PHASE_GATEUP 4     /* gate/up GEMV + SwiGLU (the other experts) */
#define MOE_PHASE_PREP 5       /* down-operand preparation */
#define MOE_PHASE_DOWN_TC 6    /* busy experts' down on tcgen05 */
#define MOE_PHASE_DOWN 7       /* down GEMV (the other experts) */
#define MOE_PHASE_COMBINE 8    /* combine all-to-all (0 on one GPU) */
#define MOE_PHASE_OUTPUT 9     /* weighted combine + shared (+ residual) */
#define MOE_N_PHASES 10
/* enable > 0 turns timing on with a ring of `enable` steps (each forward call
 * records into the next slot), 0 turns it off. */
int moe_set_timing(moe_ctx *ctx, int enable);
/* Durations of the last forward call (n <= MOE_N_PHASES floats). */
int moe_get_timing(moe_ctx *ctx, float *ms, int n);
/* Durations of the `back`-th most recent call (0 = last), while it is still
 * in the ring. */
int moe_get_timing_at(moe_ctx *ctx, int back, float *ms, int n);

/* Number of kernels this library launched on the context's device since
 * creation (or the last reset). */
uint64_t moe_kernel_launches(const moe_ctx *ctx);
void moe_reset_kernel_launches(moe_ctx *ctx);
/* Weight bytes the last forward call had to read on this rank (routed experts
 * actually hit + shared + router), for roofline accounting. */
uint64_t moe_last_weight_bytes(const moe_ctx *ctx);
/* Per-layer record of the routed experts this rank read, for critical-path
 * roofline accounting over a layer stack: while d_hits (device int
 * [n_layers]) is set, every moe_forward_device / moe_forward_stack_device
 * layer writes d_hits[layer] = the number of this rank's routed experts
 * that got at least one token (a device-to-device copy on the call's stream).
 * NULL stops recording.  Changing it drops the captured CUDA graphs. */
int moe_record_expert_hits(moe_ctx *ctx, int *d_hits);

#ifdef __cplusplus
}
#endif
#endif /* MOE_CUDA_H */
