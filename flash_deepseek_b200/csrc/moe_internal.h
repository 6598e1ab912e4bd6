// moe_internal.h -- host-side view of the device pipeline of libmoe_cuda.so.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// Dispatch plan of one forward step on one GPU: (token, expert) pairs grouped
// by expert, and chunks of one expert's tokens (the unit of work of the
// expert kernels).
struct MoePlan {
    int *counts;        // [MOE_PLAN_COUNTS]: n_pairs, n_chunks, routed experts hit, -, work counters
    int *pair_expert;   // [max_pairs]  global expert id (n_experts = shared)
    int *pair_token;    // [max_pairs]  row of the activation operand
    float *pair_w;      // [max_pairs]  routing weight (1 for the shared expert)
    int *chunk_expert;  // [max_pairs]
    int *chunk_pair0;   // [max_pairs]
    int *chunk_ntok;    // [max_pairs]
    int *chunk_order;   // [max_pairs] chunk ids, most tokens first (decode plans only)
    int *slot_pair;     // [max_tokens][K+1] pair of (token, slot); slot K = shared
    int *error;         // [1] set to a non-zero code by device-side checks
};

// Where the expert weights of one layer live on this GPU.
struct MoeLayerDev {
    uint8_t *experts;       // [n_local + 1][expert_stride]; slot n_local = shared
    size_t expert_stride;
    size_t gate_bytes;      // one Q4_K [I x H] matrix
    int down_type, sh_down_type;  // 12 / 14
    int e0, n_local;        // global id of slot 0, number of routed experts here
    float *router;          // [E][H]
    float *bias;            // [E] selection bias (exp_probs_b)
    float *logit_bias;      // [E] added to the logits before the sigmoid, or nullptr
    float *norm;            // [H] or nullptr
    // TMA maps over [slot][row][byte] of this layer's weights (moe_experts.cu)
    CUtensorMap tm_gu;      // gate and up rows (2 I) of repacked Q4_K, box 144 B x 64 rows
    CUtensorMap tm_d4;      // Q4_K down rows (H), box 144 B x 128 rows
    CUtensorMap tm_d6q;     // Q6_K down, Q plane, box 192 B x 128 rows
    CUtensorMap tm_d6s;     // Q6_K down, S plane, box 16 B x 128 rows
    CUtensorMap tm_d6d;     // Q6_K down, D plane, box 2 nb_pad B x 128 rows
    CUtensorMap tm_pf6q;    // Q6_K down, Q plane, box 208 B x 128 rows (prefill: rows 208 B apart in shared memory)
    // the router weights x 2^8 as fp16 hi / lo (decode tensor-core router), rows
    // padded with zeros to a multiple of 128; box 64 columns x 128 rows
    __half *rwh, *rwl;
    CUtensorMap tm_rwh, tm_rwl;
};

struct MoeDims {
    int H, I, E, n_group, topk_group, K;
    float scale;
    int tc;  // 1: experts with more than MOE_TC tokens run on the tcgen05 kernels (moe_experts_tc.cu)
};

// Programmatic dependent launch: a forward-path kernel may start while its
// predecessor on the stream finishes; it runs only prologue work that reads
// no earlier output before moe_pdl_wait(), and lets its own successor start
// early with moe_pdl_trigger().  Without the launch attribute both are no-ops.
#define moe_pdl_wait() asm volatile("griddepcontrol.wait;\n" ::: "memory")
#define moe_pdl_trigger() asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory")

template <typename... KArgs, typename... Args>
static inline cudaError_t moe_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                         cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Codes that kernels store in MoePlan::error with atomicExch (when several
// fire, the last store is the one reported); the host turns them into
// messages when it next synchronizes.
#define MOE_DEV_ERR_INDEX 1          // routed expert index out of range
#define EX_ERR_TIMEOUT 0x7100        // expert GEMV pipeline: an mbarrier wait gave up
#define PF_ERR_TIMEOUT 0x7200        // prefill GEMM pipeline: an mbarrier wait gave up
#define PF_ERR_PAIR 0x7201           // prefill GEMM: the CTA pair's tensor-memory columns differ
#define EP_ERR_TIMEOUT 0x7300        // peer exchange: a peer's step flag did not arrive

// Raises a kernel's dynamic shared-memory limit on the current device when
// `bytes` exceeds what was set there before.  The attribute belongs to the
// device, so a process that drives contexts on several GPUs sets it on each;
// `done` is the kernel's record per device ordinal.
#define MOE_MAX_DEVICES 64
template <typename F>
inline void moe_smem_limit(F *kernel, size_t bytes, size_t (&done)[MOE_MAX_DEVICES]) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MOE_MAX_DEVICES) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        return;
    }
    if (bytes <= done[dev]) return;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess)
        done[dev] = bytes;
}

// Chunks of an expert's tokens (the unit of work of the expert GEMVs).  An
// expert with at most MOE_TC tokens is one chunk.  A busier one is, with
// MoeDims::tc set, split evenly into chunks of at most MOE_CHUNK_MAX tokens
// that run on the tcgen05 kernels (moe_experts_tc.cu); without it, into
// chunks of MOE_WIDE_TC tokens and one chunk of the remainder on the GEMVs.
// The gate/up GEMV runs a chunk on the fp16 path when it has at least
// MOE_GU_WIDE_MIN tokens, the down GEMV when it has more than MOE_TC (the
// int8-plane path otherwise).  The GEMVs take their work items from a
// counter in the plan, chunks in the order chunk_order (most tokens first;
// the first plan.counts[3] chunks are the tcgen05 kernels').
#define MOE_TC 8           // tokens of an int8-path chunk (four 8-column tiles of 2 tokens x 3 planes)
#define MOE_WIDE_TC 16     // tokens of an fp16-path chunk (four 8-column tiles of 4 tokens x 2 planes)
#define MOE_CHUNK_MAX 32   // tokens of a tcgen05 chunk
#ifndef MOE_GU_WIDE_MIN
#define MOE_GU_WIDE_MIN 7
#endif
static_assert(MOE_GU_WIDE_MIN >= 2 && MOE_GU_WIDE_MIN <= MOE_TC + 1,
              "chunks below MOE_GU_WIDE_MIN tokens run on the int8 path, which takes at most MOE_TC tokens");
__host__ __device__ __forceinline__ bool moe_gu_wide(int ntok) { return ntok >= MOE_GU_WIDE_MIN; }
__host__ __device__ __forceinline__ bool moe_dn_wide(int ntok) { return ntok > MOE_TC; }
__host__ __device__ __forceinline__ int moe_n_chunks(int n, int tc) {
    if (n <= 0) return 0;
    if (n <= MOE_TC) return 1;
    return tc ? (n + MOE_CHUNK_MAX - 1) / MOE_CHUNK_MAX : (n + MOE_WIDE_TC - 1) / MOE_WIDE_TC;
}
// chunk c of an expert with n tokens: first token (relative) and token count
__host__ __device__ __forceinline__ void moe_chunk(int n, int c, int tc, int &start, int &ntok) {
    if (n <= MOE_TC) {
        start = 0;
        ntok = n;
        return;
    }
    if (tc) {
        const int nc = (n + MOE_CHUNK_MAX - 1) / MOE_CHUNK_MAX;
        start = c * n / nc;
        ntok = (c + 1) * n / nc - start;
        return;
    }
    start = c * MOE_WIDE_TC;
    ntok = n - start < MOE_WIDE_TC ? n - start : MOE_WIDE_TC;
}
// plan.counts: [0] pairs, [1] chunks, [2] routed experts hit, [3] tcgen05
// chunks, [4] gate/up, [5] Q6_K down, [6] Q4_K down work counters (zeroed by
// the plan builder)
#define MOE_PLAN_COUNTS 8
#define MOE_ROUTER_SIMT_T 4  // decode tokens up to which the SIMT router (k_router_small) runs

#ifdef __CUDACC__
// Block-wide, after the block has written the plan's n_chunks chunks:
// chunk_order = chunk ids grouped by token count, most tokens first (so the
// GEMVs start the long items first and finish on short ones), and the work
// counters zeroed.  Every thread of the block calls it.
__device__ __forceinline__ void moe_plan_order_chunks(const MoePlan &plan, int n_chunks, int tc) {
    __shared__ int bucket[MOE_CHUNK_MAX + 1];
    for (int i = threadIdx.x; i <= MOE_CHUNK_MAX; i += blockDim.x) bucket[i] = 0;
    __syncthreads();
    for (int c = threadIdx.x; c < n_chunks; c += blockDim.x) {
        const int k = plan.chunk_ntok[c];
        atomicAdd(&bucket[k < MOE_CHUNK_MAX ? k : MOE_CHUNK_MAX], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0, n_tc = 0;
        for (int k = MOE_CHUNK_MAX; k >= 0; k--) {
            const int v = bucket[k];
            bucket[k] = acc;
            acc += v;
            if (tc && k > MOE_TC) n_tc += v;
        }
        plan.counts[3] = n_tc;
        for (int i = 4; i < MOE_PLAN_COUNTS; i++) plan.counts[i] = 0;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < n_chunks; c += blockDim.x) {
        const int k = plan.chunk_ntok[c];
        plan.chunk_order[atomicAdd(&bucket[k < MOE_CHUNK_MAX ? k : MOE_CHUNK_MAX], 1)] = c;
    }
}
#endif

// ---- launchers (moe_kernels.cu); every one counts its kernel launches ------
extern "C++" {
// logits[T][E] = x Wr^T; part: [n_split][T][E] scratch; counters: [E/32]
// zeroed ints (reset by the kernel)
void moe_launch_router_logits(const float *Wr, const float *x, int T, int H, int E, float *part, int n_split,
                              float *logits, int *counters, cudaStream_t s, uint64_t *launches);
// mode: 0 route from logits / partial logits, 1 routing given (idx_in, w_in),
// 2 shared expert only
void moe_launch_route_and_plan(const MoeDims &d, const float *part, int n_split, const float *logits,
                               const float *bias, const float *logit_bias, int mode, const int *idx_in, const float *w_in, int T,
                               int *idx_out, float *w_out, const float *x, uint8_t *xop,
                               int include_shared, int build_plan, const MoePlan &plan, int *counter,
                               cudaStream_t s, uint64_t *launches);
// xop: int8-plane operand rows (op_bytes(H) each) indexed by pair_token;
// max_chunks bounds the chunk count of the plan (grid size)
void moe_launch_gateup(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const uint8_t *xop,
                       float *act, int max_chunks, cudaStream_t s, uint64_t *launches);
void moe_launch_prep_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const float *act,
                          uint8_t *dop, int max_pairs, cudaStream_t s, uint64_t *launches);
void moe_launch_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const uint8_t *dop, float *eo,
                     int max_chunks, cudaStream_t s, uint64_t *launches);
// busy experts on tcgen05 (moe_experts_tc.cu): the plan's first counts[3]
// chunks (in chunk_order).  xtc: fp16 operand rows of their pairs (opw_bytes(H)
// each, row = pair), gathered from the token rows of xop; tm_xtc / tm_dop:
// 2-D maps over xtc / dop (moe_make_map_opw); max_pairs bounds the grid.
void moe_launch_tc_gather(const MoeDims &d, const MoePlan &plan, const uint8_t *xop, uint8_t *xtc, int max_pairs,
                          cudaStream_t s, uint64_t *launches);
void moe_launch_gateup_tc(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const CUtensorMap &tm_xtc,
                          float *act, int max_pairs, cudaStream_t s, uint64_t *launches);
void moe_launch_down_tc(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const CUtensorMap &tm_dop,
                        float *eo, int max_pairs, cudaStream_t s, uint64_t *launches);
// 2-D map over operand rows (opw_bytes(K) each, `rows` of them) for the
// tcgen05 kernels (boxes of 64 fp16 x box_rows rows, 128-byte swizzle)
int moe_make_map_opw(CUtensorMap *m, const void *base, int K, uint64_t rows);
// TMA maps of a layer (after its weights are allocated); 0 = ok
int moe_make_layer_maps(MoeLayerDev &L, const MoeDims &d);
// 2-D map over a row-major fp16 matrix [rows][cols] with 128-byte swizzle
int moe_make_map_f16_sw128(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                           uint32_t box_rows);

// ---- prefill (moe_prefill.cu) ----------------------------------------------
struct MoePrefillWs {
    int cap = 0;                 // tokens
    float *part = nullptr, *logits = nullptr, *w = nullptr, *eo = nullptr;
    int *idx = nullptr, *counters = nullptr;
    int *pcnt = nullptr, *pcur = nullptr;  // plan: per-expert counts and scatter cursors (E + 2 each)
    __half *xg = nullptr, *act = nullptr;
    __half *wh = nullptr, *wl = nullptr, *xh = nullptr, *xl = nullptr;  // fp16 hi/lo splits for the router
    // expert parallelism (world > 1): ecap rows per peer, fp16 rows out, fp32 partial sums back
    int world = 1, ecap = 0;
    size_t P = 0;                            // pairs capacity
    __half *send_xh = nullptr, *recv_xh = nullptr;
    int *send_meta = nullptr, *recv_meta = nullptr, *tok_slot = nullptr;
    float *send_y = nullptr, *recv_y = nullptr;
    int *tcount = nullptr;                   // [2 + world] token counts exchanged by the ranks
    MoePlan plan{};
    CUtensorMap tm_xg, tm_act, tm_wh, tm_wl, tm_xh, tm_xl;
};
// grows the workspace for T own tokens (world > 1: ecap rows per peer)
int moe_prefill_alloc(MoePrefillWs &ws, const MoeDims &d, int T, int world = 1, int ecap = 0);
// expert-parallel prefill steps (moe_api.cu runs the NCCL exchanges between them)
void moe_launch_pfe_dispatch(const MoeDims &d, MoePrefillWs &ws, int T, int n_local, cudaStream_t s,
                             uint64_t *launches);
void moe_launch_pfe_experts(const MoeDims &d, const MoeLayerDev &L, MoePrefillWs &ws, int T, cudaStream_t s,
                            uint64_t *launches);
void moe_launch_pfe_final(const MoeDims &d, MoePrefillWs &ws, int T, float *out, cudaStream_t s, uint64_t *launches);
void moe_prefill_free(MoePrefillWs &ws);
// the router weights' fp16 hi/lo split kept per layer (decode tensor-core router)
void moe_launch_router_split(const float *Wr, int E, int H, __half *wh, __half *wl, cudaStream_t s,
                             uint64_t *launches);
// decode router logits of T (5..64) tokens on the tensor cores into logits[T][E]
void moe_launch_router_tc(const MoeDims &d, const CUtensorMap &tm_wh, const CUtensorMap &tm_wl, const float *x,
                          int T, __half *xh, __half *xl, const CUtensorMap &tm_xh, const CUtensorMap &tm_xl,
                          float *part, int max_split, float *logits, int *error, cudaStream_t s,
                          uint64_t *launches);
// router logits of T tokens into ws.logits (tensor cores, fp16 hi/lo splits)
void moe_launch_prefill_router(const MoeDims &d, const float *Wr, MoePrefillWs &ws, const float *x, int T,
                               cudaStream_t s, uint64_t *launches);
// plan + gather + the two tcgen05 GEMMs + combine, after ws.idx / ws.w hold
// the routing of T tokens
void moe_launch_prefill_experts(const MoeDims &d, const MoeLayerDev &L, MoePrefillWs &ws, const float *x, int T,
                                float *out, cudaStream_t s, uint64_t *launches);
void moe_launch_combine(const MoeDims &d, const MoePlan &plan, const float *eo, int T, int include_routed,
                        int include_shared, const float *residual, float *out, cudaStream_t s, uint64_t *launches);
void moe_launch_rmsnorm(const float *x, const float *w, float *y, int T, int H, float eps, cudaStream_t s,
                        uint64_t *launches);
void moe_launch_dequant(int type, const uint8_t *src, float *dst, size_t n, cudaStream_t s, uint64_t *launches);
void moe_launch_q6_repack(const uint8_t *src, uint8_t *dst, int rows, int nb, int inverse, cudaStream_t s,
                          uint64_t *launches);
// in-place Q4_K qs transpose (its own inverse) of nblocks 144-byte blocks
void moe_launch_q4_repack(uint8_t *buf, size_t nblocks, cudaStream_t s, uint64_t *launches);
void moe_launch_synth_quant(int type, uint64_t seed, uint64_t stream, int rows, int cols, double sigma,
                            uint8_t *dst, cudaStream_t s, uint64_t *launches);
void moe_launch_synth_f32(uint64_t seed, uint64_t stream, size_t n, double sigma, float *dst, cudaStream_t s,
                          uint64_t *launches);
// dense FFN layers (moe_dense.cu): w = [gate Id x H][up Id x H][down H x Id]
// fp16; act [T x Id] fp32 scratch; out = residual (may be null) + FFN(x)
#define MOE_DENSE_SMEM_MAX (227 * 1024)
size_t moe_dense_smem_need(int H, int Id);
int moe_dense_shape_ok(int H, int Id);
void moe_launch_dense_ffn(const __half *w, int H, int Id, const float *x, int T, float *act, const float *residual,
                          float *out, cudaStream_t s, uint64_t *launches);
// logits [T x V] = W [V x H] fp16 . h [T x H] (moe_dense.cu)
void moe_launch_lm_head(const __half *w, int H, int V, const float *h, int T, float *logits, cudaStream_t s,
                        uint64_t *launches);
// temperature + top-p sampling (or argmax at temp <= 0) of T rows of V logits
// (moe_sample.cu); p: [T x V] fp32 scratch; ws: moe_sample_ws_bytes(T) bytes;
// row t draws the (t + 1)-th xorshift32 state after `rng`
size_t moe_sample_ws_bytes(int rows);
void moe_launch_sample(const float *logits, int T, int V, float temp, float top_p, uint32_t rng, float *p,
                       void *ws, int *tokens, cudaStream_t s, uint64_t *launches);
// n values of a GGUF tensor of `type` (device memory) to fp16; tmp holds n
// floats for Q4_K / Q6_K
void moe_launch_to_f16(int type, const void *src, __half *dst, size_t n, float *tmp, cudaStream_t s,
                       uint64_t *launches);
void moe_launch_prep_rows(const float *recv, const int *meta, int meta_w, int R, const float *local, int T, int H,
                          uint8_t *xop, cudaStream_t s, uint64_t *launches);
// expert parallel (moe_ep.cu)
void moe_launch_ep_pack(const float *x, const int *idx, const float *w, int T, int K, int H, int world, int n_local,
                        int cap, float *send_x, int *send_meta, int *tok_slot, cudaStream_t s, uint64_t *launches);
// NVLink peer-memory exchange (moe_ep.cu): mailbox base of every rank
// (peers[me] = own), byte offsets of its regions, and the step counter in
// device memory (steps completed by this rank; every kernel of a step uses
// seq = *d_seq + 1 and the buffers of parity seq & 1, and the step's last
// kernel advances it), so that a step's launches replay as a CUDA graph.
struct EpP2P {
    uint8_t *const *peers;
    size_t off_x, off_meta, off_y;
    int world, me;
    unsigned long long *d_seq;
    int *done;   // [3] block counters of the three signalling kernels
    int *error;  // plan.error: a peer's flag that did not arrive
};
void moe_launch_ep_pack_p2p(const float *x, const int *idx, const float *w, int T, int K, int H, int n_local,
                            int cap, const EpP2P &q, int *tok_slot, cudaStream_t s, uint64_t *launches);
// waits for the peers' dispatch flags, then one block builds the plan and the
// others the operand rows of the received and local rows
void moe_launch_ep_plan_rows_p2p(const MoeDims &d, const EpP2P &q, int cap, int T, int e0, int n_local,
                                 const MoePlan &plan, const float *local, uint8_t *xop, cudaStream_t s,
                                 uint64_t *launches);
void moe_launch_ep_partial_p2p(const MoeDims &d, const MoePlan &plan, const float *eo, int cap, const EpP2P &q,
                               cudaStream_t s, uint64_t *launches);
// waits for the peers' combine flags, sums, and advances the step counter
void moe_launch_ep_final_p2p(const MoeDims &d, const MoePlan &plan, const EpP2P &q, const int *tok_slot, int cap,
                             int T, const float *eo, const float *residual, float *out, cudaStream_t s,
                             uint64_t *launches);
void moe_launch_ep_plan(const MoeDims &d, const int *recv_meta, int world, int cap, int T, int e0, int n_local,
                        const MoePlan &plan, cudaStream_t s, uint64_t *launches);
void moe_launch_ep_partial(const MoeDims &d, const MoePlan &plan, const int *recv_meta, const float *eo, int rows,
                           float *out, cudaStream_t s, uint64_t *launches);
void moe_launch_ep_final(const MoeDims &d, const MoePlan &plan, const float *recv_y, const int *tok_slot, int world,
                         int cap, int T, const float *eo, const float *residual, float *out, cudaStream_t s,
                         uint64_t *launches);
}
