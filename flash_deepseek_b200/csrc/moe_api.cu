// moe_api.cu -- context, weight residency and the C ABI of libmoe_cuda.so
// (include/moe_cuda.h).  One context per GPU; expert-parallel contexts
// exchange token rows and partial sums (dispatch / combine) through
// fixed-capacity mailboxes in NVLink peer memory, or over NCCL send/recv when
// the peers cannot be mapped, so that a decode step needs no host
// synchronisation.
#include <dlfcn.h>
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include <array>
#include <initializer_list>
#include <chrono>
#include <string>
#include <thread>
#include <algorithm>
#include <vector>

#include "../../include/moe_cuda.h"
#include "moe_common.cuh"
#include "moe_internal.h"
#include "moe_nccl.h"
#include "moe_wait.h"

const MoeNccl *moe_nccl() {
    static MoeNccl api;
    static int state = 0;  // 0 unknown, 1 ok, -1 unavailable
    if (state) return state > 0 ? &api : nullptr;
    const char *env = getenv("MOE_NCCL_LIB");
    void *h = nullptr;
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // already in the process
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        fprintf(stderr, "[moe_cuda] ERROR: cannot load libnccl (set MOE_NCCL_LIB): %s\n", dlerror());
        state = -1;
        return nullptr;
    }
#define MOE_NCCL_SYM(field, name)                                                        \
    api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));                   \
    if (!api.field) {                                                                    \
        fprintf(stderr, "[moe_cuda] ERROR: libnccl lacks %s\n", name);                   \
        state = -1;                                                                      \
        return nullptr;                                                                  \
    }
    MOE_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
    MOE_NCCL_SYM(CommInitRank, "ncclCommInitRank")
    MOE_NCCL_SYM(CommDestroy, "ncclCommDestroy")
    MOE_NCCL_SYM(CommAbort, "ncclCommAbort")
    MOE_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
    MOE_NCCL_SYM(GroupStart, "ncclGroupStart")
    MOE_NCCL_SYM(GroupEnd, "ncclGroupEnd")
    MOE_NCCL_SYM(Send, "ncclSend")
    MOE_NCCL_SYM(Recv, "ncclRecv")
    MOE_NCCL_SYM(GetErrorString, "ncclGetErrorString")
#undef MOE_NCCL_SYM
    state = 1;
    return &api;
}

struct moe_ctx {
    moe_config cfg;
    MoeDims d;
    int device = 0, rank = 0, world = 1;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;
    int e0 = 0, n_local = 0;
    int max_tok = 0;   // tokens of one call on this rank
    int max_rows = 0;  // activation rows the expert kernels may see (world * max_tok)
    int max_pairs = 0;
    int n_split = 0;
    std::vector<MoeLayerDev> layers;
    std::vector<size_t> layer_down_bytes;
    // dense FFN layers (moe_dense.cu): [gate][up][down] fp16, intermediate Id
    struct DenseDev {
        __half *w = nullptr;
        int Id = 0;
    };
    std::vector<DenseDev> dense;
    float *dense_act = nullptr;  // [max_tok x Id] of the widest dense layer
    size_t dense_act_n = 0;
    // output head (lm_head, infer.m:1937-1941): fp16 [vocab x H]; sampling scratch
    __half *head_w = nullptr;
    int vocab = 0;
    float *head_logits = nullptr, *sample_p = nullptr;  // [max_tok x n] each
    int *sample_tok = nullptr;                           // [max_tok]
    void *sample_ws = nullptr;                           // moe_sample_ws_bytes(max_tok)
    size_t sample_n = 0;
    // workspace
    float *part = nullptr, *logits = nullptr, *d_in = nullptr, *d_out = nullptr, *h_post = nullptr;
    int *rl_counters = nullptr;
    int *idx = nullptr, *idx_given = nullptr;
    float *wts = nullptr, *w_given = nullptr, *bias_tmp = nullptr;
    uint8_t *xop = nullptr;   // activation operand rows (int8 planes, then fp16 planes), opx_row(H) each
    MoePlan plan{};
    int *counter = nullptr;
    float *act = nullptr, *eo = nullptr;
    uint8_t *dop = nullptr;   // down operand, opw_bytes(I) per pair (int8 or fp16 planes by chunk)
    uint8_t *xtc = nullptr;   // gate/up fp16 operand rows of the tcgen05 chunks' pairs, opw_bytes(H) per pair
    CUtensorMap tm_xtc, tm_dop;  // TMA maps of the tcgen05 kernels over xtc and dop
    // decode tensor-core router (more than MOE_ROUTER_SIMT_T tokens): the
    // tokens' fp16 hi / lo split, 128 rows (box 64 columns x 128 rows)
    __half *rxh = nullptr, *rxl = nullptr;
    CUtensorMap tm_rxh, tm_rxl;
    int *h_counts = nullptr;  // pinned [4]
    // expert-parallel buffers
    float *send_x = nullptr, *recv_x = nullptr, *send_y = nullptr, *recv_y = nullptr;
    int *send_meta = nullptr, *recv_meta = nullptr;
    float *rows_partial = nullptr;
    int *tok_slot = nullptr;
    // NVLink peer-memory exchange (moe_ep.cu): own mailbox, the peers' mapped
    // mailboxes (device array of world pointers), region offsets, step number
    bool p2p = false;
    uint8_t *mbox = nullptr;
    uint8_t **d_peers = nullptr;
    std::vector<uint8_t *> peer_map;
    size_t mb_x = 0, mb_meta = 0, mb_y = 0;
    int *ep_done = nullptr;  // [3] block counters of the pack, pre-combine and final kernels
    unsigned long long *d_seq = nullptr;  // peer-exchange steps completed by this rank (device)
    int *hits = nullptr;     // moe_record_expert_hits target, or nullptr
    bool comm_aborted = false;  // a host wait gave up on an NCCL exchange
    bool ep_failed = false;     // a peer-exchange wait gave up: the ranks are out of step
    std::string err;
    bool timing = false;
    int ring = 0, ring_pos = 0, ring_used = 0;  // per-step phase events
    std::vector<cudaEvent_t> ev;                // [ring][MOE_N_PHASES + 1]
    std::vector<uint8_t> ev_valid;
    uint64_t launches = 0;
    // replayable CUDA graphs, one per call signature: kind 0 = one layer's
    // forward (a = layer), kind 1 = a layer stack (a = first, b = count)
    struct GraphSig {
        int kind, a, b, T;
        const void *p1, *p2;
        cudaStream_t s;
        bool operator==(const GraphSig &o) const {
            return kind == o.kind && a == o.a && b == o.b && T == o.T && p1 == o.p1 && p2 == o.p2 && s == o.s;
        }
    };
    struct Graph {
        GraphSig sig;
        cudaGraphExec_t exec;
        uint64_t kernels, last_use;
    };
    std::vector<Graph> graphs;
    MoePrefillWs pf;  // prefill workspace, allocated on first use
    std::vector<GraphSig> seen;  // signatures run once directly (kernel attributes set)
    bool use_graphs = true;
    uint64_t clock = 0;
    uint64_t last_bytes = 0;
    int last_layer = -1;
};

static thread_local std::string g_create_err;

static int fail(moe_ctx *c, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (c) c->err = buf;
    fprintf(stderr, "[moe_cuda] ERROR: %s\n", buf);
    return code;
}

#define CK(call)                                                                                     \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) return fail(c, MOE_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                           __FILE__, __LINE__);                                     \
    } while (0)
#define NK(call)                                                                                     \
    do {                                                                                             \
        ncclResult_t r_ = (call);                                                                    \
        if (r_ != ncclSuccess) return fail(c, MOE_ERR_NCCL, "%s: %s", #call, moe_nccl()->GetErrorString(r_)); \
    } while (0)

// Makes the context's device current for one entry-point call and gives the
// caller back its own current device on return (nothing happens when they
// are the same device).
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess || prev == dev) prev = -1;
        else cudaSetDevice(dev);
    }
    ~DeviceScope() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

template <typename T>
static cudaError_t dmalloc(T **p, size_t n) {
    return cudaMalloc((void **)p, n * sizeof(T) + 256);
}

static size_t row_bytes(int type, int cols) {
    return (size_t)(cols / MOE_QK) * (type == MOE_TYPE_Q6_K ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
}

extern "C" {

int moe_get_unique_id(void *out) {
    const MoeNccl *nc = moe_nccl();
    if (!nc) return MOE_ERR_NCCL;
    ncclUniqueId id;
    if (nc->GetUniqueId(&id) != ncclSuccess) return MOE_ERR_NCCL;
    memcpy(out, &id, sizeof(id));
    return MOE_OK;
}

static void drop_graphs(moe_ctx *c) {
    for (auto &g : c->graphs) cudaGraphExecDestroy(g.exec);
    c->graphs.clear();
    c->seen.clear();
}

// The context's kernels run on a non-blocking stream (and on callers'
// streams), which the legacy default stream does not order against: clears
// and uploads go on the context stream, and the setup paths below wait for
// them before anything else can be launched.
static cudaError_t zero_async(moe_ctx *c, void *p, size_t bytes) { return cudaMemsetAsync(p, 0, bytes, c->stream); }
static cudaError_t upload_sync(moe_ctx *c, void *dst, const void *src, size_t bytes) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream);
    return e == cudaSuccess ? cudaStreamSynchronize(c->stream) : e;
}

static int ctx_alloc(moe_ctx *c) {
    const int T = c->max_tok, R = c->max_rows, H = c->d.H, I = c->d.I, E = c->d.E, K = c->d.K;
    c->max_pairs = R * K + T;
    c->n_split = H / MOE_QK;
    CK(dmalloc(&c->part, (size_t)c->n_split * T * E));
    CK(dmalloc(&c->logits, (size_t)T * E));
    CK(dmalloc(&c->rl_counters, (size_t)(E + 31) / 32));
    CK(zero_async(c, c->rl_counters, sizeof(int) * ((E + 31) / 32 + 64)));
    CK(dmalloc(&c->d_in, (size_t)T * H));
    CK(dmalloc(&c->d_out, (size_t)T * H));
    CK(dmalloc(&c->h_post, (size_t)T * H));
    CK(dmalloc(&c->idx, (size_t)R * K));
    CK(dmalloc(&c->wts, (size_t)R * K));
    CK(dmalloc(&c->idx_given, (size_t)R * K));
    CK(dmalloc(&c->w_given, (size_t)R * K));
    CK(dmalloc(&c->bias_tmp, (size_t)E));
    const int RT = (c->world > 1 ? R + T : R);  // EP: received rows + local rows
    CK(dmalloc(&c->xop, (size_t)RT * opx_row(H)));
    CK(zero_async(c, c->xop, (size_t)RT * opx_row(H)));
    const int P = c->max_pairs;
    CK(dmalloc(&c->plan.counts, MOE_PLAN_COUNTS));
    CK(dmalloc(&c->plan.pair_expert, P));
    CK(dmalloc(&c->plan.pair_token, P));
    CK(dmalloc(&c->plan.pair_w, P));
    CK(dmalloc(&c->plan.chunk_expert, P));
    CK(dmalloc(&c->plan.chunk_pair0, P));
    CK(dmalloc(&c->plan.chunk_ntok, P));
    CK(dmalloc(&c->plan.chunk_order, P));
    CK(dmalloc(&c->plan.slot_pair, (size_t)RT * (K + 1)));
    CK(dmalloc(&c->plan.error, 1));
    CK(zero_async(c, c->plan.error, sizeof(int)));
    CK(zero_async(c, c->plan.counts, MOE_PLAN_COUNTS * sizeof(int)));
    CK(dmalloc(&c->counter, 1));
    CK(zero_async(c, c->counter, sizeof(int)));
    CK(dmalloc(&c->act, (size_t)P * I));
    CK(dmalloc(&c->dop, (size_t)P * opw_bytes(I)));
    CK(zero_async(c, c->dop, (size_t)P * opw_bytes(I)));
    if (c->d.tc) {
        CK(dmalloc(&c->xtc, (size_t)P * opw_bytes(H)));
        CK(zero_async(c, c->xtc, (size_t)P * opw_bytes(H)));
        if (moe_make_map_opw(&c->tm_xtc, c->xtc, H, (uint64_t)P) || moe_make_map_opw(&c->tm_dop, c->dop, I, (uint64_t)P))
            return fail(c, MOE_ERR_CUDA, "tensor maps of the tcgen05 operand rows");
    }
    CK(dmalloc(&c->eo, (size_t)P * H));
    CK(cudaMallocHost((void **)&c->h_counts, 4 * sizeof(int)));
    if (c->world > 1) {
        const size_t rows = (size_t)c->world * T;
        CK(dmalloc(&c->send_x, rows * H));
        CK(dmalloc(&c->recv_x, rows * H));
        CK(dmalloc(&c->send_y, rows * H));
        CK(dmalloc(&c->recv_y, rows * H));
        CK(dmalloc(&c->send_meta, rows * (2 * K + 2)));
        CK(dmalloc(&c->recv_meta, rows * (2 * K + 2)));
        CK(dmalloc(&c->rows_partial, rows * H));
        CK(dmalloc(&c->tok_slot, (size_t)T * c->world));
    }
    if (T > MOE_ROUTER_SIMT_T) {
        // the decode tensor-core router's token split: 128 rows (the router's
        // token box), rows past the call's tokens only feed logits never read
        CK(dmalloc(&c->rxh, (size_t)128 * H));
        CK(dmalloc(&c->rxl, (size_t)128 * H));
        CK(zero_async(c, c->rxh, sizeof(__half) * 128 * (size_t)H));
        CK(zero_async(c, c->rxl, sizeof(__half) * 128 * (size_t)H));
        if (moe_make_map_f16_sw128(&c->tm_rxh, c->rxh, H, 128, 64, 128) ||
            moe_make_map_f16_sw128(&c->tm_rxl, c->rxl, H, 128, 64, 128))
            return fail(c, MOE_ERR_CUDA, "tensor maps of the router's token split");
    }
    CK(cudaStreamSynchronize(c->stream));  // the clears above, before any launch on any stream
    return MOE_OK;
}

// The layer's router weights as fp16 hi / lo x 2^8 for the decode
// tensor-core router, recomputed whenever the router weights are written (on
// the context stream, before the caller's final synchronize).
static int router_split(moe_ctx *c, MoeLayerDev &L) {
    const int E = c->d.E, H = c->d.H, Ep = (E + 127) & ~127;
    if (!L.rwh) {
        CK(dmalloc(&L.rwh, (size_t)Ep * H));
        CK(dmalloc(&L.rwl, (size_t)Ep * H));
        CK(zero_async(c, L.rwh, sizeof(__half) * (size_t)Ep * H));  // rows E .. Ep - 1 stay zero
        CK(zero_async(c, L.rwl, sizeof(__half) * (size_t)Ep * H));
        if (moe_make_map_f16_sw128(&L.tm_rwh, L.rwh, H, Ep, 64, 128) ||
            moe_make_map_f16_sw128(&L.tm_rwl, L.rwl, H, Ep, 64, 128))
            return fail(c, MOE_ERR_CUDA, "tensor maps of the router's weight split");
    }
    moe_launch_router_split(L.router, E, H, L.rwh, L.rwl, c->stream, &c->launches);
    CK(cudaGetLastError());
    return MOE_OK;
}

// Maps every peer's mailbox into this process (CUDA IPC handles exchanged
// once over NCCL).  Falls back to the NCCL send/recv exchange when a mapping
// is refused (no peer access) or MOE_EP_NCCL=1.
static int ep_p2p_init(moe_ctx *c) {
    const char *env = getenv("MOE_EP_NCCL");
    if (env && env[0] == '1') return MOE_OK;
    const int N = c->world, K = c->d.K, H = c->d.H;
    if (N > 64) return MOE_OK;
    const size_t R = (size_t)N * c->max_tok, mw = 2 + 2 * (size_t)K;
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    c->mb_x = 1024;
    c->mb_meta = c->mb_x + al(2 * R * H * sizeof(float));
    c->mb_y = c->mb_meta + al(2 * R * mw * sizeof(int));
    const size_t total = c->mb_y + 2 * R * H * sizeof(float);
    CK(cudaMalloc((void **)&c->mbox, total));
    CK(zero_async(c, c->mbox, total));
    CK(cudaMalloc((void **)&c->ep_done, 3 * sizeof(int)));
    CK(zero_async(c, c->ep_done, 3 * sizeof(int)));
    CK(cudaMalloc((void **)&c->d_seq, sizeof(unsigned long long)));
    CK(zero_async(c, c->d_seq, sizeof(unsigned long long)));
    CK(cudaStreamSynchronize(c->stream));  // cleared before a peer can map the mailbox
    CK(cudaMalloc((void **)&c->d_peers, N * sizeof(uint8_t *)));
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, c->mbox));
    uint8_t *dh = nullptr;
    CK(cudaMalloc((void **)&dh, (N + 1) * sizeof(cudaIpcMemHandle_t)));
    CK(upload_sync(c, dh, &mine, sizeof(mine)));
    NK(moe_nccl()->GroupStart());
    for (int p = 0; p < N; p++) {
        NK(moe_nccl()->Send(dh, sizeof(mine), ncclUint8, p, c->comm, c->stream));
        NK(moe_nccl()->Recv(dh + (p + 1) * sizeof(mine), sizeof(mine), ncclUint8, p, c->comm, c->stream));
    }
    NK(moe_nccl()->GroupEnd());
    std::vector<cudaIpcMemHandle_t> hs(N);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(hs.data(), dh + sizeof(mine), N * sizeof(mine), cudaMemcpyDeviceToHost));
    cudaFree(dh);
    c->peer_map.assign(N, nullptr);
    bool ok = true;
    for (int p = 0; p < N && ok; p++) {
        if (p == c->rank) { c->peer_map[p] = c->mbox; continue; }
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, hs[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
        } else {
            c->peer_map[p] = (uint8_t *)ptr;
        }
    }
    // every rank must take the same path: agree on the outcome
    int *dflag = nullptr;
    CK(cudaMalloc((void **)&dflag, (N + 1) * sizeof(int)));
    const int mine_ok = ok ? 1 : 0;
    CK(upload_sync(c, dflag, &mine_ok, sizeof(int)));
    NK(moe_nccl()->GroupStart());
    for (int p = 0; p < N; p++) {
        NK(moe_nccl()->Send(dflag, 1, ncclInt32, p, c->comm, c->stream));
        NK(moe_nccl()->Recv(dflag + 1 + p, 1, ncclInt32, p, c->comm, c->stream));
    }
    NK(moe_nccl()->GroupEnd());
    std::vector<int> oks(N);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(oks.data(), dflag + 1, N * sizeof(int), cudaMemcpyDeviceToHost));
    cudaFree(dflag);
    for (int p = 0; p < N; p++) ok = ok && oks[p];
    if (!ok) {
        for (int p = 0; p < N; p++)
            if (c->peer_map[p] && p != c->rank) cudaIpcCloseMemHandle(c->peer_map[p]);
        c->peer_map.clear();
        cudaFree(c->mbox);
        c->mbox = nullptr;
        return MOE_OK;  // the NCCL send/recv exchange
    }
    CK(upload_sync(c, c->d_peers, c->peer_map.data(), N * sizeof(uint8_t *)));
    c->p2p = true;
    return MOE_OK;
}

moe_ctx *moe_create(const moe_config *cfg, int device, int rank, int world_size, const void *uid) {
    if (!cfg) return nullptr;
    moe_ctx *c = new moe_ctx();
    c->cfg = *cfg;
    c->use_graphs = getenv("MOE_NO_GRAPHS") == nullptr;
    c->d = MoeDims{cfg->hidden, cfg->intermediate, cfg->n_experts, cfg->n_group, cfg->topk_group, cfg->top_k,
                   cfg->routed_scale, 1};
    {
        // MOE_TC=0 keeps busy experts on the GEMVs' fp16 path (16-token chunks)
        const char *e = getenv("MOE_TC");
        if (e && e[0] == '0') c->d.tc = 0;
    }
    c->device = device;
    c->rank = rank;
    c->world = world_size;
    const moe_config &k = *cfg;
    const char *bad = nullptr;
    if (k.hidden <= 0 || k.hidden % 256 || k.hidden > 32768) bad = "hidden must be a multiple of 256 in 256..32768";
    else if (k.intermediate <= 0 || k.intermediate % 256 || k.intermediate > 32768)
        bad = "intermediate must be a multiple of 256 in 256..32768";
    else if (k.n_experts <= 0 || k.n_experts > 1024) bad = "n_experts must be in 1..1024";
    else if (k.n_group <= 0 || k.n_group > 64 || k.n_experts % k.n_group) bad = "n_group must divide n_experts (<= 64)";
    else if (k.topk_group <= 0 || k.topk_group > k.n_group) bad = "topk_group must be in 1..n_group";
    else if (k.top_k <= 0 || k.top_k > MOE_MAX_K) bad = "top_k must be in 1..16";
    else if (k.top_k > k.topk_group * (k.n_experts / k.n_group)) bad = "top_k exceeds the experts of the selected groups";
    else if (k.n_layers <= 0) bad = "n_layers must be positive";
    else if (k.max_tokens <= 0 || k.max_tokens > 64) bad = "max_tokens must be in 1..64";
    else if (world_size <= 0 || rank < 0 || rank >= world_size) bad = "bad rank / world_size";
    else if (k.n_experts % world_size) bad = "world_size must divide n_experts";
    else if (world_size > 1 && (size_t)world_size * k.max_tokens > 1024) bad = "world_size * max_tokens exceeds 1024";
    if (bad) {
        fprintf(stderr, "[moe_cuda] ERROR: moe_create: %s\n", bad);
        delete c;
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        fprintf(stderr, "[moe_cuda] ERROR: moe_create: cudaSetDevice(%d) failed\n", device);
        delete c;
        return nullptr;
    }
    c->n_local = k.n_experts / world_size;
    c->e0 = rank * c->n_local;
    c->max_tok = k.max_tokens;
    c->max_rows = world_size * k.max_tokens;
    c->layers.assign(k.n_layers, MoeLayerDev{});
    c->dense.assign(k.n_layers, moe_ctx::DenseDev{});
    c->layer_down_bytes.assign(k.n_layers, 0);
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess || ctx_alloc(c) != MOE_OK) {
        fprintf(stderr, "[moe_cuda] ERROR: moe_create: allocation failed: %s\n", c->err.c_str());
        moe_destroy(c);
        return nullptr;
    }
    if (world_size > 1) {
        if (!uid) {
            fprintf(stderr, "[moe_cuda] ERROR: moe_create: world_size > 1 needs a unique id\n");
            moe_destroy(c);
            return nullptr;
        }
        ncclUniqueId id;
        memcpy(&id, uid, sizeof(id));
        const MoeNccl *nc = moe_nccl();
        if (!nc || nc->CommInitRank(&c->comm, world_size, id, rank) != ncclSuccess) {
            fprintf(stderr, "[moe_cuda] ERROR: moe_create: ncclCommInitRank failed\n");
            c->comm = nullptr;
            moe_destroy(c);
            return nullptr;
        }
        if (ep_p2p_init(c) != MOE_OK) {
            fprintf(stderr, "[moe_cuda] ERROR: moe_create: %s\n", c->err.c_str());
            moe_destroy(c);
            return nullptr;
        }
    }
    return c;
}

void moe_destroy(moe_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (size_t p = 0; p < c->peer_map.size(); p++)
        if (c->peer_map[p] && (int)p != c->rank) cudaIpcCloseMemHandle(c->peer_map[p]);
    cudaFree(c->mbox);
    cudaFree(c->d_peers);
    cudaFree(c->ep_done);
    cudaFree(c->d_seq);
    if (c->comm) moe_nccl()->CommDestroy(c->comm);
    for (cudaEvent_t e : c->ev) cudaEventDestroy(e);
    for (auto &g : c->graphs) cudaGraphExecDestroy(g.exec);
    moe_prefill_free(c->pf);
    cudaFree(c->pf.tcount);
    for (auto &L : c->layers) {
        cudaFree(L.experts);
        cudaFree(L.router);
        cudaFree(L.rwh);
        cudaFree(L.rwl);
        cudaFree(L.bias);
        cudaFree(L.logit_bias);
        cudaFree(L.norm);
    }
    for (auto &D : c->dense) cudaFree(D.w);
    cudaFree(c->dense_act);
    cudaFree(c->head_w);
    cudaFree(c->head_logits);
    cudaFree(c->sample_p);
    cudaFree(c->sample_tok);
    cudaFree(c->sample_ws);
    void *bufs[] = {c->part, c->logits, c->rl_counters, c->d_in, c->d_out, c->h_post, c->idx, c->wts, c->idx_given, c->w_given, c->bias_tmp, c->xop, c->plan.counts,
                    c->plan.pair_expert, c->plan.pair_token, c->plan.pair_w, c->plan.chunk_expert,
                    c->plan.chunk_pair0, c->plan.chunk_ntok, c->plan.chunk_order, c->plan.slot_pair, c->plan.error, c->counter, c->act,
                    c->dop, c->xtc, c->rxh, c->rxl, c->eo, c->send_x, c->recv_x, c->send_y, c->recv_y, c->send_meta,
                    c->recv_meta, c->rows_partial, c->tok_slot};
    for (void *b : bufs) cudaFree(b);
    if (c->h_counts) cudaFreeHost(c->h_counts);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

const char *moe_last_error(const moe_ctx *c) { return c ? c->err.c_str() : "null context"; }
void *moe_stream(moe_ctx *c) { return c ? (void *)c->stream : nullptr; }
int moe_rank(const moe_ctx *c) { return c ? c->rank : -1; }
int moe_world_size(const moe_ctx *c) { return c ? c->world : -1; }
uint64_t moe_kernel_launches(const moe_ctx *c) { return c ? c->launches : 0; }
void moe_reset_kernel_launches(moe_ctx *c) {
    if (c) c->launches = 0;
}

// ------------------------------------------------------------------ weights
static int layer_alloc(moe_ctx *c, int layer, int down_type, int sh_down_type) {
    if (layer < 0 || layer >= (int)c->layers.size()) return fail(c, MOE_ERR_ARG, "layer %d out of range", layer);
    if ((down_type != MOE_TYPE_Q4_K && down_type != MOE_TYPE_Q6_K) ||
        (sh_down_type != MOE_TYPE_Q4_K && sh_down_type != MOE_TYPE_Q6_K))
        return fail(c, MOE_ERR_ARG, "down types must be Q4_K (12) or Q6_K (14)");
    if ((down_type == MOE_TYPE_Q6_K || sh_down_type == MOE_TYPE_Q6_K) && (c->d.I / MOE_QK) % 8)
        return fail(c, MOE_ERR_ARG, "Q6_K down needs intermediate %% 2048 == 0");
    CK(cudaSetDevice(c->device));
    MoeLayerDev &L = c->layers[layer];
    const int H = c->d.H, I = c->d.I, E = c->d.E;
    cudaFree(c->dense[layer].w);  // a slot holds a MoE block or a dense FFN
    c->dense[layer] = moe_ctx::DenseDev{};
    L.gate_bytes = row_bytes(MOE_TYPE_Q4_K, H) * I;
    const size_t db = row_bytes(down_type, I) * H, sdb = row_bytes(sh_down_type, I) * H;
    const size_t stride = (2 * L.gate_bytes + (db > sdb ? db : sdb) + 255) & ~(size_t)255;
    if (!L.experts || L.expert_stride != stride) {
        cudaFree(L.experts);
        L.experts = nullptr;
        CK(cudaMalloc((void **)&L.experts, stride * (c->n_local + 1)));
    }
    L.expert_stride = stride;
    L.down_type = down_type;
    L.sh_down_type = sh_down_type;
    L.e0 = c->e0;
    L.n_local = c->n_local;
    if (!L.router) CK(cudaMalloc((void **)&L.router, sizeof(float) * (size_t)E * H));
    if (!L.bias) CK(cudaMalloc((void **)&L.bias, sizeof(float) * E));
    c->layer_down_bytes[layer] = db;
    drop_graphs(c);
    const int mrc = moe_make_layer_maps(L, c->d);
    if (mrc) return fail(c, MOE_ERR_CUDA, "TMA tensor map of layer %d failed (%d)", layer, mrc);
    return MOE_OK;
}

// copies one down matrix (GGUF bytes, device or host) into its slot
static int put_down(moe_ctx *c, uint8_t *dst, const void *src, int type, bool src_host, uint8_t *tmp) {
    const int H = c->d.H, I = c->d.I;
    const size_t bytes = row_bytes(type, I) * H;
    if (type == MOE_TYPE_Q4_K) {
        CK(cudaMemcpyAsync(dst, src, bytes, src_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                           c->stream));
        moe_launch_q4_repack(dst, (size_t)H * (I / MOE_QK), c->stream, &c->launches);
        CK(cudaGetLastError());
        return MOE_OK;
    }
    const uint8_t *s = (const uint8_t *)src;
    if (src_host) {
        CK(cudaMemcpyAsync(tmp, src, bytes, cudaMemcpyHostToDevice, c->stream));
        s = tmp;
    }
    moe_launch_q6_repack(s, dst, H, I / MOE_QK, 0, c->stream, &c->launches);
    CK(cudaGetLastError());
    return MOE_OK;
}

// slice: the expert tensors hold only this rank's experts (e0 .. e0 + n_local - 1)
static int load_layer_impl(moe_ctx *c, int layer, const void *gate_exps, const void *up_exps, const void *down_exps,
                           int down_type, const float *router_w, const float *bias, const void *sh_gate,
                           const void *sh_up, const void *sh_down, int sh_down_type, bool slice) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    if (!gate_exps || !up_exps || !down_exps || !router_w || !sh_gate || !sh_up || !sh_down)
        return fail(c, MOE_ERR_ARG, "moe_load_layer: null weight pointer");
    int rc = layer_alloc(c, layer, down_type, sh_down_type);
    if (rc) return rc;
    MoeLayerDev &L = c->layers[layer];
    const int H = c->d.H, I = c->d.I, E = c->d.E;
    const size_t gb = L.gate_bytes, db = row_bytes(down_type, I) * H;
    uint8_t *tmp = nullptr;
    CK(cudaMalloc((void **)&tmp, row_bytes(MOE_TYPE_Q6_K, I) * H));
    for (int j = 0; j <= c->n_local; j++) {
        uint8_t *dst = L.experts + (size_t)j * L.expert_stride;
        const bool sh = j == c->n_local;
        const int e = slice ? j : c->e0 + j;  // index inside the tensors given
        const uint8_t *g = sh ? (const uint8_t *)sh_gate : (const uint8_t *)gate_exps + (size_t)e * gb;
        const uint8_t *u = sh ? (const uint8_t *)sh_up : (const uint8_t *)up_exps + (size_t)e * gb;
        const uint8_t *dn = sh ? (const uint8_t *)sh_down : (const uint8_t *)down_exps + (size_t)e * db;
        cudaError_t e1 = cudaMemcpyAsync(dst, g, gb, cudaMemcpyHostToDevice, c->stream);
        cudaError_t e2 = cudaMemcpyAsync(dst + gb, u, gb, cudaMemcpyHostToDevice, c->stream);
        if (e1 != cudaSuccess || e2 != cudaSuccess) { cudaFree(tmp); return fail(c, MOE_ERR_CUDA, "weight copy failed"); }
        moe_launch_q4_repack(dst, 2 * (size_t)c->d.I * (c->d.H / MOE_QK), c->stream, &c->launches);
        rc = put_down(c, dst + 2 * gb, dn, sh ? sh_down_type : down_type, true, tmp);
        if (rc) { cudaFree(tmp); return rc; }
        cudaStreamSynchronize(c->stream);  // tmp is reused by the next expert
    }
    cudaFree(tmp);
    CK(cudaMemcpyAsync(L.router, router_w, sizeof(float) * (size_t)E * H, cudaMemcpyHostToDevice, c->stream));
    if (bias) CK(cudaMemcpyAsync(L.bias, bias, sizeof(float) * E, cudaMemcpyHostToDevice, c->stream));
    else CK(cudaMemsetAsync(L.bias, 0, sizeof(float) * E, c->stream));
    const int src = router_split(c, L);
    if (src) return src;
    CK(cudaStreamSynchronize(c->stream));
    return MOE_OK;
}

int moe_load_layer(moe_ctx *c, int layer, const void *gate_exps, const void *up_exps, const void *down_exps,
                   int down_type, const float *router_w, const float *bias, const void *sh_gate, const void *sh_up,
                   const void *sh_down, int sh_down_type) {
    return load_layer_impl(c, layer, gate_exps, up_exps, down_exps, down_type, router_w, bias, sh_gate, sh_up,
                           sh_down, sh_down_type, false);
}

int moe_load_layer_shard(moe_ctx *c, int layer, const void *gate_slice, const void *up_slice, const void *down_slice,
                         int down_type, const float *router_w, const float *bias, const void *sh_gate,
                         const void *sh_up, const void *sh_down, int sh_down_type) {
    return load_layer_impl(c, layer, gate_slice, up_slice, down_slice, down_type, router_w, bias, sh_gate, sh_up,
                           sh_down, sh_down_type, true);
}

int moe_shard_range(const moe_ctx *c, size_t per_expert_bytes, size_t *offset, size_t *bytes) {
    if (!c || !offset || !bytes) return MOE_ERR_ARG;
    *offset = (size_t)c->e0 * per_expert_bytes;
    *bytes = (size_t)c->n_local * per_expert_bytes;
    return MOE_OK;
}

int moe_load_layer_packed(moe_ctx *c, int layer, const void *blob, size_t expert_size, const float *router_w,
                          const float *bias, const void *sh_gate, const void *sh_up, const void *sh_down,
                          int sh_down_type) {
    if (!c || !blob) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    const int H = c->d.H, I = c->d.I;
    const size_t gb = row_bytes(MOE_TYPE_Q4_K, H) * I;
    int down_type;
    // down type inferred from the per-expert size (infer.m:1814-1821)
    if (expert_size == 2 * gb + row_bytes(MOE_TYPE_Q6_K, I) * H) down_type = MOE_TYPE_Q6_K;
    else if (expert_size == 2 * gb + row_bytes(MOE_TYPE_Q4_K, I) * H) down_type = MOE_TYPE_Q4_K;
    else return fail(c, MOE_ERR_ARG, "packed expert size %zu matches neither Q4_K nor Q6_K down", expert_size);
    int rc = layer_alloc(c, layer, down_type, sh_down_type);
    if (rc) return rc;
    MoeLayerDev &L = c->layers[layer];
    uint8_t *tmp = nullptr;
    CK(cudaMalloc((void **)&tmp, row_bytes(MOE_TYPE_Q6_K, I) * H));
    for (int j = 0; j <= c->n_local; j++) {
        uint8_t *dst = L.experts + (size_t)j * L.expert_stride;
        const bool sh = j == c->n_local;
        const uint8_t *src = (const uint8_t *)blob + (size_t)(c->e0 + j) * expert_size;
        cudaError_t e1 = cudaMemcpyAsync(dst, sh ? sh_gate : src, gb, cudaMemcpyHostToDevice, c->stream);
        cudaError_t e2 = cudaMemcpyAsync(dst + gb, sh ? sh_up : src + gb, gb, cudaMemcpyHostToDevice, c->stream);
        if (e1 != cudaSuccess || e2 != cudaSuccess) { cudaFree(tmp); return fail(c, MOE_ERR_CUDA, "weight copy failed"); }
        moe_launch_q4_repack(dst, 2 * (size_t)c->d.I * (c->d.H / MOE_QK), c->stream, &c->launches);
        rc = put_down(c, dst + 2 * gb, sh ? sh_down : src + 2 * gb, sh ? sh_down_type : down_type, true, tmp);
        if (rc) { cudaFree(tmp); return rc; }
        cudaStreamSynchronize(c->stream);
    }
    cudaFree(tmp);
    CK(cudaMemcpyAsync(L.router, router_w, sizeof(float) * (size_t)c->d.E * H, cudaMemcpyHostToDevice, c->stream));
    if (bias) CK(cudaMemcpyAsync(L.bias, bias, sizeof(float) * c->d.E, cudaMemcpyHostToDevice, c->stream));
    else CK(cudaMemsetAsync(L.bias, 0, sizeof(float) * c->d.E, c->stream));
    const int src = router_split(c, L);
    if (src) return src;
    CK(cudaStreamSynchronize(c->stream));
    return MOE_OK;
}

int moe_init_layer_synthetic(moe_ctx *c, int layer, uint64_t seed, int down_type, double w_sigma,
                             double router_sigma, double bias_sigma) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    int rc = layer_alloc(c, layer, down_type, down_type);
    if (rc) return rc;
    MoeLayerDev &L = c->layers[layer];
    const int H = c->d.H, I = c->d.I, E = c->d.E;
    uint8_t *tmp = nullptr;
    if (down_type == MOE_TYPE_Q6_K) CK(cudaMalloc((void **)&tmp, row_bytes(MOE_TYPE_Q6_K, I) * H));
    for (int j = 0; j <= c->n_local; j++) {
        uint8_t *dst = L.experts + (size_t)j * L.expert_stride;
        const int e = (j == c->n_local) ? E : c->e0 + j;
        moe_launch_synth_quant(MOE_TYPE_Q4_K, seed, synth_stream(layer, e, SYN_GATE), I, H, w_sigma, dst, c->stream,
                               &c->launches);
        moe_launch_synth_quant(MOE_TYPE_Q4_K, seed, synth_stream(layer, e, SYN_UP), I, H, w_sigma,
                               dst + L.gate_bytes, c->stream, &c->launches);
        moe_launch_q4_repack(dst, 2 * (size_t)I * (H / MOE_QK), c->stream, &c->launches);
        if (down_type == MOE_TYPE_Q6_K) {
            moe_launch_synth_quant(MOE_TYPE_Q6_K, seed, synth_stream(layer, e, SYN_DOWN), H, I, w_sigma, tmp,
                                   c->stream, &c->launches);
            moe_launch_q6_repack(tmp, dst + 2 * L.gate_bytes, H, I / MOE_QK, 0, c->stream, &c->launches);
        } else {
            moe_launch_synth_quant(MOE_TYPE_Q4_K, seed, synth_stream(layer, e, SYN_DOWN), H, I, w_sigma,
                                   dst + 2 * L.gate_bytes, c->stream, &c->launches);
            moe_launch_q4_repack(dst + 2 * L.gate_bytes, (size_t)H * (I / MOE_QK), c->stream, &c->launches);
        }
    }
    moe_launch_synth_f32(seed, synth_stream(layer, 0, SYN_ROUTER), (size_t)E * H, router_sigma, L.router, c->stream,
                         &c->launches);
    moe_launch_synth_f32(seed, synth_stream(layer, 0, SYN_BIAS), (size_t)E, bias_sigma, L.bias, c->stream,
                         &c->launches);
    CK(cudaGetLastError());
    const int src = router_split(c, L);
    const cudaError_t se = cudaStreamSynchronize(c->stream);
    if (tmp) cudaFree(tmp);
    if (src) return src;
    if (se != cudaSuccess) return fail(c, MOE_ERR_CUDA, "synthetic layer: %s", cudaGetErrorString(se));
    return MOE_OK;
}

int moe_add_router_bias(moe_ctx *c, int layer, const float *extra) {
    if (!c || !extra) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    if (layer < 0 || layer >= (int)c->layers.size() || !c->layers[layer].bias)
        return fail(c, MOE_ERR_STATE, "layer %d not loaded", layer);
    std::vector<float> b(c->d.E);
    CK(cudaMemcpy(b.data(), c->layers[layer].bias, sizeof(float) * c->d.E, cudaMemcpyDeviceToHost));
    for (int e = 0; e < c->d.E; e++) b[e] += extra[e];
    CK(upload_sync(c, c->layers[layer].bias, b.data(), sizeof(float) * c->d.E));
    return MOE_OK;
}

int moe_set_logit_bias(moe_ctx *c, int layer, const float *lb) {
    if (!c) return MOE_ERR_ARG;
    drop_graphs(c);  // the kernels take this layer's pointers by value
    if (layer < 0 || layer >= (int)c->layers.size() || !c->layers[layer].router)
        return fail(c, MOE_ERR_STATE, "layer %d not loaded", layer);
    DeviceScope ds(c->device);
    MoeLayerDev &L = c->layers[layer];
    if (!lb) {
        cudaFree(L.logit_bias);
        L.logit_bias = nullptr;
        return MOE_OK;
    }
    if (!L.logit_bias) CK(cudaMalloc((void **)&L.logit_bias, sizeof(float) * c->d.E));
    CK(upload_sync(c, L.logit_bias, lb, sizeof(float) * c->d.E));
    return MOE_OK;
}

int moe_set_norm_weight(moe_ctx *c, int layer, const float *w) {
    if (!c || !w) return MOE_ERR_ARG;
    drop_graphs(c);  // the kernels take this layer's pointers by value
    if (layer < 0 || layer >= (int)c->layers.size()) return fail(c, MOE_ERR_ARG, "layer %d out of range", layer);
    DeviceScope ds(c->device);
    MoeLayerDev &L = c->layers[layer];
    if (!L.norm) CK(cudaMalloc((void **)&L.norm, sizeof(float) * c->d.H));
    CK(upload_sync(c, L.norm, w, sizeof(float) * c->d.H));
    return MOE_OK;
}

// ------------------------------------------------------------ dense layers
static size_t type_bytes(int type, size_t n) {
    switch (type) {
    case MOE_TYPE_F32: return n * 4;
    case MOE_TYPE_F16:
    case MOE_TYPE_BF16: return n * 2;
    case MOE_TYPE_Q4_K: return n / MOE_QK * MOE_Q4K_BYTES;
    case MOE_TYPE_Q6_K: return n / MOE_QK * MOE_Q6K_BYTES;
    default: return 0;
    }
}

// fp16 storage and activation scratch of dense layer `layer`; frees the
// slot's MoE experts
static int dense_alloc(moe_ctx *c, int layer, int Id) {
    if (layer < 0 || layer >= (int)c->layers.size()) return fail(c, MOE_ERR_ARG, "layer %d out of range", layer);
    if (!moe_dense_shape_ok(c->d.H, Id))
        return fail(c, MOE_ERR_ARG, "dense FFN needs hidden %% 256 == 0, intermediate %% 256 == 0 and %zu bytes of "
                                    "activations per pass within shared memory (hidden %d, intermediate %d)",
                    moe_dense_smem_need(c->d.H, Id), c->d.H, Id);
    CK(cudaStreamSynchronize(c->stream));
    drop_graphs(c);
    MoeLayerDev &L = c->layers[layer];
    cudaFree(L.experts);
    L.experts = nullptr;
    moe_ctx::DenseDev &D = c->dense[layer];
    if (!D.w || D.Id != Id) {
        cudaFree(D.w);
        D.w = nullptr;
        CK(cudaMalloc((void **)&D.w, 3 * (size_t)Id * c->d.H * sizeof(__half)));
    }
    D.Id = Id;
    const size_t act_n = (size_t)c->max_tok * Id;
    if (act_n > c->dense_act_n) {
        cudaFree(c->dense_act);
        c->dense_act = nullptr;
        c->dense_act_n = 0;
        CK(cudaMalloc((void **)&c->dense_act, act_n * sizeof(float)));
        c->dense_act_n = act_n;
    }
    return MOE_OK;
}

int moe_load_dense_layer(moe_ctx *c, int layer, int Id, const void *gate, int gate_type, const void *up, int up_type,
                         const void *down, int down_type) {
    if (!c || !gate || !up || !down) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    const size_t n = (size_t)Id * c->d.H;
    const int types[3] = {gate_type, up_type, down_type};
    for (int t : types)
        if (!type_bytes(t, 256) || Id <= 0)
            return fail(c, MOE_ERR_ARG, "dense matrices must be F32 (0), F16 (1), BF16 (30), Q4_K (12) or Q6_K (14)");
    int rc = dense_alloc(c, layer, Id);
    if (rc) return rc;
    const void *src[3] = {gate, up, down};
    size_t raw = 0;
    bool quant = false;
    for (int t : types) {
        raw = std::max(raw, type_bytes(t, n));
        quant |= t == MOE_TYPE_Q4_K || t == MOE_TYPE_Q6_K;
    }
    uint8_t *tmp = nullptr;
    float *tf = nullptr;
    CK(cudaMalloc((void **)&tmp, raw));
    if (quant && cudaMalloc((void **)&tf, n * sizeof(float)) != cudaSuccess) {
        cudaFree(tmp);
        return fail(c, MOE_ERR_CUDA, "dense layer %d: no room for the dequant scratch", layer);
    }
    cudaError_t e = cudaSuccess;
    for (int m = 0; m < 3 && e == cudaSuccess; m++) {
        e = cudaMemcpyAsync(tmp, src[m], type_bytes(types[m], n), cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) {
            moe_launch_to_f16(types[m], tmp, c->dense[layer].w + m * n, n, tf, c->stream, &c->launches);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);  // tmp is reused by the next matrix
    }
    cudaFree(tmp);
    cudaFree(tf);
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "dense layer %d: %s", layer, cudaGetErrorString(e));
    return MOE_OK;
}

int moe_init_dense_synthetic(moe_ctx *c, int layer, int Id, uint64_t seed, double w_sigma) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    int rc = dense_alloc(c, layer, Id);
    if (rc) return rc;
    const size_t n = (size_t)Id * c->d.H;
    float *tf = nullptr;
    CK(cudaMalloc((void **)&tf, n * sizeof(float)));
    const int kinds[3] = {SYN_GATE, SYN_UP, SYN_DOWN};
    cudaError_t e = cudaSuccess;
    for (int m = 0; m < 3 && e == cudaSuccess; m++) {
        moe_launch_synth_f32(seed, synth_stream(layer, c->d.E + 1, kinds[m]), n, w_sigma, tf, c->stream,
                             &c->launches);
        moe_launch_to_f16(MOE_TYPE_F32, tf, c->dense[layer].w + m * n, n, nullptr, c->stream, &c->launches);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tf);
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "synthetic dense layer %d: %s", layer, cudaGetErrorString(e));
    return MOE_OK;
}

static int check_dense(moe_ctx *c, int layer) {
    if (layer < 0 || layer >= (int)c->dense.size() || !c->dense[layer].w)
        return fail(c, MOE_ERR_STATE, "dense layer %d not loaded", layer);
    return MOE_OK;
}

int moe_read_dense_weight(moe_ctx *c, int layer, int which, void *dst, size_t dst_size) {
    if (!c || !dst || which < 0 || which > 2) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    int rc = check_dense(c, layer);
    if (rc) return rc;
    const size_t n = (size_t)c->dense[layer].Id * c->d.H;
    if (dst_size < n * sizeof(__half)) return fail(c, MOE_ERR_ARG, "dst_size %zu < %zu", dst_size, n * 2);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(dst, c->dense[layer].w + which * n, n * sizeof(__half), cudaMemcpyDeviceToHost));
    return MOE_OK;
}

// ---------------------------------------------------------- output head
// sampling scratch for rows of n values: logits and probabilities [max_tok x n]
static int sample_scratch(moe_ctx *c, int n) {
    if ((size_t)n <= c->sample_n) return MOE_OK;
    cudaFree(c->head_logits);
    cudaFree(c->sample_p);
    cudaFree(c->sample_tok);
    c->head_logits = c->sample_p = nullptr;
    c->sample_tok = nullptr;
    c->sample_n = 0;
    const size_t m = (size_t)c->max_tok * n;
    CK(cudaMalloc((void **)&c->head_logits, m * sizeof(float)));
    CK(cudaMalloc((void **)&c->sample_p, m * sizeof(float)));
    CK(cudaMalloc((void **)&c->sample_tok, c->max_tok * sizeof(int)));
    if (!c->sample_ws) CK(cudaMalloc(&c->sample_ws, moe_sample_ws_bytes(c->max_tok)));
    c->sample_n = n;
    return MOE_OK;
}

static int head_alloc(moe_ctx *c, int vocab) {
    if (vocab <= 0 || c->d.H % 256) return fail(c, MOE_ERR_ARG, "lm_head needs vocab > 0 and hidden %% 256 == 0");
    CK(cudaStreamSynchronize(c->stream));
    drop_graphs(c);
    if (!c->head_w || c->vocab != vocab) {
        cudaFree(c->head_w);
        c->head_w = nullptr;
        c->vocab = 0;
        CK(cudaMalloc((void **)&c->head_w, (size_t)vocab * c->d.H * sizeof(__half)));
    }
    c->vocab = vocab;
    return sample_scratch(c, vocab);
}

int moe_load_lm_head(moe_ctx *c, int vocab, const void *w, int type) {
    if (!c || !w) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    const size_t n = (size_t)vocab * c->d.H;
    if (!type_bytes(type, 256) || vocab <= 0)
        return fail(c, MOE_ERR_ARG, "lm_head must be F32 (0), F16 (1), BF16 (30), Q4_K (12) or Q6_K (14)");
    int rc = head_alloc(c, vocab);
    if (rc) return rc;
    const bool quant = type == MOE_TYPE_Q4_K || type == MOE_TYPE_Q6_K;
    uint8_t *tmp = nullptr;
    float *tf = nullptr;
    CK(cudaMalloc((void **)&tmp, type_bytes(type, n)));
    if (quant && cudaMalloc((void **)&tf, n * sizeof(float)) != cudaSuccess) {
        cudaFree(tmp);
        return fail(c, MOE_ERR_CUDA, "lm_head: no room for the dequant scratch");
    }
    cudaError_t e = cudaMemcpyAsync(tmp, w, type_bytes(type, n), cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        moe_launch_to_f16(type, tmp, c->head_w, n, tf, c->stream, &c->launches);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    cudaFree(tf);
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "lm_head: %s", cudaGetErrorString(e));
    return MOE_OK;
}

int moe_init_lm_head_synthetic(moe_ctx *c, int vocab, uint64_t seed, double w_sigma) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    int rc = head_alloc(c, vocab);
    if (rc) return rc;
    const size_t n = (size_t)vocab * c->d.H;
    float *tf = nullptr;
    CK(cudaMalloc((void **)&tf, n * sizeof(float)));
    moe_launch_synth_f32(seed, synth_stream(0, c->d.E + 2, SYN_GATE), n, w_sigma, tf, c->stream, &c->launches);
    moe_launch_to_f16(MOE_TYPE_F32, tf, c->head_w, n, nullptr, c->stream, &c->launches);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tf);
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "synthetic lm_head: %s", cudaGetErrorString(e));
    return MOE_OK;
}

int moe_read_lm_head(moe_ctx *c, void *dst, size_t dst_size) {
    if (!c || !dst) return MOE_ERR_ARG;
    if (!c->head_w) return fail(c, MOE_ERR_STATE, "lm_head not loaded");
    DeviceScope ds(c->device);
    const size_t bytes = (size_t)c->vocab * c->d.H * sizeof(__half);
    if (dst_size < bytes) return fail(c, MOE_ERR_ARG, "dst_size %zu < %zu", dst_size, bytes);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(dst, c->head_w, bytes, cudaMemcpyDeviceToHost));
    return MOE_OK;
}

size_t moe_expert_bytes(const moe_ctx *c, int layer) {
    if (!c || layer < 0 || layer >= (int)c->layers.size() || !c->layers[layer].experts) return 0;
    return 2 * c->layers[layer].gate_bytes + c->layer_down_bytes[layer];
}

int moe_read_expert(moe_ctx *c, int layer, int expert, void *dst, size_t dst_size) {
    if (!c || !dst) return MOE_ERR_ARG;
    if (layer < 0 || layer >= (int)c->layers.size() || !c->layers[layer].experts)
        return fail(c, MOE_ERR_STATE, "layer %d not loaded", layer);
    MoeLayerDev &L = c->layers[layer];
    int j;
    if (expert == c->d.E) j = c->n_local;
    else if (expert >= c->e0 && expert < c->e0 + c->n_local) j = expert - c->e0;
    else return fail(c, MOE_ERR_ARG, "expert %d not held by rank %d", expert, c->rank);
    const int ty = expert == c->d.E ? L.sh_down_type : L.down_type;
    const size_t db = row_bytes(ty, c->d.I) * c->d.H;
    if (dst_size < 2 * L.gate_bytes + db) return fail(c, MOE_ERR_ARG, "moe_read_expert: buffer too small");
    DeviceScope ds(c->device);
    const uint8_t *src = L.experts + (size_t)j * L.expert_stride;
    // undo the load-time repacks in a device copy: Q4_K qs transpose (its
    // own inverse) of gate, up and a Q4_K down; Q6_K planes -> GGUF blocks
    uint8_t *tmp = nullptr;
    const size_t total = 2 * L.gate_bytes + db;
    CK(cudaMalloc((void **)&tmp, total));
    cudaError_t e1 = cudaMemcpyAsync(tmp, src, 2 * L.gate_bytes, cudaMemcpyDeviceToDevice, c->stream);
    moe_launch_q4_repack(tmp, 2 * (size_t)c->d.I * (c->d.H / MOE_QK), c->stream, &c->launches);
    if (ty == MOE_TYPE_Q4_K) {
        if (e1 == cudaSuccess)
            e1 = cudaMemcpyAsync(tmp + 2 * L.gate_bytes, src + 2 * L.gate_bytes, db, cudaMemcpyDeviceToDevice,
                                 c->stream);
        moe_launch_q4_repack(tmp + 2 * L.gate_bytes, (size_t)c->d.H * (c->d.I / MOE_QK), c->stream, &c->launches);
    } else {
        moe_launch_q6_repack(src + 2 * L.gate_bytes, tmp + 2 * L.gate_bytes, c->d.H, c->d.I / MOE_QK, 1, c->stream,
                             &c->launches);
    }
    cudaError_t e2 = cudaStreamSynchronize(c->stream);
    cudaError_t e3 = cudaMemcpy(dst, tmp, total, cudaMemcpyDeviceToHost);
    cudaFree(tmp);
    if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess)
        return fail(c, MOE_ERR_CUDA, "moe_read_expert: unpack failed");
    return MOE_OK;
}

int moe_write_layer_packed(moe_ctx *c, int layer, const char *path) {
    if (!c || !path) return MOE_ERR_ARG;
    if (layer < 0 || layer >= (int)c->layers.size() || !c->layers[layer].experts)
        return fail(c, MOE_ERR_STATE, "layer %d not loaded", layer);
    const size_t es = moe_expert_bytes(c, layer);
    FILE *f = fopen(path, "r+b");
    if (!f) f = fopen(path, "w+b");
    if (!f) return fail(c, MOE_ERR_ARG, "moe_write_layer_packed: cannot open %s", path);
    std::vector<uint8_t> buf(es);
    int rc = MOE_OK;
    // the file holds all n_experts experts (a rank writes only its own range)
    if (fseeko(f, (off_t)((size_t)c->d.E * es) - 1, SEEK_SET) != 0 || fgetc(f) == EOF) {
        if (fseeko(f, (off_t)((size_t)c->d.E * es) - 1, SEEK_SET) != 0 || fputc(0, f) == EOF)
            rc = fail(c, MOE_ERR_ARG, "moe_write_layer_packed: cannot size %s", path);
    }
    for (int j = 0; j < c->n_local && rc == MOE_OK; j++) {
        const int e = c->e0 + j;
        rc = moe_read_expert(c, layer, e, buf.data(), es);
        if (rc == MOE_OK && (fseeko(f, (off_t)((size_t)e * es), SEEK_SET) != 0 || fwrite(buf.data(), 1, es, f) != es))
            rc = fail(c, MOE_ERR_ARG, "moe_write_layer_packed: write to %s failed", path);
    }
    if (fclose(f) != 0 && rc == MOE_OK) rc = fail(c, MOE_ERR_ARG, "moe_write_layer_packed: closing %s failed", path);
    return rc;
}

// ------------------------------------------------------------------ forward
// records the boundary before phase `ph` (MOE_N_PHASES = end of the step)
static void mark(moe_ctx *c, int ph, cudaStream_t s) {
    if (!c->timing) return;
    const size_t i = (size_t)c->ring_pos * (MOE_N_PHASES + 1) + ph;
    cudaEventRecord(c->ev[i], s);
    c->ev_valid[i] = 1;
}
static void mark_begin(moe_ctx *c) {
    if (!c->timing) return;
    c->ring_pos = (c->ring_pos + 1) % c->ring;
    if (c->ring_used < c->ring) c->ring_used++;
    for (int p = 0; p <= MOE_N_PHASES; p++) c->ev_valid[(size_t)c->ring_pos * (MOE_N_PHASES + 1) + p] = 0;
}

static int check_layer(moe_ctx *c, int layer) {
    if (layer < 0 || layer >= (int)c->layers.size() || !c->layers[layer].experts)
        return fail(c, MOE_ERR_STATE, "layer %d not loaded", layer);
    return MOE_OK;
}

// Router logits of T tokens into c->logits: the SIMT router for up to
// MOE_ROUTER_SIMT_T tokens (one pass over the fp32 rows), else the tensor-core
// router on the layer's kept hi / lo split (fp32 accuracy, ~3x fewer
// microseconds at 64 tokens).
static void launch_router(moe_ctx *c, const MoeLayerDev &L, const float *x, int T, cudaStream_t s) {
    const MoeDims &d = c->d;
    if (T > MOE_ROUTER_SIMT_T && L.rwh && c->rxh)
        moe_launch_router_tc(d, L.tm_rwh, L.tm_rwl, x, T, c->rxh, c->rxl, c->tm_rxh, c->tm_rxl, c->part, c->n_split,
                             c->logits, c->plan.error, s, &c->launches);
    else
        moe_launch_router_logits(L.router, x, T, d.H, d.E, c->part, c->n_split, c->logits, c->rl_counters, s,
                                 &c->launches);
}

// experts + combine over the activation rows in `x` (rows = tokens on one GPU)
static int run_local(moe_ctx *c, int layer, const float *x, int T, const int *idx_in, const float *w_in,
                     int routed, int with_shared, const float *residual, float *out, cudaStream_t s) {
    MoeLayerDev &L = c->layers[layer];
    const MoeDims &d = c->d;
    const int mode = !routed ? 2 : (idx_in ? 1 : 0);
    mark_begin(c);
    mark(c, MOE_PHASE_ROUTER, s);
    if (mode == 0) launch_router(c, L, x, T, s);
    mark(c, MOE_PHASE_ROUTE, s);
    moe_launch_route_and_plan(d, nullptr, 0, c->logits, L.bias, L.logit_bias, mode, idx_in, w_in, T, c->idx, c->wts,
                              x, c->xop, with_shared, 1, c->plan, c->counter, s, &c->launches);
    // a chunk holds at least one pair (the GEMV grids are sized by this bound)
    const int max_chunks = std::min(T * d.K + T, (T * d.K + T + MOE_TC - 1) / MOE_TC + d.E + 1);
    // an expert gets at most T tokens: with more than MOE_TC there can be
    // tcgen05 chunks
    const bool tc = d.tc && T > MOE_TC;
    const int P = T * d.K + T;
    mark(c, MOE_PHASE_GATEUP_TC, s);
    if (tc) {
        moe_launch_tc_gather(d, c->plan, c->xop, c->xtc, P, s, &c->launches);
        moe_launch_gateup_tc(d, L, c->plan, c->tm_xtc, c->act, P, s, &c->launches);
    }
    mark(c, MOE_PHASE_GATEUP, s);
    moe_launch_gateup(d, L, c->plan, c->xop, c->act,
                      max_chunks, s, &c->launches);
    mark(c, MOE_PHASE_PREP, s);
    moe_launch_prep_down(d, L, c->plan, c->act, c->dop, P, s, &c->launches);
    mark(c, MOE_PHASE_DOWN_TC, s);
    if (tc) moe_launch_down_tc(d, L, c->plan, c->tm_dop, c->eo, P, s, &c->launches);
    mark(c, MOE_PHASE_DOWN, s);
    moe_launch_down(d, L, c->plan, c->dop, c->eo, max_chunks, s, &c->launches);
    mark(c, MOE_PHASE_OUTPUT, s);
    moe_launch_combine(d, c->plan, c->eo, T, routed, with_shared, residual, out, s, &c->launches);
    mark(c, MOE_N_PHASES, s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
    c->last_layer = layer;
    return MOE_OK;
}

// Expert-parallel step: route local tokens, dispatch rows to the ranks that
// own their experts, run the local experts on received rows (+ shared expert
// on local rows), pre-combine per row, return the partials, sum them in rank
// order.
static int run_ep(moe_ctx *c, int layer, const float *x, int T, const int *idx_in, const float *w_in,
                  const float *residual, float *out, cudaStream_t s) {
    MoeLayerDev &L = c->layers[layer];
    const MoeDims &d = c->d;
    const int N = c->world, cap = c->max_tok, R = N * cap, mw = 2 + 2 * d.K;
    const int mode = idx_in ? 1 : 0;
    if (c->comm_aborted) return fail(c, MOE_ERR_STATE, "an exchange failed and the communicator was aborted");
    if (c->ep_failed)
        return fail(c, MOE_ERR_STATE, "a peer exchange timed out earlier; the ranks are out of step (recreate the context)");
    mark_begin(c);
    mark(c, MOE_PHASE_ROUTER, s);
    if (mode == 0 && T > 0) launch_router(c, L, x, T, s);
    mark(c, MOE_PHASE_ROUTE, s);
    if (T > 0)
        moe_launch_route_and_plan(d, nullptr, 0, c->logits, L.bias, L.logit_bias, mode, idx_in, w_in, T, c->idx,
                                  c->wts, x, nullptr, 0, 0, c->plan, c->counter, s, &c->launches);
    mark(c, MOE_PHASE_DISPATCH, s);
    const int P = R * d.K + T;
    const int max_chunks = std::min(P, (P + MOE_TC - 1) / MOE_TC + d.E + 1);
    // a routed expert gets at most R received rows, the shared one T local rows
    const bool tc = d.tc && (R > MOE_TC || T > MOE_TC);
    if (c->p2p) {
        // peer-memory exchange: no host step in between, the step number
        // lives on the device (the launches replay as a graph)
        const EpP2P q{c->d_peers, c->mb_x, c->mb_meta, c->mb_y, N, c->rank, c->d_seq, c->ep_done, c->plan.error};
        moe_launch_ep_pack_p2p(x, c->idx, c->wts, T, d.K, d.H, c->n_local, cap, q, c->tok_slot, s, &c->launches);
        moe_launch_ep_plan_rows_p2p(d, q, cap, T, c->e0, c->n_local, c->plan, x, c->xop, s, &c->launches);
        mark(c, MOE_PHASE_GATEUP_TC, s);
        if (tc) {
            moe_launch_tc_gather(d, c->plan, c->xop, c->xtc, P, s, &c->launches);
            moe_launch_gateup_tc(d, L, c->plan, c->tm_xtc, c->act, P, s, &c->launches);
        }
        mark(c, MOE_PHASE_GATEUP, s);
        moe_launch_gateup(d, L, c->plan, c->xop, c->act, max_chunks, s, &c->launches);
        mark(c, MOE_PHASE_PREP, s);
        moe_launch_prep_down(d, L, c->plan, c->act, c->dop, P, s, &c->launches);
        mark(c, MOE_PHASE_DOWN_TC, s);
        if (tc) moe_launch_down_tc(d, L, c->plan, c->tm_dop, c->eo, P, s, &c->launches);
        mark(c, MOE_PHASE_DOWN, s);
        moe_launch_down(d, L, c->plan, c->dop, c->eo, max_chunks, s, &c->launches);
        mark(c, MOE_PHASE_COMBINE, s);
        moe_launch_ep_partial_p2p(d, c->plan, c->eo, cap, q, s, &c->launches);
        moe_launch_ep_final_p2p(d, c->plan, q, c->tok_slot, cap, T, c->eo, residual, out, s, &c->launches);
        mark(c, MOE_PHASE_OUTPUT, s);
        mark(c, MOE_N_PHASES, s);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
        c->last_layer = layer;
        return MOE_OK;
    }
    {
        moe_launch_ep_pack(x, c->idx, c->wts, T, d.K, d.H, N, c->n_local, cap, c->send_x, c->send_meta, c->tok_slot,
                           s, &c->launches);
        NK(moe_nccl()->GroupStart());
        for (int p = 0; p < N; p++) {
            NK(moe_nccl()->Send(c->send_x + (size_t)p * cap * d.H, (size_t)cap * d.H, ncclFloat32, p, c->comm, s));
            NK(moe_nccl()->Recv(c->recv_x + (size_t)p * cap * d.H, (size_t)cap * d.H, ncclFloat32, p, c->comm, s));
            NK(moe_nccl()->Send(c->send_meta + (size_t)p * cap * mw, (size_t)cap * mw, ncclInt32, p, c->comm, s));
            NK(moe_nccl()->Recv(c->recv_meta + (size_t)p * cap * mw, (size_t)cap * mw, ncclInt32, p, c->comm, s));
        }
        NK(moe_nccl()->GroupEnd());
    }
    moe_launch_ep_plan(d, c->recv_meta, N, cap, T, c->e0, c->n_local, c->plan, s, &c->launches);
    moe_launch_prep_rows(c->recv_x, c->recv_meta, mw, R, x, T, d.H, c->xop, s, &c->launches);
    mark(c, MOE_PHASE_GATEUP_TC, s);
    if (tc) {
        moe_launch_tc_gather(d, c->plan, c->xop, c->xtc, P, s, &c->launches);
        moe_launch_gateup_tc(d, L, c->plan, c->tm_xtc, c->act, P, s, &c->launches);
    }
    mark(c, MOE_PHASE_GATEUP, s);
    moe_launch_gateup(d, L, c->plan, c->xop, c->act,
                      max_chunks, s, &c->launches);
    mark(c, MOE_PHASE_PREP, s);
    moe_launch_prep_down(d, L, c->plan, c->act, c->dop, P, s, &c->launches);
    mark(c, MOE_PHASE_DOWN_TC, s);
    if (tc) moe_launch_down_tc(d, L, c->plan, c->tm_dop, c->eo, P, s, &c->launches);
    mark(c, MOE_PHASE_DOWN, s);
    moe_launch_down(d, L, c->plan, c->dop, c->eo, max_chunks, s, &c->launches);
    mark(c, MOE_PHASE_COMBINE, s);
    {
        moe_launch_ep_partial(d, c->plan, c->recv_meta, c->eo, R, c->send_y, s, &c->launches);
        NK(moe_nccl()->GroupStart());
        for (int p = 0; p < N; p++) {
            NK(moe_nccl()->Send(c->send_y + (size_t)p * cap * d.H, (size_t)cap * d.H, ncclFloat32, p, c->comm, s));
            NK(moe_nccl()->Recv(c->recv_y + (size_t)p * cap * d.H, (size_t)cap * d.H, ncclFloat32, p, c->comm, s));
        }
        NK(moe_nccl()->GroupEnd());
    }
    mark(c, MOE_PHASE_OUTPUT, s);
    if (T > 0)
        moe_launch_ep_final(d, c->plan, c->recv_y, c->tok_slot, N, cap, T, c->eo, residual, out, s, &c->launches);
    mark(c, MOE_N_PHASES, s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
    c->last_layer = layer;
    return MOE_OK;
}

// Runs `body` (a sequence of launches on stream s) as a CUDA graph: a
// signature seen before is replayed (captured on its second call, when every
// kernel attribute is already set).  Direct launches while the per-phase
// timing ring is on, when the caller is capturing the stream itself, or on
// the NCCL exchange path.  On the expert-parallel peer-memory path every
// rank makes the same calls, so every rank captures and replays the same
// sequences; the step number the kernels need is in device memory.
}  // extern "C"
template <typename F>
static int run_graphed(moe_ctx *c, const moe_ctx::GraphSig &sig, cudaStream_t s, F &&body) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (!c->use_graphs || c->timing || (c->world > 1 && !c->p2p) || cudaStreamIsCapturing(s, &cs) != cudaSuccess ||
        cs != cudaStreamCaptureStatusNone)
        return body();
    c->clock++;
    for (auto &g : c->graphs)
        if (g.sig == sig) {
            g.last_use = c->clock;
            CK(cudaGraphLaunch(g.exec, s));
            c->launches += g.kernels;
            return MOE_OK;
        }
    bool seen = false;
    for (auto &x : c->seen) seen = seen || x == sig;
    if (!seen) {  // first call: run directly (sets kernel attributes)
        if (c->seen.size() > 64) c->seen.erase(c->seen.begin());
        c->seen.push_back(sig);
        return body();
    }
    const uint64_t k0 = c->launches;
    CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    const int rc = body();
    cudaGraph_t graph = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(s, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (ec != cudaSuccess || !graph) return fail(c, MOE_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ec));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ei != cudaSuccess) return fail(c, MOE_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ei));
    if (c->graphs.size() >= 32) {  // drop the least recently used
        size_t lru = 0;
        for (size_t i = 1; i < c->graphs.size(); i++)
            if (c->graphs[i].last_use < c->graphs[lru].last_use) lru = i;
        cudaGraphExecDestroy(c->graphs[lru].exec);
        c->graphs.erase(c->graphs.begin() + lru);
    }
    c->graphs.push_back({sig, exec, c->launches - k0, c->clock});
    CK(cudaGraphLaunch(exec, s));
    return MOE_OK;
}

extern "C" {

// an expert-parallel context refuses work after a failed exchange (checked
// on the host before any launch, graph replays included)
static int ep_usable(moe_ctx *c) {
    if (c->world == 1) return MOE_OK;
    if (c->comm_aborted) return fail(c, MOE_ERR_STATE, "an exchange failed and the communicator was aborted");
    if (c->ep_failed)
        return fail(c, MOE_ERR_STATE, "a peer exchange timed out earlier; the ranks are out of step (recreate the context)");
    return MOE_OK;
}

// d_hits[layer] = routed experts of this rank hit by the layer that just ran
// (plan count 2), or 0 when the layer did not run here.
static int record_hits(moe_ctx *c, int layer, bool ran, cudaStream_t s) {
    if (!c->hits) return MOE_OK;
    if (ran) CK(cudaMemcpyAsync(c->hits + layer, c->plan.counts + 2, sizeof(int), cudaMemcpyDeviceToDevice, s));
    else CK(cudaMemsetAsync(c->hits + layer, 0, sizeof(int), s));
    return MOE_OK;
}

int moe_ep_peer_memory(const moe_ctx *c) { return c && c->p2p ? 1 : 0; }

int moe_record_expert_hits(moe_ctx *c, int *d_hits) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    drop_graphs(c);
    c->hits = d_hits;
    return MOE_OK;
}

int moe_forward_device(moe_ctx *c, int layer, const float *d_h, int T, float *d_out, int *d_idx, float *d_w,
                       void *stream) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    if (T > 0 && (!d_h || !d_out)) return fail(c, MOE_ERR_ARG, "moe_forward_device: null input or output");
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    rc = ep_usable(c);
    if (rc) return rc;
    if (c->world == 1 && T == 0) return record_hits(c, layer, false, s);
    // every rank of an expert-parallel context joins, even with T == 0
    const moe_ctx::GraphSig sig{0, layer, 0, T, d_h, d_out, s};
    rc = run_graphed(c, sig, s, [&]() {
        return c->world > 1 ? run_ep(c, layer, d_h, T, nullptr, nullptr, nullptr, d_out, s)
                            : run_local(c, layer, d_h, T, nullptr, nullptr, 1, 1, nullptr, d_out, s);
    });
    if (rc) return rc;
    if (d_idx) CK(cudaMemcpyAsync(d_idx, c->idx, sizeof(int) * T * c->d.K, cudaMemcpyDeviceToDevice, s));
    if (d_w) CK(cudaMemcpyAsync(d_w, c->wts, sizeof(float) * T * c->d.K, cudaMemcpyDeviceToDevice, s));
    return record_hits(c, layer, true, s);
}

// Host wait for stream s.  A step that ran NCCL (the expert-parallel
// prefill, or the decode exchange when the peers could not be mapped) has no
// bounded wait of its own, so the host polls the communicator's
// asynchronous error while it waits and gives up after MOE_EP_TIMEOUT_S
// seconds (default 120): the communicator is then aborted, which ends its
// kernels, and the context answers every later call with an error.
static int stream_wait(moe_ctx *c, cudaStream_t s, bool nccl_in_step) {
    if (!nccl_in_step || !c->comm) {
        CK(cudaStreamSynchronize(s));
        return MOE_OK;
    }
    const char *env = getenv("MOE_EP_TIMEOUT_S");
    const double limit = env && atof(env) > 0 ? atof(env) : 120.0;
    cudaError_t qerr = cudaSuccess;
    ncclResult_t ae = ncclSuccess;
    const MoeWaitOutcome o = moe_wait_poll(
        [&]() {
            qerr = cudaStreamQuery(s);
            return qerr == cudaSuccess ? 0 : qerr == cudaErrorNotReady ? 1 : 2;
        },
        [&]() {
            return moe_nccl()->CommGetAsyncError(c->comm, &ae) == ncclSuccess && ae != ncclSuccess &&
                   ae != ncclInProgress;
        },
        [&]() {
            moe_nccl()->CommAbort(c->comm);
            c->comm = nullptr;
            c->comm_aborted = true;
        },
        limit);
    switch (o) {
        case MOE_WAIT_DONE: return MOE_OK;
        case MOE_WAIT_STREAM_ERROR: return fail(c, MOE_ERR_CUDA, "stream wait: %s", cudaGetErrorString(qerr));
        case MOE_WAIT_NCCL_ERROR:
            return fail(c, MOE_ERR_NCCL, "NCCL error during the exchange: %s; communicator aborted",
                        moe_nccl()->GetErrorString(ae));
        default:
            return fail(c, MOE_ERR_NCCL,
                        "exchange did not finish within %.0f s (a peer rank stopped calling); communicator aborted",
                        limit);
    }
}

// Reads and clears the device error words that the kernels set (decode plan
// and prefill plan) once the context stream has finished.  A peer-exchange
// timeout leaves the ranks out of step (the step numbers have advanced on
// this rank), so it also marks the context: every later expert-parallel
// call is refused.
static int take_device_error(moe_ctx *c) {
    int err[2] = {0, 0};
    CK(cudaMemcpy(&err[0], c->plan.error, sizeof(int), cudaMemcpyDeviceToHost));
    if (c->pf.plan.error) CK(cudaMemcpy(&err[1], c->pf.plan.error, sizeof(int), cudaMemcpyDeviceToHost));
    for (int i = 0; i < 2; i++) {
        const int e = err[i];
        if (!e) continue;
        // cleared before the next call's kernels (on any stream) can set it again
        if (zero_async(c, i == 0 ? c->plan.error : c->pf.plan.error, sizeof(int)) == cudaSuccess)
            cudaStreamSynchronize(c->stream);
        if (e == EP_ERR_TIMEOUT) {
            c->ep_failed = true;
            return fail(c, MOE_ERR_TIMEOUT, "peer exchange wait timed out (a peer rank stopped calling)");
        }
        if (e == EX_ERR_TIMEOUT) return fail(c, MOE_ERR_TIMEOUT, "expert pipeline wait timed out");
        if (e == PF_ERR_TIMEOUT) return fail(c, MOE_ERR_TIMEOUT, "prefill pipeline wait timed out");
        if (e == PF_ERR_PAIR) return fail(c, MOE_ERR_CUDA, "prefill CTA pair: tensor-memory allocations differ");
        if (e == MOE_DEV_ERR_INDEX) return fail(c, MOE_ERR_ARG, "expert index out of range in routing");
        return fail(c, MOE_ERR_CUDA, "device error code 0x%x", e);
    }
    return MOE_OK;
}

// True when the decode step's exchange runs over NCCL (no bounded wait).
static bool step_uses_nccl(const moe_ctx *c) { return c->world > 1 && !c->p2p; }

// Copies device results into caller memory.  When the step ran NCCL
// kernels, the host first waits with the polling wait: a copy into pageable
// memory returns only when the stream has drained, so a peer that stopped
// calling would otherwise block the host inside the copy with no limit.
struct HostCopy {
    void *dst;
    const void *src;
    size_t bytes;
};
static int copy_out(moe_ctx *c, cudaStream_t s, bool nccl_in_step, std::initializer_list<HostCopy> cps) {
    if (nccl_in_step) {
        const int rc = stream_wait(c, s, true);
        if (rc) return rc;
        for (const HostCopy &h : cps)
            if (h.dst && h.bytes) CK(cudaMemcpy(h.dst, h.src, h.bytes, cudaMemcpyDeviceToHost));
        return MOE_OK;
    }
    for (const HostCopy &h : cps)
        if (h.dst && h.bytes) CK(cudaMemcpyAsync(h.dst, h.src, h.bytes, cudaMemcpyDeviceToHost, s));
    return MOE_OK;
}

static int finish_sync(moe_ctx *c) {
    {
        const int rc = stream_wait(c, c->stream, step_uses_nccl(c));
        if (rc) return rc;
    }
    return take_device_error(c);
}

int moe_check_error(moe_ctx *c) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    return finish_sync(c);
}

int moe_forward(moe_ctx *c, int layer, const float *h, int T, float *out, int *idx_out, float *w_out) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && (!h || !out)) return fail(c, MOE_ERR_ARG, "moe_forward: null input or output");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    DeviceScope ds(c->device);
    const size_t n = (size_t)T * c->d.H;
    if (n) CK(cudaMemcpyAsync(c->d_in, h, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    int rc = moe_forward_device(c, layer, c->d_in, T, c->d_out, nullptr, nullptr, nullptr);
    if (rc) return rc;
    if (n == 0) return finish_sync(c);
    rc = copy_out(c, c->stream, step_uses_nccl(c),
                  {{out, c->d_out, n * sizeof(float)},
                   {idx_out, c->idx, sizeof(int) * T * c->d.K},
                   {w_out, c->wts, sizeof(float) * T * c->d.K}});
    if (rc) return rc;
    return finish_sync(c);
}

int moe_experts_forward_device(moe_ctx *c, int layer, const float *d_h, int T, const int *d_idx, const float *d_w,
                               int K, float *d_out, void *stream) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    if (T > 0 && (!d_h || !d_idx || !d_w || !d_out))
        return fail(c, MOE_ERR_ARG, "moe_experts_forward_device: null pointer");
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (K != c->d.K) return fail(c, MOE_ERR_ARG, "K %d differs from the context's top_k %d", K, c->d.K);
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    if (c->world > 1) return fail(c, MOE_ERR_STATE, "moe_experts_forward is single-GPU (the shared expert is "
                                                     "always added on the expert-parallel path)");
    if (T == 0) return MOE_OK;
    return run_local(c, layer, d_h, T, d_idx, d_w, 1, 0, nullptr, d_out, s);
}

int moe_experts_forward(moe_ctx *c, int layer, const float *h, int T, const int *idx, const float *w, int K,
                        float *out) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && (!h || !idx || !w || !out)) return fail(c, MOE_ERR_ARG, "moe_experts_forward: null pointer");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (K != c->d.K) return fail(c, MOE_ERR_ARG, "K %d differs from the context's top_k %d", K, c->d.K);
    for (int i = 0; i < T * K; i++)
        if (idx[i] < 0 || idx[i] >= c->d.E) return fail(c, MOE_ERR_ARG, "expert index %d out of range", idx[i]);
    DeviceScope ds(c->device);
    const size_t n = (size_t)T * c->d.H;
    CK(cudaMemcpyAsync(c->d_in, h, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->idx_given, idx, sizeof(int) * T * K, cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->w_given, w, sizeof(float) * T * K, cudaMemcpyHostToDevice, c->stream));
    int rc = moe_experts_forward_device(c, layer, c->d_in, T, c->idx_given, c->w_given, K, c->d_out, nullptr);
    if (rc) return rc;
    CK(cudaMemcpyAsync(out, c->d_out, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    return finish_sync(c);
}

int moe_shared_forward(moe_ctx *c, int layer, const float *h, int T, float *sd) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && (!h || !sd)) return fail(c, MOE_ERR_ARG, "moe_shared_forward: null pointer");
    int rc = check_layer(c, layer);
    if (rc) return rc;
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (T == 0) return MOE_OK;
    DeviceScope ds(c->device);
    const size_t n = (size_t)T * c->d.H;
    CK(cudaMemcpyAsync(c->d_in, h, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    // shared only: routed slots are empty (routing given as "none")
    rc = run_local(c, layer, c->d_in, T, nullptr, nullptr, 0, 1, nullptr, c->d_out, c->stream);
    if (rc) return rc;
    CK(cudaMemcpyAsync(sd, c->d_out, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    return finish_sync(c);
}

int moe_dense_forward_device(moe_ctx *c, int layer, const float *d_h, int T, float *d_out, void *stream) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    int rc = check_dense(c, layer);
    if (rc) return rc;
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (T > 0 && (!d_h || !d_out || ((uintptr_t)d_h & 15) || ((uintptr_t)d_out & 15)))
        return fail(c, MOE_ERR_ARG, "moe_dense_forward_device: null or not 16-byte aligned buffer");
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    const moe_ctx::DenseDev &D = c->dense[layer];
    moe_launch_dense_ffn(D.w, c->d.H, D.Id, d_h, T, c->dense_act, nullptr, d_out, s, &c->launches);
    CK(cudaGetLastError());
    return MOE_OK;
}

int moe_dense_forward(moe_ctx *c, int layer, const float *h, int T, float *out) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && (!h || !out)) return fail(c, MOE_ERR_ARG, "moe_dense_forward: null pointer");
    int rc = check_dense(c, layer);
    if (rc) return rc;
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (T == 0) return MOE_OK;
    DeviceScope ds(c->device);
    const size_t n = (size_t)T * c->d.H;
    CK(cudaMemcpyAsync(c->d_in, h, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    rc = moe_dense_forward_device(c, layer, c->d_in, T, c->d_out, c->stream);
    if (rc) return rc;
    rc = copy_out(c, c->stream, false, {{out, c->d_out, n * sizeof(float)}});
    if (rc) return rc;
    return finish_sync(c);
}

int moe_lm_head_device(moe_ctx *c, const float *d_h, int T, float *d_logits, void *stream) {
    if (!c) return MOE_ERR_ARG;
    if (!c->head_w) return fail(c, MOE_ERR_STATE, "lm_head not loaded");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (T > 0 && (!d_h || !d_logits || ((uintptr_t)d_h & 15)))
        return fail(c, MOE_ERR_ARG, "moe_lm_head_device: null or not 16-byte aligned buffer");
    DeviceScope ds(c->device);
    moe_launch_lm_head(c->head_w, c->d.H, c->vocab, d_h, T, d_logits, stream ? (cudaStream_t)stream : c->stream,
                       &c->launches);
    CK(cudaGetLastError());
    return MOE_OK;
}

int moe_lm_head(moe_ctx *c, const float *h, int T, float *logits) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && (!h || !logits)) return fail(c, MOE_ERR_ARG, "moe_lm_head: null pointer");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (!c->head_w) return fail(c, MOE_ERR_STATE, "lm_head not loaded");
    if (T == 0) return MOE_OK;
    DeviceScope ds(c->device);
    CK(cudaMemcpyAsync(c->d_in, h, (size_t)T * c->d.H * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    int rc = moe_lm_head_device(c, c->d_in, T, c->head_logits, c->stream);
    if (rc) return rc;
    rc = copy_out(c, c->stream, false, {{logits, c->head_logits, (size_t)T * c->vocab * sizeof(float)}});
    if (rc) return rc;
    return finish_sync(c);
}

int moe_sample_device(moe_ctx *c, const float *d_logits, int T, int vocab, float temp, float top_p,
                      uint32_t rng_state, int *d_tokens, void *stream) {
    if (!c) return MOE_ERR_ARG;
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (vocab <= 0 || (T > 0 && (!d_logits || !d_tokens))) return fail(c, MOE_ERR_ARG, "moe_sample_device: bad argument");
    DeviceScope ds(c->device);
    int rc = sample_scratch(c, vocab);
    if (rc) return rc;
    moe_launch_sample(d_logits, T, vocab, temp, top_p, rng_state, c->sample_p, c->sample_ws, d_tokens,
                      stream ? (cudaStream_t)stream : c->stream, &c->launches);
    CK(cudaGetLastError());
    return MOE_OK;
}

uint32_t moe_rng_advance(uint32_t state, int n) {
    for (int i = 0; i < n; i++) {
        state ^= state << 13;
        state ^= state >> 17;
        state ^= state << 5;
    }
    return state;
}

int moe_sample(moe_ctx *c, const float *logits, int T, int vocab, float temp, float top_p, uint32_t *rng_state,
               int *tokens) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && (!logits || !tokens || !rng_state)) return fail(c, MOE_ERR_ARG, "moe_sample: null pointer");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (T == 0) return MOE_OK;
    DeviceScope ds(c->device);
    int rc = sample_scratch(c, vocab);
    if (rc) return rc;
    CK(cudaMemcpyAsync(c->head_logits, logits, (size_t)T * vocab * sizeof(float), cudaMemcpyHostToDevice,
                       c->stream));
    rc = moe_sample_device(c, c->head_logits, T, vocab, temp, top_p, *rng_state, c->sample_tok, c->stream);
    if (rc) return rc;
    rc = copy_out(c, c->stream, false, {{tokens, c->sample_tok, (size_t)T * sizeof(int)}});
    if (rc) return rc;
    rc = finish_sync(c);
    if (rc) return rc;
    if (temp > 0.0f) *rng_state = moe_rng_advance(*rng_state, T);  // one draw per sampled row (infer.m:447)
    return MOE_OK;
}

int moe_route(moe_ctx *c, const float *logits, const float *bias, int T, int *idx, float *w) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && (!logits || !idx || !w)) return fail(c, MOE_ERR_ARG, "moe_route: null pointer");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    if (T == 0) return MOE_OK;
    DeviceScope ds(c->device);
    const int E = c->d.E, K = c->d.K;
    float *d_lg = c->part, *d_b = nullptr;
    CK(cudaMemcpyAsync(d_lg, logits, sizeof(float) * T * E, cudaMemcpyHostToDevice, c->stream));
    if (bias) {
        d_b = c->bias_tmp;
        CK(cudaMemcpyAsync(d_b, bias, sizeof(float) * E, cudaMemcpyHostToDevice, c->stream));
    }
    moe_launch_route_and_plan(c->d, nullptr, 0, d_lg, d_b, nullptr, 0, nullptr, nullptr, T, c->idx, c->wts, nullptr,
                              nullptr, 0, 0, c->plan, c->counter, c->stream, &c->launches);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(idx, c->idx, sizeof(int) * T * K, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaMemcpyAsync(w, c->wts, sizeof(float) * T * K, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return MOE_OK;
}

// Expert-parallel prefill: every rank routes its own tokens, sends each
// token's fp16 row and routing to the ranks that own its experts (fixed
// capacity: the largest token count of any rank, agreed first), runs the
// tcgen05 expert GEMMs over the rows it received, pre-combines them per row
// in slot order, sends the partial sums back, and adds them up in rank order
// plus its own shared expert.  Every rank calls, even with 0 tokens.
static int run_prefill_ep(moe_ctx *c, int layer, const float *d_h, int T, float *d_out, int *d_idx, float *d_w,
                          cudaStream_t s) {
    const MoeDims &d = c->d;
    MoeLayerDev &L = c->layers[layer];
    const int N = c->world, mw = 2 + 2 * d.K;
    if (N > 64) return fail(c, MOE_ERR_ARG, "moe_prefill: world size above 64");
    if (c->comm_aborted) return fail(c, MOE_ERR_STATE, "an exchange failed and the communicator was aborted");
    MoePrefillWs &ws = c->pf;
    if (!ws.tcount && cudaMalloc((void **)&ws.tcount, sizeof(int) * 66) != cudaSuccess)
        return fail(c, MOE_ERR_CUDA, "prefill token-count buffer");
    // the rows per peer: the largest n_tokens of any rank (one host sync)
    CK(cudaMemcpyAsync(ws.tcount, &T, sizeof(int), cudaMemcpyHostToDevice, s));
    NK(moe_nccl()->GroupStart());
    for (int p = 0; p < N; p++) {
        NK(moe_nccl()->Send(ws.tcount, 1, ncclInt32, p, c->comm, s));
        NK(moe_nccl()->Recv(ws.tcount + 2 + p, 1, ncclInt32, p, c->comm, s));
    }
    NK(moe_nccl()->GroupEnd());
    int counts[64];
    {
        const int rc = copy_out(c, s, true, {{counts, ws.tcount + 2, sizeof(int) * N}});
        if (rc) return rc;
    }
    int ecap = 1;
    for (int p = 0; p < N; p++) ecap = counts[p] > ecap ? counts[p] : ecap;
    if (moe_prefill_alloc(ws, d, T > 0 ? T : 1, N, ecap))
        return fail(c, MOE_ERR_CUDA, "prefill workspace for %d tokens x %d ranks could not be allocated", ecap, N);
    const size_t rows = (size_t)ws.ecap;
    if (T > 0) {
        moe_launch_prefill_router(d, L.router, ws, d_h, T, s, &c->launches);
        moe_launch_route_and_plan(d, nullptr, 0, ws.logits, L.bias, L.logit_bias, 0, nullptr, nullptr, T, ws.idx,
                                  ws.w, d_h, nullptr, 1, 0, ws.plan, c->counter, s, &c->launches);
    }
    moe_launch_pfe_dispatch(d, ws, T, c->n_local, s, &c->launches);
    NK(moe_nccl()->GroupStart());
    for (int p = 0; p < N; p++) {
        NK(moe_nccl()->Send(ws.send_xh + p * rows * d.H, rows * d.H, ncclFloat16, p, c->comm, s));
        NK(moe_nccl()->Recv(ws.recv_xh + p * rows * d.H, rows * d.H, ncclFloat16, p, c->comm, s));
        NK(moe_nccl()->Send(ws.send_meta + p * rows * mw, rows * mw, ncclInt32, p, c->comm, s));
        NK(moe_nccl()->Recv(ws.recv_meta + p * rows * mw, rows * mw, ncclInt32, p, c->comm, s));
    }
    NK(moe_nccl()->GroupEnd());
    moe_launch_pfe_experts(d, L, ws, T, s, &c->launches);
    NK(moe_nccl()->GroupStart());
    for (int p = 0; p < N; p++) {
        NK(moe_nccl()->Send(ws.send_y + p * rows * d.H, rows * d.H, ncclFloat32, p, c->comm, s));
        NK(moe_nccl()->Recv(ws.recv_y + p * rows * d.H, rows * d.H, ncclFloat32, p, c->comm, s));
    }
    NK(moe_nccl()->GroupEnd());
    if (T > 0) moe_launch_pfe_final(d, ws, T, d_out, s, &c->launches);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "prefill launch: %s", cudaGetErrorString(e));
    if (T > 0 && d_idx) CK(cudaMemcpyAsync(d_idx, ws.idx, sizeof(int) * T * d.K, cudaMemcpyDeviceToDevice, s));
    if (T > 0 && d_w) CK(cudaMemcpyAsync(d_w, ws.w, sizeof(float) * T * d.K, cudaMemcpyDeviceToDevice, s));
    return MOE_OK;
}

int moe_prefill_device(moe_ctx *c, int layer, const float *d_h, int T, float *d_out, int *d_idx, float *d_w,
                       void *stream) {
    if (!c) return MOE_ERR_ARG;
    if (T < 0 || (T > 0 && (!d_h || !d_out)) || (T == 0 && c->world == 1))
        return fail(c, MOE_ERR_ARG, "moe_prefill_device: need n_tokens >= 1 and buffers (0 only in expert parallelism)");
    int rc = check_layer(c, layer);
    if (rc) return rc;
    // row groups of the CTA pairs: gate/up 2 x 128 rows of I, down 2 x 256 rows of H
    if (c->d.H % 512 || c->d.I % 256 || c->d.K > 63 || c->d.E > 1024)
        return fail(c, MOE_ERR_ARG,
                    "moe_prefill needs hidden %% 512 == 0, intermediate %% 256 == 0, top_k <= 63, n_experts <= 1024");
    DeviceScope ds(c->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    if (c->world > 1) return run_prefill_ep(c, layer, d_h, T, d_out, d_idx, d_w, s);
    if (moe_prefill_alloc(c->pf, c->d, T))
        return fail(c, MOE_ERR_CUDA, "prefill workspace for %d tokens could not be allocated", T);
    MoeLayerDev &L = c->layers[layer];
    const MoeDims &d = c->d;
    moe_launch_prefill_router(d, L.router, c->pf, d_h, T, s, &c->launches);
    moe_launch_route_and_plan(d, nullptr, 0, c->pf.logits, L.bias, L.logit_bias, 0, nullptr, nullptr, T, c->pf.idx,
                              c->pf.w, d_h, nullptr, 1, 0, c->pf.plan, c->counter, s, &c->launches);
    moe_launch_prefill_experts(d, L, c->pf, d_h, T, d_out, s, &c->launches);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(c, MOE_ERR_CUDA, "prefill launch: %s", cudaGetErrorString(e));
    if (d_idx) CK(cudaMemcpyAsync(d_idx, c->pf.idx, sizeof(int) * T * d.K, cudaMemcpyDeviceToDevice, s));
    if (d_w) CK(cudaMemcpyAsync(d_w, c->pf.w, sizeof(float) * T * d.K, cudaMemcpyDeviceToDevice, s));
    return MOE_OK;
}

int moe_prefill(moe_ctx *c, int layer, const float *h, int T, float *out, int *idx_out, float *w_out) {
    if (!c) return MOE_ERR_ARG;
    if (T < 0 || (T > 0 && (!h || !out)) || (T == 0 && c->world == 1))
        return fail(c, MOE_ERR_ARG, "moe_prefill: need n_tokens >= 1 and buffers (0 only in expert parallelism)");
    DeviceScope ds(c->device);
    if (T == 0) {  // a rank without tokens still takes part in the exchanges
        const int rc = moe_prefill_device(c, layer, nullptr, 0, nullptr, nullptr, nullptr, nullptr);
        const int wrc = stream_wait(c, c->stream, c->world > 1);
        return rc ? rc : wrc;
    }
    const size_t n = (size_t)T * c->d.H;
    float *dh = nullptr, *dout = nullptr;
    CK(cudaMalloc((void **)&dh, n * sizeof(float)));
    if (cudaMalloc((void **)&dout, n * sizeof(float)) != cudaSuccess) {
        cudaFree(dh);
        return fail(c, MOE_ERR_CUDA, "moe_prefill: out of memory");
    }
    int rc = MOE_OK;
    if (cudaMemcpyAsync(dh, h, n * sizeof(float), cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        rc = fail(c, MOE_ERR_CUDA, "moe_prefill: copy in");
    if (!rc) rc = moe_prefill_device(c, layer, dh, T, dout, nullptr, nullptr, nullptr);
    // with expert parallelism the host waits (polling, bounded) before it
    // copies into the caller's memory
    if (!rc)
        rc = copy_out(c, c->stream, c->world > 1,
                      {{out, dout, n * sizeof(float)},
                       {idx_out, c->pf.idx, sizeof(int) * T * c->d.K},
                       {w_out, c->pf.w, sizeof(float) * T * c->d.K}});
    const int wrc = c->comm_aborted ? MOE_ERR_NCCL : stream_wait(c, c->stream, c->world > 1);
    if (wrc == MOE_OK) {  // after an abort the buffers may still be in use
        cudaFree(dh);
        cudaFree(dout);
    }
    if (rc) return rc;
    if (wrc) return wrc;
    return take_device_error(c);
}

int moe_forward_stack_device(moe_ctx *c, int first, int n_layers, float *d_hidden, int T, void *stream) {
    if (!c) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    if (T > 0 && !d_hidden) return fail(c, MOE_ERR_ARG, "moe_forward_stack_device: null hidden");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    if (T > 0 && ((uintptr_t)d_hidden & 15)) return fail(c, MOE_ERR_ARG, "hidden buffer not 16-byte aligned");
    bool any_moe = false;
    for (int l = first; l < first + n_layers; l++) {
        const bool dense = l >= 0 && l < (int)c->dense.size() && c->dense[l].w;
        const int rc = dense ? MOE_OK : check_layer(c, l);
        if (rc) return rc;
        any_moe |= !dense;
    }
    int rc = any_moe ? ep_usable(c) : MOE_OK;
    if (rc) return rc;
    // the whole stack is one launch sequence (one graph once replayed)
    const moe_ctx::GraphSig sig{1, first, n_layers, T, d_hidden, nullptr, s};
    return run_graphed(c, sig, s, [&]() {
        for (int l = first; l < first + n_layers; l++) {
            int r = MOE_OK;
            if (T > 0)
                moe_launch_rmsnorm(d_hidden, c->layers[l].norm, c->h_post, T, c->d.H, c->cfg.rms_eps, s,
                                   &c->launches);
            if (c->dense[l].w) {  // every rank runs its own tokens on its copy of the layer
                moe_launch_dense_ffn(c->dense[l].w, c->d.H, c->dense[l].Id, c->h_post, T, c->dense_act, d_hidden,
                                     d_hidden, s, &c->launches);
                if (c->hits) CK(cudaMemsetAsync(c->hits + l, 0, sizeof(int), s));
                continue;
            }
            if (c->world > 1) r = run_ep(c, l, c->h_post, T, nullptr, nullptr, d_hidden, d_hidden, s);
            else if (T > 0) r = run_local(c, l, c->h_post, T, nullptr, nullptr, 1, 1, d_hidden, d_hidden, s);
            if (r) return r;
            r = record_hits(c, l, c->world > 1 || T > 0, s);
            if (r) return r;
        }
        return MOE_OK;
    });
}

int moe_forward_stack(moe_ctx *c, int first, int n_layers, float *hidden, int T) {
    if (!c) return MOE_ERR_ARG;
    if (T > 0 && !hidden) return fail(c, MOE_ERR_ARG, "moe_forward_stack: null hidden");
    if (T < 0 || T > c->max_tok) return fail(c, MOE_ERR_ARG, "n_tokens %d exceeds max_tokens %d", T, c->max_tok);
    DeviceScope ds(c->device);
    const size_t n = (size_t)T * c->d.H;
    if (n) CK(cudaMemcpyAsync(c->d_in, hidden, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    int rc = moe_forward_stack_device(c, first, n_layers, c->d_in, T, nullptr);
    if (rc) return rc;
    rc = copy_out(c, c->stream, step_uses_nccl(c), {{hidden, c->d_in, n * sizeof(float)}});
    if (rc) return rc;
    return finish_sync(c);
}

int moe_set_timing(moe_ctx *c, int enable) {
    if (!c || enable < 0) return MOE_ERR_ARG;
    drop_graphs(c);
    DeviceScope ds(c->device);
    if (enable > 0 && enable != c->ring) {
        for (cudaEvent_t e : c->ev) cudaEventDestroy(e);
        c->ev.assign((size_t)enable * (MOE_N_PHASES + 1), nullptr);
        c->ev_valid.assign(c->ev.size(), 0);
        for (auto &e : c->ev) CK(cudaEventCreate(&e));
        c->ring = enable;
        c->ring_pos = enable - 1;
        c->ring_used = 0;
    }
    c->timing = enable > 0;
    return MOE_OK;
}

int moe_get_timing_at(moe_ctx *c, int back, float *ms, int n) {
    if (!c || !ms) return MOE_ERR_ARG;
    DeviceScope ds(c->device);
    if (!c->timing || c->ring == 0) return fail(c, MOE_ERR_STATE, "timing is not enabled");
    if (back < 0 || back >= c->ring_used) return fail(c, MOE_ERR_ARG, "step %d is not in the timing ring", back);
    const int slot = ((c->ring_pos - back) % c->ring + c->ring) % c->ring;
    cudaEvent_t *ev = &c->ev[(size_t)slot * (MOE_N_PHASES + 1)];
    const uint8_t *valid = &c->ev_valid[(size_t)slot * (MOE_N_PHASES + 1)];
    for (int p = MOE_N_PHASES; p >= 0; p--)
        if (valid[p]) { CK(cudaEventSynchronize(ev[p])); break; }
    for (int p = 0; p < n && p < MOE_N_PHASES; p++) {
        ms[p] = 0.0f;
        if (!valid[p]) continue;
        int q = p + 1;
        while (q <= MOE_N_PHASES && !valid[q]) q++;
        if (q > MOE_N_PHASES) continue;
        CK(cudaEventElapsedTime(&ms[p], ev[p], ev[q]));
    }
    return MOE_OK;
}

int moe_get_timing(moe_ctx *c, float *ms, int n) { return moe_get_timing_at(c, 0, ms, n); }

uint64_t moe_last_weight_bytes(const moe_ctx *cc) {
    moe_ctx *c = const_cast<moe_ctx *>(cc);
    if (!c || c->last_layer < 0) return 0;
    DeviceScope ds(c->device);
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return 0;
    int counts[4] = {0, 0, 0, 0};
    if (cudaMemcpy(counts, c->plan.counts, sizeof(counts), cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    const MoeLayerDev &L = c->layers[c->last_layer];
    const size_t eb = 2 * L.gate_bytes + c->layer_down_bytes[c->last_layer];
    const size_t sb = 2 * L.gate_bytes + row_bytes(L.sh_down_type, c->d.I) * c->d.H;
    return (uint64_t)counts[2] * eb + sb + sizeof(float) * ((size_t)c->d.E * c->d.H + c->d.E);
}

// ------------------------------------------------------------------ codec
static int dequant_host(int type, const void *src, float *dst, size_t n) {
    moe_ctx *c = nullptr;
    if (!src || !dst || n % MOE_QK) return fail(c, MOE_ERR_ARG, "dequantize: n must be a multiple of 256");
    const size_t nb = n / MOE_QK, bytes = nb * (type == MOE_TYPE_Q6_K ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
    uint8_t *ds = nullptr;
    float *dd = nullptr;
    CK(cudaMalloc((void **)&ds, bytes + 16));
    if (cudaMalloc((void **)&dd, n * sizeof(float)) != cudaSuccess) { cudaFree(ds); return MOE_ERR_CUDA; }
    int rc = MOE_OK;
    if (cudaMemcpy(ds, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) rc = MOE_ERR_CUDA;
    if (!rc) {
        moe_launch_dequant(type, ds, dd, n, 0, nullptr);
        if (cudaGetLastError() != cudaSuccess || cudaMemcpy(dst, dd, n * sizeof(float), cudaMemcpyDeviceToHost) !=
                                                     cudaSuccess)
            rc = MOE_ERR_CUDA;
    }
    cudaFree(ds);
    cudaFree(dd);
    return rc;
}
int moe_dequantize_row_q4_K(const void *src, float *dst, size_t n) { return dequant_host(MOE_TYPE_Q4_K, src, dst, n); }
int moe_dequantize_row_q6_K(const void *src, float *dst, size_t n) { return dequant_host(MOE_TYPE_Q6_K, src, dst, n); }

}  // extern "C"
