// moe_ep.cu -- expert-parallel dispatch / combine kernels (one process per GPU,
// experts sharded n_experts / world per rank, router and shared expert
// replicated).  The exchange runs inside the kernels that produce the data,
// as stores into the peers' mailboxes in NVLink peer memory (second half of
// this file), or, when the peers cannot be mapped, as NCCL send/recv between
// fixed-capacity buffers (moe_api.cu); either way a step needs no host
// synchronisation.
//
// Row space of the expert kernels on rank r (world N, capacity cap = max
// tokens per rank):
//   rows [p*cap, p*cap + cap)   activations received from rank p
//   rows [N*cap, N*cap + T)     this rank's own tokens (shared expert)
// Metadata of a dispatched row: [valid, src_token, idx[K], w_bits[K]].
#include <stdio.h>

#include "moe_common.cuh"
#include "moe_internal.h"

#define LAUNCH_COUNT(p) \
    do {                \
        if (p) (*(p))++; \
    } while (0)

// Per-peer masks of the local tokens that route to at least one expert of
// that peer (T <= 64).
__device__ __forceinline__ unsigned long long peer_mask(const int *__restrict__ idx, int T, int K, int n_local,
                                                        int p) {
    unsigned long long m = 0ull;
    for (int t = 0; t < T; t++)
        for (int k = 0; k < K; k++)
            if (idx[t * K + k] / n_local == p) { m |= 1ull << t; break; }
    return m;
}

// grid = T blocks (+1 block that clears the unused slots' valid flags)
__global__ void k_ep_pack(const float *__restrict__ x, const int *__restrict__ idx, const float *__restrict__ w,
                          int T, int K, int H, int world, int n_local, int cap, float *__restrict__ send_x,
                          int *__restrict__ send_meta, int *__restrict__ tok_slot) {
    __shared__ unsigned long long pm[64];
    const int meta_w = 2 + 2 * K;
    for (int p = threadIdx.x; p < world; p += blockDim.x) pm[p] = peer_mask(idx, T, K, n_local, p);
    __syncthreads();
    if (blockIdx.x == T) {  // clear the valid flag of unused slots
        for (int s = threadIdx.x; s < world * cap; s += blockDim.x) {
            const int p = s / cap, i = s % cap;
            if (i >= __popcll(pm[p])) send_meta[(size_t)s * meta_w] = 0;
        }
        return;
    }
    const int t = blockIdx.x;
    for (int p = 0; p < world; p++) {
        const bool hit = (pm[p] >> t) & 1ull;
        const int slot = hit ? __popcll(pm[p] & ((1ull << t) - 1ull)) : -1;
        if (threadIdx.x == 0) tok_slot[t * world + p] = slot;
        if (!hit) continue;
        const size_t row = (size_t)p * cap + slot;
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * H);
        float4 *dst = reinterpret_cast<float4 *>(send_x + row * H);
        for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
        int *m = send_meta + row * meta_w;
        if (threadIdx.x == 0) { m[0] = 1; m[1] = t; }
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            m[2 + k] = idx[t * K + k];
            m[2 + K + k] = __float_as_int(w[t * K + k]);
        }
    }
}

// Plan over the received rows (experts this rank owns) + the shared expert on
// the local rows, by one block; mask = dynamic shared memory of
// (E+1) * MW * 8 bytes.
__device__ void ep_plan_block(const MoeDims &d, const int *__restrict__ recv_meta, int world, int cap, int T, int e0,
                              int n_local, const MoePlan &plan, unsigned long long *mask) {
    __shared__ int cnt[1025], off[1026], coff[1026];
    __shared__ int wsum[3][32], carry[3];
    const int E = d.E, K = d.K, NE = E + 1;
    const int R = world * cap, RT = R + T;
    const int MW = (RT + 63) / 64;
    const int meta_w = 2 + 2 * K;
    for (int e = threadIdx.x; e < NE; e += blockDim.x) cnt[e] = 0;
    for (int i = threadIdx.x; i < NE * MW; i += blockDim.x) mask[i] = 0ull;
    __syncthreads();
    for (int p = threadIdx.x; p < R * K; p += blockDim.x) {
        const int r = p / K, k = p % K;
        const int *m = recv_meta + (size_t)r * meta_w;
        if (!m[0]) continue;
        const int e = m[2 + k];
        if (e < 0 || e >= E) { atomicExch(plan.error, MOE_DEV_ERR_INDEX); continue; }
        if (e < e0 || e >= e0 + n_local) continue;
        atomicAdd(&cnt[e], 1);
        atomicOr(&mask[(size_t)e * MW + (r >> 6)], 1ull << (r & 63));
    }
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const int r = R + t;
        atomicOr(&mask[(size_t)E * MW + (r >> 6)], 1ull << (r & 63));
    }
    if (threadIdx.x == 0) cnt[E] = T;
    if (threadIdx.x == 0) carry[0] = carry[1] = carry[2] = 0;
    __syncthreads();
    // exclusive scans (pairs, chunks, routed experts hit)
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    for (int base = 0; base < NE; base += blockDim.x) {
        const int e = base + threadIdx.x;
        int v[3] = {0, 0, 0};
        if (e < NE) {
            v[0] = cnt[e];
            v[1] = moe_n_chunks(cnt[e], d.tc);
            v[2] = (e < E && cnt[e] > 0) ? 1 : 0;
        }
        int inc[3];
#pragma unroll
        for (int q = 0; q < 3; q++) {
            int xv = v[q];
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, xv, o);
                if (lane >= o) xv += y;
            }
            inc[q] = xv;
            if (lane == 31) wsum[q][wid] = xv;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
#pragma unroll
            for (int q = 0; q < 3; q++) {
                int xv = threadIdx.x < nwarp ? wsum[q][threadIdx.x] : 0;
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, xv, o);
                    if (threadIdx.x >= o) xv += y;
                }
                if (threadIdx.x < nwarp) wsum[q][threadIdx.x] = xv;
            }
        }
        __syncthreads();
        int excl[3];
#pragma unroll
        for (int q = 0; q < 3; q++) excl[q] = carry[q] + (wid ? wsum[q][wid - 1] : 0) + inc[q] - v[q];
        if (e < NE) { off[e] = excl[0]; coff[e] = excl[1]; }
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) {
#pragma unroll
            for (int q = 0; q < 3; q++) carry[q] = excl[q] + v[q];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        plan.counts[0] = carry[0];
        plan.counts[1] = carry[1];
        plan.counts[2] = carry[2];
    }
    __syncthreads();
    // pairs: position = offset of the expert + earlier rows of that expert
    for (int p = threadIdx.x; p < R * K; p += blockDim.x) {
        const int r = p / K, k = p % K;
        const int *m = recv_meta + (size_t)r * meta_w;
        int pos = -1;
        const int e = m[0] ? m[2 + k] : -1;
        if (m[0] && e >= e0 && e < e0 + n_local && e < E) {
            const unsigned long long *me = mask + (size_t)e * MW;
            int before = 0;
            for (int wv = 0; wv < (r >> 6); wv++) before += __popcll(me[wv]);
            before += __popcll(me[r >> 6] & ((1ull << (r & 63)) - 1ull));
            pos = off[e] + before;
            plan.pair_expert[pos] = e;
            plan.pair_token[pos] = r;
            plan.pair_w[pos] = __int_as_float(m[2 + K + k]);
        }
        plan.slot_pair[(size_t)r * (K + 1) + k] = pos;
    }
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const int pos = off[E] + t, r = R + t;
        plan.pair_expert[pos] = E;
        plan.pair_token[pos] = r;
        plan.pair_w[pos] = 1.0f;
        plan.slot_pair[(size_t)r * (K + 1) + K] = pos;
    }
    for (int e = threadIdx.x; e < NE; e += blockDim.x) {
        const int n = cnt[e];
        const int nc = moe_n_chunks(n, d.tc);
        for (int c = 0; c < nc; c++) {
            int start, nt;
            moe_chunk(n, c, d.tc, start, nt);
            const int ci = coff[e] + c;
            plan.chunk_expert[ci] = e;
            plan.chunk_pair0[ci] = off[e] + start;
            plan.chunk_ntok[ci] = nt;
        }
    }
    __syncthreads();
    moe_plan_order_chunks(plan, carry[1], d.tc);
}

__global__ void __launch_bounds__(512) k_ep_plan(MoeDims d, const int *__restrict__ recv_meta, int world, int cap,
                                                 int T, int e0, int n_local, MoePlan plan) {
    extern __shared__ unsigned long long ep_mask[];  // [E+1][MW]
    ep_plan_block(d, recv_meta, world, cap, T, e0, n_local, plan, ep_mask);
}

// Pre-combine on the expert side: partial[r] = sum over the slots of received
// row r whose expert lives here, in slot order, of w_k * eo.
__global__ void k_ep_partial(MoeDims d, MoePlan plan, const int *__restrict__ recv_meta, const float *__restrict__ eo,
                             int rows, float *__restrict__ out) {
    const int r = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows || i >= d.H) return;
    const int K = d.K;
    if (!recv_meta[(size_t)r * (2 + 2 * K)]) return;
    float acc = 0.0f;
    for (int k = 0; k < K; k++) {
        const int p = plan.slot_pair[(size_t)r * (K + 1) + k];
        if (p < 0) continue;
        acc = fmaf(plan.pair_w[p], eo[(size_t)p * d.H + i], acc);
    }
    out[(size_t)r * d.H + i] = acc;
}

// Owner side: out[t] = sum over ranks (rank order) of the returned partials +
// shared expert (+ residual).
__global__ void k_ep_final(MoeDims d, MoePlan plan, const float *__restrict__ recv_y, const int *__restrict__ tok_slot,
                           int world, int cap, int T, const float *__restrict__ eo, const float *__restrict__ residual,
                           float *__restrict__ out) {
    const int t = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= d.H) return;
    float acc = 0.0f;
    for (int p = 0; p < world; p++) {
        const int s = tok_slot[t * world + p];
        if (s >= 0) acc = acc + recv_y[((size_t)p * cap + s) * d.H + i];
    }
    const int sp = plan.slot_pair[(size_t)(world * cap + t) * (d.K + 1) + d.K];
    acc = acc + eo[(size_t)sp * d.H + i];
    if (residual) acc = residual[(size_t)t * d.H + i] + acc;
    out[(size_t)t * d.H + i] = acc;
}

void moe_launch_ep_pack(const float *x, const int *idx, const float *w, int T, int K, int H, int world, int n_local,
                        int cap, float *send_x, int *send_meta, int *tok_slot, cudaStream_t s, uint64_t *launches) {
    k_ep_pack<<<T + 1, 256, 0, s>>>(x, idx, w, T, K, H, world, n_local, cap, send_x, send_meta, tok_slot);
    LAUNCH_COUNT(launches);
}

void moe_launch_ep_plan(const MoeDims &d, const int *recv_meta, int world, int cap, int T, int e0, int n_local,
                        const MoePlan &plan, cudaStream_t s, uint64_t *launches) {
    const int MW = (world * cap + T + 63) / 64;
    const size_t smem = sizeof(unsigned long long) * (size_t)(d.E + 1) * MW;
    static size_t attr[MOE_MAX_DEVICES];
    if (smem > 48 * 1024) moe_smem_limit(k_ep_plan, smem, attr);
    k_ep_plan<<<1, 512, smem, s>>>(d, recv_meta, world, cap, T, e0, n_local, plan);
    LAUNCH_COUNT(launches);
}

void moe_launch_ep_partial(const MoeDims &d, const MoePlan &plan, const int *recv_meta, const float *eo, int rows,
                           float *out, cudaStream_t s, uint64_t *launches) {
    dim3 grid((d.H + 255) / 256, rows);
    k_ep_partial<<<grid, 256, 0, s>>>(d, plan, recv_meta, eo, rows, out);
    LAUNCH_COUNT(launches);
}

void moe_launch_ep_final(const MoeDims &d, const MoePlan &plan, const float *recv_y, const int *tok_slot, int world,
                         int cap, int T, const float *eo, const float *residual, float *out, cudaStream_t s,
                         uint64_t *launches) {
    dim3 grid((d.H + 255) / 256, T);
    k_ep_final<<<grid, 256, 0, s>>>(d, plan, recv_y, tok_slot, world, cap, T, eo, residual, out);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// NVLink peer-memory exchange.  Every rank owns a mailbox (one allocation,
// mapped into every peer with CUDA IPC):
//   [flags: dispatch[64], combine[64] (u64 step numbers)]
//   [recv_x  (2 parities) [world*cap][H] fp32]
//   [recv_meta (2)        [world*cap][2+2K] int]
//   [recv_y  (2)          [world*cap][H] fp32]
// The pack kernel stores each token row straight into the mailboxes of the
// ranks that own its experts, and the pre-combine kernel stores each partial
// row straight into the mailbox of the token's rank: the copy is part of the
// kernel that produces the data, there is no separate collective.  When a
// kernel's blocks are done (every thread fences its stores at system scope),
// its last block writes the step number into the matching flag of every
// peer (release, system scope).  The consumers wait (acquire, bounded) for
// the flags of all peers: the plan / operand kernel for the dispatch flags,
// the final sum for the combine flags.  Buffers alternate by step parity: a
// rank cannot reach step n + 2 before every peer has finished consuming step
// n (it needs their step n + 1 partials first).  The step number lives in
// device memory (EpP2P::d_seq): every kernel of a step reads seq = *d_seq +
// 1, and the final sum's last block stores seq, so a step's launches carry
// no per-step host arguments and replay as a CUDA graph.
// ===========================================================================
#define EP_WAIT_NS 2000000000ull

__device__ __forceinline__ unsigned long long ep_ld_acquire(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ep_st_release(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ep_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// the step this launch belongs to
__device__ __forceinline__ unsigned long long ep_step(const EpP2P &q) { return *q.d_seq + 1ull; }

__device__ bool ep_wait_flags(const unsigned long long *flags, int world, unsigned long long seq, int *error);
// the whole block waits: thread 0 acquires the flags (system scope), the
// block barrier then orders every thread's later reads after the peers'
// released stores
__device__ __forceinline__ void ep_block_wait(const unsigned long long *flags, int world, unsigned long long seq,
                                              int *error) {
    if (threadIdx.x == 0) ep_wait_flags(flags, world, seq, error);
    __syncthreads();
}

// every thread: wait until flags[p] >= seq for all p < world (bounded; a
// wait that another thread of the step already gave up on is not repeated)
__device__ bool ep_wait_flags(const unsigned long long *flags, int world, unsigned long long seq, int *error) {
    const unsigned long long t0 = ep_now();
    for (int p = 0; p < world; p++)
        while (ep_ld_acquire(flags + p) < seq) {
            if (*reinterpret_cast<volatile int *>(error) == EP_ERR_TIMEOUT) return false;
            if (ep_now() - t0 > EP_WAIT_NS) {
                atomicExch(error, EP_ERR_TIMEOUT);
                return false;
            }
        }
    return true;
}

// after the block's stores: the last block of the grid raises flags[me] = seq
// in every peer's mailbox (flag_off = byte offset of the flag array).  The
// block barrier orders every thread's stores before thread 0's system-scope
// fence, which is cumulative, so one fence per block publishes them all (the
// pattern of a cooperative grid barrier).
__device__ void ep_signal(const EpP2P &q, size_t flag_off, int *done, unsigned long long seq) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned int nblk = gridDim.x * gridDim.y;
        if (atomicAdd(done, 1) == (int)nblk - 1) {
            *done = 0;  // stream order keeps the next launch behind this reset
            __threadfence_system();
            for (int p = 0; p < q.world; p++)
                ep_st_release(reinterpret_cast<unsigned long long *>(q.peers[p] + flag_off) + q.me, seq);
        }
    }
}

// grid = T blocks (+1 that clears the unused rows' valid flags on every peer)
__global__ void k_ep_pack_p2p(const float *__restrict__ x, const int *__restrict__ idx, const float *__restrict__ w,
                              int T, int K, int H, int n_local, int cap, EpP2P q, int *__restrict__ tok_slot) {
    __shared__ unsigned long long pm[64];
    const unsigned long long seq = ep_step(q);
    const int parity = (int)(seq & 1ull);
    const int world = q.world, meta_w = 2 + 2 * K;
    const size_t R = (size_t)world * cap;
    for (int p = threadIdx.x; p < world; p += blockDim.x) pm[p] = peer_mask(idx, T, K, n_local, p);
    __syncthreads();
    if (blockIdx.x == T) {
        for (int s = threadIdx.x; s < world * cap; s += blockDim.x) {
            const int p = s / cap, i = s % cap;
            if (i >= __popcll(pm[p])) {
                int *meta = reinterpret_cast<int *>(q.peers[p] + q.off_meta) + (size_t)parity * R * meta_w;
                meta[((size_t)q.me * cap + i) * meta_w] = 0;
            }
        }
    } else {
        const int t = blockIdx.x;
        for (int p = 0; p < world; p++) {
            const bool hit = (pm[p] >> t) & 1ull;
            const int slot = hit ? __popcll(pm[p] & ((1ull << t) - 1ull)) : -1;
            if (threadIdx.x == 0) tok_slot[t * world + p] = slot;
            if (!hit) continue;
            const size_t row = (size_t)parity * R + (size_t)q.me * cap + slot;
            const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * H);
            float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(q.peers[p] + q.off_x) + row * H);
            for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
            int *m = reinterpret_cast<int *>(q.peers[p] + q.off_meta) + row * meta_w;
            if (threadIdx.x == 0) { m[0] = 1; m[1] = t; }
            for (int k = threadIdx.x; k < K; k += blockDim.x) {
                m[2 + k] = idx[t * K + k];
                m[2 + K + k] = __float_as_int(w[t * K + k]);
            }
        }
    }
    ep_signal(q, 0, q.done, seq);
}

// After the peers' dispatch flags: block 0 builds the plan over the received
// rows (experts of this rank) and the local rows (shared expert); block
// 1 + r builds the operand of row r (received rows [0, R) whose slot is in
// use, then the T local rows).  Dynamic shared memory: the plan's masks.
__global__ void __launch_bounds__(512) k_ep_plan_rows_p2p(MoeDims d, EpP2P q, int cap, int T, int e0, int n_local,
                                                          MoePlan plan, const float *__restrict__ local,
                                                          uint8_t *__restrict__ xop) {
    extern __shared__ unsigned long long ep_mask2[];
    const unsigned long long seq = ep_step(q);
    const int parity = (int)(seq & 1ull);
    const int R = q.world * cap, meta_w = 2 + 2 * d.K;
    const uint8_t *own = q.peers[q.me];
    ep_block_wait(reinterpret_cast<const unsigned long long *>(own), q.world, seq, q.error);
    const int *meta = reinterpret_cast<const int *>(own + q.off_meta) + (size_t)parity * R * meta_w;
    if (blockIdx.x == 0) {
        ep_plan_block(d, meta, q.world, cap, T, e0, n_local, plan, ep_mask2);
        return;
    }
    const int r = blockIdx.x - 1;
    if (r < R && !__ldcg(meta + (size_t)r * meta_w)) return;
    const float *recv = reinterpret_cast<const float *>(own + q.off_x) + (size_t)parity * R * d.H;
    uint8_t *row = xop + (size_t)r * opx_row(d.H);
    build_op_rows(r < R ? recv + (size_t)r * d.H : local + (size_t)(r - R) * d.H, d.H, row, row + op_bytes(d.H), 4);
}

// pre-combine (k_ep_partial's sum) stored straight into the token rank's
// mailbox: received row r = (source p, slot s) -> p's recv_y row me*cap + s
__global__ void k_ep_partial_p2p(MoeDims d, MoePlan plan, const float *__restrict__ eo, int cap, EpP2P q) {
    const unsigned long long seq = ep_step(q);
    const int parity = (int)(seq & 1ull);
    const int r = blockIdx.y, i4 = blockIdx.x * blockDim.x + threadIdx.x;  // float4 column
    const int K = d.K;
    const size_t R = (size_t)q.world * cap;
    const int *recv_meta = reinterpret_cast<const int *>(q.peers[q.me] + q.off_meta) + (size_t)parity * R * (2 + 2 * K);
    if (i4 < d.H / 4 && recv_meta[(size_t)r * (2 + 2 * K)]) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int k = 0; k < K; k++) {
            const int p = plan.slot_pair[(size_t)r * (K + 1) + k];
            if (p < 0) continue;
            const float wp = plan.pair_w[p];
            const float4 e = reinterpret_cast<const float4 *>(eo + (size_t)p * d.H)[i4];
            acc.x = fmaf(wp, e.x, acc.x);
            acc.y = fmaf(wp, e.y, acc.y);
            acc.z = fmaf(wp, e.z, acc.z);
            acc.w = fmaf(wp, e.w, acc.w);
        }
        const int src = r / cap, s = r % cap;
        float *y = reinterpret_cast<float *>(q.peers[src] + q.off_y) + (size_t)parity * R * d.H;
        reinterpret_cast<float4 *>(y + ((size_t)q.me * cap + s) * d.H)[i4] = acc;
    }
    ep_signal(q, 64 * sizeof(unsigned long long), q.done + 1, seq);
}

// After the peers' combine flags: out[t] = sum over ranks (rank order) of the
// returned partials + shared expert (+ residual); then the last block stores
// the step number (the step is complete on this rank).  grid.y = max(T, 1).
__global__ void k_ep_final_p2p(MoeDims d, MoePlan plan, EpP2P q, const int *__restrict__ tok_slot, int cap, int T,
                               const float *__restrict__ eo, const float *__restrict__ residual,
                               float *__restrict__ out) {
    const unsigned long long seq = ep_step(q);
    const int parity = (int)(seq & 1ull);
    const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint8_t *own = q.peers[q.me];
    ep_block_wait(reinterpret_cast<const unsigned long long *>(own) + 64, q.world, seq, q.error);
    if (t < T && i < d.H) {
        const size_t R = (size_t)q.world * cap;
        const float *recv_y = reinterpret_cast<const float *>(own + q.off_y) + (size_t)parity * R * d.H;
        float acc = 0.0f;
        for (int p = 0; p < q.world; p++) {
            const int s = tok_slot[t * q.world + p];
            if (s >= 0) acc = acc + __ldcg(recv_y + ((size_t)p * cap + s) * d.H + i);
        }
        const int sp = plan.slot_pair[(size_t)(q.world * cap + t) * (d.K + 1) + d.K];
        acc = acc + eo[(size_t)sp * d.H + i];
        if (residual) acc = residual[(size_t)t * d.H + i] + acc;
        out[(size_t)t * d.H + i] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int nblk = gridDim.x * gridDim.y;
        if (atomicAdd(q.done + 2, 1) == (int)nblk - 1) {  // every block has read the step number
            q.done[2] = 0;
            *q.d_seq = seq;
        }
    }
}

void moe_launch_ep_pack_p2p(const float *x, const int *idx, const float *w, int T, int K, int H, int n_local,
                            int cap, const EpP2P &q, int *tok_slot, cudaStream_t s, uint64_t *launches) {
    k_ep_pack_p2p<<<T + 1, 256, 0, s>>>(x, idx, w, T, K, H, n_local, cap, q, tok_slot);
    LAUNCH_COUNT(launches);
}

void moe_launch_ep_plan_rows_p2p(const MoeDims &d, const EpP2P &q, int cap, int T, int e0, int n_local,
                                 const MoePlan &plan, const float *local, uint8_t *xop, cudaStream_t s,
                                 uint64_t *launches) {
    const int R = q.world * cap;
    const int MW = (R + T + 63) / 64;
    const size_t smem = sizeof(unsigned long long) * (size_t)(d.E + 1) * MW;
    static size_t attr[MOE_MAX_DEVICES];
    if (smem > 48 * 1024) moe_smem_limit(k_ep_plan_rows_p2p, smem, attr);
    k_ep_plan_rows_p2p<<<1 + R + T, 512, smem, s>>>(d, q, cap, T, e0, n_local, plan, local, xop);
    LAUNCH_COUNT(launches);
}

void moe_launch_ep_partial_p2p(const MoeDims &d, const MoePlan &plan, const float *eo, int cap, const EpP2P &q,
                               cudaStream_t s, uint64_t *launches) {
    dim3 grid((d.H / 4 + 255) / 256, q.world * cap);  // H % 256 == 0 (checked at create)
    k_ep_partial_p2p<<<grid, 256, 0, s>>>(d, plan, eo, cap, q);
    LAUNCH_COUNT(launches);
}

void moe_launch_ep_final_p2p(const MoeDims &d, const MoePlan &plan, const EpP2P &q, const int *tok_slot, int cap,
                             int T, const float *eo, const float *residual, float *out, cudaStream_t s,
                             uint64_t *launches) {
    dim3 grid((d.H + 255) / 256, T > 0 ? T : 1);
    k_ep_final_p2p<<<grid, 256, 0, s>>>(d, plan, q, tok_slot, cap, T, eo, residual, out);
    LAUNCH_COUNT(launches);
}
