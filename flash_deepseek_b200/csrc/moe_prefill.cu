// moe_prefill.cu -- the MoE block for many tokens at once (prefill), on the
// fifth-generation tensor cores (tcgen05).
//
// With ~128 tokens per expert the expert products are real matrix products
// (C = W X^T, M = weight rows, N = tokens, K = hidden or intermediate), so
// the weights are dequantized once per tile into fp16 tiles that feed
// tcgen05.mma, with the fp32 accumulator in tensor memory:
//   plan     counting sort of the (token, slot) pairs by expert; an
//            expert's pairs split evenly into tiles of <= 160
//   gather   fp16 copy of each pair's token row, pairs grouped by expert
//   gemm1    gate/up rows (2 blocks of 64 + 64 per CTA, a CTA pair per
//            tile) x <= 160 pairs, SwiGLU in the epilogue
//            (infer.m:378-383), act in fp16
//   gemm2    down rows (2 blocks of 128 per CTA) x <= 160 pairs, fp32
//            expert outputs
//   combine  slot order, then the shared expert (infer.m:1915-1922)
// Differences from the reference's fp32 dot: weights and activations are
// rounded to fp16 (11-bit significands) before the fp32-accumulated product.
//
// GEMM CTA (one per SM, two SMs of a TPC per tile as a cta_group::2 pair):
// warp 0 streams the raw Q4_K / Q6_K tiles of its own rows, one super-block
// per stage; warp 2 streams its half of the pairs' 64-column activation
// slices (TMA, 128-byte swizzle) into a ring of 10 KB stages; warp 1 of the
// leader runs the MMA loop, one elected lane issuing each M = 256 pair MMA
// (both row blocks share every activation stage).  12 warps
// dequantize: warp (q, g) writes the K atoms g, g + 3, ... through A stage g
// for tensor-memory lanes 32q .. 32q + 31 straight into tensor memory
// (tcgen05.st), so
// the A operand never touches shared memory, and the MMA reads A from tensor
// memory and B from shared memory; the same warps run the epilogue.  All
// hand-offs are mbarriers; every wait gives up after about a second and
// records an error instead of hanging, and a producer that gives up first
// waits (bounded) for the copies it issued.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdio.h>

#include "../../include/moe_cuda.h"
#include "moe_common.cuh"
#include "moe_internal.h"
#include "moe_umma.cuh"

#define PF_TILE 128                // weight rows per accumulator block of one CTA (the pair MMA has M = 256)
#define PF_RB 2                    // row blocks per CTA: 2 x 128 rows share each activation stage
#define PF_TILE_N 160              // pairs per tile (pair MMA N <= 160, a multiple of 32)
#define PF_ATOM 16384              // one 128-row x 128-byte tile (64 columns of K; router stages)
#define PF_BST (PF_TILE_N / 2 * 128)  // one activation stage of a CTA: its half of the pairs x 128 B
#define PF_BOX16 2048              // one 16-row activation box (2 swizzle atoms of 8 rows)
#define PF_NSA 3                   // A stages in tensor memory (PF_RB x 32 columns each, after the accumulators)
#define PF_NSB 8                   // activation stages
#define PF_Q6_ROW 208              // Q6_K Q-plane row stride in shared memory (192 B used)
#define PF_RAW_Q4 (PF_RB * 128 * 144)                  // PF_RB x 128 Q4_K rows of one super-block
#define PF_RAW_Q6 (PF_RB * 128 * (PF_Q6_ROW + 16))     // Q planes of both blocks, then their scale planes
#define PF_RAW_NS_Q4 3             // raw super-block stages
#define PF_RAW_NS_Q6 2
#define PF_RAW_NS_MAX 3
#define PF_DQ_WARPS (4 * PF_NSA)                    // dequantize + epilogue (warps 3 ..): 4 per A stage
#define PF_DQ_WARP0 3                               // warps 0-2: weight TMA, MMA, activation TMA
#define PF_THREADS (32 * (PF_DQ_WARP0 + PF_DQ_WARPS))

#define LAUNCH_COUNT(p) \
    do {                \
        if (p) (*(p))++; \
    } while (0)

// exact float of a small non-negative integer (< 2^23)
__device__ __forceinline__ float pf_i2f(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }
__device__ __forceinline__ uint32_t pf_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// ===========================================================================
// plan: counting sort of the (token, slot) pairs by expert, in three
// launches (count, offsets + tile list, scatter).  Pair order inside an
// expert follows arrival; every pair's result depends on its own token and
// expert only (each MMA column is an independent dot product), so the output
// does not.  cnt[E + 1] / cur[E + 1] are zero between calls.
// ===========================================================================
#define PF_PLAN_PAIRS 2048  // pairs per block of the count and scatter kernels

__global__ void __launch_bounds__(256) k_pf_count(MoeDims d, const int *__restrict__ idx, int n, int *__restrict__ cnt,
                                                  int *__restrict__ error) {
    __shared__ int h[1025];
    for (int e = threadIdx.x; e < d.E; e += blockDim.x) h[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * PF_PLAN_PAIRS, p1 = min(n, p0 + PF_PLAN_PAIRS);
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const int e = idx[p];
        if (e < 0 || e >= d.E) { atomicExch(error, MOE_DEV_ERR_INDEX); continue; }
        atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < d.E; e += blockDim.x)
        if (h[e]) atomicAdd(&cnt[e], h[e]);
}

// one block: expert offsets (routed experts, then the shared expert's T
// pairs), the tile list, the scatter cursors; clears cnt for the next call
__global__ void __launch_bounds__(1024) k_pf_offsets(MoeDims d, int T, int *__restrict__ cnt, int *__restrict__ cur,
                                                     MoePlan plan) {
    __shared__ int c[1025], off[1026], toff[1026];
    const int E = d.E, NE = E + 1;
    for (int e = threadIdx.x; e < E; e += blockDim.x) { c[e] = cnt[e]; cnt[e] = 0; }
    if (threadIdx.x == 0) c[E] = T;
    __syncthreads();
    if (threadIdx.x == 0) {
        int a = 0, b = 0;
        for (int e = 0; e < NE; e++) {
            off[e] = a;
            toff[e] = b;
            a += c[e];
            b += (c[e] + PF_TILE_N - 1) / PF_TILE_N;  // tiles of the expert
        }
        plan.counts[0] = a;
        plan.counts[1] = b;
        plan.counts[2] = off[E];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < NE; e += blockDim.x) {
        cur[e] = off[e];
        // the expert's pairs split evenly (sizes differ by at most one), so no
        // tile is a small remainder that pays for a whole dequantization
        const int nt = (c[e] + PF_TILE_N - 1) / PF_TILE_N;
        for (int k = 0; k < nt; k++) {
            const int a = (int)((long long)k * c[e] / nt), z = (int)((long long)(k + 1) * c[e] / nt);
            plan.chunk_expert[toff[e] + k] = e;
            plan.chunk_pair0[toff[e] + k] = off[e] + a;
            plan.chunk_ntok[toff[e] + k] = z - a;
        }
    }
}

// pairs of PF_PLAN_PAIRS per block: a block reserves each expert's range
// with one global atomic, then places its pairs inside it
__global__ void __launch_bounds__(256) k_pf_scatter(MoeDims d, const int *__restrict__ idx,
                                                    const float *__restrict__ w, int T, int *__restrict__ cur,
                                                    MoePlan plan) {
    __shared__ int h[1025], base[1025];
    const int E = d.E, K = d.K, n = T * K;
    for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * PF_PLAN_PAIRS, p1 = min(n, p0 + PF_PLAN_PAIRS);
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const int e = idx[p];
        if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        base[e] = h[e] ? atomicAdd(&cur[e], h[e]) : 0;
        h[e] = 0;
    }
    __syncthreads();
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const int t = p / K, k = p % K, e = idx[p];
        if (e < 0 || e >= E) { plan.slot_pair[t * (K + 1) + k] = -1; continue; }
        const int pos = base[e] + atomicAdd(&h[e], 1);
        plan.pair_expert[pos] = e;
        plan.pair_token[pos] = t;
        plan.pair_w[pos] = w[p];
        plan.slot_pair[t * (K + 1) + k] = pos;
    }
    // the shared expert's pairs: token order after the routed pairs
    const int sh0 = plan.counts[2];
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
        const int pos = sh0 + t;
        plan.pair_expert[pos] = E;
        plan.pair_token[pos] = t;
        plan.pair_w[pos] = 1.0f;
        plan.slot_pair[t * (K + 1) + K] = pos;
    }
}

// fp16 rows of the pairs, token-major: block t copies token t's fp16 row
// (xh = half(x), written by the router's split) to each of its K + 1 pair
// rows, xg[p] = half(x[token(p)])
__global__ void __launch_bounds__(256) k_prefill_gather(const __half *__restrict__ xh, int H, int K, MoePlan plan,
                                                        __half *__restrict__ xg) {
    __shared__ int pos[64];
    const int t = blockIdx.x;
    if (threadIdx.x <= K) pos[threadIdx.x] = plan.slot_pair[t * (K + 1) + threadIdx.x];
    __syncthreads();
    const uint4 *src = reinterpret_cast<const uint4 *>(xh + (size_t)t * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
        const uint4 v = __ldg(src + i);
        for (int k = 0; k <= K; k++)
            if (pos[k] >= 0) reinterpret_cast<uint4 *>(xg + (size_t)pos[k] * H)[i] = v;
    }
}

// combine (infer.m:1915-1922), token-major: out[t] = sum_k w_k eo[pair(t, k)]
// in slot order, then + the shared expert's row -- the same fp32 operations
// in the same order as the decode combine, four columns per thread
__global__ void __launch_bounds__(256) k_prefill_combine(MoeDims d, MoePlan plan, const float *__restrict__ eo,
                                                         float *__restrict__ out) {
    __shared__ int pos[64];
    __shared__ float wk[64];
    const int t = blockIdx.x, K = d.K, H = d.H;
    if (threadIdx.x <= K) {
        const int p = plan.slot_pair[t * (K + 1) + threadIdx.x];
        pos[threadIdx.x] = p;
        wk[threadIdx.x] = p >= 0 ? plan.pair_w[p] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int k = 0; k < K; k++) {
            if (pos[k] < 0) continue;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(eo + (size_t)pos[k] * H) + i);
            const float wv = wk[k];
            acc = make_float4(fmaf(wv, v.x, acc.x), fmaf(wv, v.y, acc.y), fmaf(wv, v.z, acc.z), fmaf(wv, v.w, acc.w));
        }
        const float4 sv = __ldg(reinterpret_cast<const float4 *>(eo + (size_t)pos[K] * H) + i);
        reinterpret_cast<float4 *>(out + (size_t)t * H)[i] =
            make_float4(acc.x + sv.x, acc.y + sv.y, acc.z + sv.z, acc.w + sv.w);
    }
}

// ===========================================================================
// dequantization of one 64-column A atom of one weight row into 32 registers
// (fp16 pairs, k = 2c and 2c + 1 in register c), written to tensor memory by
// the caller.  fp16 arithmetic with exact intermediate steps:
//   - a byte permute puts two weight bytes under the fp16 exponent of 1024
//     (0x64 high bytes); masking keeps the low nibble (1024 + q) or the high
//     nibble in place (1024 + 16 q), exact;
//   - Q4_K, w = d*sc*q - dmin*m: p = fma(1024 + q, sc, -1024 sc) = q*sc
//     exactly (<= 945; the high nibble uses sc/16 and -64 sc); then
//     fma(d, p, -dm_hi) - dm_lo with dmin*m = dm_hi + dm_lo split into two
//     fp16 values (exact), so the result is rounded on the scale of w itself;
//   - Q6_K, w = d*sc*(q - 32): (1024 + q) - 1056 = q - 32 exactly; then
//     fma(q - 32, fs_hi, (q - 32) * fs_lo) with d*sc = fs_hi + fs_lo.
// ===========================================================================
__device__ __forceinline__ uint32_t pf_h2u(__half2 h) { return *reinterpret_cast<const uint32_t *>(&h); }
__device__ __forceinline__ __half2 pf_u2h(uint32_t u) { return *reinterpret_cast<const __half2 *>(&u); }
__device__ __forceinline__ uint32_t pf_dup(float x) { return pf_h2u(__float2half2_rn(x)); }
// (hi, lo) fp16 pair of an fp32 value with <= 22 significant bits: hi + lo == x
__device__ __forceinline__ void pf_split(float x, uint32_t &hi, uint32_t &lo) {
    const float h = __half2float(__float2half_rn(x));
    hi = pf_dup(h);
    lo = pf_dup(x - h);
}

// the constants of Q4_K atom g (sub-blocks 2g, 2g + 1):
// {sc0, -1024 sc0, -dm0_hi, -dm0_lo, sc1/16, -64 sc1, -dm1_hi, -dm1_lo}
__device__ __forceinline__ void pf_q4_consts(uint4 h, int g, uint32_t (&c)[8]) {
    const float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
    int sc0 = 0, m0 = 0, sc1 = 0, m1 = 0;
    if (g == 0) { q4_scale_min<0>(h, sc0, m0); q4_scale_min<1>(h, sc1, m1); }
    else if (g == 1) { q4_scale_min<2>(h, sc0, m0); q4_scale_min<3>(h, sc1, m1); }
    else if (g == 2) { q4_scale_min<4>(h, sc0, m0); q4_scale_min<5>(h, sc1, m1); }
    else { q4_scale_min<6>(h, sc0, m0); q4_scale_min<7>(h, sc1, m1); }
    c[0] = pf_dup((float)sc0);
    c[1] = pf_dup(-1024.0f * (float)sc0);
    pf_split(-dmin * (float)m0, c[2], c[3]);
    c[4] = pf_dup(0.0625f * (float)sc1);
    c[5] = pf_dup(-64.0f * (float)sc1);
    pf_split(-dmin * (float)m1, c[6], c[7]);
}

// two weights: fp16 pair (1024 + v) or (1024 + 16 v) -> d * sc * v - dm
__device__ __forceinline__ uint32_t pf_q4_pair(uint32_t x, __half2 d2, const uint32_t *c) {
    const __half2 p = __hfma2(pf_u2h(x), pf_u2h(c[0]), pf_u2h(c[1]));  // v * sc, exact
    return pf_h2u(__hadd2(__hfma2(p, d2, pf_u2h(c[2])), pf_u2h(c[3])));
}

// Q4_K atom g of one row: w[2t], w[2t + 1] = old qs bytes 32 g + 8 t .. + 7
// (at 16 + 32 t + 8 g of the repacked block); low nibbles are k = 8 t + i
// (registers 4t ..), high nibbles k = 32 + 8 t + i (registers 16 + 4t ..).
__device__ __forceinline__ void pf_deq_q4(const uint32_t (&w)[8], __half2 d2, const uint32_t (&c)[8],
                                          uint32_t (&v)[32]) {
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t x01 = __byte_perm(w[2 * t + h], 0x64u, 0x4140u);  // bytes 0, 1 under 0x64
            const uint32_t x23 = __byte_perm(w[2 * t + h], 0x64u, 0x4342u);
            v[4 * t + 2 * h] = pf_q4_pair(x01 & 0xFF0FFF0Fu, d2, c);
            v[4 * t + 2 * h + 1] = pf_q4_pair(x23 & 0xFF0FFF0Fu, d2, c);
            v[16 + 4 * t + 2 * h] = pf_q4_pair(x01 & 0xFFF0FFF0u, d2, c + 4);
            v[16 + 4 * t + 2 * h + 1] = pf_q4_pair(x23 & 0xFFF0FFF0u, d2, c + 4);
        }
}

// the constants of Q6_K atom g (sub-blocks 4g .. 4g + 3): {fs_hi, fs_lo} x 4
// with fs = d * sc (exact in fp32)
__device__ __forceinline__ void pf_q6_consts(float d6, uint32_t sc4, uint32_t (&c)[8]) {
#pragma unroll
    for (int u = 0; u < 4; u++) pf_split(d6 * (float)(int8_t)(sc4 >> (8 * u)), c[2 * u], c[2 * u + 1]);
}

// Q6_K atom A of one row (sub-blocks 4A + s4, half h = A / 2): q[6t + ..] =
// lane chunk t's ql words s4 = 0..3 and qh words 0, 1 of half h (the high
// bit of every qh pair stored inverted, so the 6-bit field nib | qh2 << 4 is
// q ^ 32; one more xor restores q).  k = 16 s4 + 4 t + i -> register
// 8 s4 + 2 t + i / 2.
template <int A>
__device__ __forceinline__ void pf_deq_q6(const uint32_t (&q)[24], const uint32_t (&c)[8], uint32_t (&v)[32]) {
    const __half2 off = pf_u2h(0x64206420u);  // 1056 = 1024 + 32
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int s4 = 0; s4 < 4; s4++) {
            const int sp = 4 * (A & 1) + s4, f = sp >> 1;
            const uint32_t W = q[6 * t + s4];
            const uint32_t Hq = q[6 * t + 4 + (s4 & 1)];
            const uint32_t nib = (sp < 4 ? W : W >> 4) & 0x0F0F0F0Fu;
            const uint32_t hb = (2 * f <= 4 ? Hq << (4 - 2 * f) : Hq >> (2 * f - 4)) & 0x30303030u;
            const uint32_t q6 = nib | (hb ^ 0x20202020u);  // four values q in bytes
            const __half2 fh = pf_u2h(c[2 * s4]), fl = pf_u2h(c[2 * s4 + 1]);
            const __half2 v01 = __hsub2(pf_u2h(__byte_perm(q6, 0x64u, 0x4140u)), off);  // q - 32, exact
            const __half2 v23 = __hsub2(pf_u2h(__byte_perm(q6, 0x64u, 0x4342u)), off);
            v[8 * s4 + 2 * t] = pf_h2u(__hfma2(v01, fh, __hmul2(v01, fl)));
            v[8 * s4 + 2 * t + 1] = pf_h2u(__hfma2(v23, fh, __hmul2(v23, fl)));
        }
}

// ===========================================================================
// GEMM.  MODE 0: gate/up (Q4_K) -> act (fp16, SwiGLU); 1: down Q4_K -> eo;
// 2: down Q6_K -> eo.  Persistent 2-CTA clusters (a CTA pair on one TPC):
// cluster c takes the work items c, c + clusters, ... in order; item =
// tile x pair row group (PR per tile), tile = (expert, <= PF_TILE_N pairs).
// In a pair, CTA r holds row group 2 x pair row group + r (PF_RB row blocks
// of 128 accumulator rows; MODE 0: a block is 64 gate rows + the matching 64
// up rows).  Each pair MMA (M = 256: block b of both CTAs) takes the first
// half of the tile's pairs from the leader's activation stage and the second
// half from the peer's, so each SM streams half of the tile's activations per
// K step, and each stage feeds PF_RB pair MMAs.  The clusters resident at one
// time work on neighbouring items (a few tiles), so each tile's activation
// slices are read from DRAM once and then hit in L2.  Every role keeps its
// ring positions across items: the weight and activation producers run ahead
// into the next item while the last MMAs and the epilogue of the current one
// run, and each dequantizing group writes its first A stage of the next item
// before it reads back the previous item's accumulator, so the MMAs restart
// as soon as the accumulator has been read (acc_empty).
// ===========================================================================
struct PfItem {
    int e, p0, ntile, slot, rg, npair;
};

// the item's tile and rows; false for a tile of the other down type (the
// shared and the routed experts may differ), which every role skips alike
template <int MODE>
__device__ __forceinline__ bool pf_item(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, int item, int PR,
                                        uint32_t rank, PfItem &it) {
    const int tile = item / PR;
    it.e = plan.chunk_expert[tile];
    if (MODE > 0 && ((it.e == d.E) ? L.sh_down_type : L.down_type) != (MODE == 2 ? MOE_TYPE_Q6_K : MOE_TYPE_Q4_K))
        return false;
    it.p0 = plan.chunk_pair0[tile];
    it.ntile = plan.chunk_ntok[tile];
    it.slot = it.e == d.E ? L.n_local : it.e - L.e0;
    it.rg = 2 * (item % PR) + (int)rank;
    it.npair = (it.ntile + 31) & ~31;  // pair MMA N (a multiple of 32); N / 2 pairs per CTA
    return true;
}

// uses of A stage s per item: the atoms i < n_atoms with i % PF_NSA == s
__device__ __forceinline__ int pf_stage_uses(int n_atoms, int s) { return (n_atoms - s + PF_NSA - 1) / PF_NSA; }

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PF_THREADS, 1)
    k_prefill_gemm(MoeDims d, const __grid_constant__ MoeLayerDev L, MoePlan plan,
                   const __grid_constant__ CUtensorMap tmB, int PR, __half *__restrict__ act, float *__restrict__ eo) {
    constexpr int RAW = MODE == 2 ? PF_RAW_Q6 : PF_RAW_Q4;
    constexpr int RAW_NS = MODE == 2 ? PF_RAW_NS_Q6 : PF_RAW_NS_Q4;
    constexpr int QB = MODE == 2 ? 128 * PF_Q6_ROW : 128 * 144;  // one block's Q bytes in a raw stage
    extern __shared__ uint8_t pf_raw[];
    uint8_t *sm = pf_raw + ((1024u - (umma_smem_u32(pf_raw) & 1023u)) & 1023u);
    uint8_t *sb = sm, *sr = sm + PF_NSB * PF_BST;
    // Q6_K d planes of the blocks (PF_RB x 128 rows x 2 nb_pad bytes), two
    // buffers by item parity: the producer refills one only after the raw
    // ring shows every warp past the item that read it (NB >= RAW_NS)
    uint8_t *sd = sr + RAW_NS * RAW;
    __shared__ __align__(8) uint64_t raw_full[PF_RAW_NS_MAX], raw_empty[PF_RAW_NS_MAX], a_full[PF_NSA], a_empty[PF_NSA],
        b_full[PF_NSB], b_empty[PF_NSB], acc_full, acc_empty;
    __shared__ uint32_t tmem_base;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the pair MMAs
    const int cl = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    const int K = MODE == 0 ? d.H : d.I, NB = K / MOE_QK, n_atoms = 4 * NB;
    const int nbp = q6r_nb_pad(NB), dpl = PF_RB * 256 * nbp;  // bytes of one d-plane buffer
    const int n_items = plan.counts[1] * PR;                   // the same in both CTAs
    if (tid == 0) {
        // raw_empty: 4 atoms x 4 lane-quarter warps per super-block.  a_full /
        // b_full / acc_empty are used in the leader: 4 dequantizing warps of
        // each CTA; the leader's expect_tx (both CTAs' copies complete on it);
        // every dequantizing warp of both CTAs.  The empty barriers and
        // acc_full of both CTAs receive the leader's commits (tcgen05.commit
        // to both).
        for (int i = 0; i < RAW_NS; i++) { tc_mbar_init(&raw_full[i], 1); tc_mbar_init(&raw_empty[i], 16); }
        for (int i = 0; i < PF_NSA; i++) { tc_mbar_init(&a_full[i], 8); tc_mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < PF_NSB; i++) { tc_mbar_init(&b_full[i], 1); tc_mbar_init(&b_empty[i], 1); }
        tc_mbar_init(&acc_full, 1);
        tc_mbar_init(&acc_empty, 2 * PF_DQ_WARPS);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    // tensor memory (the same columns in both CTAs): accumulator b in columns
    // [PF_TILE_N b, + PF_TILE_N), A stage s of block b in [2 PF_TILE_N + 64 s + 32 b, + 32)
    if (warp == 1) tmem_alloc_pair(&tmem_base, 512);
    tmem_fence_before();
    cluster_sync_all();
    tmem_fence_after();
    const uint32_t tmem = tmem_base, tmem_a = tmem_base + PF_RB * PF_TILE_N;
    // the pair MMAs address both CTAs' tensor memory with the leader's columns
    bool ok = cluster_ld_u32(cluster_map(&tmem_base, rank ^ 1u)) == tmem;
    if (!ok && tid == 0) atomicExch(plan.error, PF_ERR_PAIR);

    if (!ok) {
        // nothing issued: both CTAs go straight to the teardown
    } else if (warp == 0) {
        // weight producer: the raw tiles of this CTA's blocks, one super-block
        // per stage, RAW_NS ahead (the warp loops together, one elected lane
        // issues the copies)
        const uint32_t leader = elect_one();
        int gs = 0, jn = 0;  // super-blocks issued, items taken
        for (int item = cl; item < n_items && ok; item += ncl) {
            PfItem it;
            if (!pf_item<MODE>(d, L, plan, item, PR, rank, it)) continue;
            for (int sbk = 0; sbk < NB; sbk++, gs++) {
                const int rs = gs % RAW_NS;
                if (!tc_wait_warp(&raw_empty[rs], ((gs / RAW_NS) & 1) ^ 1)) { ok = false; break; }
                uint8_t *r = sr + rs * RAW;
                if (leader) {
                    tc_expect(&raw_full[rs], RAW + (MODE == 2 && sbk == 0 ? dpl : 0));
#pragma unroll
                    for (int b = 0; b < PF_RB; b++) {
                        const int blk = PF_RB * it.rg + b;
                        if (MODE == 0) {
                            tc_tma3(r + b * QB, &L.tm_gu, sbk * MOE_Q4K_BYTES, blk * 64, it.slot, &raw_full[rs]);
                            tc_tma3(r + b * QB + 64 * MOE_Q4K_BYTES, &L.tm_gu, sbk * MOE_Q4K_BYTES, d.I + blk * 64,
                                    it.slot, &raw_full[rs]);
                        } else if (MODE == 1) {
                            tc_tma3(r + b * QB, &L.tm_d4, sbk * MOE_Q4K_BYTES, blk * 128, it.slot, &raw_full[rs]);
                        } else {
                            tc_tma3(r + b * QB, &L.tm_pf6q, sbk * 192, blk * 128, it.slot, &raw_full[rs]);
                            tc_tma3(r + PF_RB * QB + b * 2048, &L.tm_d6s, sbk * 16, blk * 128, it.slot, &raw_full[rs]);
                            if (sbk == 0)
                                tc_tma3(sd + (jn & 1) * dpl + b * 256 * nbp, &L.tm_d6d, 0, blk * 128, it.slot,
                                        &raw_full[rs]);
                        }
                    }
                }
            }
            jn++;
        }
        if (!ok && leader) {
            atomicExch(plan.error, PF_ERR_TIMEOUT);
            tc_drain(raw_full, gs, RAW_NS);
        }
    } else if (warp == 2) {
        // activation producer: this CTA's half of the tile's pairs (16-row
        // boxes), PF_NSB atoms ahead.  The copies of both CTAs complete on the
        // leader's b_full, where the leader expects the bytes of both halves.
        // Only the boxes that reach the tile's pairs are loaded: the rows of a
        // half past them (N is rounded up to 32) keep stale values, which
        // reach only accumulator columns that are never stored (column n of
        // D depends on row n of B alone).
        const uint32_t leader = elect_one();
        int gb = 0;  // atoms issued
        for (int item = cl; item < n_items && ok; item += ncl) {
            PfItem it;
            if (!pf_item<MODE>(d, L, plan, item, PR, rank, it)) continue;
            const int nhalf = it.npair / 2, y0 = it.p0 + (int)rank * nhalf;
            // 16-row boxes of each half that hold pairs of the tile
            const int real0 = min(it.ntile, nhalf), real1 = max(it.ntile - nhalf, 0);
            const int nb0 = (real0 + 15) / 16, nb1 = (real1 + 15) / 16, nbox = rank ? nb1 : nb0;
            for (int i = 0; i < n_atoms; i++, gb++) {
                const int st = gb % PF_NSB;
                if (!tc_wait_warp(&b_empty[st], ((gb / PF_NSB) & 1) ^ 1)) { ok = false; break; }
                if (leader) {
                    if (rank == 0) tc_expect(&b_full[st], (nb0 + nb1) * PF_BOX16);
                    const uint32_t bar = cluster_map(&b_full[st], 0);
                    for (int bx = 0; bx < nbox; bx++)
                        tc_tma2_pair(sb + st * PF_BST + bx * PF_BOX16, &tmB, 64 * i, y0 + 16 * bx, bar);
                }
            }
        }
        if (!ok && leader) {
            atomicExch(plan.error, PF_ERR_TIMEOUT);
            // the leader waits (bounded) for the last stages; the peer's copies
            // complete on the leader's barriers, and a peer that gave up here
            // issued its last copy at least one wait limit earlier
            if (rank == 0) tc_drain(b_full, gb, PF_NSB);
        }
    } else if (warp == 1) {
        if (rank == 0) {
            // MMA issuer (leader): the whole warp runs the loop, one elected lane
            // issues each MMA and commit; the operands are broadcast from lane 0 so
            // that they sit in uniform registers and the MMAs issue back to back.
            // The commits arrive on the barrier of the same address in both CTAs.
            const uint32_t td = __shfl_sync(0xffffffffu, tmem, 0), ta0 = __shfl_sync(0xffffffffu, tmem_a, 0);
            int gb = 0, jn = 0;  // atoms consumed, items taken
            for (int item = cl; item < n_items && ok; item += ncl) {
                PfItem it;
                if (!pf_item<MODE>(d, L, plan, item, PR, rank, it)) continue;
                const uint32_t idesc = __shfl_sync(0xffffffffu, umma_idesc_f16(2 * PF_TILE, it.npair), 0);
                // the previous item's accumulator has been read by every epilogue warp
                if (!tc_wait_warp(&acc_empty, (jn & 1) ^ 1)) { ok = false; break; }
                tmem_fence_after();
                for (int i = 0; i < n_atoms; i++, gb++) {
                    const int sa = i % PF_NSA, sbq = gb % PF_NSB;
                    const int use = jn * pf_stage_uses(n_atoms, sa) + i / PF_NSA;
                    if (!tc_wait_warp(&a_full[sa], use & 1) || !tc_wait_warp(&b_full[sbq], (gb / PF_NSB) & 1)) {
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const uint64_t bdesc =
                        umma_desc_sw128(__shfl_sync(0xffffffffu, umma_smem_u32(sb + sbq * PF_BST), 0));
                    const uint32_t ta = __shfl_sync(0xffffffffu, ta0 + 64 * sa, 0);
                    const uint32_t acc = __shfl_sync(0xffffffffu, i, 0) != 0 ? 1u : 0u;
#pragma unroll
                    for (int b = 0; b < PF_RB; b++)
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)  // +32 B of K per step: +2 in the descriptor's address field
                            umma_f16_ta_pair_warp(td + PF_TILE_N * b, ta + 32 * b + 8 * kk,
                                                  bdesc + (uint64_t)(2 * kk), idesc, (acc | kk) ? 1u : 0u);
                    umma_commit_pair_warp(&a_empty[sa]);
                    umma_commit_pair_warp(&b_empty[sbq]);
                }
                if (!ok) break;
                umma_commit_pair_warp(&acc_full);
                jn++;
            }
            if (!ok) {
                // the MMAs already issued finish before tensor memory is freed:
                // one more commit completes phase jn of acc_full after all of them
                if (lane == 0) atomicExch(plan.error, PF_ERR_TIMEOUT);
                umma_commit_pair_warp(&acc_full);
                tc_wait_warp(&acc_full, jn & 1);
            }
        }
    } else {
        // dequantization: warp (q = warp % 4, g) owns tensor-memory lanes
        // 32 q .. 32 q + 31 (A rows; lane = row) of both blocks, and atoms
        // i = g, g + PF_NSA, g + 2 PF_NSA, ... (K order) of every item, all of
        // them through A stage g.  A stage has one producer group that takes
        // its uses in order, so a parity wait on it is never a whole phase
        // early; every group meets every super-block (4 consecutive atoms
        // cover all residues mod PF_NSA), in order, so the raw-stage waits are
        // exact too.  The same warps run the epilogue of each item, after
        // their first A stage of the next item.
        const int q = warp & 3, g = (warp - PF_DQ_WARP0) >> 2, row = 32 * q + lane;
        int rraw = row;  // raw tile row (inside a block) holding A row `row`
        if (MODE == 0) {
            const int h = (row >> 4) & 1, i = row & 15;  // row = 32 q + 16 h + i
            rraw = h * 64 + 16 * q + i;                   // gate rows first, then up rows
        }
        const uint32_t tlane = (uint32_t)(32 * q) << 16;
        const int uses = pf_stage_uses(n_atoms, g);
        const int sub = (warp - PF_DQ_WARP0) >> 2;  // epilogue: column chunks alternate between the groups
        const uint32_t acc_empty_leader = cluster_map(&acc_empty, 0);
        // epilogue of item P (the jp-th taken): this warp reads tensor-memory
        // lanes 32 (warp % 4) .. + 31 of both accumulators, then releases them
        auto epilogue = [&](const PfItem &P, int jp) -> bool {
            if (!tc_wait_warp(&acc_full, jp & 1)) return false;
            tmem_fence_after();
#pragma unroll 1
            for (int b = 0; b < PF_RB; b++) {
                const int blk = PF_RB * P.rg + b;
                for (int c = 16 * sub; c < P.ntile; c += 16 * (PF_DQ_WARPS / 4)) {
                    float v[16];
                    tmem_ld16(tmem + PF_TILE_N * b + ((uint32_t)(32 * q) << 16) + c, v);
                    if (MODE == 0) {
                        // lanes 0-15: gate rows, 16-31: the matching up rows
                        const int i = lane & 15, rI = blk * 64 + 16 * q + i;
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            // silu(g) * u with the fast exponential and division: the
                            // result is rounded to fp16 (2^-11), far above their error
                            const float u = __shfl_xor_sync(0xffffffffu, v[j], 16);
                            if (lane < 16 && c + j < P.ntile)
                                act[(size_t)(P.p0 + c + j) * d.I + rI] =
                                    __float2half_rn(__fdividef(v[j], 1.0f + __expf(-v[j])) * u);
                        }
                    } else {
                        const int rH = blk * 128 + 32 * q + lane;
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            if (c + j < P.ntile) eo[(size_t)(P.p0 + c + j) * d.H + rH] = v[j];
                    }
                }
            }
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) tc_arrive_cluster(acc_empty_leader);
            return true;
        };
        int gs0 = 0, jn = 0;  // first super-block of the item in the raw ring, items taken
        PfItem prev{};
        bool pending = false;  // prev's epilogue not yet run
        for (int item = cl; item < n_items && ok; item += ncl) {
            PfItem it;
            if (!pf_item<MODE>(d, L, plan, item, PR, rank, it)) continue;
            const uint8_t *dplane = sd + (jn & 1) * dpl;
            for (int i = g, j = 0; i < n_atoms; i += PF_NSA, j++) {
                const int sbk = i >> 2, ga = i & 3, gs = gs0 + sbk;  // super-block, atom inside it
                const int rs = gs % RAW_NS;
                if (!tc_wait_warp(&raw_full[rs], (gs / RAW_NS) & 1)) { ok = false; break; }
                const uint8_t *r = sr + rs * RAW;
                // atom ga of this lane's rows in both blocks, dequantized into
                // registers before the tensor-memory stage is waited for
                uint32_t v[PF_RB][32];
#pragma unroll
                for (int b = 0; b < PF_RB; b++) {
                    uint32_t c[8];
                    if constexpr (MODE == 2) {
                        // chunk t: ql words s4 = 0..3 and qh words 0, 1 of half ga / 2
                        // (bytes 0-23 or 24-47 of the chunk: a 16-byte and an 8-byte load)
                        uint32_t w[24];
#pragma unroll
                        for (int t = 0; t < 4; t++) {
                            const uint8_t *cp = r + b * QB + rraw * PF_Q6_ROW + 48 * t;
                            if (ga < 2) {
                                const uint4 x = *reinterpret_cast<const uint4 *>(cp);
                                const uint2 y = *reinterpret_cast<const uint2 *>(cp + 16);
                                w[6 * t] = x.x; w[6 * t + 1] = x.y; w[6 * t + 2] = x.z; w[6 * t + 3] = x.w;
                                w[6 * t + 4] = y.x; w[6 * t + 5] = y.y;
                            } else {
                                const uint2 x = *reinterpret_cast<const uint2 *>(cp + 24);
                                const uint4 y = *reinterpret_cast<const uint4 *>(cp + 32);
                                w[6 * t] = x.x; w[6 * t + 1] = x.y; w[6 * t + 2] = y.x; w[6 * t + 3] = y.y;
                                w[6 * t + 4] = y.z; w[6 * t + 5] = y.w;
                            }
                        }
                        const uint32_t sc4 =
                            reinterpret_cast<const uint32_t *>(r + PF_RB * QB + b * 2048 + rraw * 16)[ga];
                        const float d6 =
                            __half2float(reinterpret_cast<const __half *>(dplane + b * 256 * nbp)[rraw * nbp + sbk]);
                        pf_q6_consts(d6, sc4, c);
                        if (ga == 0) pf_deq_q6<0>(w, c, v[b]);
                        else if (ga == 1) pf_deq_q6<1>(w, c, v[b]);
                        else if (ga == 2) pf_deq_q6<2>(w, c, v[b]);
                        else pf_deq_q6<3>(w, c, v[b]);
                    } else {
                        const uint8_t *blk = r + b * QB + rraw * MOE_Q4K_BYTES;
                        const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
                        uint32_t w[8];
#pragma unroll
                        for (int t = 0; t < 4; t++) {
                            const uint2 x = *reinterpret_cast<const uint2 *>(blk + 16 + 32 * t + 8 * ga);
                            w[2 * t] = x.x;
                            w[2 * t + 1] = x.y;
                        }
                        pf_q4_consts(hd, ga, c);
                        pf_deq_q4(w, pf_u2h(__byte_perm(hd.x, 0, 0x1010)), c, v[b]);  // d in both halves
                    }
                }
                // all reads of the stage are done (their values are consumed): the
                // proxy fence orders them before the next TMA write into it
                fence_async_smem();
                __syncwarp();
                if (lane == 0) tc_arrive(&raw_empty[rs]);
                if (!tc_wait_warp(&a_empty[g], ((jn * uses + j) & 1) ^ 1)) { ok = false; break; }
                tmem_fence_after();
#pragma unroll
                for (int b = 0; b < PF_RB; b++) tmem_st32(tmem_a + tlane + 64 * g + 32 * b, v[b]);
                tmem_wait_st();
                tmem_fence_before();
                __syncwarp();
                if (lane == 0) tc_arrive_cluster(cluster_map(&a_full[g], 0));  // the leader's barrier
                if (j == 0 && pending) {
                    // the previous item's epilogue, now that this group's first
                    // stage of this item is written
                    if (!epilogue(prev, jn - 1)) { ok = false; break; }
                    pending = false;
                }
            }
            prev = it;
            pending = true;
            gs0 += NB;
            jn++;
        }
        if (ok && pending && !epilogue(prev, jn - 1)) ok = false;
        if (!ok && lane == 0) atomicExch(plan.error, PF_ERR_TIMEOUT);
    }
    // teardown: every thread of both CTAs arrives (no access from the other CTA
    // after this), then each CTA frees its tensor memory
    tmem_fence_before();
    __syncwarp();
    cluster_sync_all();
    if (warp == 1) tmem_free_pair(tmem, 512);
}

// ===========================================================================
// router logits for many tokens on the tensor cores, to fp32 accuracy:
// logits = W x with W (E x H) and x (T x H) fp32 (the reference's fp32 sgemv,
// infer.m:1881).  Both are split into fp16 pairs, W * 256 = Wh + Wl and
// x = xh + xl (each hi/lo pair holds 22 significant bits; the scale 2^8 is
// exact and keeps Wl out of the fp16 subnormal range), and
//   256 W x = Wh xh + Wh xl + Wl xh   (+ Wl xl, below 2^-22 relative, dropped)
// with fp16 x fp16 products exact in the fp32 accumulator.  The CTA computes
// 128 experts x 128 tokens over one of nsplit slices of K (nsplit sized so
// that the grid covers the SMs); the slices are summed in a fixed order and
// scaled by 1/256 (exact).
// ===========================================================================
#define RT_NS 3
#define RT_THREADS 192  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
#define RT_SCALE 256.0f

// dst_hi = half(src * scale), dst_lo = half(src * scale - dst_hi), n % 4 == 0
__global__ void __launch_bounds__(256) k_pf_split(const float *__restrict__ src, size_t n, float scale,
                                                  __half *__restrict__ hi, __half *__restrict__ lo) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(src) + i);
        const float a[4] = {v.x * scale, v.y * scale, v.z * scale, v.w * scale};
        __half h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            h[j] = __float2half_rn(a[j]);
            l[j] = __float2half_rn(a[j] - __half2float(h[j]));
        }
        reinterpret_cast<uint2 *>(hi)[i] = make_uint2(pf_h2u(__halves2half2(h[0], h[1])), pf_h2u(__halves2half2(h[2], h[3])));
        reinterpret_cast<uint2 *>(lo)[i] = make_uint2(pf_h2u(__halves2half2(l[0], l[1])), pf_h2u(__halves2half2(l[2], l[3])));
    }
}

// part[split][t][e] for 128 experts (blockIdx.x) x 128 tokens (blockIdx.y),
// K slice blockIdx.z of nsplit
__global__ void __launch_bounds__(RT_THREADS, 1)
    k_pf_router(int T, int H, int E, int nsplit, const __grid_constant__ CUtensorMap tm_wh, const __grid_constant__ CUtensorMap tm_wl,
                const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                float *__restrict__ part, int *__restrict__ error) {
    extern __shared__ uint8_t rt_raw[];
    uint8_t *sm = rt_raw + ((1024u - (umma_smem_u32(rt_raw) & 1023u)) & 1023u);  // RT_NS stages of 4 boxes
    __shared__ __align__(8) uint64_t full[RT_NS], empty[RT_NS], acc_full;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = 128 * blockIdx.x, n0 = 128 * blockIdx.y, split = blockIdx.z;
    const int na = H / 64 / nsplit, a0 = na * split;
    if (tid == 0) {
        for (int i = 0; i < RT_NS; i++) { tc_mbar_init(&full[i], 1); tc_mbar_init(&empty[i], 1); }
        tc_mbar_init(&acc_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&tmem_base, 128);
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = tmem_base;
    bool ok = true;
    if (warp == 0) {
        const uint32_t leader = elect_one();
        int issued = 0;
        for (int i = 0; i < na && ok; i++) {
            const int st = i % RT_NS;
            if (!tc_wait_warp(&empty[st], ((i / RT_NS) & 1) ^ 1)) { ok = false; break; }
            if (leader) {
                uint8_t *b = sm + st * 4 * PF_ATOM;
                const int kx = 64 * (a0 + i);
                tc_expect(&full[st], 4 * PF_ATOM);
                tc_tma2(b, &tm_wh, kx, m0, &full[st]);
                tc_tma2(b + PF_ATOM, &tm_wl, kx, m0, &full[st]);
                tc_tma2(b + 2 * PF_ATOM, &tm_xh, kx, n0, &full[st]);
                tc_tma2(b + 3 * PF_ATOM, &tm_xl, kx, n0, &full[st]);
            }
            issued = i + 1;
        }
        if (!ok && leader) {
            atomicExch(error, PF_ERR_TIMEOUT);
            tc_drain(full, issued, RT_NS);
        }
    } else if (warp == 1) {
        const uint32_t idesc = umma_idesc_f16(128, 128);
        for (int i = 0; i < na && ok; i++) {
            const int st = i % RT_NS;
            if (!tc_wait_warp(&full[st], (i / RT_NS) & 1)) { ok = false; break; }
            tmem_fence_after();
            const uint32_t b = umma_smem_u32(sm + st * 4 * PF_ATOM);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint64_t wh = umma_desc_sw128(b + 32 * kk), wl = umma_desc_sw128(b + PF_ATOM + 32 * kk);
                const uint64_t xh = umma_desc_sw128(b + 2 * PF_ATOM + 32 * kk), xl = umma_desc_sw128(b + 3 * PF_ATOM + 32 * kk);
                umma_f16_warp(tmem, wh, xh, idesc, (i | kk) != 0);
                umma_f16_warp(tmem, wh, xl, idesc, 1);
                umma_f16_warp(tmem, wl, xh, idesc, 1);
            }
            umma_commit_warp(&empty[st]);
        }
        umma_commit_warp(&acc_full);
        if (!ok) {
            if (lane == 0) atomicExch(error, PF_ERR_TIMEOUT);
            tc_wait_warp(&acc_full, 0);
        }
    } else {
        // tensor-memory lanes 32 (warp % 4) .. + 31 = experts, columns = tokens
        if (tc_wait_warp(&acc_full, 0)) {
            tmem_fence_after();
            const int q = warp & 3, e = m0 + 32 * q + lane;
            for (int c = 0; c < 128; c += 16) {
                if (n0 + c >= T) break;
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c, v);
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (n0 + c + j < T && e < E) part[((size_t)split * T + n0 + c + j) * E + e] = v[j];
            }
        } else if (lane == 0) {
            atomicExch(error, PF_ERR_TIMEOUT);
        }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 1) tmem_free(tmem, 128);
}

// logits = (part[0] + part[1] + ...) / 256, in slice order
__global__ void __launch_bounds__(256) k_pf_router_sum(const float *__restrict__ part, size_t n, int nsplit,
                                                       float *__restrict__ logits) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float a = part[i];
        // the partials loaded 8 at a time (one L2 round trip per 8 slices),
        // added one by one in slice order
        for (int k = 1; k < nsplit; k += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = k + u < nsplit ? part[(size_t)(k + u) * n + i] : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (k + u < nsplit) a += v[u];
        }
        logits[i] = a * (1.0f / RT_SCALE);
    }
}

void moe_launch_prefill_router(const MoeDims &d, const float *Wr, MoePrefillWs &ws, const float *x, int T,
                               cudaStream_t s, uint64_t *launches) {
    const size_t nw = (size_t)d.E * d.H, nx = (size_t)T * d.H;
    k_pf_split<<<(unsigned)((nw / 4 + 255) / 256), 256, 0, s>>>(Wr, nw, RT_SCALE, ws.wh, ws.wl);
    k_pf_split<<<(unsigned)((nx / 4 + 255) / 256 < 148 * 16 ? (nx / 4 + 255) / 256 : 148 * 16), 256, 0, s>>>(
        x, nx, 1.0f, ws.xh, ws.xl);
    const size_t smem = 1024 + (size_t)RT_NS * 4 * PF_ATOM;
    static size_t attr[MOE_MAX_DEVICES];
    moe_smem_limit(k_pf_router, smem, attr);
    // K slices: a power of two dividing H / 64, up to 16, until the grid covers the SMs
    const int tiles = ((d.E + 127) / 128) * ((T + 127) / 128);
    int nsplit = 1;
    while (nsplit < 16 && tiles * nsplit < 148 && (d.H / 64) % (2 * nsplit) == 0) nsplit *= 2;
    k_pf_router<<<dim3((d.E + 127) / 128, (T + 127) / 128, nsplit), RT_THREADS, smem, s>>>(
        T, d.H, d.E, nsplit, ws.tm_wh, ws.tm_wl, ws.tm_xh, ws.tm_xl, ws.part, ws.plan.error);
    const size_t nl = (size_t)T * d.E;
    k_pf_router_sum<<<(unsigned)((nl + 255) / 256), 256, 0, s>>>(ws.part, nl, nsplit, ws.logits);
    if (launches) *launches += 4;
}

// The router weights' fp16 hi/lo split (x 2^8, the same split as the
// prefill router's), kept per layer for the decode path: wh / wl hold E rows
// of H (rows up to the 128-row box padded with zeros by the caller).
void moe_launch_router_split(const float *Wr, int E, int H, __half *wh, __half *wl, cudaStream_t s,
                             uint64_t *launches) {
    const size_t nw = (size_t)E * H;
    k_pf_split<<<(unsigned)((nw / 4 + 255) / 256), 256, 0, s>>>(Wr, nw, RT_SCALE, wh, wl);
    LAUNCH_COUNT(launches);
}

// Decode router logits of 5..64 tokens on the tensor cores: x split into fp16
// hi/lo (xh / xl: 128 rows, tm_xh / tm_xl over them), the three-MMA router
// against the layer's kept split, K slices summed in a fixed order into
// logits[T][E].  max_split bounds the slices (the part buffer holds
// max_split x T x E); the slice count is the largest divisor of H / 64 within
// it, so that the router CTAs cover more SMs.
void moe_launch_router_tc(const MoeDims &d, const CUtensorMap &tm_wh, const CUtensorMap &tm_wl, const float *x,
                          int T, __half *xh, __half *xl, const CUtensorMap &tm_xh, const CUtensorMap &tm_xl,
                          float *part, int max_split, float *logits, int *error, cudaStream_t s,
                          uint64_t *launches) {
    const size_t nx = (size_t)T * d.H;
    const size_t gx = (nx / 4 + 255) / 256;
    k_pf_split<<<(unsigned)(gx < 148 * 16 ? gx : 148 * 16), 256, 0, s>>>(x, nx, 1.0f, xh, xl);
    const size_t smem = 1024 + (size_t)RT_NS * 4 * PF_ATOM;
    static size_t attr[MOE_MAX_DEVICES];
    moe_smem_limit(k_pf_router, smem, attr);
    const int na = d.H / 64;
    int nsplit = 1;
    for (int k = max_split < na ? max_split : na; k >= 1; k--)
        if (na % k == 0) { nsplit = k; break; }
    k_pf_router<<<dim3((d.E + 127) / 128, (T + 127) / 128, nsplit), RT_THREADS, smem, s>>>(
        T, d.H, d.E, nsplit, tm_wh, tm_wl, tm_xh, tm_xl, part, error);
    const size_t nl = (size_t)T * d.E;
    k_pf_router_sum<<<(unsigned)((nl + 255) / 256), 256, 0, s>>>(part, nl, nsplit, logits);
    if (launches) *launches += 3;
}

// ===========================================================================
// expert parallelism for prefill (one process per GPU, experts sharded
// n_experts / world per rank, router and shared expert replicated).  Row
// space on rank r (world N, ecap rows per peer):
//   rows [p*ecap, p*ecap + ecap)  fp16 token rows received from rank p
//   rows [N*ecap, N*ecap + T)     this rank's own tokens (shared expert)
// Metadata of a sent row: [valid, src_token, idx[K], w_bits[K]].  The
// exchanges are NCCL send/recv of fixed-size buffers (moe_api.cu).
// ===========================================================================

// block p: tok_slot[t][p] = position of token t among the rows sent to rank
// p (tokens with at least one expert there, in token order) or -1; clears
// the valid flag of the unused rows
__global__ void __launch_bounds__(1024) k_pfe_slots(const int *__restrict__ idx, int T, int K, int n_local, int N,
                                                    int ecap, int *__restrict__ tok_slot, int *__restrict__ send_meta) {
    __shared__ int wsum[32], carry;
    const int p = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < T; base += blockDim.x) {
        const int t = base + threadIdx.x;
        int hit = 0;
        if (t < T)
            for (int k = 0; k < K; k++) {
                const int e = idx[t * K + k];
                if (e >= 0 && e / n_local == p) hit = 1;
            }
        int x = hit;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[wid] = x;
        __syncthreads();
        if (wid == 0) {
            int v = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += y;
            }
            wsum[lane] = v;
        }
        __syncthreads();
        const int excl = carry + (wid ? wsum[wid - 1] : 0) + x - hit;
        if (t < T) tok_slot[t * N + p] = hit ? excl : -1;
        __syncthreads();
        if (threadIdx.x == 0) carry += wsum[(blockDim.x >> 5) - 1];
        __syncthreads();
    }
    const int mw = 2 + 2 * K;
    for (int r = carry + threadIdx.x; r < ecap; r += blockDim.x) send_meta[((size_t)p * ecap + r) * mw] = 0;
}

// token t: its fp16 row and metadata to every rank it routes to
__global__ void __launch_bounds__(256) k_pfe_pack(const __half *__restrict__ xh, const int *__restrict__ idx,
                                                  const float *__restrict__ w, int K, int H, int N, int ecap,
                                                  const int *__restrict__ tok_slot, __half *__restrict__ send_xh,
                                                  int *__restrict__ send_meta) {
    const int t = blockIdx.x, mw = 2 + 2 * K;
    const uint4 *src = reinterpret_cast<const uint4 *>(xh + (size_t)t * H);
    for (int p = 0; p < N; p++) {
        const int sl = tok_slot[t * N + p];
        if (sl < 0) continue;
        const size_t row = (size_t)p * ecap + sl;
        uint4 *dst = reinterpret_cast<uint4 *>(send_xh + row * H);
        for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = __ldg(src + i);
        int *m = send_meta + row * mw;
        if (threadIdx.x == 0) { m[0] = 1; m[1] = t; }
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            m[2 + k] = idx[t * K + k];
            m[2 + K + k] = __float_as_int(w[t * K + k]);
        }
    }
}

// pairs (received row, expert of this rank) per expert, PF_PLAN_PAIRS per block
__global__ void __launch_bounds__(256) k_pfe_count(MoeDims d, const int *__restrict__ recv_meta, int R, int e0,
                                                   int n_local, int *__restrict__ cnt, int *__restrict__ error) {
    __shared__ int h[1025];
    const int K = d.K, mw = 2 + 2 * K;
    for (int e = threadIdx.x; e < d.E; e += blockDim.x) h[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * PF_PLAN_PAIRS, p1 = min(R * K, p0 + PF_PLAN_PAIRS);
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const int *m = recv_meta + (size_t)(p / K) * mw;
        if (!m[0]) continue;
        const int e = m[2 + p % K];
        if (e < 0 || e >= d.E) { atomicExch(error, MOE_DEV_ERR_INDEX); continue; }
        if (e >= e0 && e < e0 + n_local) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < d.E; e += blockDim.x)
        if (h[e]) atomicAdd(&cnt[e], h[e]);
}

__global__ void __launch_bounds__(256) k_pfe_scatter(MoeDims d, const int *__restrict__ recv_meta, int R, int T,
                                                     int e0, int n_local, int *__restrict__ cur, MoePlan plan) {
    __shared__ int h[1025], base[1025];
    const int E = d.E, K = d.K, mw = 2 + 2 * K;
    for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * PF_PLAN_PAIRS, p1 = min(R * K, p0 + PF_PLAN_PAIRS);
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const int *m = recv_meta + (size_t)(p / K) * mw;
        const int e = m[0] ? m[2 + p % K] : -1;
        if (e >= e0 && e < e0 + n_local && e < E) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        base[e] = h[e] ? atomicAdd(&cur[e], h[e]) : 0;
        h[e] = 0;
    }
    __syncthreads();
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const int r = p / K, k = p % K;
        const int *m = recv_meta + (size_t)r * mw;
        const int e = m[0] ? m[2 + k] : -1;
        int pos = -1;
        if (e >= e0 && e < e0 + n_local && e < E) {
            pos = base[e] + atomicAdd(&h[e], 1);
            plan.pair_expert[pos] = e;
            plan.pair_token[pos] = r;
            plan.pair_w[pos] = __int_as_float(m[2 + K + k]);
        }
        plan.slot_pair[(size_t)r * (K + 1) + k] = pos;
        if (k == 0) plan.slot_pair[(size_t)r * (K + 1) + K] = -1;
    }
    // own tokens: the shared expert only (their routed pairs come back through the exchange)
    const int sh0 = plan.counts[2];
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
        const int pos = sh0 + t, r = R + t;
        plan.pair_expert[pos] = E;
        plan.pair_token[pos] = r;
        plan.pair_w[pos] = 1.0f;
        for (int k = 0; k < K; k++) plan.slot_pair[(size_t)r * (K + 1) + k] = -1;
        plan.slot_pair[(size_t)r * (K + 1) + K] = pos;
    }
}

// row r of the row space to each of its pair rows
__global__ void __launch_bounds__(256) k_pfe_gather(const __half *__restrict__ recv_xh, const __half *__restrict__ xh,
                                                    int R, int H, int K, MoePlan plan, __half *__restrict__ xg) {
    __shared__ int pos[64];
    __shared__ int any;
    const int r = blockIdx.x;
    if (threadIdx.x == 0) any = 0;
    __syncthreads();
    if (threadIdx.x <= K) {
        pos[threadIdx.x] = plan.slot_pair[(size_t)r * (K + 1) + threadIdx.x];
        if (pos[threadIdx.x] >= 0) any = 1;
    }
    __syncthreads();
    if (!any) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(r < R ? recv_xh + (size_t)r * H : xh + (size_t)(r - R) * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
        const uint4 v = __ldg(src + i);
        for (int k = 0; k <= K; k++)
            if (pos[k] >= 0) reinterpret_cast<uint4 *>(xg + (size_t)pos[k] * H)[i] = v;
    }
}

// pre-combine on the expert side: send_y[r] = sum over the slots of received
// row r whose expert lives here, in slot order, of w_k * eo
__global__ void __launch_bounds__(256) k_pfe_partial(MoeDims d, MoePlan plan, const int *__restrict__ recv_meta,
                                                     const float *__restrict__ eo, float *__restrict__ send_y) {
    __shared__ int pos[64];
    __shared__ float wk[64];
    const int r = blockIdx.x, K = d.K, H = d.H;
    if (!recv_meta[(size_t)r * (2 + 2 * K)]) return;
    if (threadIdx.x < K) {
        const int p = plan.slot_pair[(size_t)r * (K + 1) + threadIdx.x];
        pos[threadIdx.x] = p;
        wk[threadIdx.x] = p >= 0 ? plan.pair_w[p] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int k = 0; k < K; k++) {
            if (pos[k] < 0) continue;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(eo + (size_t)pos[k] * H) + i);
            const float wv = wk[k];
            acc = make_float4(fmaf(wv, v.x, acc.x), fmaf(wv, v.y, acc.y), fmaf(wv, v.z, acc.z), fmaf(wv, v.w, acc.w));
        }
        reinterpret_cast<float4 *>(send_y + (size_t)r * H)[i] = acc;
    }
}

// owner side: out[t] = sum over ranks (rank order) of the returned partials
// + the shared expert
__global__ void __launch_bounds__(256) k_pfe_final(MoeDims d, MoePlan plan, const float *__restrict__ recv_y,
                                                   const int *__restrict__ tok_slot, int N, int ecap, int R,
                                                   const float *__restrict__ eo, float *__restrict__ out) {
    __shared__ int sl[64];
    __shared__ int sp;
    const int t = blockIdx.x, H = d.H;
    if (threadIdx.x < N) sl[threadIdx.x] = tok_slot[t * N + threadIdx.x];
    if (threadIdx.x == 0) sp = plan.slot_pair[(size_t)(R + t) * (d.K + 1) + d.K];
    __syncthreads();
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int p = 0; p < N; p++) {
            if (sl[p] < 0) continue;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(recv_y + ((size_t)p * ecap + sl[p]) * H) + i);
            acc = make_float4(acc.x + v.x, acc.y + v.y, acc.z + v.z, acc.w + v.w);
        }
        const float4 v = __ldg(reinterpret_cast<const float4 *>(eo + (size_t)sp * H) + i);
        reinterpret_cast<float4 *>(out + (size_t)t * H)[i] = make_float4(acc.x + v.x, acc.y + v.y, acc.z + v.z, acc.w + v.w);
    }
}

// ===========================================================================
// host side
// ===========================================================================
static size_t pf_smem(int mode, int nbp) {
    const size_t raw = mode == 2 ? PF_RAW_Q6 : PF_RAW_Q4;
    return 1024 + (size_t)PF_NSB * PF_BST + (mode == 2 ? PF_RAW_NS_Q6 : PF_RAW_NS_Q4) * raw +
           (mode == 2 ? 2 * PF_RB * 128 * 2 * (size_t)nbp : 0);  // two d-plane buffers
}

template <int MODE>
static void pf_launch(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const CUtensorMap &tmB,
                      __half *act, float *eo, int max_tiles, int row_groups, cudaStream_t s, uint64_t *launches) {
    const size_t smem = pf_smem(MODE, q6r_nb_pad(d.I / MOE_QK));
    static size_t attr[MOE_MAX_DEVICES];
    moe_smem_limit(k_prefill_gemm<MODE>, smem, attr);
    // persistent: one cluster per TPC (one CTA per SM), at most one per item
    static int n_sm[MOE_MAX_DEVICES];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= MOE_MAX_DEVICES) dev = 0;
    if (!n_sm[dev] && cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        n_sm[dev] = 148;
    const int PR = row_groups / 2;
    const long long items = (long long)max_tiles * PR;
    const int clusters = (int)std::min<long long>(std::max(n_sm[dev] / 2, 1), items);
    k_prefill_gemm<MODE><<<2 * clusters, PF_THREADS, smem, s>>>(d, L, plan, tmB, PR, act, eo);
    LAUNCH_COUNT(launches);
}

void moe_prefill_free(MoePrefillWs &ws) {
    void *b[] = {ws.part, ws.logits, ws.w, ws.eo, ws.idx, ws.counters, ws.xg, ws.act, ws.plan.counts,
                 ws.plan.pair_expert, ws.plan.pair_token, ws.plan.pair_w, ws.plan.chunk_expert, ws.plan.chunk_pair0,
                 ws.plan.chunk_ntok, ws.plan.slot_pair, ws.plan.error, ws.pcnt, ws.pcur, ws.wh, ws.wl,
                 ws.xh, ws.xl, ws.send_xh, ws.recv_xh, ws.send_meta, ws.recv_meta, ws.send_y, ws.recv_y,
                 ws.tok_slot};
    for (void *p : b) cudaFree(p);
    int *tc = ws.tcount;  // the token-count exchange buffer outlives the workspace
    ws = MoePrefillWs{};
    ws.tcount = tc;
}

int moe_prefill_alloc(MoePrefillWs &ws, const MoeDims &d, int T, int world, int ecap_req) {
    const int ecap = world > 1 ? (ecap_req + 7) & ~7 : 0;  // rows per peer in the exchange
    if (ws.cap >= T && ws.world == world && ws.ecap >= ecap) return 0;
    moe_prefill_free(ws);
    const int cap = (T + 255) & ~255;                       // own tokens
    const size_t R = (size_t)world * ecap;                  // received rows (0 on one GPU)
    const size_t rows = world > 1 ? R + cap : (size_t)cap;  // row space of the plan
    const size_t P = (world > 1 ? R * d.K + cap : (size_t)cap * (d.K + 1)) + PF_TILE_N;  // pairs (+ box slack)
    const size_t tiles = (size_t)d.E + 1 + P / PF_TILE_N + 1;
    const int nsplit = d.H / MOE_QK > 16 ? d.H / MOE_QK : 16;  // router partial slices (at most 16)
    const int mw = 2 + 2 * d.K;
    cudaError_t e = cudaSuccess;
#define PFA(ptr, bytes) \
    if (e == cudaSuccess) e = cudaMalloc((void **)&(ptr), (bytes))
    PFA(ws.part, sizeof(float) * nsplit * (size_t)cap * d.E);
    PFA(ws.logits, sizeof(float) * (size_t)cap * d.E);
    PFA(ws.idx, sizeof(int) * (size_t)cap * d.K);
    PFA(ws.w, sizeof(float) * (size_t)cap * d.K);
    PFA(ws.counters, sizeof(int) * ((size_t)(d.E + 31) / 32) * (cap / 64 + 1));
    PFA(ws.xg, sizeof(__half) * P * d.H);
    PFA(ws.act, sizeof(__half) * P * d.I);
    PFA(ws.eo, sizeof(float) * P * d.H);
    PFA(ws.plan.counts, sizeof(int) * 4);
    PFA(ws.plan.pair_expert, sizeof(int) * P);
    PFA(ws.plan.pair_token, sizeof(int) * P);
    PFA(ws.plan.pair_w, sizeof(float) * P);
    PFA(ws.plan.chunk_expert, sizeof(int) * tiles);
    PFA(ws.plan.chunk_pair0, sizeof(int) * tiles);
    PFA(ws.plan.chunk_ntok, sizeof(int) * tiles);
    PFA(ws.plan.slot_pair, sizeof(int) * rows * (d.K + 1));
    PFA(ws.plan.error, sizeof(int));
    PFA(ws.pcnt, sizeof(int) * (size_t)(d.E + 2));
    const size_t Ep = (size_t)(d.E + 127) & ~(size_t)127;  // router rows padded to the 128-row box (zero rows)
    PFA(ws.wh, sizeof(__half) * Ep * d.H);
    PFA(ws.wl, sizeof(__half) * Ep * d.H);
    PFA(ws.xh, sizeof(__half) * (size_t)cap * d.H);
    PFA(ws.xl, sizeof(__half) * (size_t)cap * d.H);
    PFA(ws.pcur, sizeof(int) * (size_t)(d.E + 2));
    if (world > 1) {
        PFA(ws.send_xh, sizeof(__half) * R * d.H);
        PFA(ws.recv_xh, sizeof(__half) * R * d.H);
        PFA(ws.send_meta, sizeof(int) * R * mw);
        PFA(ws.recv_meta, sizeof(int) * R * mw);
        PFA(ws.send_y, sizeof(float) * R * d.H);
        PFA(ws.recv_y, sizeof(float) * R * d.H);
        PFA(ws.tok_slot, sizeof(int) * (size_t)cap * world);
    }
#undef PFA
    if (e == cudaSuccess) e = cudaMemset(ws.counters, 0, sizeof(int) * ((size_t)(d.E + 31) / 32) * (cap / 64 + 1));
    if (e == cudaSuccess) e = cudaMemset(ws.plan.error, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ws.pcnt, 0, sizeof(int) * (size_t)(d.E + 2));
    if (e == cudaSuccess) e = cudaMemset(ws.wh, 0, sizeof(__half) * Ep * d.H);
    if (e == cudaSuccess) e = cudaMemset(ws.wl, 0, sizeof(__half) * Ep * d.H);
    if (e == cudaSuccess) e = cudaMemset(ws.xg, 0, sizeof(__half) * P * d.H);
    if (e == cudaSuccess) e = cudaMemset(ws.act, 0, sizeof(__half) * P * d.I);
    // the clears run on the legacy default stream, which does not order
    // against the context's non-blocking stream (nor a caller's): wait for
    // them here, or a late clear can land after the first call's kernels have
    // written wl / xg / act
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        moe_prefill_free(ws);
        return -1;
    }
    if (moe_make_map_f16_sw128(&ws.tm_xg, ws.xg, d.H, P, 64, 16) ||
        moe_make_map_f16_sw128(&ws.tm_act, ws.act, d.I, P, 64, 16) ||
        moe_make_map_f16_sw128(&ws.tm_wh, ws.wh, d.H, Ep, 64, 128) ||
        moe_make_map_f16_sw128(&ws.tm_wl, ws.wl, d.H, Ep, 64, 128) ||
        moe_make_map_f16_sw128(&ws.tm_xh, ws.xh, d.H, cap, 64, 128) ||
        moe_make_map_f16_sw128(&ws.tm_xl, ws.xl, d.H, cap, 64, 128)) {
        moe_prefill_free(ws);
        return -2;
    }
    ws.cap = cap;
    ws.world = world;
    ws.ecap = ecap;
    ws.P = P;
    return 0;
}

// tcgen05 expert GEMMs over the plan; P = pairs capacity of the workspace
static void pf_gemms(const MoeDims &d, const MoeLayerDev &L, MoePrefillWs &ws, size_t npairs, cudaStream_t s,
                     uint64_t *launches) {
    const int max_tiles = (int)(d.E + 1 + npairs / PF_TILE_N + 1);
    pf_launch<0>(d, L, ws.plan, ws.tm_xg, ws.act, nullptr, max_tiles, d.I / (64 * PF_RB), s, launches);
    if (L.down_type == MOE_TYPE_Q6_K || L.sh_down_type == MOE_TYPE_Q6_K)
        pf_launch<2>(d, L, ws.plan, ws.tm_act, nullptr, ws.eo, max_tiles, d.H / (128 * PF_RB), s, launches);
    if (L.down_type == MOE_TYPE_Q4_K || L.sh_down_type == MOE_TYPE_Q4_K)
        pf_launch<1>(d, L, ws.plan, ws.tm_act, nullptr, ws.eo, max_tiles, d.H / (128 * PF_RB), s, launches);
}

void moe_launch_pfe_dispatch(const MoeDims &d, MoePrefillWs &ws, int T, int n_local, cudaStream_t s,
                             uint64_t *launches) {
    k_pfe_slots<<<ws.world, 1024, 0, s>>>(ws.idx, T, d.K, n_local, ws.world, ws.ecap, ws.tok_slot, ws.send_meta);
    LAUNCH_COUNT(launches);
    if (T > 0) {
        k_pfe_pack<<<T, 256, 0, s>>>(ws.xh, ws.idx, ws.w, d.K, d.H, ws.world, ws.ecap, ws.tok_slot, ws.send_xh,
                                     ws.send_meta);
        LAUNCH_COUNT(launches);
    }
}

void moe_launch_pfe_experts(const MoeDims &d, const MoeLayerDev &L, MoePrefillWs &ws, int T, cudaStream_t s,
                            uint64_t *launches) {
    const int R = ws.world * ws.ecap, n = R * d.K, nblk = (n + PF_PLAN_PAIRS - 1) / PF_PLAN_PAIRS;
    k_pfe_count<<<nblk, 256, 0, s>>>(d, ws.recv_meta, R, L.e0, L.n_local, ws.pcnt, ws.plan.error);
    k_pf_offsets<<<1, 1024, 0, s>>>(d, T, ws.pcnt, ws.pcur, ws.plan);
    k_pfe_scatter<<<nblk, 256, 0, s>>>(d, ws.recv_meta, R, T, L.e0, L.n_local, ws.pcur, ws.plan);
    k_pfe_gather<<<R + T, 256, 0, s>>>(ws.recv_xh, ws.xh, R, d.H, d.K, ws.plan, ws.xg);
    if (launches) *launches += 4;
    pf_gemms(d, L, ws, (size_t)n + T, s, launches);
    k_pfe_partial<<<R, 256, 0, s>>>(d, ws.plan, ws.recv_meta, ws.eo, ws.send_y);
    LAUNCH_COUNT(launches);
}

void moe_launch_pfe_final(const MoeDims &d, MoePrefillWs &ws, int T, float *out, cudaStream_t s, uint64_t *launches) {
    k_pfe_final<<<T, 256, 0, s>>>(d, ws.plan, ws.recv_y, ws.tok_slot, ws.world, ws.ecap, ws.world * ws.ecap, ws.eo,
                                  out);
    LAUNCH_COUNT(launches);
}

void moe_launch_prefill_experts(const MoeDims &d, const MoeLayerDev &L, MoePrefillWs &ws, const float *x, int T,
                                float *out, cudaStream_t s, uint64_t *launches) {
    const int n = T * d.K, nblk = (n + PF_PLAN_PAIRS - 1) / PF_PLAN_PAIRS;
    k_pf_count<<<nblk, 256, 0, s>>>(d, ws.idx, n, ws.pcnt, ws.plan.error);
    k_pf_offsets<<<1, 1024, 0, s>>>(d, T, ws.pcnt, ws.pcur, ws.plan);
    k_pf_scatter<<<nblk, 256, 0, s>>>(d, ws.idx, ws.w, T, ws.pcur, ws.plan);
    k_prefill_gather<<<T, 256, 0, s>>>(ws.xh, d.H, d.K, ws.plan, ws.xg);
    if (launches) *launches += 4;
    pf_gemms(d, L, ws, (size_t)T * (d.K + 1), s, launches);
    k_prefill_combine<<<T, 256, 0, s>>>(d, ws.plan, ws.eo, out);
    LAUNCH_COUNT(launches);
}
