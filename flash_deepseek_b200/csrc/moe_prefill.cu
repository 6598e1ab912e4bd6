// moe_prefill.cu -- the MoE block for many tokens at once (prefill), on the
// fifth-generation tensor cores (tcgen05).
//
// With ~128 tokens per expert the expert products are real matrix products
// (C = W X^T, M = weight rows, N = tokens, K = hidden or intermediate), so
// the weights are dequantized once per tile into fp16 shared-memory tiles
// that feed tcgen05.mma, with the fp32 accumulator in tensor memory:
//   plan     counting sort of the (token, slot) pairs by expert, tiles of
//            <= 128 pairs per expert
//   gather   fp16 copy of each pair's token row, pairs grouped by expert
//   gemm1    gate/up rows (64 + 64 per tile) x 128 pairs, SwiGLU in the
//            epilogue (infer.m:378-383), act in fp16
//   gemm2    down rows (128 per tile) x 128 pairs, fp32 expert outputs
//   combine  slot order, then the shared expert (infer.m:1915-1922)
// Differences from the reference's fp32 dot: weights and activations are
// rounded to fp16 (11-bit significands) before the fp32-accumulated product.
//
// GEMM CTA: warp 0 issues TMA copies (raw Q4_K / Q6_K tiles of one
// super-block, and the pairs' 64-column activation slices with the 128-byte
// swizzle), warp 1 owns tensor memory and issues the MMAs from one thread,
// warps 2-5 dequantize one weight row each into the swizzled A tile and,
// after the last k step, run the epilogue from tensor memory.  All hand-offs
// are mbarriers; every wait gives up after about a second and records an
// error instead of hanging.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdio.h>

#include "../../include/moe_cuda.h"
#include "moe_common.cuh"
#include "moe_internal.h"
#include "moe_umma.cuh"

#define PF_TILE 128                // pairs per tile (MMA N) and weight rows per tile (MMA M)
#define PF_NS 4                    // k-atom stages (64 columns of K each)
#define PF_ATOM 16384              // 128 rows x 128 B
#define PF_RAW_NS 2                // raw super-block stages
#define PF_RAW_Q4 (128 * 144)      // 128 Q4_K rows of one super-block
#define PF_RAW_Q6 (128 * 192 + 128 * 16)
#define PF_THREADS 192
#define PF_WAIT_CYCLES (1ll << 31)
#define PF_ERR_TIMEOUT 0x7200

#define LAUNCH_COUNT(p) \
    do {                \
        if (p) (*(p))++; \
    } while (0)

__device__ __forceinline__ void pf_mbar_init(uint64_t *b, int n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(umma_smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void pf_expect(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(umma_smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void pf_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(umma_smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool pf_wait(uint64_t *b, uint32_t parity) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(umma_smem_u32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > PF_WAIT_CYCLES) return false;
    }
}
__device__ __forceinline__ void pf_tma3(void *dst, const CUtensorMap *m, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];\n" ::"r"(umma_smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(umma_smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void pf_tma2(void *dst, const CUtensorMap *m, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
            "r"(umma_smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(umma_smem_u32(bar))
        : "memory");
}
// exact float of a small non-negative integer (< 2^23)
__device__ __forceinline__ float pf_i2f(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }
__device__ __forceinline__ uint32_t pf_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// ===========================================================================
// plan: counting sort of the pairs by expert (one block).  Pair order inside
// an expert follows arrival; every pair's result depends on its own token
// and expert only, so the output does not.
// ===========================================================================
__global__ void __launch_bounds__(1024) k_prefill_plan(MoeDims d, const int *__restrict__ idx,
                                                       const float *__restrict__ w, int T, MoePlan plan) {
    __shared__ int cnt[1025], off[1026], fill[1025], toff[1026];
    const int E = d.E, K = d.K, NE = E + 1;
    for (int e = threadIdx.x; e < NE; e += blockDim.x) cnt[e] = fill[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < T * K; p += blockDim.x) {
        const int e = idx[p];
        if (e < 0 || e >= E) { atomicExch(plan.error, 1); continue; }
        atomicAdd(&cnt[e], 1);
    }
    if (threadIdx.x == 0) cnt[E] = T;
    __syncthreads();
    if (threadIdx.x == 0) {
        int a = 0, b = 0;
        for (int e = 0; e < NE; e++) {
            off[e] = a;
            toff[e] = b;
            a += cnt[e];
            b += (cnt[e] + PF_TILE - 1) / PF_TILE;
        }
        off[NE] = a;
        toff[NE] = b;
        plan.counts[0] = a;
        plan.counts[1] = b;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < NE; e += blockDim.x)
        for (int c = 0; c * PF_TILE < cnt[e]; c++) {
            plan.chunk_expert[toff[e] + c] = e;
            plan.chunk_pair0[toff[e] + c] = off[e] + c * PF_TILE;
            plan.chunk_ntok[toff[e] + c] = min(PF_TILE, cnt[e] - c * PF_TILE);
        }
    for (int p = threadIdx.x; p < T * K; p += blockDim.x) {
        const int t = p / K, k = p % K, e = idx[p];
        if (e < 0 || e >= E) { plan.slot_pair[t * (K + 1) + k] = -1; continue; }
        const int pos = off[e] + atomicAdd(&fill[e], 1);
        plan.pair_expert[pos] = e;
        plan.pair_token[pos] = t;
        plan.pair_w[pos] = w[p];
        plan.slot_pair[t * (K + 1) + k] = pos;
    }
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const int pos = off[E] + t;
        plan.pair_expert[pos] = E;
        plan.pair_token[pos] = t;
        plan.pair_w[pos] = 1.0f;
        plan.slot_pair[t * (K + 1) + K] = pos;
    }
}

// fp16 rows of the pairs' tokens: xg[p] = half(x[token(p)])
__global__ void __launch_bounds__(256) k_prefill_gather(const float *__restrict__ x, int H, MoePlan plan,
                                                        __half *__restrict__ xg) {
    const int n = plan.counts[0];
    for (int p = blockIdx.x; p < n; p += gridDim.x) {
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)plan.pair_token[p] * H);
        uint2 *dst = reinterpret_cast<uint2 *>(xg + (size_t)p * H);
        for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
            const float4 v = __ldg(src + i);
            dst[i] = make_uint2(pf_h2(v.x, v.y), pf_h2(v.z, v.w));
        }
    }
}

// ===========================================================================
// dequantization of one weight row into one 64-column A atom (thread = row)
// ===========================================================================
// Q4_K, repacked block (header + transposed qs): atom a = weights
// [64 a, 64 a + 64) of the super-block: low nibbles of old bytes 32 a + l
// (sub-block 2a) and high nibbles (sub-block 2a + 1); old byte 32 a + 8 t + i
// sits at 16 + 32 t + 8 a + i.
__device__ __forceinline__ void pf_deq_q4(const uint8_t *blk, int a, uint8_t *atom, int row) {
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const float d = __half2float(__ushort_as_half((uint16_t)(hd.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(hd.x >> 16)));
    const uint8_t *q = blk + 4;  // 12 scale bytes (get_scale_min_k4, quant.c:26-34)
    int sc0, m0, sc1, m1;
    {
        const int j0 = 2 * a, j1 = 2 * a + 1;
        if (j0 < 4) { sc0 = q[j0] & 63; m0 = q[j0 + 4] & 63; }
        else { sc0 = (q[j0 + 4] & 0xF) | ((q[j0 - 4] >> 6) << 4); m0 = (q[j0 + 4] >> 4) | ((q[j0] >> 6) << 4); }
        if (j1 < 4) { sc1 = q[j1] & 63; m1 = q[j1 + 4] & 63; }
        else { sc1 = (q[j1 + 4] & 0xF) | ((q[j1 - 4] >> 6) << 4); m1 = (q[j1 + 4] >> 4) | ((q[j1] >> 6) << 4); }
    }
    const float ds0 = d * (float)sc0, dm0 = dmin * (float)m0, ds1 = d * (float)sc1, dm1 = dmin * (float)m1;
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const uint2 wv = *reinterpret_cast<const uint2 *>(blk + 16 + 32 * t + 8 * a);
        const uint32_t wd[2] = {wv.x, wv.y};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int b = 0; b < 4; b += 2) {
                const uint32_t q0 = (wd[h] >> (8 * b)) & 0xFFu, q1 = (wd[h] >> (8 * b + 8)) & 0xFFu;
                lo[2 * h + b / 2] = pf_h2(fmaf(pf_i2f(q0 & 0xFu), ds0, -dm0), fmaf(pf_i2f(q1 & 0xFu), ds0, -dm0));
                hi[2 * h + b / 2] = pf_h2(fmaf(pf_i2f(q0 >> 4), ds1, -dm1), fmaf(pf_i2f(q1 >> 4), ds1, -dm1));
            }
        *reinterpret_cast<uint4 *>(atom + sw128_offset(row, 8 * t)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4 *>(atom + sw128_offset(row, 32 + 8 * t)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    }
}

// Q6_K, repacked planes: rq = this row's 192-byte Q part of the super-block
// (lane chunk t: per half h, ql words w at 24 h + 4 w, qh words at
// 24 h + 16 + 4 w', high bit of every qh pair stored inverted), sc = its 16
// scales, d = its fp16 d.  Atom a covers weights [64 a, 64 a + 64).
__device__ __forceinline__ void pf_deq_q6(const uint8_t *rq, const int8_t *sc, float d, int a, uint8_t *atom,
                                          int row) {
    const int h = a >> 1, wp = a & 1;
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int g = 0; g < 2; g++) {
            const uint32_t hq = *reinterpret_cast<const uint32_t *>(rq + 48 * t + 24 * h + 16 + 4 * g) ^ 0xAAAAAAAAu;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const uint32_t W = *reinterpret_cast<const uint32_t *>(rq + 48 * t + 24 * h + 8 * u + 4 * g);
                const int which = 2 * wp + u;
                const float f = d * (float)sc[8 * h + 2 * which + g];
                float v[4];
#pragma unroll
                for (int bb = 0; bb < 4; bb++) {
                    const uint32_t q6 = ((W >> (8 * bb + 4 * wp)) & 0xFu) | (((hq >> (8 * bb + 2 * which)) & 3u) << 4);
                    v[bb] = f * (pf_i2f(q6) - 32.0f);
                }
                const int c = 4 * u + 2 * g + (t >> 1);
                *reinterpret_cast<uint2 *>(atom + sw128_offset(row, 8 * c) + 8 * (t & 1)) =
                    make_uint2(pf_h2(v[0], v[1]), pf_h2(v[2], v[3]));
            }
        }
}

// ===========================================================================
// GEMM.  MODE 0: gate/up (Q4_K) -> act (fp16, SwiGLU); 1: down Q4_K -> eo;
// 2: down Q6_K -> eo.  blockIdx.x = tile (expert, <= 128 pairs), blockIdx.y
// = row block.
// ===========================================================================
template <int MODE>
__global__ void __launch_bounds__(PF_THREADS, 1)
    k_prefill_gemm(MoeDims d, const __grid_constant__ MoeLayerDev L, MoePlan plan,
                   const __grid_constant__ CUtensorMap tmB, __half *__restrict__ act, float *__restrict__ eo) {
    constexpr int RAW = MODE == 2 ? PF_RAW_Q6 : PF_RAW_Q4;
    extern __shared__ uint8_t pf_raw[];
    uint8_t *sm = pf_raw + ((1024u - (umma_smem_u32(pf_raw) & 1023u)) & 1023u);
    uint8_t *sa = sm, *sb = sm + PF_NS * PF_ATOM, *sr = sm + 2 * PF_NS * PF_ATOM;
    uint8_t *sd = sr + PF_RAW_NS * RAW;  // Q6_K d plane of the tile (rows x 2 nb_pad bytes)
    __shared__ __align__(8) uint64_t raw_full[PF_RAW_NS], raw_empty[PF_RAW_NS], a_full[PF_NS], b_full[PF_NS],
        ab_empty[PF_NS], acc_full;
    __shared__ uint32_t tmem_base;
    __shared__ int s_skip;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, rb = blockIdx.y;
    if (tid == 0) {
        int skip = tile >= plan.counts[1];
        if (!skip && MODE > 0) {
            const int e = plan.chunk_expert[tile];
            skip = ((e == d.E) ? L.sh_down_type : L.down_type) != (MODE == 2 ? MOE_TYPE_Q6_K : MOE_TYPE_Q4_K);
        }
        s_skip = skip;
    }
    __syncthreads();
    if (s_skip) return;
    const int e = plan.chunk_expert[tile], p0 = plan.chunk_pair0[tile], ntile = plan.chunk_ntok[tile];
    const int slot = e == d.E ? L.n_local : e - L.e0;
    const int K = MODE == 0 ? d.H : d.I, NB = K / MOE_QK, n_atoms = 4 * NB;
    const int nbp = q6r_nb_pad(NB);
    if (tid == 0) {
        for (int i = 0; i < PF_RAW_NS; i++) { pf_mbar_init(&raw_full[i], 1); pf_mbar_init(&raw_empty[i], 4); }
        for (int i = 0; i < PF_NS; i++) {
            pf_mbar_init(&a_full[i], 4);
            pf_mbar_init(&b_full[i], 1);
            pf_mbar_init(&ab_empty[i], 1);
        }
        pf_mbar_init(&acc_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&tmem_base, PF_TILE);
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = tmem_base;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            for (int sbk = 0; sbk < NB && ok; sbk++) {
                const int rs = sbk % PF_RAW_NS;
                if (!pf_wait(&raw_empty[rs], ((sbk / PF_RAW_NS) & 1) ^ 1)) { ok = false; break; }
                uint8_t *r = sr + rs * RAW;
                if (MODE == 0) {
                    pf_expect(&raw_full[rs], RAW);
                    pf_tma3(r, &L.tm_gu, sbk * MOE_Q4K_BYTES, rb * 64, slot, &raw_full[rs]);
                    pf_tma3(r + 64 * MOE_Q4K_BYTES, &L.tm_gu, sbk * MOE_Q4K_BYTES, d.I + rb * 64, slot, &raw_full[rs]);
                } else if (MODE == 1) {
                    pf_expect(&raw_full[rs], RAW);
                    pf_tma3(r, &L.tm_d4, sbk * MOE_Q4K_BYTES, rb * 128, slot, &raw_full[rs]);
                } else {
                    pf_expect(&raw_full[rs], RAW + (sbk == 0 ? 128 * 2 * nbp : 0));
                    pf_tma3(r, &L.tm_d6q, sbk * 192, rb * 128, slot, &raw_full[rs]);
                    pf_tma3(r + 128 * 192, &L.tm_d6s, sbk * 16, rb * 128, slot, &raw_full[rs]);
                    if (sbk == 0) pf_tma3(sd, &L.tm_d6d, 0, rb * 128, slot, &raw_full[rs]);
                }
                for (int a = 0; a < 4; a++) {
                    const int i = 4 * sbk + a, st = i % PF_NS;
                    if (!pf_wait(&ab_empty[st], ((i / PF_NS) & 1) ^ 1)) { ok = false; break; }
                    pf_expect(&b_full[st], PF_ATOM);
                    pf_tma2(sb + st * PF_ATOM, &tmB, sbk * MOE_QK + 64 * a, p0, &b_full[st]);
                }
            }
            if (!ok) atomicExch(plan.error, PF_ERR_TIMEOUT);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(PF_TILE, PF_TILE);
            for (int i = 0; i < n_atoms && ok; i++) {
                const int st = i % PF_NS;
                const uint32_t ph = (i / PF_NS) & 1;
                if (!pf_wait(&a_full[st], ph) || !pf_wait(&b_full[st], ph)) { ok = false; break; }
                tmem_fence_after();
                const uint32_t a0 = umma_smem_u32(sa + st * PF_ATOM), b0 = umma_smem_u32(sb + st * PF_ATOM);
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    umma_f16(tmem, umma_desc_sw128(a0 + 32 * kk), umma_desc_sw128(b0 + 32 * kk), idesc,
                             (i | kk) != 0);
                umma_commit(&ab_empty[st]);
            }
            if (ok) umma_commit(&acc_full);
            else atomicExch(plan.error, PF_ERR_TIMEOUT);
        }
    } else {
        // dequantization: thread = A row
        const int row = tid - 64;
        int rraw;  // raw tile row holding A row `row`
        if (MODE == 0) {
            const int q = row >> 5, h = (row >> 4) & 1, i = row & 15;  // row = 32 q + 16 h + i
            rraw = h * 64 + 16 * q + i;                                // gate rows first, then up rows
        } else {
            rraw = row;
        }
        for (int sbk = 0; sbk < NB && ok; sbk++) {
            const int rs = sbk % PF_RAW_NS;
            if (!pf_wait(&raw_full[rs], (sbk / PF_RAW_NS) & 1)) { ok = false; break; }
            const uint8_t *r = sr + rs * RAW;
            float d6 = 0.0f;
            if (MODE == 2) d6 = __half2float(reinterpret_cast<const __half *>(sd)[rraw * nbp + sbk]);
            for (int a = 0; a < 4; a++) {
                const int i = 4 * sbk + a, st = i % PF_NS;
                if (!pf_wait(&ab_empty[st], ((i / PF_NS) & 1) ^ 1)) { ok = false; break; }
                uint8_t *atom = sa + st * PF_ATOM;
                if (MODE == 2)
                    pf_deq_q6(r + rraw * 192, reinterpret_cast<const int8_t *>(r + 128 * 192 + rraw * 16), d6, a,
                              atom, row);
                else
                    pf_deq_q4(r + rraw * MOE_Q4K_BYTES, a, atom, row);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) pf_arrive(&a_full[st]);
            }
            __syncwarp();
            if (lane == 0) pf_arrive(&raw_empty[rs]);
        }
        // epilogue: this warp reads tensor-memory lanes 32 (warp % 4) .. + 31
        if (ok && pf_wait(&acc_full, 0)) {
            tmem_fence_after();
            const int q = warp & 3;
            for (int c = 0; c < PF_TILE; c += 16) {
                if (c >= ntile) break;
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c, v);
                if (MODE == 0) {
                    // lanes 0-15: gate rows, 16-31: the matching up rows
                    const int i = lane & 15, rI = rb * 64 + 16 * q + i;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const float u = __shfl_xor_sync(0xffffffffu, v[j], 16);
                        if (lane < 16 && c + j < ntile)
                            act[(size_t)(p0 + c + j) * d.I + rI] = __float2half_rn((v[j] / (1.0f + expf(-v[j]))) * u);
                    }
                } else {
                    const int rH = rb * 128 + 32 * q + lane;
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (c + j < ntile) eo[(size_t)(p0 + c + j) * d.H + rH] = v[j];
                }
            }
        } else if (lane == 0) {
            atomicExch(plan.error, PF_ERR_TIMEOUT);
        }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 1) tmem_free(tmem, PF_TILE);
}

// ===========================================================================
// host side
// ===========================================================================
static size_t pf_smem(int mode, int nbp) {
    const size_t raw = mode == 2 ? PF_RAW_Q6 : PF_RAW_Q4;
    return 1024 + 2 * (size_t)PF_NS * PF_ATOM + PF_RAW_NS * raw + (mode == 2 ? 128 * 2 * (size_t)nbp : 0);
}

template <int MODE>
static void pf_launch(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const CUtensorMap &tmB,
                      __half *act, float *eo, int max_tiles, int row_blocks, cudaStream_t s, uint64_t *launches) {
    const size_t smem = pf_smem(MODE, q6r_nb_pad(d.I / MOE_QK));
    static size_t attr = 0;
    if (smem > attr) {
        cudaFuncSetAttribute(k_prefill_gemm<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = smem;
    }
    k_prefill_gemm<MODE><<<dim3(max_tiles, row_blocks), PF_THREADS, smem, s>>>(d, L, plan, tmB, act, eo);
    LAUNCH_COUNT(launches);
}

void moe_prefill_free(MoePrefillWs &ws) {
    void *b[] = {ws.part, ws.logits, ws.w, ws.eo, ws.idx, ws.counters, ws.xg, ws.act, ws.plan.counts,
                 ws.plan.pair_expert, ws.plan.pair_token, ws.plan.pair_w, ws.plan.chunk_expert, ws.plan.chunk_pair0,
                 ws.plan.chunk_ntok, ws.plan.slot_pair, ws.plan.error};
    for (void *p : b) cudaFree(p);
    ws = MoePrefillWs{};
}

int moe_prefill_alloc(MoePrefillWs &ws, const MoeDims &d, int T) {
    if (ws.cap >= T) return 0;
    moe_prefill_free(ws);
    const int cap = (T + 255) & ~255;
    const size_t P = (size_t)cap * (d.K + 1) + PF_TILE;  // pairs (+ slack rows for the last TMA box)
    const size_t tiles = (size_t)d.E + 1 + P / PF_TILE + 1;
    const int nsplit = d.H / MOE_QK;
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
    PFA(ws.plan.slot_pair, sizeof(int) * (size_t)cap * (d.K + 1));
    PFA(ws.plan.error, sizeof(int));
#undef PFA
    if (e == cudaSuccess) e = cudaMemset(ws.counters, 0, sizeof(int) * ((size_t)(d.E + 31) / 32) * (cap / 64 + 1));
    if (e == cudaSuccess) e = cudaMemset(ws.plan.error, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ws.xg, 0, sizeof(__half) * P * d.H);
    if (e == cudaSuccess) e = cudaMemset(ws.act, 0, sizeof(__half) * P * d.I);
    if (e != cudaSuccess) {
        moe_prefill_free(ws);
        return -1;
    }
    if (moe_make_map_f16_sw128(&ws.tm_xg, ws.xg, d.H, P, 64, PF_TILE) ||
        moe_make_map_f16_sw128(&ws.tm_act, ws.act, d.I, P, 64, PF_TILE)) {
        moe_prefill_free(ws);
        return -2;
    }
    ws.cap = cap;
    return 0;
}

void moe_launch_prefill_experts(const MoeDims &d, const MoeLayerDev &L, MoePrefillWs &ws, const float *x, int T,
                                float *out, cudaStream_t s, uint64_t *launches) {
    k_prefill_plan<<<1, 1024, 0, s>>>(d, ws.idx, ws.w, T, ws.plan);
    LAUNCH_COUNT(launches);
    const int P = T * (d.K + 1);
    k_prefill_gather<<<P < 148 * 8 ? P : 148 * 8, 256, 0, s>>>(x, d.H, ws.plan, ws.xg);
    LAUNCH_COUNT(launches);
    const int max_tiles = d.E + 1 + P / PF_TILE + 1;
    pf_launch<0>(d, L, ws.plan, ws.tm_xg, ws.act, nullptr, max_tiles, d.I / 64, s, launches);
    if (L.down_type == MOE_TYPE_Q6_K || L.sh_down_type == MOE_TYPE_Q6_K)
        pf_launch<2>(d, L, ws.plan, ws.tm_act, nullptr, ws.eo, max_tiles, d.H / 128, s, launches);
    if (L.down_type == MOE_TYPE_Q4_K || L.sh_down_type == MOE_TYPE_Q4_K)
        pf_launch<1>(d, L, ws.plan, ws.tm_act, nullptr, ws.eo, max_tiles, d.H / 128, s, launches);
    moe_launch_combine(d, ws.plan, ws.eo, T, 1, 1, nullptr, out, s, launches);
}
