// moe_dense.cu -- the dense FFN of DeepSeek-V3's first layers (0-2), the
// other FFN half of a decoder layer next to the MoE block (infer.m:1852-1868).
//
// Weights are kept as fp16 in HBM, rounded from whatever the GGUF holds
// (F32, F16, BF16, Q4_K, Q6_K) the way the reference's dequant_tensor_f16
// does (infer.m:314-348, 519-538); activations stay fp32 and the products
// accumulate in fp32, as mv_f16 (infer.m:459-516) and silu_mul
// (infer.m:378-383) do.
//
//   k_dense_gateup  g = Wg x, u = Wu x, act = silu(g) * u   (fp32 [T x Id])
//   k_dense_down    out = Wd act (+ residual)               (fp32 [T x H])
//
// Decode is a pass over 3 * Id * H * 2 bytes of weights (DeepSeek-V3:
// 792.7 MB per layer), so both kernels are HBM streams: one warp per output
// row, 16-byte non-allocating weight loads, several in flight per lane, the
// tokens' activations staged once per CTA in shared memory, persistent CTAs
// sized by occupancy over all SMs; each CTA issues its first weight loads
// before it stages the activations.  Up to DN_TT_GU (gate/up) and DN_TT_D
// (down) tokens share one weight pass; larger batches take more passes.
#include <cuda_fp16.h>
#include <math.h>

#include "../../include/moe_cuda.h"
#include "moe_common.cuh"
#include "moe_internal.h"

#define LAUNCH_COUNT(p) \
    do {                \
        if (p) (*(p))++; \
    } while (0)

namespace {

constexpr int DN_WARPS = 8;
constexpr int DN_THREADS = DN_WARPS * 32;
constexpr int DN_TT_GU = 4;   // tokens per weight pass, gate/up
constexpr int DN_TT_D = 2;    // tokens per weight pass, down
constexpr int DN_U_GU = 4;    // 16-byte loads in flight per lane and matrix, gate/up
constexpr int DN_VD = 9;      // 16-byte loads in flight per lane, down (one row's share when Id <= 18432)
constexpr int DN_RPC_MAX = 128;  // hidden rows per CTA of the down kernel, at most

__device__ __forceinline__ uint4 ld_weight16(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// acc += sum over the 8 halves of w times the 8 floats lo[0..4), hi[0..4)
// (a lane's activations sit in two 16-byte pieces 512 bytes apart; see
// stage_rows)
__device__ __forceinline__ float dot8(const uint4 &w, const float *lo, float acc) {
    const float4 x0 = *reinterpret_cast<const float4 *>(lo);
    const float4 x1 = *reinterpret_cast<const float4 *>(lo + 128);
    const float2 w0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
    const float2 w1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
    const float2 w2 = __half22float2(*reinterpret_cast<const __half2 *>(&w.z));
    const float2 w3 = __half22float2(*reinterpret_cast<const __half2 *>(&w.w));
    acc = fmaf(w0.x, x0.x, acc);
    acc = fmaf(w0.y, x0.y, acc);
    acc = fmaf(w1.x, x0.z, acc);
    acc = fmaf(w1.y, x0.w, acc);
    acc = fmaf(w2.x, x1.x, acc);
    acc = fmaf(w2.y, x1.y, acc);
    acc = fmaf(w3.x, x1.z, acc);
    acc = fmaf(w3.y, x1.w, acc);
    return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// the tokens [t0, t0 + tt) of x [T x cols] into shared memory (cols % 256 ==
// 0), DN_STAGE loads in flight per thread.  Within each 256-float chunk the
// floats 8 l .. 8 l + 3 go to 4 l and 8 l + 4 .. 8 l + 7 to 128 + 4 l, so that
// lane l of a warp reading its 8 floats touches two 16-byte pieces that sit
// next to its neighbours' (no bank conflicts).
constexpr int DN_STAGE = 4;
__device__ __forceinline__ void stage_rows(float *xs, const float *__restrict__ x, int t0, int tt, int cols) {
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t0 * cols);
    float4 *dst = reinterpret_cast<float4 *>(xs);
    const int n4 = tt * cols / 4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += DN_STAGE * blockDim.x) {
        float4 v[DN_STAGE];
#pragma unroll
        for (int j = 0; j < DN_STAGE; j++)
            if (i0 + j * (int)blockDim.x < n4) v[j] = src[i0 + j * blockDim.x];
#pragma unroll
        for (int j = 0; j < DN_STAGE; j++) {
            const int q = i0 + j * blockDim.x;
            if (q < n4) dst[(q & ~63) | ((q & 1) << 5) | ((q >> 1) & 31)] = v[j];
        }
    }
}

// One warp per output row r: g = Wg[r] . x (and u = Wu[r] . x when GLU) for up
// to DN_TT_GU tokens per pass; GLU writes act[t][r] = g / (1 + exp(-g)) * u
// (infer.m:378-383), else act[t][r] = g.  Lane l reads the 16-byte vectors
// l, l + 32, ... of the rows (H % 256 == 0).
template <bool GLU>
__device__ __forceinline__ void dense_rows(const __half *__restrict__ Wg, const __half *__restrict__ Wu,
                                           const float *__restrict__ x, int T, int H, int Id,
                                           float *__restrict__ act) {
    constexpr int U = GLU ? DN_U_GU : 7;   // 16-byte loads in flight per lane (7 divides H / 256 = 28)
    extern __shared__ float4 dn_smem[];
    float *xs = reinterpret_cast<float *>(dn_smem);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nv = H >> 8;
    const int r_first = blockIdx.x * DN_WARPS + warp;
    for (int t0 = 0; t0 < T; t0 += DN_TT_GU) {
        const int tt = min(DN_TT_GU, T - t0);
        // the first row's first vectors are in flight while x is staged
        uint4 g[U], u[GLU ? U : 1];
        const bool pre = r_first < Id && nv >= U;
        if (pre) {
#pragma unroll
            for (int j = 0; j < U; j++) {
                g[j] = ld_weight16(reinterpret_cast<const uint4 *>(Wg + (size_t)r_first * H) + lane + j * 32);
                if constexpr (GLU) u[j] = ld_weight16(reinterpret_cast<const uint4 *>(Wu + (size_t)r_first * H) + lane + j * 32);
            }
        }
        __syncthreads();
        stage_rows(xs, x, t0, tt, H);
        __syncthreads();
        for (int r = r_first; r < Id; r += gridDim.x * DN_WARPS) {
            float ag[DN_TT_GU], au[DN_TT_GU];
#pragma unroll
            for (int t = 0; t < DN_TT_GU; t++) ag[t] = au[t] = 0.0f;
            const uint4 *pg = reinterpret_cast<const uint4 *>(Wg + (size_t)r * H) + lane;
            const uint4 *pu = reinterpret_cast<const uint4 *>(Wu + (size_t)r * H) + lane;
            const float *xl = xs + lane * 4;
            int i = 0;
            for (; i + U <= nv; i += U) {
                if (!(pre && r == r_first && i == 0)) {
#pragma unroll
                    for (int j = 0; j < U; j++) {
                        g[j] = ld_weight16(pg + (i + j) * 32);
                        if constexpr (GLU) u[j] = ld_weight16(pu + (i + j) * 32);
                    }
                }
#pragma unroll
                for (int j = 0; j < U; j++)
#pragma unroll
                    for (int t = 0; t < DN_TT_GU; t++)
                        if (t < tt) {
                            const float *xp = xl + (size_t)t * H + (i + j) * 256;
                            ag[t] = dot8(g[j], xp, ag[t]);
                            if constexpr (GLU) au[t] = dot8(u[j], xp, au[t]);
                        }
            }
            for (; i < nv; i++) {
                const uint4 g1 = ld_weight16(pg + i * 32);
                uint4 u1 = g1;
                if (GLU) u1 = ld_weight16(pu + i * 32);
#pragma unroll
                for (int t = 0; t < DN_TT_GU; t++)
                    if (t < tt) {
                        const float *xp = xl + (size_t)t * H + i * 256;
                        ag[t] = dot8(g1, xp, ag[t]);
                        if (GLU) au[t] = dot8(u1, xp, au[t]);
                    }
            }
#pragma unroll
            for (int t = 0; t < DN_TT_GU; t++)
                if (t < tt) {
                    const float gs = warp_sum(ag[t]);
                    if (GLU) {
                        const float us = warp_sum(au[t]);
                        if (lane == 0) act[(size_t)(t0 + t) * Id + r] = (gs / (1.0f + expf(-gs))) * us;
                    } else if (lane == 0) {
                        act[(size_t)(t0 + t) * Id + r] = gs;
                    }
                }
        }
    }
}

__global__ void __launch_bounds__(DN_THREADS, 2) k_dense_gateup(const __half *__restrict__ Wg,
                                                             const __half *__restrict__ Wu,
                                                             const float *__restrict__ x, int T, int H, int Id,
                                                             float *__restrict__ act) {
    dense_rows<true>(Wg, Wu, x, T, H, Id, act);
}

// logits[t][v] = W[v] . h[t] over fp16 W [V x H] (lm_head, infer.m:1937-1941)
__global__ void __launch_bounds__(DN_THREADS, 2) k_lm_head(const __half *__restrict__ W,
                                                        const float *__restrict__ h, int T, int H, int V,
                                                        float *__restrict__ logits) {
    dense_rows<false>(W, nullptr, h, T, H, V, logits);
}

// CTA b owns the hidden rows [H b / G, H (b + 1) / G) (G CTAs, at most
// DN_RPC_MAX rows each); warp w covers the 16-byte vectors w * 32 + lane +
// 256 i of every one of them, so that the rows divide evenly over the CTAs
// whatever H / (warps on the GPU) is.  Partial sums meet in shared memory and
// are added in warp order: out[t][r] = (residual[t][r]) + Wd[r] . act[t] for
// up to DN_TT_D tokens per pass (Id % 256 == 0).  residual may be out itself
// (the layer stack's hidden state): each element is read and written by the
// same thread.
__global__ void __launch_bounds__(DN_THREADS, 3) k_dense_down(const __half *__restrict__ Wd,
                                                           const float *__restrict__ act, int T, int H, int Id,
                                                           int rpc, const float *residual, float *out) {
    extern __shared__ float4 dn_smem[];
    const int tt_max = min(T, DN_TT_D);
    float *part = reinterpret_cast<float *>(dn_smem);        // [DN_WARPS][rpc][tt_max]
    float *as = part + DN_WARPS * rpc * tt_max;              // [tt][Id], 16-byte aligned (rpc * tt_max * 32 B)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = (int)((long long)H * blockIdx.x / gridDim.x);
    const int r1 = (int)((long long)H * (blockIdx.x + 1) / gridDim.x);
    const int nv32 = Id >> 3;                      // 16-byte vectors per row
    const int base = warp * 32 + lane;
    const int cnt = nv32 > base ? (nv32 - base + 255) >> 8 : 0;   // this lane's vectors per row (warp-uniform)
    for (int t0 = 0; t0 < T; t0 += DN_TT_D) {
        const int tt = min(DN_TT_D, T - t0);
        // the first row's weights are in flight while the activations are staged
        uint4 w[DN_VD];
        if (r0 < r1) {
            const uint4 *pw = reinterpret_cast<const uint4 *>(Wd + (size_t)r0 * Id) + base;
#pragma unroll
            for (int j = 0; j < DN_VD; j++)
                if (j < cnt) w[j] = ld_weight16(pw + j * 256);
        }
        __syncthreads();
        stage_rows(as, act, t0, tt, Id);
        __syncthreads();
        for (int r = r0; r < r1; r++) {
            float acc[DN_TT_D];
#pragma unroll
            for (int t = 0; t < DN_TT_D; t++) acc[t] = 0.0f;
            const uint4 *pw = reinterpret_cast<const uint4 *>(Wd + (size_t)r * Id) + base;
            const float *al = as + warp * 256 + lane * 4;   // vector base + 256 i sits in chunk warp + 8 i
            for (int i0 = 0; i0 < cnt; i0 += DN_VD) {
                if (r != r0 || i0 != 0) {
#pragma unroll
                    for (int j = 0; j < DN_VD; j++)
                        if (i0 + j < cnt) w[j] = ld_weight16(pw + (i0 + j) * 256);
                }
#pragma unroll
                for (int j = 0; j < DN_VD; j++)
                    if (i0 + j < cnt)
#pragma unroll
                        for (int t = 0; t < DN_TT_D; t++)
                            if (t < tt) acc[t] = dot8(w[j], al + (size_t)t * Id + (i0 + j) * 2048, acc[t]);
            }
#pragma unroll
            for (int t = 0; t < DN_TT_D; t++)
                if (t < tt) {
                    const float v = warp_sum(acc[t]);
                    if (lane == 0) part[(warp * rpc + (r - r0)) * tt_max + t] = v;
                }
        }
        __syncthreads();
        for (int k = threadIdx.x; k < (r1 - r0) * tt; k += blockDim.x) {
            const int rl = k / tt, t = k - rl * tt;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < DN_WARPS; w++) v += part[(w * rpc + rl) * tt_max + t];
            const size_t o = (size_t)(t0 + t) * H + r0 + rl;
            out[o] = residual ? residual[o] + v : v;
        }
    }
}

// GGUF tensor values to fp16 (RNE): F32 / BF16 sources, or fp32 from the
// Q4_K / Q6_K dequant twins
__global__ void k_f32_to_f16(const float *__restrict__ src, __half *__restrict__ dst, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}
__global__ void k_bf16_to_f16(const uint16_t *__restrict__ src, __half *__restrict__ dst, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(__uint_as_float((uint32_t)src[i] << 16));
}

int dense_sms() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// persistent CTAs: as many as fit on every SM with this much shared memory
int dense_ctas(const void *fn, size_t smem) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, DN_THREADS, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    return per_sm * dense_sms();
}

}  // namespace

size_t moe_dense_smem_need(int H, int Id) {
    (void)H;
    const size_t a = (size_t)DN_TT_GU * H * sizeof(float);
    const size_t b = (size_t)DN_TT_D * Id * sizeof(float) + (size_t)DN_WARPS * DN_RPC_MAX * DN_TT_D * sizeof(float);
    return a > b ? a : b;
}

int moe_dense_shape_ok(int H, int Id) {
    return H > 0 && Id > 0 && H % 256 == 0 && Id % 256 == 0 && moe_dense_smem_need(H, Id) <= MOE_DENSE_SMEM_MAX;
}

void moe_launch_dense_ffn(const __half *w, int H, int Id, const float *x, int T, float *act, const float *residual,
                          float *out, cudaStream_t s, uint64_t *launches) {
    if (T <= 0) return;
    const __half *Wg = w, *Wu = w + (size_t)Id * H, *Wd = w + 2 * (size_t)Id * H;
    const int ttg = min(T, DN_TT_GU), ttd = min(T, DN_TT_D);
    const size_t sg = (size_t)ttg * H * sizeof(float);
    static size_t done_gu[MOE_MAX_DEVICES], done_d[MOE_MAX_DEVICES];
    moe_smem_limit(k_dense_gateup, sg, done_gu);
    const int gg = min(dense_ctas((const void *)k_dense_gateup, sg), (Id + DN_WARPS - 1) / DN_WARPS);
    // down: as many CTAs as fit with their activations and partial sums (the
    // partials grow as the CTAs get fewer, so settle the count in two rounds)
    const size_t sd_act = (size_t)ttd * Id * sizeof(float);
    moe_smem_limit(k_dense_down, sd_act + (size_t)DN_WARPS * DN_RPC_MAX * DN_TT_D * sizeof(float), done_d);
    int gd = H;
    size_t sd = 0;
    int rpc = 1;
    for (int round = 0; round < 2; round++) {
        const size_t guess = sd_act + (size_t)DN_WARPS * (round ? rpc : 1) * ttd * sizeof(float);
        gd = min(dense_ctas((const void *)k_dense_down, guess), H);
        gd = max(gd, (H + DN_RPC_MAX - 1) / DN_RPC_MAX);
        rpc = (H + gd - 1) / gd;
        sd = sd_act + (size_t)DN_WARPS * rpc * ttd * sizeof(float);
    }
    // (launched as programmatic dependents, with the first weight loads ahead
    // of the wait, the step measured 3 % slower: plain launches)
    k_dense_gateup<<<gg, DN_THREADS, sg, s>>>(Wg, Wu, x, T, H, Id, act);
    LAUNCH_COUNT(launches);
    k_dense_down<<<gd, DN_THREADS, sd, s>>>(Wd, act, T, H, Id, rpc, residual, out);
    LAUNCH_COUNT(launches);
}

void moe_launch_lm_head(const __half *w, int H, int V, const float *h, int T, float *logits, cudaStream_t s,
                        uint64_t *launches) {
    if (T <= 0) return;
    const size_t sg = (size_t)min(T, DN_TT_GU) * H * sizeof(float);
    static size_t done[MOE_MAX_DEVICES];
    moe_smem_limit(k_lm_head, sg, done);
    const int g = min(dense_ctas((const void *)k_lm_head, sg), (V + DN_WARPS - 1) / DN_WARPS);
    k_lm_head<<<g, DN_THREADS, sg, s>>>(w, h, T, H, V, logits);
    LAUNCH_COUNT(launches);
}

void moe_launch_to_f16(int type, const void *src, __half *dst, size_t n, float *tmp, cudaStream_t s,
                       uint64_t *launches) {
    const int grid = 4 * dense_sms();
    if (type == MOE_TYPE_F16) {
        cudaMemcpyAsync(dst, src, n * sizeof(__half), cudaMemcpyDeviceToDevice, s);
        return;
    }
    if (type == MOE_TYPE_BF16) {
        k_bf16_to_f16<<<grid, 256, 0, s>>>((const uint16_t *)src, dst, n);
        LAUNCH_COUNT(launches);
        return;
    }
    const float *f = (const float *)src;
    if (type == MOE_TYPE_Q4_K || type == MOE_TYPE_Q6_K) {
        moe_launch_dequant(type, (const uint8_t *)src, tmp, n, s, launches);
        f = tmp;
    }
    k_f32_to_f16<<<grid, 256, 0, s>>>(f, dst, n);
    LAUNCH_COUNT(launches);
}
