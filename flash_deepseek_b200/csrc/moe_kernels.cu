// moe_kernels.cu -- device kernels of the DeepSeek-V3/R1 MoE block for B200.
//
//   router logits   fp32 [T x H] x [H x E], split over H into partial sums
//   route + plan    sigmoid, grouped top-k (infer.m:920-991), dispatch plan,
//                   activation operand of the gate/up GEMV
//   gate/up         grouped Q4_K GEMV with SwiGLU epilogue (infer.m:1564-1568)
//   prep_down       activation operand of the down GEMV
//   down            grouped Q6_K / Q4_K GEMV (infer.m:1570, 1611)
//   combine         sum_k w_k eo_k in slot order + shared (infer.m:1915-1922)
//   codec / synth   dequant twins of quant.c, generator + quantizer, repack
#include <math.h>
#include <stdio.h>

#include "moe_common.cuh"
#include "moe_internal.h"

#define LAUNCH_COUNT(p) \
    do {                \
        if (p) (*(p))++; \
    } while (0)

static int g_num_sms = 0;
static int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

size_t moe_q4op_halves(int K) { return q4op_halves(K); }
size_t moe_q6op_halves(int K) { return q6op_halves(K); }

// ===========================================================================
// codec: device twins of quant.c (bit exact; explicit _rn ops, no contraction)
// ===========================================================================
__global__ void k_dequant_q4k(const uint8_t *__restrict__ src, float *__restrict__ y, size_t nblocks) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // one (block, chunk) per thread
    if (i >= nblocks * 4) return;
    const size_t b = i >> 2;
    const int c = (int)(i & 3);
    const uint8_t *p = src + b * MOE_Q4K_BYTES;
    const float d = h2f_bits((uint16_t)(p[0] | (p[1] << 8)));
    const float dmin = h2f_bits((uint16_t)(p[2] | (p[3] << 8)));
    const uint8_t *q = p + 4;
    int s0, m0, s1, m1;
    // scale_min_k4 (quant.c:26-34) for slots 2c and 2c+1
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const int j = 2 * c + u;
        int sc, mn;
        if (j < 4) { sc = q[j] & 63; mn = q[j + 4] & 63; }
        else { sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4); mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
        if (u == 0) { s0 = sc; m0 = mn; } else { s1 = sc; m1 = mn; }
    }
    const float d1 = __fmul_rn(d, (float)s0), n1 = __fmul_rn(dmin, (float)m0);
    const float d2 = __fmul_rn(d, (float)s1), n2 = __fmul_rn(dmin, (float)m1);
    const uint8_t *qs = p + 16 + 32 * c;
    float *yy = y + b * MOE_QK + 64 * c;
    for (int l = 0; l < 32; l++) {
        yy[l] = __fsub_rn(__fmul_rn(d1, (float)(qs[l] & 0x0F)), n1);
        yy[32 + l] = __fsub_rn(__fmul_rn(d2, (float)(qs[l] >> 4)), n2);
    }
}

__global__ void k_dequant_q6k(const uint8_t *__restrict__ src, float *__restrict__ y, size_t nblocks) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // one (block, half) per thread
    if (i >= nblocks * 2) return;
    const size_t b = i >> 1;
    const int h = (int)(i & 1);
    const uint8_t *p = src + b * MOE_Q6K_BYTES;
    const float d = h2f_bits((uint16_t)(p[208] | (p[209] << 8)));
    const uint8_t *ql = p + 64 * h, *qh = p + 128 + 32 * h;
    const int8_t *sc = (const int8_t *)(p + 192 + 8 * h);
    float *yy = y + b * MOE_QK + 128 * h;
    for (int l = 0; l < 32; l++) {
        const int is = l / 16;
        const int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
        const int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
        const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        yy[l] = __fmul_rn(__fmul_rn(d, (float)sc[is + 0]), (float)q1);
        yy[l + 32] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2]), (float)q2);
        yy[l + 64] = __fmul_rn(__fmul_rn(d, (float)sc[is + 4]), (float)q3);
        yy[l + 96] = __fmul_rn(__fmul_rn(d, (float)sc[is + 6]), (float)q4);
    }
}

void moe_launch_dequant(int type, const uint8_t *src, float *dst, size_t n, cudaStream_t s, uint64_t *launches) {
    const size_t nb = n / MOE_QK;
    if (nb == 0) return;
    if (type == 14) {
        const size_t work = nb * 2;
        k_dequant_q6k<<<(unsigned)((work + 255) / 256), 256, 0, s>>>(src, dst, nb);
    } else {
        const size_t work = nb * 4;
        k_dequant_q4k<<<(unsigned)((work + 255) / 256), 256, 0, s>>>(src, dst, nb);
    }
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// Q6_K repack (lossless byte permutation) and its inverse.
// ===========================================================================
__global__ void k_q6_repack(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int rows, int nb,
                            int inverse) {
    const size_t nblocks = (size_t)rows * nb;
    const int nbp = q6r_nb_pad(nb);
    for (size_t b = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; b < nblocks;
         b += (size_t)gridDim.x * (blockDim.x / 32)) {
        const int lane = threadIdx.x & 31;
        const size_t row = b / nb, sb = b % nb;
        uint8_t *rq = (inverse ? (uint8_t *)src : dst) + b * 192;
        uint8_t *rs = (inverse ? (uint8_t *)src : dst) + q6r_plane_s_off(rows, nb) + b * 16;
        uint8_t *rd = (inverse ? (uint8_t *)src : dst) + q6r_plane_d_off(rows, nb) + (row * nbp + sb) * 2;
        uint8_t *g = (inverse ? dst : (uint8_t *)src) + b * MOE_Q6K_BYTES;
        for (int p = lane; p < 192; p += 32) {
            const int sbyte = q6r_src_byte(p);
            if (inverse) g[sbyte] = rq[p]; else rq[p] = g[sbyte];
        }
        if (lane < 16) {
            if (inverse) g[192 + lane] = rs[lane]; else rs[lane] = g[192 + lane];
        } else if (lane < 18) {
            if (inverse) g[208 + lane - 16] = rd[lane - 16]; else rd[lane - 16] = g[208 + lane - 16];
        }
        // pad entries of the d plane (nb not a multiple of 8) stay zero: the
        // destination is cleared by the caller.
    }
}

void moe_launch_q6_repack(const uint8_t *src, uint8_t *dst, int rows, int nb, int inverse, cudaStream_t s,
                          uint64_t *launches) {
    const size_t nblocks = (size_t)rows * nb;
    int grid = (int)((nblocks + 7) / 8);
    if (grid > num_sms() * 16) grid = num_sms() * 16;
    if (grid < 1) grid = 1;
    k_q6_repack<<<grid, 256, 0, s>>>(src, dst, rows, nb, inverse);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// Synthetic weights: generator + quantizer (bit exact with the test oracle).
// One warp per super-block; lane l holds weights 8l .. 8l+7.
// ===========================================================================
__device__ __forceinline__ float warp_min_f(float v, int width_mask) {
    for (int o = 1; o <= width_mask; o <<= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max_f(float v, int width_mask) {
    for (int o = 1; o <= width_mask; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int clampi_d(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ void quant_q4k_warp(const float (&v)[8], uint8_t *dst, int lane, uint8_t *sq /*256 B smem*/,
                               uint8_t *ssm /*16 B smem*/) {
    // sub-block j = lane/4 (32 weights)
    float mn = v[0], mx = v[0];
#pragma unroll
    for (int i = 1; i < 8; i++) { mn = fminf(mn, v[i]); mx = fmaxf(mx, v[i]); }
    mn = warp_min_f(mn, 2);
    mx = warp_max_f(mx, 2);
    if (mn > 0.0f) mn = 0.0f;
    const float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    const float minv = -mn;
    const float max_scale = warp_max_f(scale, 16);
    const float max_min = warp_max_f(minv, 16);
    const uint16_t dh = f2h_rne_bits(__fdiv_rn(max_scale, 63.0f));
    const uint16_t mh = f2h_rne_bits(__fdiv_rn(max_min, 63.0f));
    const float d = h2f_bits(dh), dmin = h2f_bits(mh);
    const int sc = d > 0.0f ? clampi_d(q_rnd(__fdiv_rn(scale, d)), 0, 63) : 0;
    const int mm = dmin > 0.0f ? clampi_d(q_rnd(__fdiv_rn(minv, dmin)), 0, 63) : 0;
    const float ds = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)mm);
#pragma unroll
    for (int i = 0; i < 8; i++)
        sq[8 * lane + i] = (uint8_t)(ds > 0.0f ? clampi_d(q_rnd(__fdiv_rn(__fadd_rn(v[i], dm), ds)), 0, 15) : 0);
    if ((lane & 3) == 0) { ssm[lane >> 2] = (uint8_t)sc; ssm[8 + (lane >> 2)] = (uint8_t)mm; }
    __syncwarp();
    // qs byte b (b = 4*lane .. 4*lane+3): chunk c = b/32, l = b%32
    uint32_t word = 0;
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int b = 4 * lane + u, c = b >> 5, l = b & 31;
        const uint32_t byte = (uint32_t)sq[64 * c + l] | ((uint32_t)sq[64 * c + 32 + l] << 4);
        word |= byte << (8 * u);
    }
    reinterpret_cast<uint32_t *>(dst + 16)[lane] = word;
    if (lane < 4) {
        uint32_t hw;
        if (lane == 0) {
            hw = (uint32_t)dh | ((uint32_t)mh << 16);
        } else {
            hw = 0;
            for (int u = 0; u < 4; u++) {
                const int j = 4 * (lane - 1) + u;  // scale byte index 0..11
                uint32_t byte;
                if (j < 4) byte = (ssm[j] & 63) | ((ssm[j + 4] >> 4) << 6);
                else if (j < 8) byte = (ssm[8 + j - 4] & 63) | ((ssm[8 + j] >> 4) << 6);
                else byte = (ssm[j - 4] & 0xF) | ((ssm[8 + j - 4] & 0xF) << 4);
                hw |= byte << (8 * u);
            }
        }
        reinterpret_cast<uint32_t *>(dst)[lane] = hw;
    }
    __syncwarp();
}

__device__ void quant_q6k_warp(const float (&v)[8], uint8_t *dst, int lane, uint8_t *sq /*256 B*/,
                               int8_t *ssc /*16 B*/) {
    // sub-block j = lane/2 (16 weights)
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) am = fmaxf(am, fabsf(v[i]));
    am = warp_max_f(am, 1);
    const float scale = __fdiv_rn(am, 31.0f);
    const float max_scale = warp_max_f(scale, 16);
    const uint16_t dh = f2h_rne_bits(__fdiv_rn(max_scale, 127.0f));
    const float d = h2f_bits(dh);
    const int sc = d > 0.0f ? clampi_d(q_rnd(__fdiv_rn(scale, d)), 0, 127) : 0;
    const float ds = __fmul_rn(d, (float)sc);
#pragma unroll
    for (int i = 0; i < 8; i++)
        sq[8 * lane + i] = (uint8_t)((ds > 0.0f ? clampi_d(q_rnd(__fdiv_rn(v[i], ds)), -32, 31) : 0) + 32);
    if ((lane & 1) == 0) ssc[lane >> 1] = (int8_t)sc;
    __syncwarp();
    // 210 bytes: each lane builds bytes p = lane, lane+32, ... (< 210)
    for (int p = lane; p < MOE_Q6K_BYTES; p += 32) {
        uint8_t byte;
        if (p < 128) {
            const int h = p / 64, l = p % 64;
            const uint8_t *qq = sq + 128 * h;
            if (l < 32) byte = (uint8_t)((qq[l] & 0xF) | ((qq[l + 64] & 0xF) << 4));
            else byte = (uint8_t)((qq[l] & 0xF) | ((qq[l + 64] & 0xF) << 4));
        } else if (p < 192) {
            const int h = (p - 128) / 32, l = (p - 128) % 32;
            const uint8_t *qq = sq + 128 * h;
            byte = (uint8_t)((qq[l] >> 4) | ((qq[l + 32] >> 4) << 2) | ((qq[l + 64] >> 4) << 4) |
                             ((qq[l + 96] >> 4) << 6));
        } else if (p < 208) {
            byte = (uint8_t)ssc[p - 192];
        } else {
            byte = (uint8_t)(p == 208 ? (dh & 0xFF) : (dh >> 8));
        }
        dst[p] = byte;
    }
    __syncwarp();
}

__global__ void k_synth_quant(int type, uint64_t key, int rows, int cols, double sigma, uint8_t *__restrict__ dst) {
    __shared__ uint8_t sq[8][256];
    __shared__ uint8_t ssm[8][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = cols / MOE_QK;
    const size_t nblocks = (size_t)rows * nb;
    const size_t bsz = type == 14 ? MOE_Q6K_BYTES : MOE_Q4K_BYTES;
    for (size_t b = (size_t)blockIdx.x * 8 + warp; b < nblocks; b += (size_t)gridDim.x * 8) {
        const size_t row = b / nb, sb = b % nb;
        const uint64_t base = row * (uint64_t)cols + sb * MOE_QK + 8 * lane;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = synth_normal(key, base + i, sigma);
        if (type == 14) quant_q6k_warp(v, dst + b * bsz, lane, sq[warp], (int8_t *)ssm[warp]);
        else quant_q4k_warp(v, dst + b * bsz, lane, sq[warp], ssm[warp]);
    }
}

void moe_launch_synth_quant(int type, uint64_t seed, uint64_t stream, int rows, int cols, double sigma,
                            uint8_t *dst, cudaStream_t s, uint64_t *launches) {
    const uint64_t key = splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
    const size_t nblocks = (size_t)rows * (cols / MOE_QK);
    int grid = (int)((nblocks + 7) / 8);
    if (grid > num_sms() * 8) grid = num_sms() * 8;
    k_synth_quant<<<grid, 256, 0, s>>>(type, key, rows, cols, sigma, dst);
    LAUNCH_COUNT(launches);
}

__global__ void k_synth_f32(uint64_t key, size_t n, double sigma, float *__restrict__ dst) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = synth_normal(key, i, sigma);
}

void moe_launch_synth_f32(uint64_t seed, uint64_t stream, size_t n, double sigma, float *dst, cudaStream_t s,
                          uint64_t *launches) {
    const uint64_t key = splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
    int grid = (int)((n + 255) / 256);
    if (grid > num_sms() * 8) grid = num_sms() * 8;
    if (grid < 1) grid = 1;
    k_synth_f32<<<grid, 256, 0, s>>>(key, n, sigma, dst);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// Router logits: part[s][t][e] = sum_{k in split s} Wr[e][k] x[t][k].
// CTA = 32 experts x 256 k x all T tokens; thread = 4 experts x 2 tokens.
// ===========================================================================
#define RL_KS 256
#define RL_WPAD 36
__global__ void __launch_bounds__(256) k_router_logits(const float *__restrict__ Wr, const float *__restrict__ x,
                                                       int T, int H, int E, float *__restrict__ part) {
    extern __shared__ float sm[];
    float *Wt = sm;                       // [RL_KS][RL_WPAD]
    float *xt = sm + RL_KS * RL_WPAD;     // [RL_KS][64]
    const int e0 = blockIdx.x * 32, split = blockIdx.y, k0 = split * RL_KS;
    const int tid = threadIdx.x;
    // W tile: 32 rows x 256 floats, coalesced float4 loads, transposed store
    for (int i = tid; i < 32 * (RL_KS / 4); i += 256) {
        const int r = i / (RL_KS / 4), c4 = i % (RL_KS / 4);
        float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e0 + r < E) w = __ldg(reinterpret_cast<const float4 *>(Wr + (size_t)(e0 + r) * H + k0) + c4);
        Wt[(4 * c4 + 0) * RL_WPAD + r] = w.x;
        Wt[(4 * c4 + 1) * RL_WPAD + r] = w.y;
        Wt[(4 * c4 + 2) * RL_WPAD + r] = w.z;
        Wt[(4 * c4 + 3) * RL_WPAD + r] = w.w;
    }
    for (int i = tid; i < T * (RL_KS / 4); i += 256) {
        const int t = i / (RL_KS / 4), c4 = i % (RL_KS / 4);
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x + (size_t)t * H + k0) + c4);
        xt[(4 * c4 + 0) * 64 + t] = v.x;
        xt[(4 * c4 + 1) * 64 + t] = v.y;
        xt[(4 * c4 + 2) * 64 + t] = v.z;
        xt[(4 * c4 + 3) * 64 + t] = v.w;
    }
    __syncthreads();
    const int eg = tid >> 5, tg = tid & 31;
    const bool t0ok = tg < T, t1ok = tg + 32 < T;
    if (!t0ok) return;
    float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
#pragma unroll 4
    for (int k = 0; k < RL_KS; k++) {
        const float4 w = *reinterpret_cast<const float4 *>(Wt + k * RL_WPAD + 4 * eg);
        const float xa = xt[k * 64 + tg], xb = t1ok ? xt[k * 64 + tg + 32] : 0.f;
        acc[0][0] = fmaf(w.x, xa, acc[0][0]); acc[0][1] = fmaf(w.x, xb, acc[0][1]);
        acc[1][0] = fmaf(w.y, xa, acc[1][0]); acc[1][1] = fmaf(w.y, xb, acc[1][1]);
        acc[2][0] = fmaf(w.z, xa, acc[2][0]); acc[2][1] = fmaf(w.z, xb, acc[2][1]);
        acc[3][0] = fmaf(w.w, xa, acc[3][0]); acc[3][1] = fmaf(w.w, xb, acc[3][1]);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int e = e0 + 4 * eg + u;
        if (e >= E) continue;
        part[((size_t)split * T + tg) * E + e] = acc[u][0];
        if (t1ok) part[((size_t)split * T + tg + 32) * E + e] = acc[u][1];
    }
}

void moe_launch_router_logits(const float *Wr, const float *x, int T, int H, int E, float *part, int n_split,
                              cudaStream_t s, uint64_t *launches) {
    dim3 grid((E + 31) / 32, n_split);
    const size_t smem = sizeof(float) * (RL_KS * RL_WPAD + RL_KS * 64);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_router_logits, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = true;
    }
    k_router_logits<<<grid, 256, smem, s>>>(Wr, x, T, H, E, part);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// Activation operands
// ===========================================================================
__device__ __forceinline__ float block_max_abs(const float *x, int n, float *red /*[32]*/) {
    float m = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}

// power-of-two scale s with max|x| * s in (2^9, 2^10]; returns s, sets *inv.
__device__ __forceinline__ float op_scale(float amax, float *inv) {
    if (!(amax > 0.0f) || !isfinite(amax)) { *inv = 1.0f; return 1.0f; }
    int ex;
    frexpf(amax, &ex);  // amax = m 2^ex, m in [0.5, 1)
    int e = 10 - ex;
    if (e > 120) e = 120;
    if (e < -120) e = -120;
    *inv = ldexpf(1.0f, -e);
    return ldexpf(1.0f, e);
}

__device__ __forceinline__ void split_hl(float v, __half &hi, __half &lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
}

// Q4_K operand of one K-vector (all threads of the block).
__device__ void build_q4op(const float *__restrict__ x, int K, float s, __half *__restrict__ op) {
    const int NB = K / MOE_QK;
    for (int ent = threadIdx.x; ent < NB * Q4OP_STEPS * 4; ent += blockDim.x) {
        const int sb = ent / (Q4OP_STEPS * 4), m = (ent / 4) % Q4OP_STEPS, t = ent % 4;
        __half *o = op + ((size_t)sb * Q4OP_STEPS + m) * 32 + t * 4;
        const float *xb = x + sb * MOE_QK;
        if (m < 16) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                __half hi, lo;
                split_hl(__fmul_rn(xb[q4k_k(m, t, j)], s), hi, lo);
                o[j] = hi;
                o[16 + j] = lo;
            }
        } else {
            const int sa = q4k_min_sub(t);
#pragma unroll
            for (int u = 0; u < 2; u++) {
                float acc = 0.0f;
                for (int i = 0; i < 32; i++) {
                    __half hi, lo;
                    split_hl(__fmul_rn(xb[32 * (sa + u) + i], s), hi, lo);
                    acc = __fadd_rn(acc, __fadd_rn(__half2float(hi), __half2float(lo)));
                }
                __half hi, lo;
                split_hl(acc, hi, lo);
                o[u] = hi;
                o[16 + u] = lo;
            }
            o[2] = o[3] = o[18] = o[19] = __float2half_rn(0.0f);
        }
    }
}

// Q6_K operand of one K-vector plus the C-fold term per 16-weight sub-block.
__device__ void build_q6op(const float *__restrict__ x, int K, float s, __half *__restrict__ op,
                           float *__restrict__ cf) {
    const int NB = K / MOE_QK;
    for (int ent = threadIdx.x; ent < NB * 16 * 4; ent += blockDim.x) {
        const int sb = ent / 64, st = (ent / 4) % 16, t = ent % 4;
        __half *o = op + ((size_t)sb * 16 + st) * 32 + t * 4;
        const float *xb = x + sb * MOE_QK;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            __half hi, lo;
            split_hl(__fmul_rn(xb[q6k_k(st, t, j)], s), hi, lo);
            o[j] = hi;
            o[16 + j] = lo;
        }
    }
    for (int e = threadIdx.x; e < NB * 16; e += blockDim.x) {
        const int sb = e / 16, st = e % 16;
        const float *xb = x + sb * MOE_QK + 16 * st;
        float acc = 0.0f;
        for (int i = 0; i < 16; i++) {
            __half hi, lo;
            split_hl(__fmul_rn(xb[i], s), hi, lo);
            acc = __fadd_rn(acc, __fadd_rn(__half2float(hi), __half2float(lo)));
        }
        // low sub-blocks (s' < 4) decode to 1024 + q6, high ones to 1024 + 16 q6
        const float off = ((st & 7) < 4) ? -1056.0f : -1536.0f;
        cf[e] = __fmul_rn(off, acc);
    }
}

// ===========================================================================
// Route + plan.  Grid = T blocks of 256 threads (one thread per expert).
// ===========================================================================
struct RouteArgs {
    MoeDims d;
    const float *part;  int n_split;   // partial logits or nullptr
    const float *logits;               // full logits [T][E] or nullptr
    const float *bias;
    const int *idx_in; const float *w_in;  // given routing (mode 1)
    int mode;                              // 0 route, 1 routing given, 2 shared expert only
    int T;
    int *idx_out; float *w_out;
    const float *x; __half *xop; float *x_inv;   // x operand (may be nullptr)
    int include_shared, build_plan;
    MoePlan plan;
    int *counter;
};

__device__ void build_plan_block(const RouteArgs &a) {
    // one block, any blockDim >= 32
    __shared__ int cnt[1025], off[1026], coff[1026];
    __shared__ unsigned long long mask[1025];
    const int E = a.d.E, K = a.d.K, T = a.T;
    const int NE = E + 1;
    for (int e = threadIdx.x; e < NE; e += blockDim.x) { cnt[e] = 0; mask[e] = 0ull; }
    __syncthreads();
    const int n_routed = a.mode == 2 ? 0 : T * K;
    for (int p = threadIdx.x; p < n_routed; p += blockDim.x) {
        const int t = p / K;
        const int e = __ldcg(a.idx_out + p);
        if (e < 0 || e >= E) { atomicExch(a.plan.error, 1); continue; }
        atomicAdd(&cnt[e], 1);
        atomicOr(&mask[e], 1ull << t);
    }
    if (threadIdx.x == 0 && a.include_shared) {
        cnt[E] = T;
        mask[E] = (T >= 64) ? ~0ull : ((1ull << T) - 1ull);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int o = 0, c = 0, act = 0;
        for (int e = 0; e < NE; e++) {
            off[e] = o; coff[e] = c;
            o += cnt[e];
            c += (cnt[e] + MOE_TC - 1) / MOE_TC;
            if (e < E && cnt[e] > 0) act++;
        }
        off[NE] = o; coff[NE] = c;
        a.plan.counts[0] = o;
        a.plan.counts[1] = c;
        a.plan.counts[2] = act;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < n_routed; p += blockDim.x) {
        const int t = p / K, k = p % K;
        const int e = __ldcg(a.idx_out + p);
        if (e < 0 || e >= E) {  // flagged above; the combine skips the slot
            a.plan.slot_pair[t * (K + 1) + k] = -1;
            continue;
        }
        const int pos = off[e] + __popcll(mask[e] & ((1ull << t) - 1ull));
        a.plan.pair_expert[pos] = e;
        a.plan.pair_token[pos] = t;
        a.plan.pair_w[pos] = __ldcg(a.w_out + p);
        a.plan.slot_pair[t * (K + 1) + k] = pos;
    }
    if (a.include_shared) {
        for (int t = threadIdx.x; t < T; t += blockDim.x) {
            const int pos = off[E] + t;
            a.plan.pair_expert[pos] = E;
            a.plan.pair_token[pos] = t;
            a.plan.pair_w[pos] = 1.0f;
            a.plan.slot_pair[t * (K + 1) + K] = pos;
        }
    }
    for (int e = threadIdx.x; e < NE; e += blockDim.x) {
        const int n = cnt[e];
        for (int c = 0; c * MOE_TC < n; c++) {
            const int ci = coff[e] + c;
            a.plan.chunk_expert[ci] = e;
            a.plan.chunk_pair0[ci] = off[e] + c * MOE_TC;
            a.plan.chunk_ntok[ci] = min(MOE_TC, n - c * MOE_TC);
        }
    }
}

__global__ void __launch_bounds__(256) k_route_plan(RouteArgs a) {
    __shared__ float score[1024], choice[1024];
    __shared__ float gs[64];
    __shared__ float red[32];
    __shared__ int is_last;
    const int t = blockIdx.x;
    const int E = a.d.E, K = a.d.K, G = a.d.n_group, TG = a.d.topk_group;
    const int per = E / G;
    if (a.mode == 0) {
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            float lg;
            if (a.logits) lg = a.logits[(size_t)t * E + e];
            else {
                lg = 0.0f;
                for (int s = 0; s < a.n_split; s++) lg += a.part[((size_t)s * a.T + t) * E + e];
            }
            const float sc = 1.0f / (1.0f + expf(-lg));  // sigmoidf, infer.m:376
            score[e] = sc;
            choice[e] = sc + (a.bias ? a.bias[e] : 0.0f);
        }
        __syncthreads();
        // group score = top1 + top2 (strict '>', infer.m:931-941)
        for (int g = threadIdx.x; g < G; g += blockDim.x) {
            float t1 = -1e30f, t2 = -1e30f;
            for (int e = 0; e < per; e++) {
                const float s = choice[g * per + e];
                if (s > t1) { t2 = t1; t1 = s; }
                else if (s > t2) t2 = s;
            }
            gs[g] = t1 + t2;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            // top groups by repeated argmax, lowest index wins (infer.m:944-954)
            unsigned long long taken = 0ull;
            for (int k = 0; k < TG; k++) {
                int best = -1;
                float bs = -1e30f;
                for (int g = 0; g < G; g++)
                    if (!((taken >> g) & 1ull) && gs[g] > bs) { bs = gs[g]; best = g; }
                if (best >= 0) taken |= 1ull << best;
            }
            // top-K in slot order (infer.m:966-980): scan experts ascending,
            // replace the first minimum slot when strictly greater.
            float key[MOE_MAX_K];
            int idx[MOE_MAX_K];
            for (int k = 0; k < K; k++) { key[k] = -1e30f; idx[k] = 0; }
            int mk = 0;
            float mkey = -1e30f;
            for (int g = 0; g < G; g++) {
                if (!((taken >> g) & 1ull)) continue;
                for (int e = g * per; e < (g + 1) * per; e++) {
                    const float c = choice[e];
                    if (c > mkey) {
                        key[mk] = c;
                        idx[mk] = e;
                        mk = 0;
                        mkey = key[0];
                        for (int k = 1; k < K; k++)
                            if (key[k] < mkey) { mkey = key[k]; mk = k; }
                    }
                }
            }
            float w[MOE_MAX_K], s = 0.0f;
            for (int k = 0; k < K; k++) { w[k] = score[idx[k]]; s += w[k]; }
            if (s > 0.0f) {
                const float f = a.d.scale / s;
                for (int k = 0; k < K; k++) w[k] *= f;
            }
            for (int k = 0; k < K; k++) {
                a.idx_out[t * K + k] = idx[k];
                a.w_out[t * K + k] = w[k];
            }
        }
    } else if (a.mode == 1 && threadIdx.x < K) {
        a.idx_out[t * K + threadIdx.x] = a.idx_in[t * K + threadIdx.x];
        a.w_out[t * K + threadIdx.x] = a.w_in[t * K + threadIdx.x];
    }

    // activation operand of this token for the gate/up GEMV
    if (a.xop) {
        const float *xr = a.x + (size_t)t * a.d.H;
        const float amax = block_max_abs(xr, a.d.H, red);
        float inv;
        const float s = op_scale(amax, &inv);
        build_q4op(xr, a.d.H, s, a.xop + (size_t)t * q4op_halves(a.d.H));
        if (threadIdx.x == 0) a.x_inv[t] = inv;
    }
    if (!a.build_plan) return;
    // last block to finish builds the plan for all tokens
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = (atomicAdd(a.counter, 1) == a.T - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    build_plan_block(a);
    if (threadIdx.x == 0) *a.counter = 0;
}

void moe_launch_route_and_plan(const MoeDims &d, const float *part, int n_split, const float *logits,
                               const float *bias, int mode, const int *idx_in, const float *w_in, int T,
                               int *idx_out, float *w_out, const float *x, __half *xop, float *x_inv,
                               int include_shared, int build_plan, const MoePlan &plan, int *counter,
                               cudaStream_t s, uint64_t *launches) {
    RouteArgs a;
    a.d = d; a.part = part; a.n_split = n_split; a.logits = logits; a.bias = bias;
    a.idx_in = idx_in; a.w_in = w_in; a.mode = mode; a.T = T; a.idx_out = idx_out; a.w_out = w_out;
    a.x = x; a.xop = xop; a.x_inv = x_inv; a.include_shared = include_shared; a.build_plan = build_plan;
    a.plan = plan; a.counter = counter;
    k_route_plan<<<T, 256, 0, s>>>(a);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// Q4_K warp tile: rows (r0+g, r0+g+8) of one matrix over super-blocks
// [sb0, sb1) against up to 4*NT activation vectors.  Lane (g = lane/4,
// t = lane%4).  For each super-block the lane loads 2 x 16 B of nibbles per
// row plus the 16-byte header, decodes the weights of each MMA step to
// sc*q in fp16 (exact: HFMA2 of the 1024+q magic), accumulates
// P1 = sum sc*q*x and P2 = sum m*X (min term) on the tensor core and flushes
// acc += d*P1 - dmin*P2 (quant.c:36-61 algebra, fp32).
// ===========================================================================
struct Q4Hdr {
    __half2 sc[4], nsc[4];
    uint32_t m2;
    float d, dmin;
};

__device__ __forceinline__ void q4_decode_hdr(const uint4 h, int t, Q4Hdr &o) {
    const int q = t >> 1;
    o.d = h2f_bits((uint16_t)(h.x & 0xFFFFu));
    o.dmin = h2f_bits((uint16_t)(h.x >> 16));
    const uint32_t a0 = h.y >> (16 * q), a1 = h.z >> (16 * q), a2 = h.w >> (16 * q);
    const uint32_t sc_lo = a0 & 0x3F3Fu, m_lo = a1 & 0x3F3Fu;
    const uint32_t sc_hi = (a2 & 0x0F0Fu) | ((a0 >> 2) & 0x3030u);
    const uint32_t m_hi = ((a2 >> 4) & 0x0F0Fu) | ((a1 >> 2) & 0x3030u);
    const __half2 k1024 = __float2half2_rn(1024.0f), km1024 = __float2half2_rn(-1024.0f);
    o.sc[0] = __hsub2(u32_as_h2(__byte_perm(sc_lo, 0x6464u, 0x4040u)), k1024);
    o.sc[1] = __hsub2(u32_as_h2(__byte_perm(sc_lo, 0x6464u, 0x4141u)), k1024);
    o.sc[2] = __hsub2(u32_as_h2(__byte_perm(sc_hi, 0x6464u, 0x4040u)), k1024);
    o.sc[3] = __hsub2(u32_as_h2(__byte_perm(sc_hi, 0x6464u, 0x4141u)), k1024);
#pragma unroll
    for (int u = 0; u < 4; u++) o.nsc[u] = __hmul2(o.sc[u], km1024);
    const uint32_t mw = (t & 1) ? m_hi : m_lo;
    o.m2 = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(mw, 0x6464u, 0x4140u)), k1024));
}

// sc*q for the two nibbles at bits [0,4) and [16,20) of w (exact fp16)
__device__ __forceinline__ uint32_t q4_dq(uint32_t w, __half2 sc, __half2 nsc) {
    const uint32_t h = (w & 0x000F000Fu) | 0x64006400u;
    return h2_as_u32(__hfma2(u32_as_h2(h), sc, nsc));
}

template <int NT>
__device__ __forceinline__ void q4k_warp_rows(const uint8_t *__restrict__ rg, const uint8_t *__restrict__ rg8,
                                              int sb0, int sb1, const __half *const (&opb)[NT], const bool (&bok)[NT],
                                              float (&acc)[NT][2], int t) {
#pragma unroll 1
    for (int sb = sb0; sb < sb1; ++sb) {
        const uint8_t *bg = rg + (size_t)sb * MOE_Q4K_BYTES, *bg8 = rg8 + (size_t)sb * MOE_Q4K_BYTES;
        const uint4 hg = ldg_stream16(bg), hg8 = ldg_stream16(bg8);
        uint4 qg[2], qg8[2];
        qg[0] = ldg_stream16(bg + 16 + 16 * t);
        qg[1] = ldg_stream16(bg + 80 + 16 * t);
        qg8[0] = ldg_stream16(bg8 + 16 + 16 * t);
        qg8[1] = ldg_stream16(bg8 + 80 + 16 * t);
        Q4Hdr Hg, Hg8;
        q4_decode_hdr(hg, t, Hg);
        q4_decode_hdr(hg8, t, Hg8);
        float p1[NT][4], p2[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
            for (int c = 0; c < 4; c++) p1[n][c] = 0.0f;
        const __half *opsb[NT];
#pragma unroll
        for (int n = 0; n < NT; n++) opsb[n] = opb[n] + (size_t)sb * Q4OP_HALVES_PER_SB;
#pragma unroll
        for (int r = 0; r < 2; r++) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t wg = (i == 0) ? qg[r].x : (i == 1) ? qg[r].y : (i == 2) ? qg[r].z : qg[r].w;
                const uint32_t wg8 = (i == 0) ? qg8[r].x : (i == 1) ? qg8[r].y : (i == 2) ? qg8[r].z : qg8[r].w;
#pragma unroll
                for (int hi = 0; hi < 2; hi++) {
                    const int m = 8 * r + 2 * i + hi, u = 2 * r + hi;
                    const uint32_t a0 = q4_dq(wg >> (4 * hi), Hg.sc[u], Hg.nsc[u]);
                    const uint32_t a2 = q4_dq(wg >> (8 + 4 * hi), Hg.sc[u], Hg.nsc[u]);
                    const uint32_t a1 = q4_dq(wg8 >> (4 * hi), Hg8.sc[u], Hg8.nsc[u]);
                    const uint32_t a3 = q4_dq(wg8 >> (8 + 4 * hi), Hg8.sc[u], Hg8.nsc[u]);
#pragma unroll
                    for (int n = 0; n < NT; n++) {
                        uint2 b = make_uint2(0u, 0u);
                        if (bok[n]) b = ldg_op8(opsb[n] + m * 32);
                        mma_f16_16816(p1[n], a0, a1, a2, a3, b.x, b.y, p1[n][0], p1[n][1], p1[n][2], p1[n][3]);
                    }
                }
            }
        }
#pragma unroll
        for (int n = 0; n < NT; n++) {
            uint2 b = make_uint2(0u, 0u);
            if (bok[n]) b = ldg_op8(opsb[n] + 16 * 32);
            mma_f16_16816(p2[n], Hg.m2, Hg8.m2, 0u, 0u, b.x, b.y, 0.f, 0.f, 0.f, 0.f);
            acc[n][0] = fmaf(Hg.d, p1[n][0] + p1[n][1], fmaf(-Hg.dmin, p2[n][0] + p2[n][1], acc[n][0]));
            acc[n][1] = fmaf(Hg8.d, p1[n][2] + p1[n][3], fmaf(-Hg8.dmin, p2[n][2] + p2[n][3], acc[n][1]));
        }
    }
}

// ===========================================================================
// Q6_K warp tile (repacked layout): one MMA per 16-weight sub-block with the
// -32 offset and the decode magic folded into the C operand, flushed as
// acc += d*sc*D (quant.c:63-92 algebra, fp32).
// ===========================================================================
template <int NT>
__device__ __forceinline__ void q6k_warp_rows(const uint8_t *__restrict__ W, int rows, int nb, int row_g,
                                              const __half *const (&opb)[NT], const bool (&bok)[NT],
                                              const float *const (&cfb)[NT], const bool (&cok)[NT],
                                              float (&acc)[NT][2], int t) {
    const int row_g8 = row_g + 8;
    const int nbp = q6r_nb_pad(nb);
    const uint8_t *qpl = W, *spl = W + q6r_plane_s_off(rows, nb);
    const uint16_t *dpl = reinterpret_cast<const uint16_t *>(W + q6r_plane_d_off(rows, nb));
#pragma unroll 1
    for (int sb = 0; sb < nb; ++sb) {
        const uint8_t *qg = qpl + ((size_t)row_g * nb + sb) * 192 + 48 * t;
        const uint8_t *qg8 = qpl + ((size_t)row_g8 * nb + sb) * 192 + 48 * t;
        uint4 ug[3], ug8[3];
#pragma unroll
        for (int v = 0; v < 3; v++) {
            ug[v] = ldg_stream16(qg + 16 * v);
            ug8[v] = ldg_stream16(qg8 + 16 * v);
        }
        const uint4 sg = ldg_stream16(spl + ((size_t)row_g * nb + sb) * 16);
        const uint4 sg8 = ldg_stream16(spl + ((size_t)row_g8 * nb + sb) * 16);
        const float dg = h2f_bits(__ldg(dpl + (size_t)row_g * nbp + sb));
        const float dg8 = h2f_bits(__ldg(dpl + (size_t)row_g8 * nbp + sb));
        // words [h][0..3] = ql, [h][4..5] = qh
        const uint32_t wg[2][6] = {{ug[0].x, ug[0].y, ug[0].z, ug[0].w, ug[1].x, ug[1].y},
                                   {ug[1].z, ug[1].w, ug[2].x, ug[2].y, ug[2].z, ug[2].w}};
        const uint32_t wg8[2][6] = {{ug8[0].x, ug8[0].y, ug8[0].z, ug8[0].w, ug8[1].x, ug8[1].y},
                                    {ug8[1].z, ug8[1].w, ug8[2].x, ug8[2].y, ug8[2].z, ug8[2].w}};
        const uint32_t sgw[4] = {sg.x, sg.y, sg.z, sg.w}, sg8w[4] = {sg8.x, sg8.y, sg8.z, sg8.w};
        const size_t sbo = (size_t)sb * Q6OP_HALVES_PER_SB;
#pragma unroll
        for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int sp = 0; sp < 8; sp++) {
                const int s = 8 * h + sp;
                const bool hiT = sp >= 4;
                const int f = sp >> 1;
                const uint32_t M1 = hiT ? 0x00F000F0u : 0x000F000Fu;
                const uint32_t M2 = hiT ? 0x03000300u : 0x00300030u;
                const int she = (f & 1) ? 2 : 4, sho = (f & 1) ? 6 : 4;
                const uint32_t Wg = wg[h][sp & 3], Hg = wg[h][4 + (sp & 1)];
                const uint32_t Wg8 = wg8[h][sp & 3], Hg8 = wg8[h][4 + (sp & 1)];
                const uint32_t a0 = (Wg & M1) | ((Hg << she) & M2) | 0x64006400u;
                const uint32_t a2 = ((Wg >> 8) & M1) | ((Hg >> sho) & M2) | 0x64006400u;
                const uint32_t a1 = (Wg8 & M1) | ((Hg8 << she) & M2) | 0x64006400u;
                const uint32_t a3 = ((Wg8 >> 8) & M1) | ((Hg8 >> sho) & M2) | 0x64006400u;
                const float fs = hiT ? 0.0625f : 1.0f;
                const float dsg = dg * fs * (float)(int8_t)(sgw[s >> 2] >> (8 * (s & 3)));
                const float dsg8 = dg8 * fs * (float)(int8_t)(sg8w[s >> 2] >> (8 * (s & 3)));
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    uint2 b = make_uint2(0u, 0u);
                    if (bok[n]) b = ldg_op8(opb[n] + sbo + s * 32);
                    const float cf = cok[n] ? __ldg(cfb[n] + sb * 16 + s) : 0.0f;
                    float dd[4];
                    mma_f16_16816(dd, a0, a1, a2, a3, b.x, b.y, cf, 0.f, cf, 0.f);
                    acc[n][0] = fmaf(dsg, dd[0] + dd[1], acc[n][0]);
                    acc[n][1] = fmaf(dsg8, dd[2] + dd[3], acc[n][1]);
                }
            }
        }
    }
}

__device__ __forceinline__ int expert_slot(const MoeLayerDev &L, int E, int e) {
    return e == E ? L.n_local : e - L.e0;
}

// ===========================================================================
// gate/up: CTA item = (chunk, 64 rows); warp w: row tile w&3, K half w>>2.
// act[pair][row] = silu(gate) * up  (infer.m:378-383)
// ===========================================================================
#define GU_NT 2
__global__ void __launch_bounds__(256, 2) k_gateup(MoeDims d, MoeLayerDev L, MoePlan plan,
                                                   const __half *__restrict__ xop, const float *__restrict__ x_inv,
                                                   float *__restrict__ act) {
    __shared__ float red[2][2][MOE_ROWS_GU][MOE_TC + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int rt = warp & 3, kh = warp >> 2;
    const int n_chunks = plan.counts[1];
    const int n_rg = d.I / MOE_ROWS_GU;
    const int n_items = n_chunks * n_rg;
    const int NB = d.H / MOE_QK, nbh = NB / 2;
    const int sb0 = kh ? nbh : 0, sb1 = kh ? NB : nbh;
    const size_t rowb = (size_t)NB * MOE_Q4K_BYTES;
    const size_t opstride = q4op_halves(d.H);
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int rgi = item / n_chunks, c = item % n_chunks;
        const int e = plan.chunk_expert[c], p0 = plan.chunk_pair0[c], ntok = plan.chunk_ntok[c];
        const uint8_t *ex = L.experts + (size_t)expert_slot(L, d.E, e) * L.expert_stride;
        const int r0 = rgi * MOE_ROWS_GU + rt * 16;
        const __half *opb[GU_NT];
        bool bok[GU_NT];
#pragma unroll
        for (int n = 0; n < GU_NT; n++) {
            const int tk = 4 * n + (g >> 1);
            bok[n] = tk < ntok;
            const int tok = bok[n] ? plan.pair_token[p0 + tk] : 0;
            opb[n] = xop + (size_t)tok * opstride + (g & 1) * 16 + t * 4;
        }
#pragma unroll 1
        for (int mat = 0; mat < 2; mat++) {
            const uint8_t *Wm = ex + (size_t)mat * L.gate_bytes;
            float acc[GU_NT][2];
#pragma unroll
            for (int n = 0; n < GU_NT; n++) acc[n][0] = acc[n][1] = 0.0f;
            q4k_warp_rows<GU_NT>(Wm + (size_t)(r0 + g) * rowb, Wm + (size_t)(r0 + g + 8) * rowb, sb0, sb1, opb, bok,
                                 acc, t);
#pragma unroll
            for (int n = 0; n < GU_NT; n++) {
                red[kh][mat][rt * 16 + g][4 * n + t] = acc[n][0];
                red[kh][mat][rt * 16 + g + 8][4 * n + t] = acc[n][1];
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < MOE_ROWS_GU * ntok; i += blockDim.x) {
            const int row = i / ntok, tk = i % ntok;
            const int pair = p0 + tk;
            const float inv = x_inv[plan.pair_token[pair]];
            const float gv = (red[0][0][row][tk] + red[1][0][row][tk]) * inv;
            const float uv = (red[0][1][row][tk] + red[1][1][row][tk]) * inv;
            act[(size_t)pair * d.I + rgi * MOE_ROWS_GU + row] = (gv / (1.0f + expf(-gv))) * uv;
        }
        __syncthreads();
    }
}

void moe_launch_gateup(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const __half *xop,
                       const float *x_inv, float *act, int max_items, cudaStream_t s, uint64_t *launches) {
    int grid = num_sms() * 2;
    if (grid > max_items) grid = max_items;
    if (grid < 1) grid = 1;
    k_gateup<<<grid, 256, 0, s>>>(d, L, plan, xop, x_inv, act);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// down operand: per pair, scale + hi/lo split of act into the layout of the
// expert's down type.
// ===========================================================================
__global__ void __launch_bounds__(256) k_prep_down(MoeDims d, MoeLayerDev L, MoePlan plan,
                                                   const float *__restrict__ act, __half *__restrict__ dop,
                                                   float *__restrict__ dcf, float *__restrict__ d_inv) {
    __shared__ float red[32];
    const int n_pairs = plan.counts[0];
    const size_t opst = q4op_halves(d.I) > q6op_halves(d.I) ? q4op_halves(d.I) : q6op_halves(d.I);
    for (int p = blockIdx.x; p < n_pairs; p += gridDim.x) {
        const float *a = act + (size_t)p * d.I;
        const float amax = block_max_abs(a, d.I, red);
        float inv;
        const float s = op_scale(amax, &inv);
        const int e = plan.pair_expert[p];
        const int ty = (e == d.E) ? L.sh_down_type : L.down_type;
        if (ty == 14) build_q6op(a, d.I, s, dop + (size_t)p * opst, dcf + (size_t)p * (d.I / MOE_QK) * 16);
        else build_q4op(a, d.I, s, dop + (size_t)p * opst);
        if (threadIdx.x == 0) d_inv[p] = inv;
        __syncthreads();
    }
}

void moe_launch_prep_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const float *act,
                          __half *dop, float *dcf, float *d_inv, int max_pairs, cudaStream_t s,
                          uint64_t *launches) {
    int grid = max_pairs;
    if (grid > num_sms() * 4) grid = num_sms() * 4;
    if (grid < 1) grid = 1;
    k_prep_down<<<grid, 256, 0, s>>>(d, L, plan, act, dop, dcf, d_inv);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// down: warp task = (chunk, 16 rows of H); eo[pair][row]
// ===========================================================================
#define DN_NT 2
__global__ void __launch_bounds__(256, 2) k_down(MoeDims d, MoeLayerDev L, MoePlan plan,
                                                 const __half *__restrict__ dop, const float *__restrict__ dcf,
                                                 const float *__restrict__ d_inv, float *__restrict__ eo) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nw = gridDim.x * (blockDim.x >> 5);
    const int n_chunks = plan.counts[1];
    const int n_rt = d.H / 16;
    const int n_tasks = n_chunks * n_rt;
    const int NB = d.I / MOE_QK;
    const size_t opst = q4op_halves(d.I) > q6op_halves(d.I) ? q4op_halves(d.I) : q6op_halves(d.I);
    for (int task = gw; task < n_tasks; task += nw) {
        const int rt = task / n_chunks, c = task % n_chunks;
        const int e = plan.chunk_expert[c], p0 = plan.chunk_pair0[c], ntok = plan.chunk_ntok[c];
        const uint8_t *Wd = L.experts + (size_t)expert_slot(L, d.E, e) * L.expert_stride + 2 * L.gate_bytes;
        const int ty = (e == d.E) ? L.sh_down_type : L.down_type;
        const int r0 = rt * 16;
        const __half *opb[DN_NT];
        const float *cfb[DN_NT];
        bool bok[DN_NT], cok[DN_NT];
#pragma unroll
        for (int n = 0; n < DN_NT; n++) {
            const int tb = 4 * n + (g >> 1), tc = 4 * n + t;
            bok[n] = tb < ntok;
            cok[n] = tc < ntok;
            opb[n] = dop + (size_t)(p0 + (bok[n] ? tb : 0)) * opst + (g & 1) * 16 + t * 4;
            cfb[n] = dcf + (size_t)(p0 + (cok[n] ? tc : 0)) * NB * 16;
        }
        float acc[DN_NT][2];
#pragma unroll
        for (int n = 0; n < DN_NT; n++) acc[n][0] = acc[n][1] = 0.0f;
        if (ty == 14) {
            q6k_warp_rows<DN_NT>(Wd, d.H, NB, r0 + g, opb, bok, cfb, cok, acc, t);
        } else {
            const size_t rowb = (size_t)NB * MOE_Q4K_BYTES;
            q4k_warp_rows<DN_NT>(Wd + (size_t)(r0 + g) * rowb, Wd + (size_t)(r0 + g + 8) * rowb, 0, NB, opb, bok,
                                 acc, t);
        }
#pragma unroll
        for (int n = 0; n < DN_NT; n++) {
            if (!cok[n]) continue;
            const int pair = p0 + 4 * n + t;
            const float inv = d_inv[pair];
            eo[(size_t)pair * d.H + r0 + g] = acc[n][0] * inv;
            eo[(size_t)pair * d.H + r0 + g + 8] = acc[n][1] * inv;
        }
    }
}

void moe_launch_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const __half *dop,
                     const float *dcf, const float *d_inv, float *eo, int max_items, cudaStream_t s,
                     uint64_t *launches) {
    int grid = num_sms() * 2;
    const int need = (max_items + 7) / 8;
    if (grid > need) grid = need;
    if (grid < 1) grid = 1;
    k_down<<<grid, 256, 0, s>>>(d, L, plan, dop, dcf, d_inv, eo);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// combine: out[t] = (sum_k w_k eo_k in slot order) + shared (+ residual)
// ===========================================================================
__global__ void k_combine(MoeDims d, MoePlan plan, const float *__restrict__ eo, int T, int include_routed,
                          int include_shared, const float *__restrict__ residual, float *__restrict__ out) {
    const int t = blockIdx.y;
    const int K = d.K, KR = include_routed ? d.K : 0;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= d.H) return;
    float acc = 0.0f;
    for (int k = 0; k < KR; k++) {
        const int p = plan.slot_pair[t * (K + 1) + k];
        if (p < 0) continue;
        acc = fmaf(plan.pair_w[p], eo[(size_t)p * d.H + i], acc);
    }
    if (include_shared) acc = acc + eo[(size_t)plan.slot_pair[t * (K + 1) + K] * d.H + i];
    if (residual) acc = residual[(size_t)t * d.H + i] + acc;
    out[(size_t)t * d.H + i] = acc;
}

void moe_launch_combine(const MoeDims &d, const MoePlan &plan, const float *eo, int T, int include_routed,
                        int include_shared, const float *residual, float *out, cudaStream_t s, uint64_t *launches) {
    dim3 grid((d.H + 255) / 256, T);
    k_combine<<<grid, 256, 0, s>>>(d, plan, eo, T, include_routed, include_shared, residual, out);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// RMSNorm (infer.m:369-374): y = x * (1/sqrtf(mean(x^2) + eps)) * w
// ===========================================================================
__global__ void k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ y, int H,
                          float eps) {
    __shared__ float red[32];
    const float *xr = x + (size_t)blockIdx.x * H;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(red[0] / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = xr[i] * inv;
        y[(size_t)blockIdx.x * H + i] = w ? v * w[i] : v;
    }
}

void moe_launch_rmsnorm(const float *x, const float *w, float *y, int T, int H, float eps, cudaStream_t s,
                        uint64_t *launches) {
    k_rmsnorm<<<T, 256, 0, s>>>(x, w, y, H, eps);
    LAUNCH_COUNT(launches);
}
