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
size_t moe_dop_bytes(int K) { return dop_bytes(K); }

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
#define RL_WPAD (RL_KS + 4)
__global__ void __launch_bounds__(256) k_router_logits(const float *__restrict__ Wr, const float *__restrict__ x,
                                                       int T, int H, int E, float *__restrict__ part,
                                                       float *__restrict__ logits, int *__restrict__ counters) {
    extern __shared__ float sm[];
    float *Ws = sm;                       // [32 experts][RL_WPAD] row-major (k contiguous)
    float *xt = sm + 32 * RL_WPAD;        // [RL_KS][64] (tokens contiguous)
    const int e0 = blockIdx.x * 32, split = blockIdx.y, k0 = split * RL_KS;
    const int tid = threadIdx.x;
    // W tile: 8 coalesced float4 loads in flight per thread, then float4 stores
    {
        float4 wv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = tid + 256 * u, r = i / (RL_KS / 4), c4 = i % (RL_KS / 4);
            wv[u] = e0 + r < E ? __ldg(reinterpret_cast<const float4 *>(Wr + (size_t)(e0 + r) * H + k0) + c4)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = tid + 256 * u, r = i / (RL_KS / 4), c4 = i % (RL_KS / 4);
            *reinterpret_cast<float4 *>(Ws + r * RL_WPAD + 4 * c4) = wv[u];
        }
    }
    const int eg = tid >> 5, tg = tid & 31;
    const bool small = T <= 4;
    if (small) {
        // few tokens: x row-major, lane = 8 consecutive k, warp-reduced
        for (int i = tid; i < T * (RL_KS / 4); i += 256) {
            const int t = i / (RL_KS / 4), c4 = i % (RL_KS / 4);
            *reinterpret_cast<float4 *>(xt + t * RL_KS + 4 * c4) =
                __ldg(reinterpret_cast<const float4 *>(x + (size_t)t * H + k0) + c4);
        }
        __syncthreads();
        float accs[4][4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const float4 w0 = *reinterpret_cast<const float4 *>(Ws + (4 * eg + u) * RL_WPAD + 8 * tg);
            const float4 w1 = *reinterpret_cast<const float4 *>(Ws + (4 * eg + u) * RL_WPAD + 8 * tg + 4);
#pragma unroll
            for (int t = 0; t < 4; t++) {
                float v = 0.0f;
                if (t < T) {
                    const float4 x0 = *reinterpret_cast<const float4 *>(xt + t * RL_KS + 8 * tg);
                    const float4 x1 = *reinterpret_cast<const float4 *>(xt + t * RL_KS + 8 * tg + 4);
                    v = w0.x * x0.x + w0.y * x0.y + w0.z * x0.z + w0.w * x0.w + w1.x * x1.x + w1.y * x1.y +
                        w1.z * x1.z + w1.w * x1.w;
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                }
                accs[u][t] = v;
            }
        }
        if (tg == 0) {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int e = e0 + 4 * eg + u;
                if (e >= E) continue;
#pragma unroll
                for (int t = 0; t < 4; t++)
                    if (t < T) part[((size_t)split * T + t) * E + e] = accs[u][t];
            }
        }
    } else {
    // x tile transposed: consecutive threads take consecutive tokens
    for (int i = tid; i < T * (RL_KS / 4); i += 256) {
        const int c4 = i / T, t = i % T;
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x + (size_t)t * H + k0) + c4);
        xt[(4 * c4 + 0) * 64 + t] = v.x;
        xt[(4 * c4 + 1) * 64 + t] = v.y;
        xt[(4 * c4 + 2) * 64 + t] = v.z;
        xt[(4 * c4 + 3) * 64 + t] = v.w;
    }
    __syncthreads();
    // warp = 4 experts, lane = tokens tg, tg+32
    const bool t0ok = tg < T, t1ok = tg + 32 < T;
    float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
    const float *w0 = Ws + (4 * eg) * RL_WPAD;
#pragma unroll 2
    for (int k = 0; k < RL_KS; k += 4) {
        float4 w[4];
#pragma unroll
        for (int u = 0; u < 4; u++) w[u] = *reinterpret_cast<const float4 *>(w0 + u * RL_WPAD + k);  // broadcast
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float xa = xt[(k + j) * 64 + tg], xb = t1ok ? xt[(k + j) * 64 + tg + 32] : 0.f;
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float wv = j == 0 ? w[u].x : j == 1 ? w[u].y : j == 2 ? w[u].z : w[u].w;
                acc[u][0] = fmaf(wv, xa, acc[u][0]);
                acc[u][1] = fmaf(wv, xb, acc[u][1]);
            }
        }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int e = e0 + 4 * eg + u;
        if (e >= E) continue;
        if (t0ok) part[((size_t)split * T + tg) * E + e] = acc[u][0];
        if (t1ok) part[((size_t)split * T + tg + 32) * E + e] = acc[u][1];
    }
    }
    // The last split CTA of this expert group sums the partials in split
    // order (deterministic) into the final logits.
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&counters[blockIdx.x], 1) == (int)gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int ns = gridDim.y;
    for (int i = tid; i < T * 32; i += 256) {
        const int t = i / 32, e = e0 + i % 32;
        if (e >= E) continue;
        float v = 0.0f;
#pragma unroll 4
        for (int sp = 0; sp < ns; sp++) v += __ldcg(part + ((size_t)sp * T + t) * E + e);
        logits[(size_t)t * E + e] = v;
    }
    if (tid == 0) counters[blockIdx.x] = 0;
}

void moe_launch_router_logits(const float *Wr, const float *x, int T, int H, int E, float *part, int n_split,
                              float *logits, int *counters, cudaStream_t s, uint64_t *launches) {
    dim3 grid((E + 31) / 32, n_split);
    const size_t smem = sizeof(float) * (32 * RL_WPAD + RL_KS * 64);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_router_logits, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = true;
    }
    k_router_logits<<<grid, 256, smem, s>>>(Wr, x, T, H, E, part, logits, counters);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// Activation operands
// ===========================================================================
// Copies a row of n floats (n % 4 == 0, 16-byte aligned) to shared memory
// with up to 8 float4 loads in flight per thread, then syncs the block.
__device__ __forceinline__ void stage_row(const float *__restrict__ x, int n, float *__restrict__ xs) {
    const float4 *src = reinterpret_cast<const float4 *>(x);
    float4 *dst = reinterpret_cast<float4 *>(xs);
    const int n4 = n / 4, step = blockDim.x;
    for (int base = 0; base < n4; base += 8 * step) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = base + u * step + threadIdx.x;
            if (i < n4) v[u] = __ldg(src + i);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = base + u * step + threadIdx.x;
            if (i < n4) dst[i] = v[u];
        }
    }
    __syncthreads();
}

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

// power-of-two scale s with max|x| * s in [2^(top-1), 2^top); returns s, sets
// *inv = 1/s.  top = 10 for the fp16 operand (sub-block sums stay below
// 65504), 20 for the int8-plane operand (|x * s| < 2^20).
__device__ __forceinline__ float op_scale(float amax, float *inv, int top = 10) {
    if (!(amax > 0.0f) || !isfinite(amax)) { *inv = 1.0f; return 1.0f; }
    int ex;
    frexpf(amax, &ex);  // amax = m 2^ex, m in [0.5, 1)
    int e = top - ex;
    if (e > 120) e = 120;
    if (e < -120) e = -120;
    *inv = ldexpf(1.0f, -e);
    return ldexpf(1.0f, e);
}

__device__ __forceinline__ void split_hl(float v, __half &hi, __half &lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
}

// Q4_K operand of one K-vector (all threads of the block).  xsum: smem
// scratch of K/32 floats for the sub-block sums.
__device__ void build_q4op(const float *__restrict__ x, int K, float s, __half *__restrict__ op,
                           float *__restrict__ xsum) {
    const int NB = K / MOE_QK;
    for (int sub = threadIdx.x; sub < K / 32; sub += blockDim.x) {
        float acc = 0.0f;
        for (int i = 0; i < 32; i++) {
            __half hi, lo;
            split_hl(__fmul_rn(x[32 * sub + i], s), hi, lo);
            acc = __fadd_rn(acc, __fadd_rn(__half2float(hi), __half2float(lo)));
        }
        xsum[sub] = acc;
    }
    __syncthreads();
    const __half z = __float2half_rn(0.0f);
    for (int ent = threadIdx.x; ent < NB * 4 * Q4OP_STEPS; ent += blockDim.x) {
        const int sb = ent / (4 * Q4OP_STEPS), t = (ent / Q4OP_STEPS) % 4, m = ent % Q4OP_STEPS;
        __half *o = op + (size_t)sb * Q4OP_HALVES_PER_SB + t * Q4OP_LANE_HALVES + m * 4;  // part 0 (hi)
        __half *o1 = o + 4 * Q4OP_LANE_HALVES;                                                // part 1 (lo)
        const float *xb = x + sb * MOE_QK;
        if (m < 16) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                __half hi, lo;
                split_hl(__fmul_rn(xb[q4k_k(m, t, j)], s), hi, lo);
                o[j] = hi;
                o1[j] = lo;
            }
        } else if (m == 16) {
            const int sa = q4k_min_sub(t);
#pragma unroll
            for (int u = 0; u < 2; u++) {
                __half hi, lo;
                split_hl(xsum[sb * 8 + sa + u], hi, lo);
                o[u] = hi;
                o1[u] = lo;
            }
            o[2] = o[3] = o1[2] = o1[3] = z;
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) o[j] = o1[j] = z;
        }
    }
}

// Q6_K operand: 21-bit fixed point x * 2^e split into three int8 planes.
__device__ void build_q6i(const float *__restrict__ x, int K, float s, int8_t *__restrict__ op) {
    const int NB = K / MOE_QK;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const int v = __float2int_rn(__fmul_rn(x[k], s));  // |v| <= 2^20
        const int sb = k / MOE_QK, w = k % MOE_QK, st = w / 16, t = (w / 4) % 4, i = w % 4;
        const size_t off = ((size_t)sb * 4 + t) * 64 + st * 4 + i;
        op[off] = (int8_t)(v & 127);
        op[(size_t)NB * Q6I_BYTES_PER_SB + off] = (int8_t)((v >> 7) & 127);
        op[(size_t)2 * NB * Q6I_BYTES_PER_SB + off] = (int8_t)(v >> 14);
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
    const float *logit_bias;               // added to the logits before the sigmoid (or nullptr)
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
    // exclusive scans of the pair counts and chunk counts over experts
    __shared__ int wsum[3][32], carry[3];
    if (threadIdx.x == 0) carry[0] = carry[1] = carry[2] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    for (int base = 0; base < NE; base += blockDim.x) {
        const int e = base + threadIdx.x;
        int v[3] = {0, 0, 0};
        if (e < NE) {
            v[0] = cnt[e];
            v[1] = (cnt[e] + MOE_TC - 1) / MOE_TC;
            v[2] = (e < E && cnt[e] > 0) ? 1 : 0;
        }
        int inc[3];
#pragma unroll
        for (int q = 0; q < 3; q++) {
            int x = v[q];
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            inc[q] = x;
            if (lane == 31) wsum[q][wid] = x;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
#pragma unroll
            for (int q = 0; q < 3; q++) {
                int x = threadIdx.x < nwarp ? wsum[q][threadIdx.x] : 0;
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, x, o);
                    if (threadIdx.x >= o) x += y;
                }
                if (threadIdx.x < nwarp) wsum[q][threadIdx.x] = x;  // inclusive warp totals
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
        off[NE] = carry[0];
        coff[NE] = carry[1];
        a.plan.counts[0] = carry[0];
        a.plan.counts[1] = carry[1];
        a.plan.counts[2] = carry[2];
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
    __shared__ float xsum[1024];  // sub-block sums of the operand (H <= 32768)
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
            if (a.logit_bias) lg += a.logit_bias[e];
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
            // replace the first minimum slot when strictly greater.  The K
            // slots stay in registers (fully unrolled over MOE_MAX_K).
            float key[MOE_MAX_K];
            int idx[MOE_MAX_K];
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; k++) { key[k] = -1e30f; idx[k] = 0; }
            int mk = 0;
            float mkey = -1e30f;
            for (int g = 0; g < G; g++) {
                if (!((taken >> g) & 1ull)) continue;
                for (int e = g * per; e < (g + 1) * per; e++) {
                    const float c = choice[e];
                    if (c > mkey) {
#pragma unroll
                        for (int k = 0; k < MOE_MAX_K; k++)
                            if (k == mk) { key[k] = c; idx[k] = e; }
                        mk = 0;
                        mkey = key[0];
#pragma unroll
                        for (int k = 1; k < MOE_MAX_K; k++)
                            if (k < K && key[k] < mkey) { mkey = key[k]; mk = k; }
                    }
                }
            }
            float w[MOE_MAX_K], s = 0.0f;
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; k++)
                if (k < K) { w[k] = score[idx[k]]; s += w[k]; }
            const float f = s > 0.0f ? a.d.scale / s : 1.0f;
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; k++)
                if (k < K) {
                    a.idx_out[t * K + k] = idx[k];
                    a.w_out[t * K + k] = s > 0.0f ? w[k] * f : w[k];
                }
        }
    } else if (a.mode == 1 && threadIdx.x < K) {
        a.idx_out[t * K + threadIdx.x] = a.idx_in[t * K + threadIdx.x];
        a.w_out[t * K + threadIdx.x] = a.w_in[t * K + threadIdx.x];
    }

    // activation operand of this token for the gate/up GEMV
    if (a.xop) {
        extern __shared__ float xrow[];  // [H]
        stage_row(a.x + (size_t)t * a.d.H, a.d.H, xrow);
        const float *xr = xrow;
        const float amax = block_max_abs(xr, a.d.H, red);
        float inv;
        const float s = op_scale(amax, &inv);
        build_q4op(xr, a.d.H, s, a.xop + (size_t)t * q4op_halves(a.d.H), xsum);
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
                               const float *bias, const float *logit_bias, int mode, const int *idx_in, const float *w_in, int T,
                               int *idx_out, float *w_out, const float *x, __half *xop, float *x_inv,
                               int include_shared, int build_plan, const MoePlan &plan, int *counter,
                               cudaStream_t s, uint64_t *launches) {
    RouteArgs a;
    a.d = d; a.part = part; a.n_split = n_split; a.logits = logits; a.bias = bias; a.logit_bias = logit_bias;
    a.idx_in = idx_in; a.w_in = w_in; a.mode = mode; a.T = T; a.idx_out = idx_out; a.w_out = w_out;
    a.x = x; a.xop = xop; a.x_inv = x_inv; a.include_shared = include_shared; a.build_plan = build_plan;
    a.plan = plan; a.counter = counter;
    const size_t smem = xop ? sizeof(float) * (size_t)d.H : 0;
    static size_t attr = 0;
    if (smem > attr) {
        cudaFuncSetAttribute(k_route_plan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = smem;
    }
    k_route_plan<<<T, 256, smem, s>>>(a);
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

// Scales of the four sub-blocks lane t decodes (u = 2r + hi -> sub-block
// 4r + 2(t/2) + hi, quant.c:26-34) as half2 pairs, with the magic offsets of
// the low-nibble (1024) and high-nibble (64) decodes; m2 = the two minimums
// lane t supplies to the min-term MMA.
__device__ __forceinline__ void q4_decode_hdr(const uint4 h, int t, Q4Hdr &o) {
    const int q = t >> 1;
    o.d = h2f_bits((uint16_t)(h.x & 0xFFFFu));
    o.dmin = h2f_bits((uint16_t)(h.x >> 16));
    const uint32_t a0 = h.y >> (16 * q), a1 = h.z >> (16 * q), a2 = h.w >> (16 * q);
    const uint32_t sc_lo = a0 & 0x3F3Fu, m_lo = a1 & 0x3F3Fu;
    const uint32_t sc_hi = (a2 & 0x0F0Fu) | ((a0 >> 2) & 0x3030u);
    const uint32_t m_hi = ((a2 >> 4) & 0x0F0Fu) | ((a1 >> 2) & 0x3030u);
    const __half2 k1024 = __float2half2_rn(1024.0f), km1024 = __float2half2_rn(-1024.0f),
                  km64 = __float2half2_rn(-64.0f);
    o.sc[0] = __hsub2(u32_as_h2(__byte_perm(sc_lo, 0x6464u, 0x4040u)), k1024);
    o.sc[1] = __hsub2(u32_as_h2(__byte_perm(sc_lo, 0x6464u, 0x4141u)), k1024);
    o.sc[2] = __hsub2(u32_as_h2(__byte_perm(sc_hi, 0x6464u, 0x4040u)), k1024);
    o.sc[3] = __hsub2(u32_as_h2(__byte_perm(sc_hi, 0x6464u, 0x4141u)), k1024);
    o.nsc[0] = __hmul2(o.sc[0], km1024);
    o.nsc[1] = __hmul2(o.sc[1], km64);
    o.nsc[2] = __hmul2(o.sc[2], km1024);
    o.nsc[3] = __hmul2(o.sc[3], km64);
    const uint32_t mw = (t & 1) ? m_hi : m_lo;
    o.m2 = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(mw, 0x6464u, 0x4140u)), k1024));
}

// sc*q (exact fp16) of the low nibbles at bits [0,4) and [16,20) of w: the
// half with bits 0x6400 | q is 1024 + q.
__device__ __forceinline__ uint32_t q4_dq_lo(uint32_t w, __half2 sc, __half2 nsc1024) {
    return h2_as_u32(__hfma2(u32_as_h2((w & 0x000F000Fu) | 0x64006400u), sc, nsc1024));
}
// ... of the high nibbles at bits [4,8) and [20,24) without a shift: the
// half with bits 0x5400 | (q << 4) is 64 + q.
__device__ __forceinline__ uint32_t q4_dq_hi(uint32_t w, __half2 sc, __half2 nsc64) {
    return h2_as_u32(__hfma2(u32_as_h2((w & 0x00F000F0u) | 0x54005400u), sc, nsc64));
}

// raw bytes of one Q4_K super-block for rows g and g+8 of one lane
struct Q4Raw {
    uint4 hg, hg8, qg[2], qg8[2];
};

// ring slot of a lane: word k of stage `slot` at wsm[(slot * W + k) * 32 + lane]
__device__ __forceinline__ void q4_issue(uint4 *wsm, int slot, int lane, const uint8_t *__restrict__ rg,
                                         const uint8_t *__restrict__ rg8, int sb, int t) {
    const uint8_t *bg = rg + (size_t)sb * MOE_Q4K_BYTES, *bg8 = rg8 + (size_t)sb * MOE_Q4K_BYTES;
    uint4 *w = wsm + slot * MOE_Q4_WORDS * 32 + lane;
    cp_async16(w + 0 * 32, bg);
    cp_async16(w + 1 * 32, bg8);
    cp_async16(w + 2 * 32, bg + 16 + 16 * t);
    cp_async16(w + 3 * 32, bg + 80 + 16 * t);
    cp_async16(w + 4 * 32, bg8 + 16 + 16 * t);
    cp_async16(w + 5 * 32, bg8 + 80 + 16 * t);
}

__device__ __forceinline__ void q4_read(Q4Raw &r, const uint4 *wsm, int slot, int lane) {
    const uint4 *w = wsm + slot * MOE_Q4_WORDS * 32 + lane;
    r.hg = w[0];
    r.hg8 = w[32];
    r.qg[0] = w[64];
    r.qg[1] = w[96];
    r.qg8[0] = w[128];
    r.qg8[1] = w[160];
}

__device__ __forceinline__ uint32_t u4c(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// One Q4_K super-block of rows (g, g+8) against NT 8-column tiles (4 vectors
// x {hi, lo}).  opb[n] points at this lane's fragment stream of tile n (a
// zero stream for empty columns).
template <int NT>
__device__ __forceinline__ void q4_compute(const Q4Raw &R, int sb, const __half *const (&opb)[NT],
                                           float (&acc)[NT][2], int t) {
    Q4Hdr Hg, Hg8;
    q4_decode_hdr(R.hg, t, Hg);
    q4_decode_hdr(R.hg8, t, Hg8);
    float p1[NT][4], p2[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++)
#pragma unroll
        for (int c = 0; c < 4; c++) p1[n][c] = 0.0f;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        uint4 B[NT][4];  // steps 8r .. 8r+7 of this lane: 64 bytes
#pragma unroll
        for (int n = 0; n < NT; n++) {
            const uint4 *bp = reinterpret_cast<const uint4 *>(opb[n] + (size_t)sb * Q4OP_HALVES_PER_SB + r * 32);
#pragma unroll
            for (int q = 0; q < 4; q++) B[n][q] = ldg_op16(bp + q);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t wg = u4c(R.qg[r], i), wg8 = u4c(R.qg8[r], i);
            const uint32_t wg_s = wg >> 8, wg8_s = wg8 >> 8;
            const int ul = 2 * r, uh = 2 * r + 1;
            // low nibbles (step 2i) then high nibbles (step 2i + 1)
            const uint32_t l0 = q4_dq_lo(wg, Hg.sc[ul], Hg.nsc[ul]), l2 = q4_dq_lo(wg_s, Hg.sc[ul], Hg.nsc[ul]);
            const uint32_t l1 = q4_dq_lo(wg8, Hg8.sc[ul], Hg8.nsc[ul]), l3 = q4_dq_lo(wg8_s, Hg8.sc[ul], Hg8.nsc[ul]);
            const uint32_t h0 = q4_dq_hi(wg, Hg.sc[uh], Hg.nsc[uh]), h2 = q4_dq_hi(wg_s, Hg.sc[uh], Hg.nsc[uh]);
            const uint32_t h1 = q4_dq_hi(wg8, Hg8.sc[uh], Hg8.nsc[uh]), h3 = q4_dq_hi(wg8_s, Hg8.sc[uh], Hg8.nsc[uh]);
#pragma unroll
            for (int n = 0; n < NT; n++) {
                const uint4 &b = B[n][i];
                mma_f16_16816(p1[n], l0, l1, l2, l3, b.x, b.y, p1[n][0], p1[n][1], p1[n][2], p1[n][3]);
                mma_f16_16816(p1[n], h0, h1, h2, h3, b.z, b.w, p1[n][0], p1[n][1], p1[n][2], p1[n][3]);
            }
        }
    }
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const uint4 b = ldg_op16(opb[n] + (size_t)sb * Q4OP_HALVES_PER_SB + 64);  // steps 16 (min) and 17 (pad)
        mma_f16_16816(p2[n], Hg.m2, Hg8.m2, 0u, 0u, b.x, b.y, 0.f, 0.f, 0.f, 0.f);
        acc[n][0] = fmaf(Hg.d, p1[n][0] + p1[n][1], fmaf(-Hg.dmin, p2[n][0] + p2[n][1], acc[n][0]));
        acc[n][1] = fmaf(Hg8.d, p1[n][2] + p1[n][3], fmaf(-Hg8.dmin, p2[n][2] + p2[n][3], acc[n][1]));
    }
}

// Per-lane cp.async pipeline: MOE_STAGES - 1 super-blocks in flight while
// the current one is decoded.  wsm = this warp's ring [MOE_STAGES][6][32].
template <int NT>
__device__ __forceinline__ void q4k_warp_rows(const uint8_t *__restrict__ rg, const uint8_t *__restrict__ rg8,
                                              int sb0, int sb1, const __half *const (&opb)[NT],
                                              float (&acc)[NT][2], int t, int lane, uint4 *wsm) {
#pragma unroll
    for (int s = 0; s < MOE_STAGES - 1; s++) {
        if (sb0 + s < sb1) q4_issue(wsm, s, lane, rg, rg8, sb0 + s, t);
        cp_async_commit();
    }
    int slot = 0, nslot = MOE_STAGES - 1;
#pragma unroll 1
    for (int sb = sb0; sb < sb1; ++sb) {
        if (sb + MOE_STAGES - 1 < sb1) q4_issue(wsm, nslot, lane, rg, rg8, sb + MOE_STAGES - 1, t);
        cp_async_commit();
        cp_async_wait<MOE_STAGES - 1>();
        Q4Raw R;
        q4_read(R, wsm, slot, lane);
        q4_compute<NT>(R, sb, opb, acc, t);
        slot = (slot + 1 == MOE_STAGES) ? 0 : slot + 1;
        nslot = (nslot + 1 == MOE_STAGES) ? 0 : nslot + 1;
    }
    cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Q6_K (repacked planes) against the int8-plane operand.  Per 16-weight
// sub-block s: A = q6 as u8 (nibble | 2 high bits << 4, exact), one u8 x s8
// MMA for sum q6*x and one s8 x s8 MMA with A = -32 everywhere for -32*sum x,
// both into the same int32 tile; flushed as acc += sc_s * D (exact int32).
// At the end of each super-block acc_f += d * acc (fp32).
// ---------------------------------------------------------------------------
struct Q6Raw {
    uint4 ug[3], ug8[3], sg, sg8;
};

__device__ __forceinline__ void q6_issue(uint4 *wsm, int slot, int lane, const uint8_t *__restrict__ qpl,
                                         const uint8_t *__restrict__ spl, int nb, int row_g, int sb, int t) {
    const uint8_t *qg = qpl + ((size_t)row_g * nb + sb) * 192 + 48 * t;
    const uint8_t *qg8 = qpl + ((size_t)(row_g + 8) * nb + sb) * 192 + 48 * t;
    uint4 *w = wsm + slot * MOE_Q6_WORDS * 32 + lane;
#pragma unroll
    for (int v = 0; v < 3; v++) {
        cp_async16(w + v * 32, qg + 16 * v);
        cp_async16(w + (3 + v) * 32, qg8 + 16 * v);
    }
    cp_async16(w + 6 * 32, spl + ((size_t)row_g * nb + sb) * 16);
    cp_async16(w + 7 * 32, spl + ((size_t)(row_g + 8) * nb + sb) * 16);
}

__device__ __forceinline__ void q6_read(Q6Raw &r, const uint4 *wsm, int slot, int lane) {
    const uint4 *w = wsm + slot * MOE_Q6_WORDS * 32 + lane;
#pragma unroll
    for (int v = 0; v < 3; v++) {
        r.ug[v] = w[v * 32];
        r.ug8[v] = w[(3 + v) * 32];
    }
    r.sg = w[6 * 32];
    r.sg8 = w[7 * 32];
}

// u8 q6 values (one byte per weight) of sub-block sp of a half: nibble word W,
// qh word Hw (bit pair sp/2 of every byte)
template <int SP>
__device__ __forceinline__ uint32_t q6_a(uint32_t W, uint32_t Hw) {
    const uint32_t nib = SP < 4 ? (W & 0x0F0F0F0Fu) : ((W >> 4) & 0x0F0F0F0Fu);
    const int f = SP >> 1;
    const uint32_t hs = f == 0 ? (Hw << 4) : f == 1 ? (Hw << 2) : f == 2 ? Hw : (Hw >> 2);
    return nib | (hs & 0x30303030u);
}

template <int NT>
__device__ __forceinline__ void q6i_compute(const Q6Raw &R, int sb, const int8_t *const (&opb)[NT],
                                            int (&acc)[NT][4]) {
    const uint32_t wg[2][6] = {{R.ug[0].x, R.ug[0].y, R.ug[0].z, R.ug[0].w, R.ug[1].x, R.ug[1].y},
                               {R.ug[1].z, R.ug[1].w, R.ug[2].x, R.ug[2].y, R.ug[2].z, R.ug[2].w}};
    const uint32_t wg8[2][6] = {{R.ug8[0].x, R.ug8[0].y, R.ug8[0].z, R.ug8[0].w, R.ug8[1].x, R.ug8[1].y},
                                {R.ug8[1].z, R.ug8[1].w, R.ug8[2].x, R.ug8[2].y, R.ug8[2].z, R.ug8[2].w}};
    const uint32_t sgw[4] = {R.sg.x, R.sg.y, R.sg.z, R.sg.w}, sg8w[4] = {R.sg8.x, R.sg8.y, R.sg8.z, R.sg8.w};
    const uint32_t NEG32 = 0xE0E0E0E0u;
    uint4 Bq[NT];  // fragments of the current quarter; the next quarter's are loaded one quarter ahead
#pragma unroll
    for (int n = 0; n < NT; n++) Bq[n] = ldg_op16(opb[n] + (size_t)sb * Q6I_BYTES_PER_SB);
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int qd = 0; qd < 2; qd++) {  // quarter: steps 8h + 4qd .. +3
            uint4 B[NT], Bn[NT];
#pragma unroll
            for (int n = 0; n < NT; n++) {
                B[n] = Bq[n];
                if (2 * h + qd < 3) Bn[n] = ldg_op16(opb[n] + (size_t)sb * Q6I_BYTES_PER_SB + (2 * h + qd + 1) * 16);
            }
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int sp = 4 * qd + j, s = 8 * h + sp;
                uint32_t a0, a1;
#define Q6A(SPV)                                                   \
    a0 = q6_a<SPV>(wg[h][(SPV)&3], wg[h][4 + ((SPV)&1)]);          \
    a1 = q6_a<SPV>(wg8[h][(SPV)&3], wg8[h][4 + ((SPV)&1)]);
                switch (sp) {
                    case 0: Q6A(0) break;
                    case 1: Q6A(1) break;
                    case 2: Q6A(2) break;
                    case 3: Q6A(3) break;
                    case 4: Q6A(4) break;
                    case 5: Q6A(5) break;
                    case 6: Q6A(6) break;
                    default: Q6A(7) break;
                }
#undef Q6A
                int scg, scg8;
                switch (s & 3) {
                    case 0: scg = sext_byte<0>(sgw[s >> 2]); scg8 = sext_byte<0>(sg8w[s >> 2]); break;
                    case 1: scg = sext_byte<1>(sgw[s >> 2]); scg8 = sext_byte<1>(sg8w[s >> 2]); break;
                    case 2: scg = sext_byte<2>(sgw[s >> 2]); scg8 = sext_byte<2>(sg8w[s >> 2]); break;
                    default: scg = sext_byte<3>(sgw[s >> 2]); scg8 = sext_byte<3>(sg8w[s >> 2]); break;
                }
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    const uint32_t b = u4c(B[n], j);
                    int dd[4];
                    mma_u8s8_16816(dd, a0, a1, b, 0, 0, 0, 0);
                    mma_s8s8_16816(dd, NEG32, NEG32, b, dd[0], dd[1], dd[2], dd[3]);
                    acc[n][0] += scg * dd[0];
                    acc[n][1] += scg * dd[1];
                    acc[n][2] += scg8 * dd[2];
                    acc[n][3] += scg8 * dd[3];
                }
            }
#pragma unroll
            for (int n = 0; n < NT; n++)
                if (2 * h + qd < 3) Bq[n] = Bn[n];
        }
    }
}

template <int NT>
__device__ __forceinline__ void q6k_warp_rows(const uint8_t *__restrict__ W, int rows, int nb, int row_g,
                                              const int8_t *const (&opb)[NT], float (&accf)[NT][4], int t,
                                              int lane, uint4 *wsm) {
    const int nbp = q6r_nb_pad(nb);
    const uint8_t *qpl = W, *spl = W + q6r_plane_s_off(rows, nb);
    const uint16_t *dpl = reinterpret_cast<const uint16_t *>(W + q6r_plane_d_off(rows, nb));
#pragma unroll
    for (int s = 0; s < MOE_STAGES - 1; s++) {
        if (s < nb) q6_issue(wsm, s, lane, qpl, spl, nb, row_g, s, t);
        cp_async_commit();
    }
    // d of the first 8 super-blocks of both rows in one 16-byte load each
    const uint4 dv = __ldg(reinterpret_cast<const uint4 *>(dpl + (size_t)row_g * nbp));
    const uint4 dv8 = __ldg(reinterpret_cast<const uint4 *>(dpl + (size_t)(row_g + 8) * nbp));
    int slot = 0, nslot = MOE_STAGES - 1;
#pragma unroll 1
    for (int sb = 0; sb < nb; ++sb) {
        if (sb + MOE_STAGES - 1 < nb) q6_issue(wsm, nslot, lane, qpl, spl, nb, row_g, sb + MOE_STAGES - 1, t);
        cp_async_commit();
        float dg, dg8;
        if (sb < 8) {
            const uint32_t w = u4c(dv, sb >> 1), w8 = u4c(dv8, sb >> 1);
            dg = h2f_bits((uint16_t)((sb & 1) ? (w >> 16) : (w & 0xFFFFu)));
            dg8 = h2f_bits((uint16_t)((sb & 1) ? (w8 >> 16) : (w8 & 0xFFFFu)));
        } else {
            dg = h2f_bits(__ldg(dpl + (size_t)row_g * nbp + sb));
            dg8 = h2f_bits(__ldg(dpl + (size_t)(row_g + 8) * nbp + sb));
        }
        cp_async_wait<MOE_STAGES - 1>();
        Q6Raw R;
        q6_read(R, wsm, slot, lane);
        int acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0;
        q6i_compute<NT>(R, sb, opb, acc);
#pragma unroll
        for (int n = 0; n < NT; n++) {
            accf[n][0] = fmaf(dg, (float)acc[n][0], accf[n][0]);
            accf[n][1] = fmaf(dg, (float)acc[n][1], accf[n][1]);
            accf[n][2] = fmaf(dg8, (float)acc[n][2], accf[n][2]);
            accf[n][3] = fmaf(dg8, (float)acc[n][3], accf[n][3]);
        }
        slot = (slot + 1 == MOE_STAGES) ? 0 : slot + 1;
        nslot = (nslot + 1 == MOE_STAGES) ? 0 : nslot + 1;
    }
    cp_async_wait<0>();
}

__device__ __forceinline__ int expert_slot(const MoeLayerDev &L, int E, int e) {
    return e == E ? L.n_local : e - L.e0;
}

// ===========================================================================
// gate/up: CTA item = (chunk, 64 rows); warp w: row tile w&3, K half w>>2.
// act[pair][row] = silu(gate) * up  (infer.m:378-383)
// ===========================================================================
template <int NT>
__device__ __forceinline__ void gateup_item(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan,
                                            const __half *__restrict__ xop, const __half *__restrict__ zop, int e,
                                            int p0, int ntok, int rgi, int rt, int kh, int g, int t, int lane,
                                            uint4 *wsm, float (*red)[2][MOE_ROWS_GU][MOE_TC + 1]) {
    const int NB = d.H / MOE_QK, nbh = NB / 2;
    const int sb0 = kh ? nbh : 0, sb1 = kh ? NB : nbh;
    const size_t rowb = (size_t)NB * MOE_Q4K_BYTES;
    const size_t opstride = q4op_halves(d.H);
    const uint8_t *ex = L.experts + (size_t)expert_slot(L, d.E, e) * L.expert_stride;
    const int r0 = rgi * MOE_ROWS_GU + rt * 16;
    const int lane_off = (g & 1) * 4 * Q4OP_LANE_HALVES + t * Q4OP_LANE_HALVES;
    const __half *opb[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int tk = 4 * n + (g >> 1);
        opb[n] = (tk < ntok ? xop + (size_t)plan.pair_token[p0 + tk] * opstride : zop) + lane_off;
    }
#pragma unroll 1
    for (int mat = 0; mat < 2; mat++) {
        const uint8_t *Wm = ex + (size_t)mat * L.gate_bytes;
        float acc[NT][2];
#pragma unroll
        for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = 0.0f;
        q4k_warp_rows<NT>(Wm + (size_t)(r0 + g) * rowb, Wm + (size_t)(r0 + g + 8) * rowb, sb0, sb1, opb, acc, t,
                          lane, wsm);
#pragma unroll
        for (int n = 0; n < NT; n++) {
            red[kh][mat][rt * 16 + g][4 * n + t] = acc[n][0];
            red[kh][mat][rt * 16 + g + 8][4 * n + t] = acc[n][1];
        }
    }
}

__global__ void __launch_bounds__(256, 2) k_gateup(MoeDims d, MoeLayerDev L, MoePlan plan,
                                                   const __half *__restrict__ xop, const __half *__restrict__ zop,
                                                   const float *__restrict__ x_inv, float *__restrict__ act) {
    __shared__ float red[2][2][MOE_ROWS_GU][MOE_TC + 1];
    extern __shared__ uint4 ring[];  // [8 warps][MOE_STAGES][6][32]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    uint4 *wsm = ring + (size_t)warp * MOE_STAGES * MOE_Q4_WORDS * 32;
    const int rt = warp & 3, kh = warp >> 2;
    const int n_chunks = plan.counts[1];
    const int n_rg = d.I / MOE_ROWS_GU;
    const int n_items = n_chunks * n_rg;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int rgi = item / n_chunks, c = item % n_chunks;
        const int e = plan.chunk_expert[c], p0 = plan.chunk_pair0[c], ntok = plan.chunk_ntok[c];
        if (ntok <= 4) gateup_item<1>(d, L, plan, xop, zop, e, p0, ntok, rgi, rt, kh, g, t, lane, wsm, red);
        else gateup_item<2>(d, L, plan, xop, zop, e, p0, ntok, rgi, rt, kh, g, t, lane, wsm, red);
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
                       const __half *zop, const float *x_inv, float *act, int max_items, cudaStream_t s,
                       uint64_t *launches) {
    int grid = num_sms() * 2;
    if (grid > max_items) grid = max_items;
    if (grid < 1) grid = 1;
    const size_t smem = sizeof(uint4) * 8 * MOE_STAGES * MOE_Q4_WORDS * 32;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = true;
    }
    k_gateup<<<grid, 256, smem, s>>>(d, L, plan, xop, zop, x_inv, act);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// down operand: per pair, scale + operand of the expert's down type
// ===========================================================================
__global__ void __launch_bounds__(256) k_prep_down(MoeDims d, MoeLayerDev L, MoePlan plan,
                                                   const float *__restrict__ act, uint8_t *__restrict__ dop,
                                                   float *__restrict__ d_inv) {
    __shared__ float red[32];
    __shared__ float xsum[1024];
    const int n_pairs = plan.counts[0];
    const size_t opst = dop_bytes(d.I);
    extern __shared__ float arow[];  // [I]
    for (int p = blockIdx.x; p < n_pairs; p += gridDim.x) {
        stage_row(act + (size_t)p * d.I, d.I, arow);
        const float *a = arow;
        const float amax = block_max_abs(a, d.I, red);
        const int e = plan.pair_expert[p];
        const int ty = (e == d.E) ? L.sh_down_type : L.down_type;
        float inv;
        if (ty == 14) {
            const float s = op_scale(amax, &inv, 20);
            build_q6i(a, d.I, s, reinterpret_cast<int8_t *>(dop + (size_t)p * opst));
        } else {
            const float s = op_scale(amax, &inv);
            build_q4op(a, d.I, s, reinterpret_cast<__half *>(dop + (size_t)p * opst), xsum);
        }
        if (threadIdx.x == 0) d_inv[p] = inv;
        __syncthreads();
    }
}

// Q4_K operand of activation rows: rows [0, R) come from `recv` (skipped when
// their metadata says the slot is empty), rows [R, R + T) from `local`.
__global__ void __launch_bounds__(256) k_prep_rows(const float *__restrict__ recv, const int *__restrict__ meta,
                                                   int meta_w, int R, const float *__restrict__ local, int H,
                                                   __half *__restrict__ xop, float *__restrict__ x_inv) {
    __shared__ float red[32];
    __shared__ float xsum[1024];
    const int r = blockIdx.x;
    if (r < R && !meta[(size_t)r * meta_w]) return;
    extern __shared__ float xrow[];  // [H]
    stage_row(r < R ? recv + (size_t)r * H : local + (size_t)(r - R) * H, H, xrow);
    const float *x = xrow;
    const float amax = block_max_abs(x, H, red);
    float inv;
    const float s = op_scale(amax, &inv);
    build_q4op(x, H, s, xop + (size_t)r * q4op_halves(H), xsum);
    if (threadIdx.x == 0) x_inv[r] = inv;
}

void moe_launch_prep_rows(const float *recv, const int *meta, int meta_w, int R, const float *local, int T, int H,
                          __half *xop, float *x_inv, cudaStream_t s, uint64_t *launches) {
    const size_t smem = sizeof(float) * (size_t)H;
    static size_t attr = 0;
    if (smem > attr) {
        cudaFuncSetAttribute(k_prep_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = smem;
    }
    k_prep_rows<<<R + T, 256, smem, s>>>(recv, meta, meta_w, R, local, H, xop, x_inv);
    LAUNCH_COUNT(launches);
}

void moe_launch_prep_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const float *act,
                          uint8_t *dop, float *d_inv, int max_pairs, cudaStream_t s, uint64_t *launches) {
    int grid = max_pairs;
    if (grid > num_sms() * 4) grid = num_sms() * 4;
    if (grid < 1) grid = 1;
    const size_t smem = sizeof(float) * (size_t)d.I;
    static size_t attr = 0;
    if (smem > attr) {
        cudaFuncSetAttribute(k_prep_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = smem;
    }
    k_prep_down<<<grid, 256, smem, s>>>(d, L, plan, act, dop, d_inv);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// down: warp task = (chunk, 16 rows of H); eo[pair][row]
// ===========================================================================
// Q6_K: n-tile n holds vectors 2n, 2n+1, three planes each (columns 0-2,
// 3-5; columns 6, 7 empty).  NT = ceil(ntok / 2).
template <int NT>
__device__ __forceinline__ void down_task_q6(const MoeDims &d, const MoeLayerDev &L, const uint8_t *__restrict__ dop,
                                             const uint8_t *__restrict__ zop, const float *__restrict__ d_inv,
                                             float *__restrict__ eo, int e, int p0, int ntok, int rt, int g, int t,
                                             int lane, uint4 *wsm) {
    const int NB = d.I / MOE_QK;
    const size_t opst = dop_bytes(d.I);
    const uint8_t *Wd = L.experts + (size_t)expert_slot(L, d.E, e) * L.expert_stride + 2 * L.gate_bytes;
    const int r0 = rt * 16;
    const int8_t *opb[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int tk = 2 * n + (g >= 3 ? 1 : 0), plane = g % 3;
        const bool ok = g < 6 && tk < ntok;
        const uint8_t *base = ok ? dop + (size_t)(p0 + tk) * opst : zop;
        opb[n] = reinterpret_cast<const int8_t *>(base + (size_t)(ok ? plane : 0) * NB * Q6I_BYTES_PER_SB + t * 64);
    }
    float accf[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) accf[n][0] = accf[n][1] = accf[n][2] = accf[n][3] = 0.0f;
    q6k_warp_rows<NT>(Wd, d.H, NB, r0 + g, opb, accf, t, lane, wsm);
    // combine the planes: column c of tile n = vector 2n + c/3, plane c%3
#pragma unroll
    for (int n = 0; n < NT; n++) {
        float va[2], vb[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {  // rows g (h=0) and g+8 (h=1)
            const float c0 = accf[n][2 * h], c1 = accf[n][2 * h + 1];
            va[h] = t == 0 ? c0 + 128.0f * c1 : (t == 1 ? 16384.0f * c0 : 0.0f);
            vb[h] = t == 1 ? c1 : (t == 2 ? 128.0f * c0 + 16384.0f * c1 : 0.0f);
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {
                va[h] += __shfl_xor_sync(0xffffffffu, va[h], o);
                vb[h] += __shfl_xor_sync(0xffffffffu, vb[h], o);
            }
        }
        if (t < 2) {
            const int tk = 2 * n + t;
            if (tk < ntok) {
                const int pair = p0 + tk;
                const float inv = d_inv[pair];
                eo[(size_t)pair * d.H + r0 + g] = (t == 0 ? va[0] : vb[0]) * inv;
                eo[(size_t)pair * d.H + r0 + g + 8] = (t == 0 ? va[1] : vb[1]) * inv;
            }
        }
    }
}

template <int NT>
__device__ __forceinline__ void down_task_q4(const MoeDims &d, const MoeLayerDev &L, const uint8_t *__restrict__ dop,
                                             const uint8_t *__restrict__ zop, const float *__restrict__ d_inv,
                                             float *__restrict__ eo, int e, int p0, int ntok, int rt, int g, int t,
                                             int lane, uint4 *wsm) {
    const int NB = d.I / MOE_QK;
    const size_t opst = dop_bytes(d.I);
    const uint8_t *Wd = L.experts + (size_t)expert_slot(L, d.E, e) * L.expert_stride + 2 * L.gate_bytes;
    const int r0 = rt * 16;
    const int lane_off = (g & 1) * 4 * Q4OP_LANE_HALVES + t * Q4OP_LANE_HALVES;
    const __half *opb[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int tb = 4 * n + (g >> 1);
        opb[n] = reinterpret_cast<const __half *>(tb < ntok ? dop + (size_t)(p0 + tb) * opst : zop) + lane_off;
    }
    float acc[NT][2];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = 0.0f;
    const size_t rowb = (size_t)NB * MOE_Q4K_BYTES;
    q4k_warp_rows<NT>(Wd + (size_t)(r0 + g) * rowb, Wd + (size_t)(r0 + g + 8) * rowb, 0, NB, opb, acc, t, lane, wsm);
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int tc = 4 * n + t;
        if (tc >= ntok) continue;
        const int pair = p0 + tc;
        const float inv = d_inv[pair];
        eo[(size_t)pair * d.H + r0 + g] = acc[n][0] * inv;
        eo[(size_t)pair * d.H + r0 + g + 8] = acc[n][1] * inv;
    }
}

// One instance per down type; chunks of the other type are skipped.
template <int TY>
__global__ void __launch_bounds__(256, 2) k_down(MoeDims d, MoeLayerDev L, MoePlan plan,
                                                 const uint8_t *__restrict__ dop, const uint8_t *__restrict__ zop,
                                                 const float *__restrict__ d_inv, float *__restrict__ eo) {
    extern __shared__ uint4 ring[];  // [8 warps][MOE_STAGES][words][32]
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    uint4 *wsm = ring + (size_t)(threadIdx.x >> 5) * MOE_STAGES * (TY == 14 ? MOE_Q6_WORDS : MOE_Q4_WORDS) * 32;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nw = gridDim.x * (blockDim.x >> 5);
    const int n_chunks = plan.counts[1];
    const int n_tasks = n_chunks * (d.H / 16);
    for (int task = gw; task < n_tasks; task += nw) {
        const int rt = task / n_chunks, c = task % n_chunks;
        const int e = plan.chunk_expert[c], p0 = plan.chunk_pair0[c], ntok = plan.chunk_ntok[c];
        if (((e == d.E) ? L.sh_down_type : L.down_type) != TY) continue;
        if (TY == 14) {
            // at most 4 vectors per pass (two 8-column tiles); a chunk of more
            // runs a second pass over the same rows (weights then come from L2)
            for (int q0 = 0; q0 < ntok; q0 += 4) {
                const int nq = min(4, ntok - q0);
                if (nq <= 2) down_task_q6<1>(d, L, dop, zop, d_inv, eo, e, p0 + q0, nq, rt, g, t, lane, wsm);
                else down_task_q6<2>(d, L, dop, zop, d_inv, eo, e, p0 + q0, nq, rt, g, t, lane, wsm);
            }
        } else {
            if (ntok <= 4) down_task_q4<1>(d, L, dop, zop, d_inv, eo, e, p0, ntok, rt, g, t, lane, wsm);
            else down_task_q4<2>(d, L, dop, zop, d_inv, eo, e, p0, ntok, rt, g, t, lane, wsm);
        }
    }
}

void moe_launch_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const uint8_t *dop,
                     const uint8_t *zop, const float *d_inv, float *eo, int max_items, cudaStream_t s,
                     uint64_t *launches) {
    int grid = num_sms() * 2;
    const int need = (max_items + 7) / 8;
    if (grid > need) grid = need;
    if (grid < 1) grid = 1;
    const size_t sm6 = sizeof(uint4) * 8 * MOE_STAGES * MOE_Q6_WORDS * 32;
    const size_t sm4 = sizeof(uint4) * 8 * MOE_STAGES * MOE_Q4_WORDS * 32;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_down<14>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm6);
        cudaFuncSetAttribute(k_down<12>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm4);
        attr = true;
    }
    if (L.down_type == 14 || L.sh_down_type == 14) {
        k_down<14><<<grid, 256, sm6, s>>>(d, L, plan, dop, zop, d_inv, eo);
        LAUNCH_COUNT(launches);
    }
    if (L.down_type == 12 || L.sh_down_type == 12) {
        k_down<12><<<grid, 256, sm4, s>>>(d, L, plan, dop, zop, d_inv, eo);
        LAUNCH_COUNT(launches);
    }
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
