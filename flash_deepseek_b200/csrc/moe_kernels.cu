// moe_kernels.cu -- device kernels of the DeepSeek-V3/R1 MoE block for B200.
//
//   router logits   fp32 [T x H] x [H x E], split over H into partial sums
//                   (one CTA per expert over the whole row for <= 4 tokens)
//   route + plan    sigmoid, grouped top-k (infer.m:920-991), dispatch plan,
//                   activation operand of the gate/up GEMV
//   prep_down       activation operand of the down GEMV
//   combine         sum_k w_k eo_k in slot order + shared (infer.m:1915-1922)
//   rmsnorm         the stack's per-layer norm (infer.m:369-374)
//   codec / synth   dequant twins of quant.c, generator + quantizer, repack
// The expert GEMVs themselves (gate/up with the SwiGLU epilogue, down) are in
// moe_experts.cu.
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
            // qh bytes are stored with the high bit of every 2-bit pair
            // inverted: the kernels then decode 4 (q ^ 32), i.e. 4 (q - 32)
            // as int8, with no separate offset term
            const uint8_t flip = sbyte >= 128 ? 0xAA : 0x00;
            if (inverse) g[sbyte] = rq[p] ^ flip; else rq[p] = g[sbyte] ^ flip;
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

// Q4_K: transpose the 4x4 grid of 8-byte qs chunks of every block (its own
// inverse; layout in moe_common.cuh).
__global__ void k_q4_repack(uint8_t *__restrict__ buf, size_t nblocks) {
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
        uint2 *qs = reinterpret_cast<uint2 *>(buf + b * MOE_Q4K_BYTES + 16);
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int t = j + 1; t < 4; t++) {
                const uint2 x = qs[4 * j + t];
                qs[4 * j + t] = qs[4 * t + j];
                qs[4 * t + j] = x;
            }
    }
}

void moe_launch_q4_repack(uint8_t *buf, size_t nblocks, cudaStream_t s, uint64_t *launches) {
    if (!nblocks) return;
    size_t grid = (nblocks + 255) / 256;
    if (grid > (size_t)num_sms() * 16) grid = (size_t)num_sms() * 16;
    k_q4_repack<<<(int)grid, 256, 0, s>>>(buf, nblocks);
    LAUNCH_COUNT(launches);
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
#define RL_MAX_SPLIT 32  // partial sums loaded together by the reducing CTA
__global__ void __launch_bounds__(256) k_router_logits(const float *__restrict__ Wr, const float *__restrict__ x,
                                                       int T_all, int H, int E, float *__restrict__ part,
                                                       float *__restrict__ logits, int *__restrict__ counters) {
    extern __shared__ float sm[];
    float *Ws = sm;                       // [32 experts][RL_WPAD] row-major (k contiguous)
    float *xt = sm + 32 * RL_WPAD;        // [RL_KS][64] (tokens contiguous)
    const int e0 = blockIdx.x * 32, split = blockIdx.y, k0 = split * RL_KS;
    // token chunk z: tokens [64 z, 64 z + T) of T_all
    const int tz0 = blockIdx.z * 64, T = min(64, T_all - tz0);
    x += (size_t)tz0 * H;
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
    // the weight tile above is constant; x comes from the previous kernel
    moe_pdl_wait();
    moe_pdl_trigger();
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
                    if (t < T) part[((size_t)split * T_all + tz0 + t) * E + e] = accs[u][t];
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
        if (t0ok) part[((size_t)split * T_all + tz0 + tg) * E + e] = acc[u][0];
        if (t1ok) part[((size_t)split * T_all + tz0 + tg + 32) * E + e] = acc[u][1];
    }
    }
    // The last split CTA of this expert group sums the partials in split
    // order (deterministic) into the final logits.
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&counters[blockIdx.z * gridDim.x + blockIdx.x], 1) == (int)gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int ns = gridDim.y;
    for (int i = tid; i < T * 32; i += 256) {
        const int t = i / 32, e = e0 + i % 32;
        if (e >= E) continue;
        // all partials in flight at once, then summed in split order
        float pv[RL_MAX_SPLIT];
#pragma unroll
        for (int sp = 0; sp < RL_MAX_SPLIT; sp++)
            pv[sp] = sp < ns ? __ldcg(part + ((size_t)sp * T_all + tz0 + t) * E + e) : 0.0f;
        float v = 0.0f;
#pragma unroll
        for (int sp = 0; sp < RL_MAX_SPLIT; sp++)
            if (sp < ns) v += pv[sp];
        for (int sp = RL_MAX_SPLIT; sp < ns; sp++) v += __ldcg(part + ((size_t)sp * T_all + tz0 + t) * E + e);
        logits[(size_t)(tz0 + t) * E + e] = v;
    }
    if (tid == 0) counters[blockIdx.z * gridDim.x + blockIdx.x] = 0;
}

// Few tokens (T <= RS_MAX_T): one CTA per expert reads the expert's whole
// router row (H fp32, all loads in flight at once) and reduces in a fixed
// order, so there is no second pass over partials.  Same fp32 dot product as
// the reference's sgemv (infer.m:1881) up to summation order.
#define RS_MAX_T MOE_ROUTER_SIMT_T
#define RS_U 8  // float4 loads in flight per thread
__global__ void __launch_bounds__(256) k_router_small(const float *__restrict__ Wr, const float *__restrict__ x, int T,
                                                      int H, int E, float *__restrict__ logits) {
    __shared__ float red[RS_MAX_T][8];
    moe_pdl_wait();
    moe_pdl_trigger();
    const int e = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const float4 *w4 = reinterpret_cast<const float4 *>(Wr + (size_t)e * H);
    float acc[RS_MAX_T] = {0.0f, 0.0f, 0.0f, 0.0f};
    // the row's loads of a thread are issued together (RS_U in flight, one
    // DRAM latency instead of one per load); the products are added in the
    // same order as one load at a time
    const int n4 = H / 4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += RS_U * blockDim.x) {
        float4 w[RS_U];
#pragma unroll
        for (int u = 0; u < RS_U; u++) {
            const int i = i0 + u * blockDim.x;
            w[u] = i < n4 ? __ldg(w4 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < RS_U; u++) {
            const int i = i0 + u * blockDim.x;
            if (i >= n4) break;
#pragma unroll
            for (int t = 0; t < RS_MAX_T; t++) {
                if (t >= T) break;
                const float4 v = __ldg(reinterpret_cast<const float4 *>(x + (size_t)t * H) + i);
                acc[t] = fmaf(w[u].x, v.x, fmaf(w[u].y, v.y, fmaf(w[u].z, v.z, fmaf(w[u].w, v.w, acc[t]))));
            }
        }
    }
#pragma unroll
    for (int t = 0; t < RS_MAX_T; t++) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[t][wid] = v;
    }
    __syncthreads();
    if (threadIdx.x < T) {
        float v = 0.0f;
        for (int w = 0; w < 8; w++) v += red[threadIdx.x][w];
        logits[(size_t)threadIdx.x * E + e] = v;
    }
}

void moe_launch_router_logits(const float *Wr, const float *x, int T, int H, int E, float *part, int n_split,
                              float *logits, int *counters, cudaStream_t s, uint64_t *launches) {
    if (T <= RS_MAX_T && H % 4 == 0) {
        moe_launch_pdl(k_router_small, dim3(E), dim3(256), 0, s, Wr, x, T, H, E, logits);
        LAUNCH_COUNT(launches);
        return;
    }
    dim3 grid((E + 31) / 32, n_split, (T + 63) / 64);
    const size_t smem = sizeof(float) * (32 * RL_WPAD + RL_KS * 64);
    static size_t attr[MOE_MAX_DEVICES];
    moe_smem_limit(k_router_logits, smem, attr);
    moe_launch_pdl(k_router_logits, grid, dim3(256), smem, s, Wr, x, T, H, E, part, logits, counters);
    LAUNCH_COUNT(launches);
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
    const float *x; uint8_t *xop;  // x operand (may be nullptr)
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
        if (e < 0 || e >= E) { atomicExch(a.plan.error, MOE_DEV_ERR_INDEX); continue; }
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
            v[1] = moe_n_chunks(cnt[e], a.d.tc);
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
        const int nc = moe_n_chunks(n, a.d.tc);
        for (int c = 0; c < nc; c++) {
            int start, nt;
            moe_chunk(n, c, a.d.tc, start, nt);
            const int ci = coff[e] + c;
            a.plan.chunk_expert[ci] = e;
            a.plan.chunk_pair0[ci] = off[e] + start;
            a.plan.chunk_ntok[ci] = nt;
        }
    }
    __syncthreads();
    moe_plan_order_chunks(a.plan, coff[NE], a.d.tc);
}

// Top groups of infer.m:944-954 (repeated argmax, the lowest index winning
// ties, only scores above -1e30 counting), with one warp: lane l ranks groups
// l and l + 32 directly -- a group is taken when its score is above -1e30 and
// fewer than TG groups come before it in (score descending, index ascending)
// order, which is the set the repeated argmax takes, in one step instead of
// TG rounds of shuffles.  NaN scores are never taken and rank no group.
__device__ __forceinline__ unsigned long long top_groups_warp(const float *gs, int G, int TG, int lane) {
    unsigned long long taken = 0ull;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int g = lane + 32 * half;
        bool take = false;
        if (g < G) {
            const float v = gs[g];
            int rank = 0;
            for (int h = 0; h < G; h++) {
                const float u = gs[h];
                rank += (u > v || (u == v && h < g)) ? 1 : 0;
            }
            take = v > -1e30f && rank < TG;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, take);
        taken |= (unsigned long long)bal << (32 * half);
    }
    return taken;
}

// order-preserving int key of a non-NaN float: a < b exactly when
// f32_ord(a) < f32_ord(b) (-0.0 below +0.0; the scores here are never -0.0)
__device__ __forceinline__ int f32_ord(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float f32_unord(int o) { return __int_as_float(o >= 0 ? o : o ^ 0x7FFFFFFF); }

// Slot-order top-K of infer.m:966-980 over the experts of the taken groups in
// ascending order: a candidate strictly greater than the current minimum
// replaces the first (lowest) slot holding that minimum.  One warp; lane k < K
// holds slot k.  Candidates are tested 32 at a time with a ballot; only the
// first one above the minimum is inserted before the rest of the batch is
// tested again against the new minimum (the minimum only grows, so earlier
// lanes stay out).  The new minimum is one warp min-reduction of the slots'
// ordered keys, its slot the first lane holding it.  On return every lane
// holds the K slots in key[] / idx[] (slot order).
__device__ __forceinline__ void topk_slots_warp(const float *choice, unsigned long long taken, int G, int per, int K,
                                                int lane, float (&key)[MOE_MAX_K], int (&idx)[MOE_MAX_K]) {
    float sv = lane < K ? -1e30f : 3.0e38f;  // lanes past K never hold the minimum
    int si = 0;
    float mkey = -1e30f;  // the current minimum
    int mk = 0;           // the first slot holding it
    for (int g = 0; g < G; g++) {
        if (!((taken >> g) & 1ull)) continue;
        for (int e0 = g * per; e0 < (g + 1) * per; e0 += 32) {
            const float c = e0 + lane < (g + 1) * per ? choice[e0 + lane] : -1e30f;
            unsigned rem = 0xffffffffu;
            for (;;) {
                const unsigned bal = __ballot_sync(0xffffffffu, c > mkey) & rem;
                if (!bal) break;
                const int f = __ffs(bal) - 1;
                const float cf = __shfl_sync(0xffffffffu, c, f);
                if (lane == mk) { sv = cf; si = e0 + f; }
                const int o = f32_ord(sv);
                const int mn = __reduce_min_sync(0xffffffffu, o);
                mk = __ffs(__ballot_sync(0xffffffffu, o == mn)) - 1;
                mkey = f32_unord(mn);
                rem = f == 31 ? 0u : (0xffffffffu << (f + 1));
            }
        }
    }
#pragma unroll
    for (int k = 0; k < MOE_MAX_K; k++) {
        key[k] = __shfl_sync(0xffffffffu, sv, k);
        idx[k] = __shfl_sync(0xffffffffu, si, k);
    }
}

// The plan of one token, written by warp 0 from its registers (all lanes hold
// the K slots and weights, routed or given): when the K experts are
// distinct, each gets one pair and one chunk of one token, in ascending
// expert order, then the shared expert's pair and chunk -- what
// build_plan_block produces for this input (chunks of equal size may take any
// order in chunk_order).  Returns false, writing nothing, when an expert
// repeats (fewer candidates than slots), which build_plan_block handles.
__device__ __forceinline__ bool plan_one_token(const RouteArgs &a, int lane, const int (&idx)[MOE_MAX_K],
                                               const float (&w)[MOE_MAX_K]) {
    const int K = a.d.K, E = a.d.E;
    int e = 0, rank = 0;
    float wk = 0.0f;
    bool dup = false;
#pragma unroll
    for (int k = 0; k < MOE_MAX_K; k++)
        if (k == lane) { e = idx[k]; wk = w[k]; }
#pragma unroll
    for (int j = 0; j < MOE_MAX_K; j++)
        if (j < K) {
            rank += idx[j] < e ? 1 : 0;
            dup |= j != lane && idx[j] == e;
        }
    if (__any_sync(0xffffffffu, lane < K && (dup || e < 0 || e >= E))) return false;
    const int n = K + (a.include_shared ? 1 : 0);
    const MoePlan &p = a.plan;
    if (lane < K) {
        p.pair_expert[rank] = e;
        p.pair_token[rank] = 0;
        p.pair_w[rank] = wk;
        p.slot_pair[lane] = rank;
        p.chunk_expert[rank] = e;
        p.chunk_pair0[rank] = rank;
        p.chunk_ntok[rank] = 1;
    } else if (lane == K && a.include_shared) {
        p.pair_expert[K] = E;
        p.pair_token[K] = 0;
        p.pair_w[K] = 1.0f;
        p.slot_pair[K] = K;
        p.chunk_expert[K] = E;
        p.chunk_pair0[K] = K;
        p.chunk_ntok[K] = 1;
    }
    if (lane < n) p.chunk_order[lane] = lane;
    // pairs, chunks, routed experts with pairs, tcgen05 chunks (none), the rest 0
    if (lane < MOE_PLAN_COUNTS) p.counts[lane] = lane == 0 ? n : lane == 1 ? n : lane == 2 ? K : 0;
    return true;
}

// The last block of the grid to finish builds the plan for all tokens.  With
// one token the routing block builds it itself, right after routing (no
// grid-wide fence and counter hand-off; usually straight from warp 0's
// registers, plan_one_token); the operand blocks then just leave.
__device__ __forceinline__ void route_plan_finish(const RouteArgs &a, int &is_last, const int &plan_done) {
    if (!a.build_plan) return;
    if (a.T == 1) {
        if (blockIdx.x != 0) return;
        __syncthreads();  // the block's own idx / w stores (and plan_done) are visible to its reads
        if (!plan_done) build_plan_block(a);
        return;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = (atomicAdd(a.counter, 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    build_plan_block(a);
    if (threadIdx.x == 0) *a.counter = 0;
}

// Grid: T routing blocks (one per token), then the operand blocks (one
// super-block of one token per warp).  The last block to finish builds the
// plan.
__global__ void __launch_bounds__(256) k_route_plan(RouteArgs a) {
    __shared__ float score[1024], choice[1024];
    __shared__ float gs[64];
    __shared__ int is_last, plan_done;
    if (threadIdx.x == 0) plan_done = 0;
    moe_pdl_wait();
    moe_pdl_trigger();
    if ((int)blockIdx.x >= a.T) {
        const int nbh = a.d.H / MOE_QK;
        const int item = ((int)blockIdx.x - a.T) * (blockDim.x >> 5) + (threadIdx.x >> 5);
        if (item < a.T * nbh) {
            // both forms of the token's super-block (the expert GEMVs pick one per chunk)
            const int tk = item / nbh, sb = item % nbh;
            const float *xs = a.x + (size_t)tk * a.d.H + (size_t)sb * MOE_QK;
            uint8_t *row = a.xop + (size_t)tk * opx_row(a.d.H);
            build_op_sb(xs, row + (size_t)sb * OPB_SB, 4, threadIdx.x & 31);
            build_opw_sb(xs, row + op_bytes(a.d.H) + (size_t)sb * OPW_SB, 4, threadIdx.x & 31);
        }
        route_plan_finish(a, is_last, plan_done);
        return;
    }
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
        // group score = top1 + top2 (strict '>', infer.m:931-941): the sum of
        // the two largest values of the group, counted with multiplicity
        if (per <= 32) {
            const int lane = threadIdx.x & 31;
            for (int g = threadIdx.x >> 5; g < G; g += blockDim.x >> 5) {
                const float v = lane < per ? choice[g * per + lane] : -1e30f;
                float m1 = v;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
                const unsigned at = __ballot_sync(0xffffffffu, v == m1);
                float m2 = (__popc(at) > 1 || lane != __ffs(at) - 1) ? v : -1e30f;
                if (__popc(at) > 1) m2 = m1;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
                if (per < 2) m2 = -1e30f;
                if (lane == 0) gs[g] = m1 + m2;
            }
        } else {
            for (int g = threadIdx.x; g < G; g += blockDim.x) {
                float t1 = -1e30f, t2 = -1e30f;
                for (int e = 0; e < per; e++) {
                    const float s = choice[g * per + e];
                    if (s > t1) { t2 = t1; t1 = s; }
                    else if (s > t2) t2 = s;
                }
                gs[g] = t1 + t2;
            }
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // top groups, then the slot-order top-K, by warp 0 (all lanes end
            // with the same slots)
            const int lane = threadIdx.x;
            const unsigned long long taken = top_groups_warp(gs, G, TG, lane);
            float key[MOE_MAX_K];
            int idx[MOE_MAX_K];
            topk_slots_warp(choice, taken, G, per, K, lane, key, idx);
            // the routing weights (every lane, the same values; lane 0 stores them)
            float w[MOE_MAX_K], s = 0.0f;
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; k++)
                if (k < K) { w[k] = score[idx[k]]; s += w[k]; }
            const float f = s > 0.0f ? a.d.scale / s : 1.0f;
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; k++)
                if (k < K) w[k] = s > 0.0f ? w[k] * f : w[k];
            if (lane == 0) {
#pragma unroll
                for (int k = 0; k < MOE_MAX_K; k++)
                    if (k < K) {
                        a.idx_out[t * K + k] = idx[k];
                        a.w_out[t * K + k] = w[k];
                    }
            }
            if (a.build_plan && a.T == 1) {
                const bool done = plan_one_token(a, lane, idx, w);
                if (lane == 0) plan_done = done ? 1 : 0;
            }
        }
    } else if (a.mode == 1 && threadIdx.x < 32) {
        // routing given: copied through; with one token warp 0 also writes the plan
        const int lane = threadIdx.x;
        int ie = 0;
        float iw = 0.0f;
        if (lane < K) {
            ie = a.idx_in[t * K + lane];
            iw = a.w_in[t * K + lane];
            a.idx_out[t * K + lane] = ie;
            a.w_out[t * K + lane] = iw;
        }
        if (a.build_plan && a.T == 1) {
            int idx[MOE_MAX_K];
            float w[MOE_MAX_K];
#pragma unroll
            for (int k = 0; k < MOE_MAX_K; k++) {
                idx[k] = __shfl_sync(0xffffffffu, ie, k);
                w[k] = __shfl_sync(0xffffffffu, iw, k);
            }
            const bool done = plan_one_token(a, lane, idx, w);
            if (lane == 0) plan_done = done ? 1 : 0;
        }
    }

    route_plan_finish(a, is_last, plan_done);
}

void moe_launch_route_and_plan(const MoeDims &d, const float *part, int n_split, const float *logits,
                               const float *bias, const float *logit_bias, int mode, const int *idx_in, const float *w_in, int T,
                               int *idx_out, float *w_out, const float *x, uint8_t *xop,
                               int include_shared, int build_plan, const MoePlan &plan, int *counter,
                               cudaStream_t s, uint64_t *launches) {
    RouteArgs a;
    a.d = d; a.part = part; a.n_split = n_split; a.logits = logits; a.bias = bias; a.logit_bias = logit_bias;
    a.idx_in = idx_in; a.w_in = w_in; a.mode = mode; a.T = T; a.idx_out = idx_out; a.w_out = w_out;
    a.x = x; a.xop = xop; a.include_shared = include_shared; a.build_plan = build_plan;
    a.plan = plan; a.counter = counter;
    const int n_op = xop ? (T * (d.H / MOE_QK) + 7) / 8 : 0;
    moe_launch_pdl(k_route_plan, dim3(T + n_op), dim3(256), 0, s, a);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// down operand: per pair, scale + operand of the expert's down type
// ===========================================================================
// The down operand of every pair: the int8 planes, or the fp16 planes when
// the pair's chunk runs on the down GEMV's fp16 path or on the tcgen05
// kernel (chunks of more than MOE_TC tokens).  One super-block of
// one pair per warp; tasks (chunk, pair slot, super-block) are spread over
// the whole grid.  Pair rows are opw_bytes(I) apart (the larger form).
__global__ void __launch_bounds__(256) k_prep_down(MoeDims d, MoeLayerDev L, MoePlan plan,
                                                   const float *__restrict__ act, uint8_t *__restrict__ dop) {
    moe_pdl_wait();
    moe_pdl_trigger();
    const int n_chunks = plan.counts[1];
    const size_t opst = opw_bytes(d.I);
    const int nb = d.I / MOE_QK, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int per_chunk = MOE_CHUNK_MAX * nb, total = n_chunks * per_chunk;
    for (int task = blockIdx.x * nw + (threadIdx.x >> 5); task < total; task += gridDim.x * nw) {
        const int c = task / per_chunk, j = (task / nb) % MOE_CHUNK_MAX, sb = task % nb;
        const int ntok = plan.chunk_ntok[c];
        if (j >= ntok) continue;
        const int e = plan.chunk_expert[c], p = plan.chunk_pair0[c] + j;
        const int style = ((e == d.E) ? L.sh_down_type : L.down_type) == 14 ? 6 : 4;
        const float *x = act + (size_t)p * d.I + (size_t)sb * MOE_QK;
        uint8_t *o = dop + (size_t)p * opst;
        if (moe_dn_wide(ntok)) build_opw_sb(x, o + (size_t)sb * OPW_SB, style, lane);
        else build_op_sb(x, o + (size_t)sb * OPB_SB, style, lane);
    }
}

// Q4_K operand rows (both forms, opx_row(H) apart) of activation rows: rows
// [0, R) come from `recv` (skipped when their metadata says the slot is
// empty), rows [R, R + T) from `local`.
__global__ void __launch_bounds__(256) k_prep_rows(const float *__restrict__ recv, const int *__restrict__ meta,
                                                   int meta_w, int R, const float *__restrict__ local, int H,
                                                   uint8_t *__restrict__ xop) {
    const int r = blockIdx.x;
    if (r < R && !meta[(size_t)r * meta_w]) return;
    uint8_t *row = xop + (size_t)r * opx_row(H);
    build_op_rows(r < R ? recv + (size_t)r * H : local + (size_t)(r - R) * H, H, row, row + op_bytes(H), 4);
}

void moe_launch_prep_rows(const float *recv, const int *meta, int meta_w, int R, const float *local, int T, int H,
                          uint8_t *xop, cudaStream_t s, uint64_t *launches) {
    k_prep_rows<<<R + T, 256, 0, s>>>(recv, meta, meta_w, R, local, H, xop);
    LAUNCH_COUNT(launches);
}

void moe_launch_prep_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const float *act,
                          uint8_t *dop, int max_pairs, cudaStream_t s, uint64_t *launches) {
    // one warp per (chunk, pair slot, super-block) task where the plan can
    // have that many, at most 2 blocks per SM
    long tasks = (long)max_pairs * MOE_CHUNK_MAX * (d.I / MOE_QK);
    int grid = (int)((tasks + 7) / 8);
    if (grid > num_sms() * 2) grid = num_sms() * 2;
    if (grid < 1) grid = 1;
    moe_launch_pdl(k_prep_down, dim3(grid), dim3(256), 0, s, d, L, plan, act, dop);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// combine: out[t] = (sum_k w_k eo_k in slot order) + shared (+ residual)
// ===========================================================================
__global__ void k_combine(MoeDims d, MoePlan plan, const float *__restrict__ eo, int T, int include_routed,
                          int include_shared, const float *__restrict__ residual, float *__restrict__ out) {
    moe_pdl_wait();
    moe_pdl_trigger();
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
    moe_launch_pdl(k_combine, grid, dim3(256), 0, s, d, plan, eo, T, include_routed, include_shared, residual, out);
    LAUNCH_COUNT(launches);
}

// ===========================================================================
// RMSNorm (infer.m:369-374): y = x * (1/sqrtf(mean(x^2) + eps)) * w
// ===========================================================================
__global__ void k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ y, int H,
                          float eps) {
    moe_pdl_wait();
    moe_pdl_trigger();
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
    moe_launch_pdl(k_rmsnorm, dim3(T), dim3(256), 0, s, x, w, y, H, eps);
    LAUNCH_COUNT(launches);
}
