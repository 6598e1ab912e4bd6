// moe_sample.cu -- the next token from the lm_head logits: the reference's
// sample_top_p (infer.m:419-456: temperature softmax, descending sort,
// nucleus cut at top_p, one xorshift32 draw scaled by the nucleus mass, walk)
// and argmax (infer.m:390-394) at temp <= 0.
//
// One CTA per token row.  Instead of sorting the vocabulary, the kernel finds
// the two places where the descending cumulative probability crosses a
// target (top_p, then the draw) by radix selection over the probabilities'
// bit patterns (positive floats order like their bits): four passes of 8-bit
// digits, each a histogram of counts and of 2^40-scaled fixed-point sums
// (integer atomics: the same sums in any order).  Equal probabilities are
// taken in index order, the order a stable sort gives.
#include <math.h>
#include <stdint.h>

#include "moe_common.cuh"
#include "moe_internal.h"

#define LAUNCH_COUNT(p) \
    do {                \
        if (p) (*(p))++; \
    } while (0)

namespace {

constexpr int SP_THREADS = 1024;
constexpr int SP_WARPS = SP_THREADS / 32;
constexpr int SP_HIST = 8;                  // histograms, each shared by 4 warps (fewer atomic conflicts)
constexpr float SP_FIX = 1099511627776.0f;  // 2^40

struct SpShared {
    unsigned int cnt[SP_HIST][256];
    unsigned long long sum[SP_HIST][256];
    float fred[SP_WARPS];
    int ired[SP_WARPS];
    unsigned int wscan[SP_WARPS];
    uint32_t pre, msk, last_cnt;
    unsigned long long above;
};

__device__ __forceinline__ unsigned long long fx(float p) { return __float2ull_rz(p * SP_FIX); }

__device__ __forceinline__ float block_max(float v, SpShared &sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) sh.fred[warp] = v;
    __syncthreads();
    v = sh.fred[0];
    for (int w = 1; w < SP_WARPS; w++) v = fmaxf(v, sh.fred[w]);
    return v;
}

// every thread gets the sum, added in warp order
__device__ __forceinline__ float block_sum(float v, SpShared &sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) sh.fred[warp] = v;
    __syncthreads();
    v = 0.0f;
    for (int w = 0; w < SP_WARPS; w++) v += sh.fred[w];
    return v;
}

// Descending over the probabilities whose key (bit pattern) is in the set
// (all of them, or those above kmin when gt): the key K at which the
// cumulative fixed-point sum first reaches `target` (the smallest key when it
// never does).  Leaves K in sh.pre, the sum over set keys above K in
// sh.above and the count of set keys equal to K in sh.last_cnt.
__device__ void radix_select(const float *__restrict__ p, int n, bool gt, uint32_t kmin,
                             unsigned long long target, SpShared &sh) {
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        sh.pre = 0;
        sh.msk = 0;
        sh.above = 0;
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int k = tid; k < SP_HIST * 256; k += SP_THREADS) {
            (&sh.cnt[0][0])[k] = 0;
            (&sh.sum[0][0])[k] = 0;
        }
        __syncthreads();
        const uint32_t pre = sh.pre, msk = sh.msk;
        for (int i = tid; i < n; i += SP_THREADS) {
            const float v = p[i];
            const uint32_t k = __float_as_uint(v);
            if ((gt && k <= kmin) || (k & msk) != pre) continue;
            const int d = (k >> shift) & 255;
            atomicAdd(&sh.cnt[warp % SP_HIST][d], 1u);
            atomicAdd(&sh.sum[warp % SP_HIST][d], fx(v));
        }
        __syncthreads();
        // fold the histograms into the first
        for (int d = tid; d < 256; d += SP_THREADS) {
            unsigned int c = 0;
            unsigned long long s = 0;
            for (int w = 0; w < SP_HIST; w++) {
                c += sh.cnt[w][d];
                s += sh.sum[w][d];
            }
            sh.cnt[0][d] = c;
            sh.sum[0][d] = s;
        }
        __syncthreads();
        if (tid == 0) {
            unsigned long long acc = sh.above;
            int pick = -1, lowest = -1;
            for (int d = 255; d >= 0; d--) {
                if (!sh.cnt[0][d]) continue;
                lowest = d;
                if (acc + sh.sum[0][d] >= target) {
                    pick = d;
                    break;
                }
                acc += sh.sum[0][d];
            }
            if (pick < 0 && lowest >= 0) {  // target not reached: the smallest key
                pick = lowest;
                acc -= sh.sum[0][lowest];
            }
            if (pick < 0) pick = 0;         // empty set (callers rule it out)
            sh.above = acc;
            sh.pre = pre | ((uint32_t)pick << shift);
            sh.msk = msk | (255u << shift);
            sh.last_cnt = sh.cnt[0][pick];
        }
        __syncthreads();
    }
}

// index of the m-th (1-based) element whose key is K, in index order
__device__ int mth_equal(const float *__restrict__ p, int n, uint32_t K, unsigned int m, SpShared &sh, int *slot) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = (n + SP_THREADS - 1) / SP_THREADS;
    const int lo = min(n, tid * chunk), hi = min(n, lo + chunk);
    unsigned int c = 0;
    for (int i = lo; i < hi; i++) c += __float_as_uint(p[i]) == K;
    unsigned int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) sh.wscan[warp] = incl;
    __syncthreads();
    unsigned int before = incl - c;
    for (int w = 0; w < warp; w++) before += sh.wscan[w];
    if (c && m > before && m <= before + c) {
        unsigned int seen = before;
        for (int i = lo; i < hi; i++)
            if (__float_as_uint(p[i]) == K && ++seen == m) {
                *slot = i;
                break;
            }
    }
    __syncthreads();
    return *slot;
}

__device__ __forceinline__ unsigned int need_count(unsigned long long target, unsigned long long above, float pk,
                                                   unsigned int cap) {
    const unsigned long long f = fx(pk);
    if (target <= above) return 1;
    if (!f) return cap;
    const unsigned long long m = (target - above + f - 1) / f;
    return (unsigned int)max(1ull, min((unsigned long long)cap, m));
}

__global__ void __launch_bounds__(SP_THREADS, 1) k_sample(const float *__restrict__ logits, int V, float temp,
                                                         float top_p, uint32_t rng, float *__restrict__ pbuf,
                                                         int *__restrict__ tokens) {
    __shared__ SpShared sh;
    __shared__ int slot;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *l = logits + (size_t)blockIdx.x * V;
    float *p = pbuf + (size_t)blockIdx.x * V;
    if (tid == 0) slot = V - 1;
    if (!(temp > 0.0f)) {
        // argmax: the first index of the largest logit (infer.m:390-394)
        float bv = l[0];
        int bi = 0;
        for (int i = tid; i < V; i += SP_THREADS)
            if (l[i] > bv) {
                bv = l[i];
                bi = i;
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            sh.fred[warp] = bv;
            sh.ired[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < SP_WARPS; w++)
                if (sh.fred[w] > bv || (sh.fred[w] == bv && sh.ired[w] < bi)) {
                    bv = sh.fred[w];
                    bi = sh.ired[w];
                }
            tokens[blockIdx.x] = bi;
        }
        return;
    }
    // softmax of logits / temp (infer.m:426-436), no contraction of the scaled subtraction
    const float inv_t = 1.0f / temp;
    float mx = -1e30f;
    for (int i = tid; i < V; i += SP_THREADS) mx = fmaxf(mx, __fmul_rn(l[i], inv_t));
    mx = block_max(mx, sh);
    float part = 0.0f;
    for (int i = tid; i < V; i += SP_THREADS) {
        const float e = expf(__fsub_rn(__fmul_rn(l[i], inv_t), mx));
        p[i] = e;
        part += e;
    }
    const float inv_s = 1.0f / block_sum(part, sh);
    for (int i = tid; i < V; i += SP_THREADS) p[i] = __fmul_rn(p[i], inv_s);
    __syncthreads();
    // nucleus (infer.m:440-445): the first key where the cumulative mass reaches top_p
    const unsigned long long t1 = (unsigned long long)((double)top_p * 1099511627776.0);
    radix_select(p, V, false, 0, t1, sh);
    const uint32_t tau = sh.pre;
    const unsigned long long above1 = sh.above;
    const unsigned int j1 = need_count(t1, above1, __uint_as_float(tau), sh.last_cnt);
    const float cum = (float)((double)(above1 + (unsigned long long)j1 * fx(__uint_as_float(tau))) /
                              1099511627776.0);
    // the draw of this row (infer.m:412-418): the (row + 1)-th xorshift32 state
    uint32_t x = rng;
    for (int t = 0; t <= (int)blockIdx.x; t++) {
        x ^= x << 13;
        x ^= x >> 17;
        x ^= x << 5;
    }
    const float r = __fmul_rn((float)(x & 0xFFFFFFu) * (1.0f / (float)0x1000000), cum);
    const unsigned long long t2 = fx(r);
    __syncthreads();
    int pick;
    if (above1 >= t2 && above1 > 0) {
        radix_select(p, V, true, tau, t2, sh);
        const uint32_t kap = sh.pre;
        const unsigned int m = need_count(t2, sh.above, __uint_as_float(kap), sh.last_cnt);
        pick = mth_equal(p, V, kap, m, sh, &slot);
    } else {
        const unsigned int m = need_count(t2, above1, __uint_as_float(tau), j1);
        pick = mth_equal(p, V, tau, m, sh, &slot);
    }
    if (tid == 0) tokens[blockIdx.x] = pick;
}

// ---------------------------------------------------------------------------
// Many-CTA form of the same selection (temp > 0): SG_CTAS CTAs per row, each
// over one slice of the vocabulary, one small kernel per histogram pass; each
// pass resolves the previous pass's digit itself (every CTA the same way) and
// CTA 0 records the state for the next launch; the histograms live in global
// memory, one per pass, with integer atomics (order-independent sums).
constexpr int SG_CTAS = 128;
constexpr int SG_THREADS = 256;

struct SmpRow {
    uint32_t pre, msk, last_cnt, tau, j1, key, m;
    int sel2;                       // the draw lies above tau: select 2 runs
    unsigned long long above, above1, t2;
};

constexpr int SG_PASSES = 8;     // four digits per selection, two selections

struct SmpWs {
    float *part_max, *part_sum;     // [T][SG_CTAS]
    unsigned int *hcnt;             // [SG_PASSES][T][256]
    unsigned long long *hsum;       // [SG_PASSES][T][256]
    unsigned int *cnt;              // [T][SG_CTAS]
    SmpRow *row;                    // [SG_PASSES + 1][T]: the state after 0..8 digits
    int T;
};

__device__ __forceinline__ void slice_of(int V, int &s0, int &s1) {
    s0 = (int)((long long)V * blockIdx.x / gridDim.x);
    s1 = (int)((long long)V * (blockIdx.x + 1) / gridDim.x);
}

// CTA-wide reductions for SG_THREADS threads; every thread gets the result
__device__ __forceinline__ float sg_max(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = red[0];
    for (int w = 1; w < SG_THREADS / 32; w++) v = fmaxf(v, red[w]);
    return v;
}
__device__ __forceinline__ float sg_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = 0.0f;
    for (int w = 0; w < SG_THREADS / 32; w++) v += red[w];
    return v;
}

// pass 0: per-slice max of logits / temp; CTA 0 of a row clears its histogram,
// state and token
__global__ void __launch_bounds__(SG_THREADS) k_sg_max(const float *__restrict__ logits, int V, float inv_t, SmpWs w,
                                                      int *__restrict__ tokens) {
    __shared__ float red[SG_THREADS / 32];
    const int t = blockIdx.y;
    const float *l = logits + (size_t)t * V;
    int s0, s1;
    slice_of(V, s0, s1);
    float mx = -1e30f;
    for (int i = s0 + threadIdx.x; i < s1; i += SG_THREADS) mx = fmaxf(mx, __fmul_rn(l[i], inv_t));
    mx = sg_max(mx, red);
    if (threadIdx.x == 0) w.part_max[t * SG_CTAS + blockIdx.x] = mx;
    if (blockIdx.x == 0) {
        for (int k = threadIdx.x; k < SG_PASSES * 256; k += SG_THREADS) {
            const size_t o = ((size_t)(k >> 8) * w.T + t) * 256 + (k & 255);
            w.hcnt[o] = 0;
            w.hsum[o] = 0;
        }
        if (threadIdx.x == 0) {
            const SmpRow r = {};
            for (int j = 0; j <= SG_PASSES; j++) w.row[(size_t)j * w.T + t] = r;
            tokens[t] = V - 1;   // replaced by k_sg_final
        }
    }
}

// pass 1: exp(logit / temp - max) into p, per-slice sums
__global__ void __launch_bounds__(SG_THREADS) k_sg_exp(const float *__restrict__ logits, int V, float inv_t, SmpWs w,
                                                      float *__restrict__ pbuf) {
    __shared__ float red[SG_THREADS / 32];
    const int t = blockIdx.y;
    const float *l = logits + (size_t)t * V;
    float *p = pbuf + (size_t)t * V;
    float mx = -1e30f;
    for (int g = 0; g < SG_CTAS; g++) mx = fmaxf(mx, w.part_max[t * SG_CTAS + g]);
    int s0, s1;
    slice_of(V, s0, s1);
    float part = 0.0f;
    for (int i = s0 + threadIdx.x; i < s1; i += SG_THREADS) {
        const float e = expf(__fsub_rn(__fmul_rn(l[i], inv_t), mx));
        p[i] = e;
        part += e;
    }
    part = sg_sum(part, red);
    if (threadIdx.x == 0) w.part_sum[t * SG_CTAS + blockIdx.x] = part;
}

// The digit of pass `pass` (0..7: selection pass / 4 + 1, shift 24 - 8 (pass
// % 4)) resolved from its histogram, on top of the state after the earlier
// digits.  After the last digit of selection 1 it forms the nucleus, the draw
// and which selection finds the token; after the last of selection 2, the
// token's key.  Every CTA that needs it computes it (the same data, the same
// result); one thread of the caller runs it on the histogram in shared memory.
__device__ SmpRow sg_resolve(SmpRow r, int pass, const unsigned int *hc, const unsigned long long *hs, float top_p,
                             uint32_t rng, int t) {
    const int sel = pass / 4 + 1, shift = 24 - 8 * (pass % 4);
    if (sel == 2 && !r.sel2) return r;
    const unsigned long long target = sel == 1 ? (unsigned long long)((double)top_p * 1099511627776.0) : r.t2;
    unsigned long long acc = r.above;
    int pick = -1, lowest = -1;
    for (int d = 255; d >= 0; d--) {
        if (!hc[d]) continue;
        lowest = d;
        if (acc + hs[d] >= target) {
            pick = d;
            break;
        }
        acc += hs[d];
    }
    if (pick < 0 && lowest >= 0) {
        pick = lowest;
        acc -= hs[lowest];
    }
    if (pick < 0) pick = 0;
    r.above = acc;
    r.pre |= (uint32_t)pick << shift;
    r.msk |= 255u << shift;
    r.last_cnt = hc[pick];
    if (shift == 0 && sel == 1) {
        r.tau = r.pre;
        r.above1 = r.above;
        r.j1 = need_count(target, r.above1, __uint_as_float(r.tau), r.last_cnt);
        const float cum = (float)((double)(r.above1 + (unsigned long long)r.j1 * fx(__uint_as_float(r.tau))) /
                                  1099511627776.0);
        uint32_t x = rng;
        for (int i = 0; i <= t; i++) {
            x ^= x << 13;
            x ^= x >> 17;
            x ^= x << 5;
        }
        const float rr = __fmul_rn((float)(x & 0xFFFFFFu) * (1.0f / (float)0x1000000), cum);
        r.t2 = fx(rr);
        r.sel2 = r.above1 >= r.t2 && r.above1 > 0;
        if (!r.sel2) {
            r.key = r.tau;
            r.m = need_count(r.t2, r.above1, __uint_as_float(r.tau), r.j1);
        }
        r.pre = r.msk = 0;
        r.above = 0;
    } else if (shift == 0 && sel == 2) {
        r.key = r.pre;
        r.m = need_count(r.t2, r.above, __uint_as_float(r.pre), r.last_cnt);
    }
    return r;
}

// The state after `npass` digits, in shared memory for the whole CTA: the
// state after npass - 1 (written by CTA 0 of the previous launch) and the
// digit of pass npass - 1 from its finished histogram.  CTA 0 stores it for
// the next launch.
__device__ void sg_state(const SmpWs &w, int npass, float top_p, uint32_t rng, SmpRow &st, unsigned int *hc,
                         unsigned long long *hs) {
    const int t = blockIdx.y;
    if (npass == 0) {
        if (threadIdx.x == 0) st = w.row[t];
        __syncthreads();
        return;
    }
    const size_t hb = ((size_t)(npass - 1) * w.T + t) * 256;
    for (int d = threadIdx.x; d < 256; d += blockDim.x) {
        hc[d] = w.hcnt[hb + d];
        hs[d] = w.hsum[hb + d];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        st = sg_resolve(w.row[(size_t)(npass - 1) * w.T + t], npass - 1, hc, hs, top_p, rng, t);
        if (blockIdx.x == 0) w.row[(size_t)npass * w.T + t] = st;
    }
    __syncthreads();
}

// histogram pass `pass` (0..7) over this CTA's slice; pass 0 first scales the
// slice to probabilities; the passes of selection 2 run only when the draw
// lies above tau
__global__ void __launch_bounds__(SG_THREADS) k_sg_hist(int V, SmpWs w, float *__restrict__ pbuf, int pass,
                                                       float top_p, uint32_t rng) {
    __shared__ unsigned int hc[256];
    __shared__ unsigned long long hs[256];
    __shared__ SmpRow st;
    const int t = blockIdx.y;
    sg_state(w, pass, top_p, rng, st, hc, hs);
    const SmpRow r = st;
    const int sel = pass / 4 + 1, shift = 24 - 8 * (pass % 4);
    if (sel == 2 && !r.sel2) return;   // CTA-uniform
    float *p = pbuf + (size_t)t * V;
    for (int d = threadIdx.x; d < 256; d += SG_THREADS) {
        hc[d] = 0;
        hs[d] = 0;
    }
    float inv_s = 0.0f;
    if (pass == 0) {
        float sum = 0.0f;
        for (int g = 0; g < SG_CTAS; g++) sum += w.part_sum[t * SG_CTAS + g];
        inv_s = 1.0f / sum;
    }
    __syncthreads();
    int s0, s1;
    slice_of(V, s0, s1);
    for (int i = s0 + threadIdx.x; i < s1; i += SG_THREADS) {
        float v = p[i];
        if (pass == 0) {
            v = __fmul_rn(v, inv_s);
            p[i] = v;
        }
        const uint32_t k = __float_as_uint(v);
        if ((sel == 2 && k <= r.tau) || (k & r.msk) != r.pre) continue;
        const int d = (k >> shift) & 255;
        atomicAdd(&hc[d], 1u);
        atomicAdd(&hs[d], fx(v));
    }
    __syncthreads();
    const size_t hb = ((size_t)pass * w.T + t) * 256;
    for (int d = threadIdx.x; d < 256; d += SG_THREADS)
        if (hc[d]) {
            atomicAdd(&w.hcnt[hb + d], hc[d]);
            atomicAdd(&w.hsum[hb + d], hs[d]);
        }
}

// the last digit resolved, then the per-slice count of the token's key
__global__ void __launch_bounds__(SG_THREADS) k_sg_count(int V, SmpWs w, const float *__restrict__ pbuf, float top_p,
                                                        uint32_t rng) {
    __shared__ unsigned int hc[256];
    __shared__ unsigned long long hs[256];
    __shared__ SmpRow st;
    __shared__ float red[SG_THREADS / 32];
    const int t = blockIdx.y;
    sg_state(w, SG_PASSES, top_p, rng, st, hc, hs);
    const uint32_t key = st.key;
    const float *p = pbuf + (size_t)t * V;
    int s0, s1;
    slice_of(V, s0, s1);
    float c = 0.0f;   // counts below 2^24: exact in fp32
    for (int i = s0 + threadIdx.x; i < s1; i += SG_THREADS) c += __float_as_uint(p[i]) == key ? 1.0f : 0.0f;
    c = sg_sum(c, red);
    if (threadIdx.x == 0) w.cnt[t * SG_CTAS + blockIdx.x] = (unsigned int)c;
}

// the slice that holds the m-th element of the key (in index order) finds it
__global__ void __launch_bounds__(SG_THREADS) k_sg_final(int V, SmpWs w, const float *__restrict__ pbuf,
                                                        int *__restrict__ tokens) {
    __shared__ unsigned int wsum[SG_THREADS / 32];
    const int t = blockIdx.y;
    const SmpRow &r = w.row[(size_t)SG_PASSES * w.T + t];
    const uint32_t key = r.key;
    const unsigned int m = r.m;
    unsigned int before = 0;
    for (int g = 0; g < (int)blockIdx.x; g++) before += w.cnt[t * SG_CTAS + g];
    const unsigned int mine = w.cnt[t * SG_CTAS + blockIdx.x];
    if (!(m > before && m <= before + mine)) return;   // CTA-uniform
    const float *p = pbuf + (size_t)t * V;
    int s0, s1;
    slice_of(V, s0, s1);
    const int per = (s1 - s0 + SG_THREADS - 1) / SG_THREADS;
    const int lo = min(s1, s0 + (int)threadIdx.x * per), hi = min(s1, lo + per);
    unsigned int c = 0;
    for (int i = lo; i < hi; i++) c += __float_as_uint(p[i]) == key;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    unsigned int b = before + incl - c;
    for (int k = 0; k < warp; k++) b += wsum[k];
    if (c && m > b && m <= b + c) {
        for (int i = lo; i < hi; i++)
            if (__float_as_uint(p[i]) == key && ++b == m) {
                tokens[t] = i;
                break;
            }
    }
}

}  // namespace

size_t moe_sample_ws_bytes(int rows) {
    return (size_t)rows * (2 * SG_CTAS * sizeof(float) +
                           SG_PASSES * 256 * (sizeof(unsigned int) + sizeof(unsigned long long)) +
                           SG_CTAS * sizeof(unsigned int) + (SG_PASSES + 1) * sizeof(SmpRow)) + 64;
}

void moe_launch_sample(const float *logits, int T, int V, float temp, float top_p, uint32_t rng, float *p,
                       void *ws, int *tokens, cudaStream_t s, uint64_t *launches) {
    if (T <= 0) return;
    if (!(temp > 0.0f) || V < 4 * SG_CTAS) {   // argmax, or a small vocabulary: one CTA per row
        k_sample<<<T, SP_THREADS, 0, s>>>(logits, V, temp, top_p, rng, p, tokens);
        LAUNCH_COUNT(launches);
        return;
    }
    // carve the workspace: 8-byte arrays first
    uint8_t *b = reinterpret_cast<uint8_t *>(ws);
    SmpWs w;
    w.T = T;
    w.hsum = reinterpret_cast<unsigned long long *>(b);
    b += (size_t)SG_PASSES * T * 256 * sizeof(unsigned long long);
    w.row = reinterpret_cast<SmpRow *>(b);
    b += (size_t)(SG_PASSES + 1) * T * sizeof(SmpRow);
    w.part_max = reinterpret_cast<float *>(b);
    b += (size_t)T * SG_CTAS * sizeof(float);
    w.part_sum = reinterpret_cast<float *>(b);
    b += (size_t)T * SG_CTAS * sizeof(float);
    w.hcnt = reinterpret_cast<unsigned int *>(b);
    b += (size_t)SG_PASSES * T * 256 * sizeof(unsigned int);
    w.cnt = reinterpret_cast<unsigned int *>(b);
    const float inv_t = 1.0f / temp;
    const dim3 grid(SG_CTAS, T);
    k_sg_max<<<grid, SG_THREADS, 0, s>>>(logits, V, inv_t, w, tokens);
    k_sg_exp<<<grid, SG_THREADS, 0, s>>>(logits, V, inv_t, w, p);
    for (int pass = 0; pass < SG_PASSES; pass++) k_sg_hist<<<grid, SG_THREADS, 0, s>>>(V, w, p, pass, top_p, rng);
    k_sg_count<<<grid, SG_THREADS, 0, s>>>(V, w, p, top_p, rng);
    k_sg_final<<<grid, SG_THREADS, 0, s>>>(V, w, p, tokens);
    const int n = 4 + SG_PASSES;
    if (launches) *launches += n;
}
