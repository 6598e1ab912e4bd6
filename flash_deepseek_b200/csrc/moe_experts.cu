// moe_experts.cu -- the grouped expert GEMVs of the MoE block on B200:
//
//   gate/up   act[p][i] = silu(Wg[e] x) * (Wu[e] x)   Q4_K  (infer.m:1564-1568,
//             expert_worker infer.m:1078-1086, silu_mul infer.m:378-383)
//   down      eo[p][h]  = Wd[e] act[p]                Q6_K or Q4_K
//             (infer.m:1570, 1087-1090)
//
// Work item = (chunk of one expert's tokens, group of rows).  A persistent
// CTA runs one producer warp and eight consumer warps over a ring of
// shared-memory stages, one stage per 256-weight super-block of K:
//   producer   waits for a free stage (mbarrier), then TMA-loads the item's
//              weight tile of that super-block (3-D tensor map over
//              [expert slot][row][byte]) and bulk-copies the chunk's
//              activation operand slice; completion is counted in bytes on
//              the stage's mbarrier
//   consumers  wait for the stage, decode the weights in registers and
//              reduce on the tensor cores, flush to fp32 once per
//              super-block, release the stage
// Two reductions, chosen per chunk (moe_internal.h):
//   int8 path  (chunks of few tokens) exact integer products of the weight
//              integers and 21-bit activation planes (moe_common.cuh); the
//              6-bit sub-block scales are applied to the int32 results
//   fp16 path  (busy experts) the sub-block scale is folded into A exactly
//              (Q4_K: q sc <= 945; Q6_K: (q - 32) sc as a rounded fp16 product
//              plus its exact residual in a second MMA on the same B), the
//              activations are fp16 hi/lo planes (22 bits), products exact,
//              fp32 accumulation; 4 tokens per 8-column tile and no per-
//              sub-block integer work, so each weight block is decoded once
//              for up to 16 tokens
// Every wait is bounded (about one second); on expiry the CTA records an
// error in plan.error and leaves, after the producer has waited (again
// bounded) for the copies it issued.
#include <cuda.h>
#include <stdio.h>

#include "../../include/moe_cuda.h"
#include "moe_common.cuh"
#include "moe_internal.h"

#define EX_CONSUMERS 8
#define EX_THREADS (32 * (EX_CONSUMERS + 1))
// operand bytes of one stage: <= MOE_TC int8-plane vectors or <= MOE_WIDE_TC fp16-plane vectors
#define EX_OPND (MOE_TC * OPB_SB > MOE_WIDE_TC * OPW_SB ? MOE_TC * OPB_SB : MOE_WIDE_TC * OPW_SB)
#define EX_WAIT_CYCLES (1ll << 31)

// gate/up: item = 64 rows of I (gate and up rows), K = H
#define GU_ROWS 64
#define GU_WBOX (GU_ROWS * MOE_Q4K_BYTES)
#define GU_STAGE (2 * GU_WBOX + EX_OPND)
#ifndef GU_NS
#define GU_NS 3
#endif
// down: item = 128 rows of H, K = I
#define DN_ROWS 128
#define DN4_WBOX (DN_ROWS * MOE_Q4K_BYTES)
#define DN4_STAGE (DN4_WBOX + EX_OPND)
#ifndef DN4_NS
#define DN4_NS 3
#endif
#define DN6_QBOX (DN_ROWS * 192)
#define DN6_SBOX (DN_ROWS * 16)
#define DN6_STAGE (DN6_QBOX + DN6_SBOX + EX_OPND)
#ifndef DN6_NS
#define DN6_NS 2
#endif

#define LAUNCH_COUNT(p) \
    do {                \
        if (p) (*(p))++; \
    } while (0)

static int ex_num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of parity `parity` to complete; false after about a
// second (the caller then reports an error instead of hanging).
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity) {
    if (mbar_try_wait(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(b, parity))
        if (clock64() - t0 > EX_WAIT_CYCLES) return false;
    return true;
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *m, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];\n" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ uint32_t u4w(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// D = A(16x32 u8, row) x B(32x8 s8, col), s32
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_s8s8_16816z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// D += A(16x16 fp16, row) x B(16x8 fp16, col), fp32 accumulators
__device__ __forceinline__ void mma_f16_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A(16x8 fp16, row) x B(8x8 fp16, col), fp32
__device__ __forceinline__ void mma_f16_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "f"(0.0f));
}
struct ExItem {
    int rg, e, slot, p0, ntok;
};
// Work item `item` = (chunk chunk_order[counts[3] + item / n_rg], row group
// item % n_rg): the row groups of one chunk are consecutive items, and the
// chunks with the most tokens come first.  The first plan.counts[3] chunks
// of the order run on the tcgen05 kernels instead.
__device__ __forceinline__ void ex_item(const MoePlan &plan, const MoeLayerDev &L, int E, int n_rg, int item,
                                        ExItem &it) {
    const int c = plan.chunk_order[plan.counts[3] + item / n_rg];
    it.rg = item % n_rg;
    it.e = plan.chunk_expert[c];
    it.p0 = plan.chunk_pair0[c];
    it.ntok = plan.chunk_ntok[c];
    it.slot = it.e == E ? L.n_local : it.e - L.e0;
}

// 1/s of the two vectors of an operand tile (2n, 2n + 1) for the lane's two
// columns 2t, 2t + 1 (columns 0-2: vector 2n, 3-5: vector 2n + 1; columns 6,
// 7 carry no vector and their results are discarded)
__device__ __forceinline__ void tile_scales(const uint8_t *tile, int t, float &i0, float &i1) {
    const float a = *reinterpret_cast<const float *>(tile + OPB_SCALE);
    const float b = *reinterpret_cast<const float *>(tile + OPB_SB + OPB_SCALE);
    i0 = t >= 2 ? b : a;
    i1 = t >= 1 ? b : a;
}

// ===========================================================================
// Q4_K super-block of two rows (A rows g, g+8) against NT operand tiles.
// A Q4_K weight is d sc q - dmin m (quant.c:36-61).  Per sub-block pair j the
// lane's qs words give q (low nibbles, u8) and 16 q (high nibbles, masked in
// place); sum_k q x is exact in int32 and scaled by sc (16 sc for the low
// sub-block) in int32; the min term sum_j m_(j/2) xsum_j is one f16 MMA over
// the operand's exact 16-value sums.  Per super-block:
//   acc_f += (d / 16) * acc_i - dmin * min_term                         (fp32)
// Operand tile n holds vectors 2n (columns 0-2 = planes) and 2n + 1 (3-5).
// ===========================================================================
template <int NT>
__device__ __forceinline__ void q4_stage(const uint8_t *rowg, const uint8_t *row8, const uint8_t *opnd, int ntok,
                                         int g, int t, float (&accf)[NT][4]) {
    // 6-bit scales, one per byte (get_scale_min_k4, quant.c:26-34)
    uint32_t scg_lo, scg_hi, sc8_lo, sc8_hi;
    {
        const uint4 hg = lds128(rowg), h8 = lds128(row8);
        scg_lo = hg.y & 0x3F3F3F3Fu;
        scg_hi = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
        sc8_lo = h8.y & 0x3F3F3F3Fu;
        sc8_hi = (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u);
    }
    // this lane's operand column: vector 2n + tsel, plane g % 3.  Columns
    // without a vector (g >= 6, or 2n + tsel >= ntok) read another slot of
    // the stage; only their own output columns see it, and those are dropped.
    const int tsel = g >= 3 ? 1 : 0;
    const uint8_t *bp = opnd + tsel * OPB_SB + (g % 3) * OPB_PLANE + 16 * t;
    int acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0;
    uint4 qw, rw;  // this lane's qs words of sub-block pairs j, j + 1 (rows g, g + 8)
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if ((j & 1) == 0) {
            qw = lds128(rowg + 16 + 32 * t + 8 * j);
            rw = lds128(row8 + 16 + 32 * t + 8 * j);
        }
        const uint32_t wg0 = j & 1 ? qw.z : qw.x, wg1 = j & 1 ? qw.w : qw.y;
        const uint32_t w80 = j & 1 ? rw.z : rw.x, w81 = j & 1 ? rw.w : rw.y;
        const uint32_t swg = j < 2 ? scg_lo : scg_hi, sw8 = j < 2 ? sc8_lo : sc8_hi;
        const int bl = 2 * (j & 1);  // byte of sub-block 2j; sub-block 2j + 1 is the next byte
        const int slg = (int)((swg >> (8 * bl)) & 0x3Fu) << 4, shg = (int)((swg >> (8 * bl + 8)) & 0x3Fu);
        const int sl8 = (int)((sw8 >> (8 * bl)) & 0x3Fu) << 4, sh8 = (int)((sw8 >> (8 * bl + 8)) & 0x3Fu);
        const uint32_t a0l = wg0 & 0x0F0F0F0Fu, a2l = wg1 & 0x0F0F0F0Fu;
        const uint32_t a1l = w80 & 0x0F0F0F0Fu, a3l = w81 & 0x0F0F0F0Fu;
        const uint32_t a0h = wg0 & 0xF0F0F0F0u, a2h = wg1 & 0xF0F0F0F0u;
        const uint32_t a1h = w80 & 0xF0F0F0F0u, a3h = w81 & 0xF0F0F0F0u;
#pragma unroll
        for (int n = 0; n < NT; n++) {
            const uint4 b = lds128(bp + 2 * n * OPB_SB + 64 * j);
            int dl[4], dh[4];
            mma_u8s8_16832(dl, a0l, a1l, a2l, a3l, b.x, b.y);
            mma_u8s8_16832(dh, a0h, a1h, a2h, a3h, b.z, b.w);
            acc[n][0] += slg * dl[0] + shg * dh[0];
            acc[n][1] += slg * dl[1] + shg * dh[1];
            acc[n][2] += sl8 * dl[2] + sh8 * dh[2];
            acc[n][3] += sl8 * dl[3] + sh8 * dh[3];
        }
    }
    // mins m_t, m_(t+4) of both rows as half2 (m, m): bytes (m, 0x64) = 1024 + m
    const uint4 hg = lds128(rowg), h8 = lds128(row8);
    const uint32_t mng_lo = hg.z & 0x3F3F3F3Fu, mng_hi = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
    const uint32_t mn8_lo = h8.z & 0x3F3F3F3Fu, mn8_hi = ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u);
    const uint32_t sel = (uint32_t)t | (4u << 4) | ((uint32_t)t << 8) | (4u << 12);
    const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
    const uint32_t ma = h2_as_u32(__hsub2(u32_as_h2(prmt(mng_lo, 0x64u, sel)), k1024));
    const uint32_t mb = h2_as_u32(__hsub2(u32_as_h2(prmt(mn8_lo, 0x64u, sel)), k1024));
    const uint32_t mc = h2_as_u32(__hsub2(u32_as_h2(prmt(mng_hi, 0x64u, sel)), k1024));
    const uint32_t md = h2_as_u32(__hsub2(u32_as_h2(prmt(mn8_hi, 0x64u, sel)), k1024));
    const float dg = h2f_bits((uint16_t)(hg.x & 0xFFFFu)) * 0.0625f, dmg = h2f_bits((uint16_t)(hg.x >> 16));
    const float d8 = h2f_bits((uint16_t)(h8.x & 0xFFFFu)) * 0.0625f, dm8 = h2f_bits((uint16_t)(h8.x >> 16));
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const uint2 xs = lds64(bp + 2 * n * OPB_SB - 8 * t + OPB_XSUM);
        float mt[4];
        mma_f16_16816(mt, ma, mb, mc, md, xs.x, xs.y, 0.f, 0.f, 0.f, 0.f);
        // 1/s of this super-block for the vector of each of the lane's columns
        float i0, i1;
        tile_scales(opnd + 2 * n * OPB_SB, t, i0, i1);
        accf[n][0] = fmaf(dg * i0, (float)acc[n][0], fmaf(-dmg * i0, mt[0], accf[n][0]));
        accf[n][1] = fmaf(dg * i1, (float)acc[n][1], fmaf(-dmg * i1, mt[1], accf[n][1]));
        accf[n][2] = fmaf(d8 * i0, (float)acc[n][2], fmaf(-dm8 * i0, mt[2], accf[n][2]));
        accf[n][3] = fmaf(d8 * i1, (float)acc[n][3], fmaf(-dm8 * i1, mt[3], accf[n][3]));
    }
}

// ===========================================================================
// Q6_K super-block of two rows against NT operand tiles.  The repacked 6-bit
// q (with the high bit of every qh pair stored inverted) is decoded to the
// byte 4 (q ^ 32), whose int8 value is exactly 4 (q - 32) (quant.c:63-92):
// one s8 x s8 MMA per 16-weight sub-block, scaled by sc in int32, and per
// super-block acc_f += (d / 4) * acc_i.
// ===========================================================================
template <int SP>
__device__ __forceinline__ uint32_t q6_a4(uint32_t W, uint32_t Hw) {
    const uint32_t nib = SP < 4 ? ((W << 2) & 0x3C3C3C3Cu) : ((W >> 2) & 0x3C3C3C3Cu);
    const int f = SP >> 1;
    const uint32_t hs = f == 0 ? (Hw << 6) : f == 1 ? (Hw << 4) : f == 2 ? (Hw << 2) : Hw;
    return nib | (hs & 0xC0C0C0C0u);
}

template <int NT>
__device__ __forceinline__ void q6_stage(const uint8_t *qg, const uint8_t *q8, const uint8_t *sg_p,
                                         const uint8_t *s8_p, float dg, float d8, const uint8_t *opnd, int ntok,
                                         int g, int t, float (&accf)[NT][4]) {
    const uint4 u0 = lds128(qg + 48 * t), u1 = lds128(qg + 48 * t + 16), u2 = lds128(qg + 48 * t + 32);
    const uint4 v0 = lds128(q8 + 48 * t), v1 = lds128(q8 + 48 * t + 16), v2 = lds128(q8 + 48 * t + 32);
    const uint32_t wg[2][6] = {{u0.x, u0.y, u0.z, u0.w, u1.x, u1.y}, {u1.z, u1.w, u2.x, u2.y, u2.z, u2.w}};
    const uint32_t w8[2][6] = {{v0.x, v0.y, v0.z, v0.w, v1.x, v1.y}, {v1.z, v1.w, v2.x, v2.y, v2.z, v2.w}};
    const uint4 sgv = lds128(sg_p), s8v = lds128(s8_p);
    const uint32_t sgw[4] = {sgv.x, sgv.y, sgv.z, sgv.w}, s8w[4] = {s8v.x, s8v.y, s8v.z, s8v.w};
    // this lane's operand column: vector 2n + tsel, plane g % 3.  Columns
    // without a vector (g >= 6, or 2n + tsel >= ntok) read another slot of
    // the stage; only their own output columns see it, and those are dropped.
    const int tsel = g >= 3 ? 1 : 0;
    const uint8_t *bp = opnd + tsel * OPB_SB + (g % 3) * OPB_PLANE + 16 * t;
    int acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int q = 0; q < 2; q++) {
            uint4 B[NT];
#pragma unroll
            for (int n = 0; n < NT; n++) B[n] = lds128(bp + 2 * n * OPB_SB + 64 * (2 * h + q));
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int sp = 4 * q + u, s = 8 * h + sp;
                uint32_t a0, a1;
#define Q6A(SPV)                                                        \
    a0 = q6_a4<SPV>(wg[h][(SPV)&3], wg[h][4 + ((SPV)&1)]);              \
    a1 = q6_a4<SPV>(w8[h][(SPV)&3], w8[h][4 + ((SPV)&1)]);
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
                int scg, sc8;
                switch (s & 3) {
                    case 0: scg = sext_byte<0>(sgw[s >> 2]); sc8 = sext_byte<0>(s8w[s >> 2]); break;
                    case 1: scg = sext_byte<1>(sgw[s >> 2]); sc8 = sext_byte<1>(s8w[s >> 2]); break;
                    case 2: scg = sext_byte<2>(sgw[s >> 2]); sc8 = sext_byte<2>(s8w[s >> 2]); break;
                    default: scg = sext_byte<3>(sgw[s >> 2]); sc8 = sext_byte<3>(s8w[s >> 2]); break;
                }
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    int dd[4];
                    mma_s8s8_16816z(dd, a0, a1, u4w(B[n], u));
                    acc[n][0] += scg * dd[0];
                    acc[n][1] += scg * dd[1];
                    acc[n][2] += sc8 * dd[2];
                    acc[n][3] += sc8 * dd[3];
                }
            }
        }
    }
    const float fg = dg * 0.25f, f8 = d8 * 0.25f;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        float i0, i1;
        tile_scales(opnd + 2 * n * OPB_SB, t, i0, i1);
        accf[n][0] = fmaf(fg * i0, (float)acc[n][0], accf[n][0]);
        accf[n][1] = fmaf(fg * i1, (float)acc[n][1], accf[n][1]);
        accf[n][2] = fmaf(f8 * i0, (float)acc[n][2], accf[n][2]);
        accf[n][3] = fmaf(f8 * i1, (float)acc[n][3], accf[n][3]);
    }
}

// Plane columns -> vector values.  Lane t holds columns 2t, 2t+1 of tile n
// for one row; vector 2n = col0 + 2^7 col1 + 2^14 col2 (lanes t = 0, 1),
// vector 2n+1 = col3 + 2^7 col4 + 2^14 col5 (lanes t = 1, 2).  Returns the
// value of vector 2n + t in lanes t = 0, 1 (every lane of the quad computes).
__device__ __forceinline__ float planes_to_vector(float c0, float c1, int t) {
    float va = t == 0 ? c0 + 128.0f * c1 : (t == 1 ? 16384.0f * c0 : 0.0f);
    float vb = t == 1 ? c1 : (t == 2 ? 128.0f * c0 + 16384.0f * c1 : 0.0f);
    va += __shfl_xor_sync(0xffffffffu, va, 1);
    vb += __shfl_xor_sync(0xffffffffu, vb, 1);
    va += __shfl_xor_sync(0xffffffffu, va, 2);
    vb += __shfl_xor_sync(0xffffffffu, vb, 2);
    return t == 0 ? va : vb;
}

// ===========================================================================
// fp16 path, Q4_K super-block of two rows (A rows g, g + 8) against NT tiles
// of 4 tokens x 2 planes (column c: token c / 2 of the tile, plane c % 2).
// A = q sc exactly in fp16: the nibble under the exponent of 1024 (1024 + q,
// or 1024 + 16 q for a high nibble masked in place), then
// fma(1024 + q, sc, -1024 sc) = q sc (or with sc / 16 and -64 sc), one
// rounding of an exact integer <= 945.  Lane t's qs bytes 8 t .. 8 t + 7 of
// sub-block pair jj give elements (0, 2), (1, 3) (k16 step 0) and (4, 6),
// (5, 7) (step 1) of the low and of the high sub-block; the operand stores
// B in the same order (style Q4, moe_common.cuh).  The min term
// sum_j m_j xsum_j is one m16n8k8 MMA over the sub-block sums.  Per
// super-block and lane column (token 4 n + t, both planes summed):
//   acc_f += (d / s) (hi + lo) - (32 dmin / s) (min_hi + min_lo)
// ===========================================================================
template <int NT>
__device__ __forceinline__ void q4w_stage(const uint8_t *rowg, const uint8_t *row8, const uint8_t *opnd, int g,
                                          int t, float (&accf)[NT][2]) {
    const uint4 hg = lds128(rowg), h8 = lds128(row8);
    // 6-bit scales of sub-blocks 0-3 / 4-7, one per byte (get_scale_min_k4, quant.c:26-34)
    const uint32_t scg[2] = {hg.y & 0x3F3F3F3Fu, (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u)};
    const uint32_t sc8[2] = {h8.y & 0x3F3F3F3Fu, (h8.w & 0x0F0F0F0Fu) | ((h8.y >> 2) & 0x30303030u)};
    // this lane's B column: token g / 2 of the tile, plane g % 2
    const uint8_t *bp = opnd + (g >> 1) * OPW_SB + (g & 1) * OPW_LO + 16 * t;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
#pragma unroll
    for (int jj = 0; jj < 4; jj++) {
        const uint2 wg = lds64(rowg + 16 + 32 * t + 8 * jj), w8 = lds64(row8 + 16 + 32 * t + 8 * jj);
        // scale constants of sub-blocks 2 jj (low nibbles) and 2 jj + 1 (high)
        uint32_t sl_g, sl_8, sh_g, sh_8;
        if ((jj & 1) == 0) {
            sl_g = byte_h2<0>(scg[jj >> 1], H2_1024); sh_g = byte_h2<1>(scg[jj >> 1], H2_1024);
            sl_8 = byte_h2<0>(sc8[jj >> 1], H2_1024); sh_8 = byte_h2<1>(sc8[jj >> 1], H2_1024);
        } else {
            sl_g = byte_h2<2>(scg[jj >> 1], H2_1024); sh_g = byte_h2<3>(scg[jj >> 1], H2_1024);
            sl_8 = byte_h2<2>(sc8[jj >> 1], H2_1024); sh_8 = byte_h2<3>(sc8[jj >> 1], H2_1024);
        }
        const uint32_t nl_g = hmul2u(sl_g, H2_M1024), nl_8 = hmul2u(sl_8, H2_M1024);
        const uint32_t nh_g = hmul2u(sh_g, H2_M64), nh_8 = hmul2u(sh_8, H2_M64);
        sh_g = hmul2u(sh_g, H2_16TH);
        sh_8 = hmul2u(sh_8, H2_16TH);
        uint32_t lo[2][4], hi[2][4];  // [row g / g + 8][(0,2) (1,3) (4,6) (5,7)]
        const uint32_t wv[2][2] = {{wg.x, wg.y}, {w8.x, w8.y}};
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint32_t sl = r ? sl_8 : sl_g, nl = r ? nl_8 : nl_g, sh = r ? sh_8 : sh_g, nh = r ? nh_8 : nh_g;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t w = wv[r][h], ws = w >> 8;
                lo[r][2 * h] = hfma2u((w & 0x000F000Fu) | H2_1024, sl, nl);
                lo[r][2 * h + 1] = hfma2u((ws & 0x000F000Fu) | H2_1024, sl, nl);
                hi[r][2 * h] = hfma2u((w & 0x00F000F0u) | H2_1024, sh, nh);
                hi[r][2 * h + 1] = hfma2u((ws & 0x00F000F0u) | H2_1024, sh, nh);
            }
        }
#pragma unroll
        for (int n = 0; n < NT; n++) {
            const uint4 bl = lds128(bp + 4 * n * OPW_SB + 128 * jj);
            const uint4 bh = lds128(bp + 4 * n * OPW_SB + 128 * jj + 64);
            mma_f16_acc(acc[n], lo[0][0], lo[1][0], lo[0][1], lo[1][1], bl.x, bl.y);
            mma_f16_acc(acc[n], lo[0][2], lo[1][2], lo[0][3], lo[1][3], bl.z, bl.w);
            mma_f16_acc(acc[n], hi[0][0], hi[1][0], hi[0][1], hi[1][1], bh.x, bh.y);
            mma_f16_acc(acc[n], hi[0][2], hi[1][2], hi[0][3], hi[1][3], bh.z, bh.w);
        }
    }
    // mins m_2t, m_2t+1 of rows g and g + 8 (A of the m16n8k8 min-term MMA)
    const uint32_t mng[2] = {hg.z & 0x3F3F3F3Fu, ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u)};
    const uint32_t mn8[2] = {h8.z & 0x3F3F3F3Fu, ((h8.w >> 4) & 0x0F0F0F0Fu) | ((h8.z >> 2) & 0x30303030u)};
    const uint32_t bsel = 2u * (uint32_t)(t & 1);
    const uint32_t msel = bsel | (4u << 4) | ((bsel + 1u) << 8) | (4u << 12);
    const uint32_t ma = hsub2u(prmt(mng[t >> 1], 0x64u, msel), H2_1024);
    const uint32_t mb = hsub2u(prmt(mn8[t >> 1], 0x64u, msel), H2_1024);
    const float dg = h2f_bits((uint16_t)(hg.x & 0xFFFFu)), dmg = 32.0f * h2f_bits((uint16_t)(hg.x >> 16));
    const float d8 = h2f_bits((uint16_t)(h8.x & 0xFFFFu)), dm8 = 32.0f * h2f_bits((uint16_t)(h8.x >> 16));
    const uint8_t *xs = opnd + (g >> 1) * OPW_SB + OPW_XSUM + 16 * (g & 1) + 4 * t;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        float mt[4];
        mma_f16_1688(mt, ma, mb, *reinterpret_cast<const uint32_t *>(xs + 4 * n * OPW_SB));
        const float inv = *reinterpret_cast<const float *>(opnd + (4 * n + t) * OPW_SB + OPW_SCALE);
        accf[n][0] = fmaf(dg * inv, acc[n][0] + acc[n][1], fmaf(-dmg * inv, mt[0] + mt[1], accf[n][0]));
        accf[n][1] = fmaf(d8 * inv, acc[n][2] + acc[n][3], fmaf(-dm8 * inv, mt[2] + mt[3], accf[n][1]));
    }
}

// ===========================================================================
// fp16 path, Q6_K super-block of two rows against NT tiles of 4 tokens x 2
// planes.  q (6 bits, from the repacked planes, high qh bit restored) under
// the exponent of 1024 minus 1056 gives Q = q - 32 exactly; v = Q sc
// (|v| <= 4096) is P = fp16(Q sc) plus R = fma(Q, sc, -P) in {-1, 0, 1}, both
// exact.  P multiplies both planes of x; R only x_hi (R x_lo is below 2^-23
// of P x), on tiles of 8 tokens whose column order (token (c / 2) + 4 (c % 2)
// of the pair of P tiles) puts in lane t the same tokens as its P columns.
// Lane t holds elements 4 t .. 4 t + 3 of every sub-block (style Q6).  Per
// super-block: acc_f += (d / s) (hi + lo + r).
// ===========================================================================
template <int NT>
__device__ __forceinline__ void q6w_stage(const uint8_t *qg, const uint8_t *q8, const uint8_t *sg_p,
                                          const uint8_t *s8_p, float dg, float d8, const uint8_t *opnd, int g, int t,
                                          float (&accf)[NT][2]) {
    const uint4 u0 = lds128(qg + 48 * t), u1 = lds128(qg + 48 * t + 16), u2 = lds128(qg + 48 * t + 32);
    const uint4 v0 = lds128(q8 + 48 * t), v1 = lds128(q8 + 48 * t + 16), v2 = lds128(q8 + 48 * t + 32);
    const uint32_t wq[2][2][6] = {{{u0.x, u0.y, u0.z, u0.w, u1.x, u1.y}, {u1.z, u1.w, u2.x, u2.y, u2.z, u2.w}},
                                  {{v0.x, v0.y, v0.z, v0.w, v1.x, v1.y}, {v1.z, v1.w, v2.x, v2.y, v2.z, v2.w}}};
    // int8 scales + 128 (bytes under 0x64 give 1152 + sc)
    const uint4 sgv = lds128(sg_p), s8v = lds128(s8_p);
    const uint32_t sw[2][4] = {{sgv.x ^ 0x80808080u, sgv.y ^ 0x80808080u, sgv.z ^ 0x80808080u, sgv.w ^ 0x80808080u},
                               {s8v.x ^ 0x80808080u, s8v.y ^ 0x80808080u, s8v.z ^ 0x80808080u, s8v.w ^ 0x80808080u}};
    const uint8_t *bp = opnd + (g >> 1) * OPW_SB + (g & 1) * OPW_LO + 16 * t;
    // R tiles: x_hi of token 8 r + (g / 2) + 4 (g % 2)
    const uint8_t *br = opnd + ((g >> 1) + 4 * (g & 1)) * OPW_SB + 16 * t;
    constexpr int NR = (NT + 1) / 2;
    float acc[NT][4], accr[NR][4];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
#pragma unroll
    for (int n = 0; n < NR; n++) accr[n][0] = accr[n][1] = accr[n][2] = accr[n][3] = 0.0f;
#pragma unroll
    for (int s2 = 0; s2 < 8; s2++) {
        uint32_t P[2][2][2], R[2][2][2];  // [sub-block even / odd][row][elements (0,1) / (2,3)]
#pragma unroll
        for (int o = 0; o < 2; o++) {
            const int s = 2 * s2 + o, h = s >> 3, sp = s & 7, f = sp >> 1;
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const uint32_t W = wq[r][h][sp & 3], Hq = wq[r][h][4 + (sp & 1)];
                const uint32_t nib = (sp < 4 ? W : W >> 4) & 0x0F0F0F0Fu;
                const uint32_t hb = (2 * f <= 4 ? Hq << (4 - 2 * f) : Hq >> (2 * f - 4)) & 0x30303030u;
                const uint32_t q6 = nib | (hb ^ 0x20202020u);  // four values q (0..63) in bytes
                uint32_t sc;
                switch (s & 3) {
                    case 0: sc = byte_h2<0>(sw[r][s >> 2], H2_1152); break;
                    case 1: sc = byte_h2<1>(sw[r][s >> 2], H2_1152); break;
                    case 2: sc = byte_h2<2>(sw[r][s >> 2], H2_1152); break;
                    default: sc = byte_h2<3>(sw[r][s >> 2], H2_1152); break;
                }
                const uint32_t q01 = hsub2u(prmt(q6, 0x64u, 0x4140u), H2_1056);  // q - 32, exact
                const uint32_t q23 = hsub2u(prmt(q6, 0x64u, 0x4342u), H2_1056);
                P[o][r][0] = hmul2u(q01, sc);
                P[o][r][1] = hmul2u(q23, sc);
                R[o][r][0] = hfma2u(q01, sc, P[o][r][0] ^ 0x80008000u);  // Q sc - P, exact
                R[o][r][1] = hfma2u(q23, sc, P[o][r][1] ^ 0x80008000u);
            }
        }
#pragma unroll
        for (int n = 0; n < NT; n++) {
            const uint4 b = lds128(bp + 4 * n * OPW_SB + 64 * s2);
            mma_f16_acc(acc[n], P[0][0][0], P[0][1][0], P[0][0][1], P[0][1][1], b.x, b.y);
            mma_f16_acc(acc[n], P[1][0][0], P[1][1][0], P[1][0][1], P[1][1][1], b.z, b.w);
        }
#pragma unroll
        for (int n = 0; n < NR; n++) {
            const uint4 b = lds128(br + 8 * n * OPW_SB + 64 * s2);
            mma_f16_acc(accr[n], R[0][0][0], R[0][1][0], R[0][0][1], R[0][1][1], b.x, b.y);
            mma_f16_acc(accr[n], R[1][0][0], R[1][1][0], R[1][0][1], R[1][1][1], b.z, b.w);
        }
    }
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const float inv = *reinterpret_cast<const float *>(opnd + (4 * n + t) * OPW_SB + OPW_SCALE);
        const float rg = accr[n >> 1][n & 1], r8 = accr[n >> 1][2 + (n & 1)];
        accf[n][0] = fmaf(dg * inv, (acc[n][0] + acc[n][1]) + rg, accf[n][0]);
        accf[n][1] = fmaf(d8 * inv, (acc[n][2] + acc[n][3]) + r8, accf[n][1]);
    }
}

// ===========================================================================
// gate/up
// ===========================================================================
template <int NT>
__device__ __forceinline__ bool gu_item(const MoeDims &d, const MoePlan &plan, float *__restrict__ act, const ExItem &it, int NB, uint8_t *sm,
                                        uint64_t *full, uint64_t *empty, uint32_t &seq, int w, int lane) {
    const int g = lane >> 2, t = lane & 3;
    float accf[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) accf[n][0] = accf[n][1] = accf[n][2] = accf[n][3] = 0.0f;
    for (int sb = 0; sb < NB; sb++, seq++) {
        const int st = seq % GU_NS;
        if (!mbar_wait(&full[st], (seq / GU_NS) & 1)) return false;
        const uint8_t *stage = sm + (size_t)st * GU_STAGE;
        q4_stage<NT>(stage + (8 * w + g) * MOE_Q4K_BYTES, stage + GU_WBOX + (8 * w + g) * MOE_Q4K_BYTES,
                     stage + 2 * GU_WBOX, it.ntok, g, t, accf);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    const int row = it.rg * GU_ROWS + 8 * w + g;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const float gv = planes_to_vector(accf[n][0], accf[n][1], t);
        const float uv = planes_to_vector(accf[n][2], accf[n][3], t);
        const int tk = 2 * n + t;
        if (t < 2 && tk < it.ntok) act[(size_t)(it.p0 + tk) * d.I + row] = (gv / (1.0f + expf(-gv))) * uv;
    }
    return true;
}

// fp16-path gate/up item: lane (g, t) ends with the gate (row g) and up
// (row g + 8) values of token 4 n + t, so SwiGLU needs no shuffle.
template <int NT>
__device__ __forceinline__ bool gu_item_w(const MoeDims &d, float *__restrict__ act, const ExItem &it, int NB,
                                          uint8_t *sm, uint64_t *full, uint64_t *empty, uint32_t &seq, int w,
                                          int lane) {
    const int g = lane >> 2, t = lane & 3;
    float accf[NT][2];
#pragma unroll
    for (int n = 0; n < NT; n++) accf[n][0] = accf[n][1] = 0.0f;
    for (int sb = 0; sb < NB; sb++, seq++) {
        const int st = seq % GU_NS;
        if (!mbar_wait(&full[st], (seq / GU_NS) & 1)) return false;
        const uint8_t *stage = sm + (size_t)st * GU_STAGE;
        q4w_stage<NT>(stage + (8 * w + g) * MOE_Q4K_BYTES, stage + GU_WBOX + (8 * w + g) * MOE_Q4K_BYTES,
                      stage + 2 * GU_WBOX, g, t, accf);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    const int row = it.rg * GU_ROWS + 8 * w + g;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int tk = 4 * n + t;
        const float gv = accf[n][0], uv = accf[n][1];
        if (tk < it.ntok) act[(size_t)(it.p0 + tk) * d.I + row] = (gv / (1.0f + expf(-gv))) * uv;
    }
    return true;
}

__device__ __forceinline__ uint8_t *align128(uint8_t *p) {
    return p + ((128u - (smem_u32(p) & 127u)) & 127u);
}

__global__ void __launch_bounds__(EX_THREADS, 2)
    k_gateup(MoeDims d, const __grid_constant__ MoeLayerDev L, MoePlan plan, const uint8_t *__restrict__ xop,
             float *__restrict__ act) {
    extern __shared__ uint8_t ex_raw[];
    __shared__ __align__(8) uint64_t full[GU_NS], empty[GU_NS];
    __shared__ int stage_item[GU_NS];  // item whose first super-block the stage holds; -1: no more items
    uint8_t *sm = align128(ex_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NB = d.H / MOE_QK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < GU_NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], EX_CONSUMERS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    moe_pdl_wait();  // the plan and the operand come from the previous kernels
    moe_pdl_trigger();
    const int n_rg = d.I / GU_ROWS;
    const int n_items = (plan.counts[1] - plan.counts[3]) * n_rg;
    uint32_t seq = 0;
    if (warp == EX_CONSUMERS) {  // producer: takes items from the plan's counter
        const size_t rowst = opx_row(d.H), wide_off = op_bytes(d.H);
        bool ok = true;
        for (;;) {
            int item = 0;
            if (lane == 0) item = atomicAdd(&plan.counts[4], 1);
            item = __shfl_sync(0xffffffffu, item, 0);
            if (item >= n_items) {  // end marker for the consumers
                const int st = seq % GU_NS;
                if (!mbar_wait(&empty[st], ((seq / GU_NS) & 1) ^ 1)) { ok = false; break; }
                if (lane == 0) {
                    stage_item[st] = -1;
                    mbar_arrive(&full[st]);
                }
                seq++;
                break;
            }
            ExItem it;
            ex_item(plan, L, d.E, n_rg, item, it);
            // the chunk's operand form: fp16 planes on the fp16 path
            const bool fp = moe_gu_wide(it.ntok);
            const uint32_t osb = fp ? OPW_SB : OPB_SB;
            const uint8_t *src = lane < it.ntok ? xop + (size_t)plan.pair_token[it.p0 + lane] * rowst +
                                                      (fp ? wide_off : 0)
                                                : nullptr;
            for (int sb = 0; sb < NB; sb++, seq++) {
                const int st = seq % GU_NS;
                if (!mbar_wait(&empty[st], ((seq / GU_NS) & 1) ^ 1)) { ok = false; break; }
                uint8_t *stage = sm + (size_t)st * GU_STAGE;
                if (lane == 0) {
                    if (sb == 0) stage_item[st] = item;
                    mbar_expect_tx(&full[st], 2 * GU_WBOX + it.ntok * osb);
                    tma_load_3d(stage, &L.tm_gu, sb * MOE_Q4K_BYTES, it.rg * GU_ROWS, it.slot, &full[st]);
                    tma_load_3d(stage + GU_WBOX, &L.tm_gu, sb * MOE_Q4K_BYTES, d.I + it.rg * GU_ROWS, it.slot,
                                &full[st]);
                }
                __syncwarp();
                if (lane < it.ntok) bulk_load(stage + 2 * GU_WBOX + lane * osb, src + (size_t)sb * osb, osb, &full[st]);
            }
            if (!ok) break;
        }
        if (!ok && lane == 0) atomicExch(plan.error, EX_ERR_TIMEOUT);
        // the copies of the last stages must land before the CTA leaves
        for (uint32_t k = seq > GU_NS ? seq - GU_NS : 0; k < seq; k++)
            if (!mbar_wait(&full[k % GU_NS], (k / GU_NS) & 1)) break;
        return;
    }
    for (;;) {  // consumers: the items in the producer's order
        const int st = seq % GU_NS;
        if (!mbar_wait(&full[st], (seq / GU_NS) & 1)) {
            if (lane == 0) atomicExch(plan.error, EX_ERR_TIMEOUT);
            return;
        }
        const int item = stage_item[st];
        if (item < 0) return;
        ExItem it;
        ex_item(plan, L, d.E, n_rg, item, it);
        bool ok;
        if (moe_gu_wide(it.ntok)) {
            switch ((it.ntok + 3) >> 2) {
                case 2: ok = gu_item_w<2>(d, act, it, NB, sm, full, empty, seq, warp, lane); break;
                case 3: ok = gu_item_w<3>(d, act, it, NB, sm, full, empty, seq, warp, lane); break;
                default: ok = gu_item_w<4>(d, act, it, NB, sm, full, empty, seq, warp, lane); break;
            }
        } else {
            switch ((it.ntok + 1) >> 1) {  // int8-path chunks have at most MOE_TC tokens
                case 1: ok = gu_item<1>(d, plan, act, it, NB, sm, full, empty, seq, warp, lane); break;
                case 2: ok = gu_item<2>(d, plan, act, it, NB, sm, full, empty, seq, warp, lane); break;
                case 3: ok = gu_item<3>(d, plan, act, it, NB, sm, full, empty, seq, warp, lane); break;
                default: ok = gu_item<4>(d, plan, act, it, NB, sm, full, empty, seq, warp, lane); break;
            }
        }
        if (!ok) {
            if (lane == 0) atomicExch(plan.error, EX_ERR_TIMEOUT);
            return;
        }
    }
}

// ===========================================================================
// down
// ===========================================================================
template <int NT, int TY>
__device__ __forceinline__ bool dn_item(const MoeDims &d, float *__restrict__ eo,
                                        const ExItem &it, int NB, int nbp, uint8_t *sm, const uint8_t *dbuf,
                                        uint64_t *full, uint64_t *empty, uint32_t &seq, int w, int lane) {
    const int g = lane >> 2, t = lane & 3;
    constexpr int NS = TY == MOE_TYPE_Q6_K ? DN6_NS : DN4_NS;
    constexpr int STAGE = TY == MOE_TYPE_Q6_K ? DN6_STAGE : DN4_STAGE;
    const int rl = 16 * w + g;  // local rows rl, rl + 8 of the item
    float accf[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) accf[n][0] = accf[n][1] = accf[n][2] = accf[n][3] = 0.0f;
    for (int sb = 0; sb < NB; sb++, seq++) {
        const int st = seq % NS;
        if (!mbar_wait(&full[st], (seq / NS) & 1)) return false;
        const uint8_t *stage = sm + (size_t)st * STAGE;
        if (TY == MOE_TYPE_Q6_K) {
            const __half *dp = reinterpret_cast<const __half *>(dbuf);
            const float dg = __half2float(dp[rl * nbp + sb]), d8 = __half2float(dp[(rl + 8) * nbp + sb]);
            q6_stage<NT>(stage + rl * 192, stage + (rl + 8) * 192, stage + DN6_QBOX + rl * 16,
                         stage + DN6_QBOX + (rl + 8) * 16, dg, d8, stage + DN6_QBOX + DN6_SBOX, it.ntok, g, t,
                         accf);
        } else {
            q4_stage<NT>(stage + rl * MOE_Q4K_BYTES, stage + (rl + 8) * MOE_Q4K_BYTES, stage + DN4_WBOX, it.ntok,
                         g, t, accf);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    const int row = it.rg * DN_ROWS + rl;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const float vg = planes_to_vector(accf[n][0], accf[n][1], t);
        const float v8 = planes_to_vector(accf[n][2], accf[n][3], t);
        const int tk = 2 * n + t;
        if (t < 2 && tk < it.ntok) {
            eo[(size_t)(it.p0 + tk) * d.H + row] = vg;
            eo[(size_t)(it.p0 + tk) * d.H + row + 8] = v8;
        }
    }
    return true;
}

// fp16-path down item (chunks of more than MOE_TC tokens)
template <int NT, int TY>
__device__ __forceinline__ bool dn_item_w(const MoeDims &d, float *__restrict__ eo, const ExItem &it, int NB,
                                          int nbp, uint8_t *sm, const uint8_t *dbuf, uint64_t *full, uint64_t *empty,
                                          uint32_t &seq, int w, int lane) {
    const int g = lane >> 2, t = lane & 3;
    constexpr int NS = TY == MOE_TYPE_Q6_K ? DN6_NS : DN4_NS;
    constexpr int STAGE = TY == MOE_TYPE_Q6_K ? DN6_STAGE : DN4_STAGE;
    const int rl = 16 * w + g;  // local rows rl, rl + 8 of the item
    float accf[NT][2];
#pragma unroll
    for (int n = 0; n < NT; n++) accf[n][0] = accf[n][1] = 0.0f;
    for (int sb = 0; sb < NB; sb++, seq++) {
        const int st = seq % NS;
        if (!mbar_wait(&full[st], (seq / NS) & 1)) return false;
        const uint8_t *stage = sm + (size_t)st * STAGE;
        if (TY == MOE_TYPE_Q6_K) {
            const __half *dp = reinterpret_cast<const __half *>(dbuf);
            const float dg = __half2float(dp[rl * nbp + sb]), d8 = __half2float(dp[(rl + 8) * nbp + sb]);
            q6w_stage<NT>(stage + rl * 192, stage + (rl + 8) * 192, stage + DN6_QBOX + rl * 16,
                          stage + DN6_QBOX + (rl + 8) * 16, dg, d8, stage + DN6_QBOX + DN6_SBOX, g, t, accf);
        } else {
            q4w_stage<NT>(stage + rl * MOE_Q4K_BYTES, stage + (rl + 8) * MOE_Q4K_BYTES, stage + DN4_WBOX, g, t, accf);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    const int row = it.rg * DN_ROWS + rl;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int tk = 4 * n + t;
        if (tk < it.ntok) {
            eo[(size_t)(it.p0 + tk) * d.H + row] = accf[n][0];
            eo[(size_t)(it.p0 + tk) * d.H + row + 8] = accf[n][1];
        }
    }
    return true;
}

// One instance per down type; chunks of the other type are skipped.
template <int TY>
__global__ void __launch_bounds__(EX_THREADS, 2)
    k_down(MoeDims d, const __grid_constant__ MoeLayerDev L, MoePlan plan, const uint8_t *__restrict__ dop,
           float *__restrict__ eo) {
    constexpr int NS = TY == MOE_TYPE_Q6_K ? DN6_NS : DN4_NS;
    constexpr int STAGE = TY == MOE_TYPE_Q6_K ? DN6_STAGE : DN4_STAGE;
    extern __shared__ uint8_t ex_raw[];
    __shared__ __align__(8) uint64_t full[NS], empty[NS];
    __shared__ int stage_item[NS];  // item whose first super-block the stage holds; -1: no more items
    uint8_t *sm = align128(ex_raw);
    const int NB = d.I / MOE_QK, nbp = q6r_nb_pad(NB);
    const int dbytes = DN_ROWS * 2 * nbp;  // per item (Q6_K d plane)
    uint8_t *dbuf0 = sm + (size_t)NS * STAGE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], EX_CONSUMERS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    // The plan (two launches older) and the weights do not depend on the
    // previous kernel, only the down operand does: the producer issues the
    // weight copies of its first NS stages before the dependency wait and
    // their operand copies after it.  The consumers only read shared memory
    // behind the full barriers.
    moe_pdl_trigger();
    const int n_rg = d.H / DN_ROWS;
    const int n_items = (plan.counts[1] - plan.counts[3]) * n_rg;
    int *counter = &plan.counts[TY == MOE_TYPE_Q6_K ? 5 : 6];
    uint32_t seq = 0, nitem = 0;
    if (warp == EX_CONSUMERS) {  // producer: takes items from the plan's counter
        const size_t opst = opw_bytes(d.I);  // pair rows of the down operand
        bool ok = true, waited = false;
        int ndef = 0, def_st[NS], def_p0[NS], def_nt[NS], def_sb[NS];
        auto issue_ops = [&](int st, int p0, int ntok, int sb) {
            if (lane < ntok) {
                const uint32_t osb = moe_dn_wide(ntok) ? OPW_SB : OPB_SB;
                uint8_t *od = sm + (size_t)st * STAGE + (TY == MOE_TYPE_Q6_K ? DN6_QBOX + DN6_SBOX : DN4_WBOX) +
                              lane * osb;
                bulk_load(od, dop + (size_t)(p0 + lane) * opst + (size_t)sb * osb, osb, &full[st]);
            }
        };
        auto flush_deferred = [&]() {
            moe_pdl_wait();
            waited = true;
            for (int k = 0; k < ndef; k++) issue_ops(def_st[k], def_p0[k], def_nt[k], def_sb[k]);
            ndef = 0;
        };
        for (;;) {
            int item = 0;
            if (lane == 0) item = atomicAdd(counter, 1);
            item = __shfl_sync(0xffffffffu, item, 0);
            if (item >= n_items) {  // end marker for the consumers
                const int st = seq % NS;
                if (!mbar_wait(&empty[st], ((seq / NS) & 1) ^ 1)) { ok = false; break; }
                if (lane == 0) {
                    stage_item[st] = -1;
                    mbar_arrive(&full[st]);
                }
                seq++;
                break;
            }
            ExItem it;
            ex_item(plan, L, d.E, n_rg, item, it);
            if (((it.e == d.E) ? L.sh_down_type : L.down_type) != TY) continue;
            uint8_t *dbuf = dbuf0 + (size_t)(nitem & 1) * dbytes;
            nitem++;
            const uint32_t osb = moe_dn_wide(it.ntok) ? OPW_SB : OPB_SB;
            for (int sb = 0; sb < NB; sb++, seq++) {
                const int st = seq % NS;
                if (!mbar_wait(&empty[st], ((seq / NS) & 1) ^ 1)) { ok = false; break; }
                uint8_t *stage = sm + (size_t)st * STAGE;
                if (lane == 0) {
                    if (sb == 0) stage_item[st] = item;
                    const int y = it.rg * DN_ROWS;
                    if (TY == MOE_TYPE_Q6_K) {
                        mbar_expect_tx(&full[st], DN6_QBOX + DN6_SBOX + it.ntok * osb + (sb == 0 ? dbytes : 0));
                        tma_load_3d(stage, &L.tm_d6q, sb * 192, y, it.slot, &full[st]);
                        tma_load_3d(stage + DN6_QBOX, &L.tm_d6s, sb * 16, y, it.slot, &full[st]);
                        if (sb == 0) tma_load_3d(dbuf, &L.tm_d6d, 0, y, it.slot, &full[st]);
                    } else {
                        mbar_expect_tx(&full[st], DN4_WBOX + it.ntok * osb);
                        tma_load_3d(stage, &L.tm_d4, sb * MOE_Q4K_BYTES, y, it.slot, &full[st]);
                    }
                }
                __syncwarp();
                if (waited) {
                    issue_ops(st, it.p0, it.ntok, sb);
                } else {
                    def_st[ndef] = st; def_p0[ndef] = it.p0; def_nt[ndef] = it.ntok; def_sb[ndef] = sb;
                    if (++ndef == NS) flush_deferred();
                }
            }
            if (!ok) break;
        }
        if (!waited) flush_deferred();
        if (!ok && lane == 0) atomicExch(plan.error, EX_ERR_TIMEOUT);
        for (uint32_t k = seq > (uint32_t)NS ? seq - NS : 0; k < seq; k++)
            if (!mbar_wait(&full[k % NS], (k / NS) & 1)) break;
        return;
    }
    moe_pdl_wait();
    for (;;) {  // consumers: the items in the producer's order
        const int st = seq % NS;
        if (!mbar_wait(&full[st], (seq / NS) & 1)) {
            if (lane == 0) atomicExch(plan.error, EX_ERR_TIMEOUT);
            return;
        }
        const int item = stage_item[st];
        if (item < 0) return;
        ExItem it;
        ex_item(plan, L, d.E, n_rg, item, it);
        const uint8_t *dbuf = dbuf0 + (size_t)(nitem & 1) * dbytes;
        nitem++;
        bool ok;
        if (moe_dn_wide(it.ntok)) {
            switch ((it.ntok + 3) >> 2) {
                case 3: ok = dn_item_w<3, TY>(d, eo, it, NB, nbp, sm, dbuf, full, empty, seq, warp, lane); break;
                default: ok = dn_item_w<4, TY>(d, eo, it, NB, nbp, sm, dbuf, full, empty, seq, warp, lane); break;
            }
        } else {
            switch ((it.ntok + 1) >> 1) {
                case 1: ok = dn_item<1, TY>(d, eo, it, NB, nbp, sm, dbuf, full, empty, seq, warp, lane); break;
                case 2: ok = dn_item<2, TY>(d, eo, it, NB, nbp, sm, dbuf, full, empty, seq, warp, lane); break;
                case 3: ok = dn_item<3, TY>(d, eo, it, NB, nbp, sm, dbuf, full, empty, seq, warp, lane); break;
                default: ok = dn_item<4, TY>(d, eo, it, NB, nbp, sm, dbuf, full, empty, seq, warp, lane); break;
            }
        }
        if (!ok) {
            if (lane == 0) atomicExch(plan.error, EX_ERR_TIMEOUT);
            return;
        }
    }
}

// ===========================================================================
// host side
// ===========================================================================
void moe_launch_gateup(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const uint8_t *xop,
                       float *act, int max_chunks, cudaStream_t s, uint64_t *launches) {
    const int max_items = max_chunks * (d.I / GU_ROWS);
    int grid = 2 * ex_num_sms();
    if (grid > max_items) grid = max_items;
    if (grid < 1) grid = 1;
    const size_t smem = (size_t)GU_NS * GU_STAGE + 128;
    static size_t attr[MOE_MAX_DEVICES];
    moe_smem_limit(k_gateup, smem, attr);
    moe_launch_pdl(k_gateup, dim3(grid), dim3(EX_THREADS), smem, s, d, L, plan, xop, act);
    LAUNCH_COUNT(launches);
}

void moe_launch_down(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const uint8_t *dop, float *eo,
                     int max_chunks, cudaStream_t s, uint64_t *launches) {
    const int max_items = max_chunks * (d.H / DN_ROWS);
    int grid = 2 * ex_num_sms();
    if (grid > max_items) grid = max_items;
    if (grid < 1) grid = 1;
    const int nbp = q6r_nb_pad(d.I / MOE_QK);
    const size_t sm6 = (size_t)DN6_NS * DN6_STAGE + 2 * (size_t)DN_ROWS * 2 * nbp + 128;
    const size_t sm4 = (size_t)DN4_NS * DN4_STAGE + 128;
    static size_t attr6[MOE_MAX_DEVICES], attr4[MOE_MAX_DEVICES];
    moe_smem_limit(k_down<MOE_TYPE_Q6_K>, sm6, attr6);
    moe_smem_limit(k_down<MOE_TYPE_Q4_K>, sm4, attr4);
    if (L.down_type == MOE_TYPE_Q6_K || L.sh_down_type == MOE_TYPE_Q6_K) {
        moe_launch_pdl(k_down<MOE_TYPE_Q6_K>, dim3(grid), dim3(EX_THREADS), sm6, s, d, L, plan, dop, eo);
        LAUNCH_COUNT(launches);
    }
    if (L.down_type == MOE_TYPE_Q4_K || L.sh_down_type == MOE_TYPE_Q4_K) {
        moe_launch_pdl(k_down<MOE_TYPE_Q4_K>, dim3(grid), dim3(EX_THREADS), sm4, s, d, L, plan, dop, eo);
        LAUNCH_COUNT(launches);
    }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
typedef CUresult (*moe_encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                        const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                        CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                        CUtensorMapFloatOOBfill);
static moe_encode_tiled_fn encode_fn() {
    static moe_encode_tiled_fn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (moe_encode_tiled_fn)p;
    }
    return fn;
}

// 3-D byte map [slots][rows][row_bytes] with a box of box_x bytes x box_y rows.
static int map3(CUtensorMap *m, const void *base, uint64_t row_bytes, uint64_t rows, uint64_t slots,
                uint64_t slot_stride, uint32_t box_x, uint32_t box_y) {
    moe_encode_tiled_fn fn = encode_fn();
    if (!fn) return -1;
    const cuuint64_t dims[3] = {row_bytes, rows, slots};
    const cuuint64_t strides[2] = {row_bytes, slot_stride};
    const cuuint32_t box[3] = {box_x, box_y, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -(int)r - 100;
}

int moe_make_map_f16_sw128(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                           uint32_t box_rows) {
    moe_encode_tiled_fn fn = encode_fn();
    if (!fn) return -1;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -(int)r - 100;
}

int moe_make_layer_maps(MoeLayerDev &L, const MoeDims &d) {
    const int H = d.H, I = d.I, NBh = H / MOE_QK, NBi = I / MOE_QK;
    const uint64_t slots = (uint64_t)L.n_local + 1;
    int rc = map3(&L.tm_gu, L.experts, (uint64_t)NBh * MOE_Q4K_BYTES, 2ull * I, slots, L.expert_stride,
                  MOE_Q4K_BYTES, GU_ROWS);
    if (rc) return rc;
    const uint8_t *down = L.experts + 2 * L.gate_bytes;
    if (L.down_type == MOE_TYPE_Q4_K || L.sh_down_type == MOE_TYPE_Q4_K) {
        rc = map3(&L.tm_d4, down, (uint64_t)NBi * MOE_Q4K_BYTES, H, slots, L.expert_stride, MOE_Q4K_BYTES, DN_ROWS);
        if (rc) return rc;
    }
    if (L.down_type == MOE_TYPE_Q6_K || L.sh_down_type == MOE_TYPE_Q6_K) {
        const int nbp = q6r_nb_pad(NBi);
        rc = map3(&L.tm_d6q, down, (uint64_t)NBi * 192, H, slots, L.expert_stride, 192, DN_ROWS);
        if (!rc)
            rc = map3(&L.tm_d6s, down + q6r_plane_s_off(H, NBi), (uint64_t)NBi * 16, H, slots, L.expert_stride, 16,
                      DN_ROWS);
        if (!rc)
            rc = map3(&L.tm_d6d, down + q6r_plane_d_off(H, NBi), (uint64_t)nbp * 2, H, slots, L.expert_stride,
                      (uint32_t)nbp * 2, DN_ROWS);
        // the prefill copies 208 bytes per row (the super-block plus 16 bytes it
        // ignores), so that rows land 208 B apart: eight consecutive rows on
        // distinct 16-byte bank groups
        if (!rc) rc = map3(&L.tm_pf6q, down, (uint64_t)NBi * 192, H, slots, L.expert_stride, 208, DN_ROWS);
        if (rc) return rc;
    }
    return 0;
}
