// moe_experts_tc.cu -- the grouped expert products of the busy experts
// (chunks of MOE_TC + 1 .. MOE_CHUNK_MAX tokens) on the fifth-generation
// tensor cores:
//
//   gate/up   act[p][i] = silu(Wg[e] x) * (Wu[e] x)   Q4_K  (infer.m:1564-1568,
//             silu_mul infer.m:378-383)
//   down      eo[p][h]  = Wd[e] act[p]                Q6_K or Q4_K (infer.m:1570)
//
// The arithmetic is that of the GEMVs' fp16 path (moe_experts.cu), so the
// products are exact: the weight integers times their 6-bit sub-block scale
// are exact fp16 values (Q4_K: q sc <= 945; Q6_K: (q - 32) sc as the rounded
// product P plus its exact residual R), the activations are the fp16 hi/lo
// planes of the operand rows (moe_common.cuh: 22 significant bits, a power-
// of-two scale per super-block), and the tensor core accumulates in fp32.
// What changes is the engine: a 128-row slice of one expert's weights is the
// A operand, written by the dequantizing warps straight into tensor memory,
// and one tcgen05.mma multiplies it with all of a chunk's tokens (N = 16 or
// 32), so each weight is decoded once per chunk of up to 32 tokens.  With A
// in tensor memory an M = 128, K = 16 MMA costs about N / 2 cycles (16 at
// N = 32, the dense fp16 peak), so the MMA warp issues from precomputed
// descriptors in unrolled code.
//
// Per super-block (256 weights of K) the MMAs leave, per row and token,
//   D   = sum_k A_k (x_hi,k + x_lo,k)            (Q6_K: + R_k x_hi,k)
//   Dn  = sum_j m_j (xsum_hi,j + xsum_lo,j)      (Q4_K: the sub-block sums / 32)
// in tensor memory, and read-back warps fold them into fp32 registers:
//   acc += (1 / s) (d D - 32 dmin Dn)            (Q6_K: (1 / s) d D)
// which is quant.c's w = d sc q - dmin m (quant.c:36-61) and w = d sc (q - 32)
// (quant.c:63-92) dotted with x.
//
// CTA (one per SM, persistent) = 15 warps:
//   warp 0      raw weight super-blocks by TMA, a ring of TC_RNS stages
//   warp 1      tensor memory owner and MMA issuer (one elected lane)
//   warp 2      the activation planes by TMA (128-byte swizzle): per super-
//               block 4 x_hi boxes, 4 x_lo boxes and the sums / scale box,
//               32 pair rows each, a ring of TC_NSB stages
//   warps 3-10  warp (q, gp) dequantizes atoms 2 gp, 2 gp + 1 (64 weights
//               each) of the 32 rows of lane quarter q into tensor memory
//   warps 11-14 warp q reads back its 32 rows' accumulators, all token
//               columns, after each super-block, and writes the outputs
// Work items (chunk, row block) are dealt to the CTAs in turn; every role
// walks the same items.  All hand-offs are mbarriers whose waits give up
// after about a second and record an error instead of hanging; a producer
// that gives up waits (bounded) for the copies it issued, and the MMA warp
// for the MMAs it issued, before tensor memory is freed.
#include <cuda.h>
#include <stdio.h>

#include "../../include/moe_cuda.h"
#include "moe_common.cuh"
#include "moe_internal.h"
#include "moe_umma.cuh"

#define TC_M 128                     // accumulator rows of an item (MMA M)
#define TC_BOX_ROWS 32               // pair rows of an activation box (MMA N <= 32)
#define TC_BOX (TC_BOX_ROWS * 128)   // 64 fp16 of K x 32 rows
#define TC_BSTAGE (9 * TC_BOX)       // (x_hi, x_lo) of atoms 0-3, then sums / scale
#define TC_NSB_MAX 4                 // activation stages (Q4_K modes: 4, Q6_K: 3, for shared memory)
#ifndef TC_RNS
#define TC_RNS 3
#endif
#define TC_DQ_WARP0 3
#define TC_DQ_WARPS 8                // warps 3-10: dequantization
#define TC_RB_WARPS 4                // warps 11-14: read-back
#define TC_THREADS (32 * (TC_DQ_WARP0 + TC_DQ_WARPS + TC_RB_WARPS))
#define TC_Q6_ROW 208                             // Q6_K Q-plane row stride in shared memory (192 B used)
#define TC_RAW_Q4 (TC_M * MOE_Q4K_BYTES)          // 128 Q4_K rows of one super-block
#define TC_RAW_Q6Q (TC_M * TC_Q6_ROW)             // Q plane of 128 Q6_K rows, then 16 scale bytes per row,
#define TC_RAW_Q6S (TC_M * 16)                    // then the rows' d planes (2 nb_pad bytes each)
#define TC_ERR_TIMEOUT 0x7400                     // plan.error code: a wait of this kernel gave up
// tensor-memory columns: accumulator buffer b at 128 b holds D (64 columns:
// the x_hi products of the 32 pair rows, then the x_lo products), Dn (32
// columns at + 64) and the min-term A of the super-block it serves (8 columns
// at + 96); the A stages follow at 256 (Q4_K: two super-blocks of 4 atoms x
// 32 columns; Q6_K: one of 4 atoms x (P + R = 64))
#define TC_TM_A 256
#define TC_TM_COLS 512

// MODE 0: gate/up (Q4_K, 64 gate rows + the matching 64 up rows per item,
// SwiGLU at the end); 1: down Q4_K; 2: down Q6_K (128 rows of H per item)
template <int MODE>
struct TcCfg {
    static constexpr bool Q6 = MODE == 2;
    static constexpr int NSS = Q6 ? 1 : 2;  // A stages of a whole super-block (4 atoms each)
    static constexpr int NSB = Q6 ? 3 : 4;  // activation stages
    static constexpr int A_COLS = Q6 ? 64 : 32;
};

struct TcItem {
    int rb, slot, p0, ntok;
};

// Item `item` of the plan: (chunk chunk_order[item / n_rb], row block
// item % n_rb).  False when the chunk's down matrix is not of this MODE's
// type (the other down kernel takes it).
template <int MODE>
__device__ __forceinline__ bool tc_item(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, int n_rb, int item,
                                        TcItem &it) {
    const int c = plan.chunk_order[item / n_rb];
    const int e = plan.chunk_expert[c];
    it.rb = item % n_rb;
    it.slot = e == d.E ? L.n_local : e - L.e0;
    it.p0 = plan.chunk_pair0[c];
    it.ntok = plan.chunk_ntok[c];
    if (MODE == 0) return true;
    const int ty = e == d.E ? L.sh_down_type : L.down_type;
    return ty == (MODE == 2 ? MOE_TYPE_Q6_K : MOE_TYPE_Q4_K);
}

// ---------------------------------------------------------------------------
// Dequantization into A columns.  Atom g of a super-block is its weights
// [64 g, 64 g + 64), in the operand's lane order (moe_common.cuh): A column c
// holds positions 2c, 2c + 1 (low half first).
//
// Q4_K (repacked block, quant.c:36-61): the lane words w[2t], w[2t + 1] are
// old qs bytes 32 g + 8 t .. + 7; low nibbles are sub-block 2g, element
// 8 t + i, high nibbles sub-block 2g + 1.  Style Q4 puts element 8 t + i at
// position 8 t + perm(i), perm = 0 2 1 3 4 6 5 7: positions (0, 1) hold
// bytes (0, 2) of the word, (2, 3) bytes (1, 3).  A = fma(1024 + q, sc,
// -1024 sc) = q sc exactly (high nibbles: 1024 + 16 q, sc / 16, -64 sc).
// sl / sh = (sc, sc) of the low / high sub-block as fp16 pairs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_deq_q4(const uint32_t (&w)[8], uint32_t sl, uint32_t sh, uint32_t (&v)[32]) {
    const uint32_t nl = hmul2u(sl, H2_M1024), nh = hmul2u(sh, H2_M64), sh16 = hmul2u(sh, H2_16TH);
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t W = w[2 * t + h], Ws = W >> 8;
            v[4 * t + 2 * h] = hfma2u((W & 0x000F000Fu) | H2_1024, sl, nl);
            v[4 * t + 2 * h + 1] = hfma2u((Ws & 0x000F000Fu) | H2_1024, sl, nl);
            v[16 + 4 * t + 2 * h] = hfma2u((W & 0x00F000F0u) | H2_1024, sh16, nh);
            v[16 + 4 * t + 2 * h + 1] = hfma2u((Ws & 0x00F000F0u) | H2_1024, sh16, nh);
        }
}

// Q6_K atom G (sub-blocks 4 G + s4) of one row, repacked (moe_common.cuh):
// q[6 t + s4] holds elements 4 t .. 4 t + 3 of sub-block s4 (low nibbles for
// even G, high for odd), q[6 t + 4 + (s4 & 1)] their high bits (the high bit
// of every pair stored inverted, so nib | qh2 << 4 is q ^ 32).  Style Q6 puts
// element 4 t + i of sub-block s4 at atom position 32 (s4 / 2) + 8 t +
// 4 (s4 % 2) + i.  Q = (1024 + q) - 1056 = q - 32 exactly, P = fp16(Q sc),
// R = fma(Q, sc, -P) (|R| <= 1, exact); sc4 = the atom's four int8 scales.
template <int G>
__device__ __forceinline__ void tc_deq_q6(const uint32_t (&q)[24], uint32_t sc4, uint32_t (&vp)[32],
                                          uint32_t (&vr)[32]) {
    const uint32_t sw = sc4 ^ 0x80808080u;  // bytes sc + 128: under 0x64 they are 1152 + sc
#pragma unroll
    for (int s4 = 0; s4 < 4; s4++) {
        uint32_t sc;
        switch (s4) {
            case 0: sc = byte_h2<0>(sw, H2_1152); break;
            case 1: sc = byte_h2<1>(sw, H2_1152); break;
            case 2: sc = byte_h2<2>(sw, H2_1152); break;
            default: sc = byte_h2<3>(sw, H2_1152); break;
        }
        const int sp = 4 * (G & 1) + s4, f = sp >> 1;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t W = q[6 * t + s4], Hq = q[6 * t + 4 + (s4 & 1)];
            const uint32_t nib = (sp < 4 ? W : W >> 4) & 0x0F0F0F0Fu;
            const uint32_t hb = (2 * f <= 4 ? Hq << (4 - 2 * f) : Hq >> (2 * f - 4)) & 0x30303030u;
            const uint32_t q6 = nib | (hb ^ 0x20202020u);  // four values q (0..63) in bytes
            const uint32_t q01 = hsub2u(prmt(q6, 0x64u, 0x4140u), H2_1056);  // q - 32, exact
            const uint32_t q23 = hsub2u(prmt(q6, 0x64u, 0x4342u), H2_1056);
            const int col = 16 * (s4 >> 1) + 4 * t + 2 * (s4 & 1);
            vp[col] = hmul2u(q01, sc);
            vp[col + 1] = hmul2u(q23, sc);
            vr[col] = hfma2u(q01, sc, vp[col] ^ 0x80008000u);  // Q sc - P
            vr[col + 1] = hfma2u(q23, sc, vp[col + 1] ^ 0x80008000u);
        }
    }
}

// The MMAs of one super-block: per atom a and K step kk, one N = 64 MMA
// over the atom's x_hi box and the x_lo box right after it (D columns 0-31:
// A x_hi, 32-63: A x_lo; Q6_K adds R x_hi into columns 0-31 with N = n),
// K = 16 per MMA, then (Q4_K) the min term Dn = (m_j, m_j) x (xsum_hi,j,
// xsum_lo,j).  Straight-line code with compile-time offsets from warp-
// uniform bases: ta0 = the step's first A atom, bdesc = the B stage's
// descriptor (a 16-byte step of its start address is +1, so +32 B is +2 and
// a 4096-byte box is +256); idesc64 / idescn = N 64 / the chunk's N.
template <bool Q6, int A_COLS>
__device__ __forceinline__ void tc_mma_step(uint32_t dm, uint32_t dn, uint32_t ta0, uint32_t tmin, uint64_t bdesc,
                                            uint32_t idesc64, uint32_t idescn) {
#pragma unroll
    for (int a = 0; a < 4; a++) {
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const uint32_t ta = ta0 + A_COLS * a + 8 * kk;
            const uint64_t bh = bdesc + (uint64_t)(256 * 2 * a + 2 * kk);
            umma_f16_ta_warp(dm, ta, bh, idesc64, (a | kk) ? 1u : 0u);
            if (Q6) umma_f16_ta_warp(dm, ta + 32, bh, idescn, 1u);
        }
    }
    if (!Q6) umma_f16_ta_warp(dn, tmin, bdesc + (uint64_t)(256 * 8), idescn, 0u);
}

// ===========================================================================
// The kernel.  blockIdx.x deals items blockIdx.x, + gridDim.x, ...; tmB maps
// the operand rows of the pairs (xtc for gate/up, dop for down); out = act
// (MODE 0, [pair][I]) or eo ([pair][H]).
// ===========================================================================
template <int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_experts_tc(MoeDims d, const __grid_constant__ MoeLayerDev L, MoePlan plan,
                 const __grid_constant__ CUtensorMap tmB, float *__restrict__ out) {
    using C = TcCfg<MODE>;
    extern __shared__ uint8_t tc_raw_smem[];
    uint8_t *sm = tc_raw_smem + ((1024u - (umma_smem_u32(tc_raw_smem) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t raw_full[TC_RNS], raw_empty[TC_RNS], b_full[TC_NSB_MAX], b_empty[TC_NSB_MAX],
        a_full[2], a_empty[2], d_full[2], d_empty[2], fin;
    __shared__ uint32_t tmem_base;
    // per step: 1/s of the box's 32 pair rows (written by the MMA warp), and
    // d, 32 dmin (Q4_K) or d (Q6_K) of the 128 rows (written by the dequant
    // warps of atom pair 0)
    __shared__ __align__(16) float inv_buf[2][TC_BOX_ROWS];
    __shared__ __align__(16) float2 dbuf[4][TC_M];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = MODE == 0 ? d.H : d.I, NB = K / MOE_QK, nbp = q6r_nb_pad(NB);
    const int n_rb = MODE == 0 ? d.I / 64 : d.H / TC_M;
    const int RAW = C::Q6 ? TC_RAW_Q6Q + TC_RAW_Q6S + TC_M * 2 * nbp : TC_RAW_Q4;
    uint8_t *sb_ring = sm, *raw_ring = sm + C::NSB * TC_BSTAGE;

    // the plan comes from earlier kernels; no tensor memory is touched before
    // they have finished
    moe_pdl_wait();
    const int n_items = plan.counts[3] * n_rb;
    if ((int)blockIdx.x >= n_items) return;
    if (tid == 0) {
        for (int i = 0; i < TC_RNS; i++) { tc_mbar_init(&raw_full[i], 1); tc_mbar_init(&raw_empty[i], TC_DQ_WARPS); }
        for (int i = 0; i < C::NSB; i++) { tc_mbar_init(&b_full[i], 1); tc_mbar_init(&b_empty[i], 1); }
        // one A hand-off per super-block: every dequant warp arrives once
        for (int i = 0; i < 2; i++) { tc_mbar_init(&a_full[i], TC_DQ_WARPS); tc_mbar_init(&a_empty[i], 1); }
        // d_full: the MMAs' commit + the MMA warp's own arrival after it wrote
        // inv_buf (and had seen the dequant warps' dbuf through a_full)
        for (int i = 0; i < 2; i++) { tc_mbar_init(&d_full[i], 2); tc_mbar_init(&d_empty[i], TC_RB_WARPS); }
        tc_mbar_init(&fin, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&tmem_base, TC_TM_COLS);
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    moe_pdl_trigger();
    const uint32_t tmem = __shfl_sync(0xffffffffu, tmem_base, 0);
    bool ok = true;

    if (warp == 0) {
        // raw weight super-blocks, TC_RNS ahead
        const uint32_t leader = elect_one();
        int s = 0;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            TcItem it;
            if (!tc_item<MODE>(d, L, plan, n_rb, item, it)) continue;
            for (int sbk = 0; sbk < NB; sbk++, s++) {
                const int rs = s % TC_RNS;
                if (!tc_wait_warp(&raw_empty[rs], ((s / TC_RNS) & 1) ^ 1)) { ok = false; break; }
                uint8_t *r = raw_ring + (size_t)rs * RAW;
                if (leader) {
                    tc_expect(&raw_full[rs], RAW);
                    if (MODE == 0) {
                        tc_tma3(r, &L.tm_gu, sbk * MOE_Q4K_BYTES, it.rb * 64, it.slot, &raw_full[rs]);
                        tc_tma3(r + 64 * MOE_Q4K_BYTES, &L.tm_gu, sbk * MOE_Q4K_BYTES, d.I + it.rb * 64, it.slot,
                                &raw_full[rs]);
                    } else if (MODE == 1) {
                        tc_tma3(r, &L.tm_d4, sbk * MOE_Q4K_BYTES, it.rb * TC_M, it.slot, &raw_full[rs]);
                    } else {
                        tc_tma3(r, &L.tm_pf6q, sbk * 192, it.rb * TC_M, it.slot, &raw_full[rs]);
                        tc_tma3(r + TC_RAW_Q6Q, &L.tm_d6s, sbk * 16, it.rb * TC_M, it.slot, &raw_full[rs]);
                        tc_tma3(r + TC_RAW_Q6Q + TC_RAW_Q6S, &L.tm_d6d, 0, it.rb * TC_M, it.slot, &raw_full[rs]);
                    }
                }
            }
        }
        if (!ok && leader) {
            atomicExch(plan.error, TC_ERR_TIMEOUT);
            tc_drain(raw_full, s, TC_RNS);
        }
    } else if (warp == 2) {
        // activation planes of the chunk's pairs (rows p0 .. p0 + 31; rows past
        // the chunk belong to other chunks and only reach columns nobody reads)
        const uint32_t leader = elect_one();
        int s = 0;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            TcItem it;
            if (!tc_item<MODE>(d, L, plan, n_rb, item, it)) continue;
            for (int sbk = 0; sbk < NB; sbk++, s++) {
                const int st = s % C::NSB;
                if (!tc_wait_warp(&b_empty[st], ((s / C::NSB) & 1) ^ 1)) { ok = false; break; }
                uint8_t *b = sb_ring + (size_t)st * TC_BSTAGE;
                if (leader) {
                    tc_expect(&b_full[st], TC_BSTAGE);
                    const int x0 = sbk * (OPW_SB / 2);
#pragma unroll
                    for (int a = 0; a < 4; a++) {
                        tc_tma2(b + 2 * a * TC_BOX, &tmB, x0 + 64 * a, it.p0, &b_full[st]);
                        tc_tma2(b + (2 * a + 1) * TC_BOX, &tmB, x0 + OPW_LO / 2 + 64 * a, it.p0, &b_full[st]);
                    }
                    tc_tma2(b + 8 * TC_BOX, &tmB, x0 + OPW_XSUM / 2, it.p0, &b_full[st]);
                }
            }
        }
        if (!ok && leader) {
            atomicExch(plan.error, TC_ERR_TIMEOUT);
            tc_drain(b_full, s, C::NSB);
        }
    } else if (warp == 1) {
        // MMA issuer: the whole warp runs the loop (uniform operands), one
        // elected lane issues each MMA and commit.  Every MMA operand is
        // broadcast from lane 0 and the MMAs of a step are straight-line code
        // with compile-time offsets, so that the operands stay in uniform
        // registers: operands the compiler cannot prove uniform made each MMA
        // several times slower to issue than the tensor core runs it.
        int s = 0;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            TcItem it;
            if (!tc_item<MODE>(d, L, plan, n_rb, item, it)) continue;
            // N = the chunk's tokens rounded up to 16 (M = 128 takes N = 16, 32)
            const uint32_t idescn = __shfl_sync(0xffffffffu, umma_idesc_f16(TC_M, (it.ntok + 15) & ~15), 0);
            constexpr uint32_t idesc64 = umma_idesc_f16(TC_M, 64);
            for (int sbk = 0; sbk < NB && ok; sbk++, s++) {
                const int st = s % C::NSB, db = s & 1;
                if (!tc_wait_warp(&b_full[st], (s / C::NSB) & 1) ||
                    !tc_wait_warp(&d_empty[db], ((s >> 1) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                uint8_t *bst = sb_ring + (size_t)st * TC_BSTAGE;
                // 1/s of pair row `lane`: fp32 at byte OPW_SCALE - OPW_XSUM = 32 of the sums box row
                inv_buf[db][lane] = *reinterpret_cast<const float *>(bst + 8 * TC_BOX + sw128_offset(lane, 16));
                // the step's four A atoms
                const int ss = s % C::NSS;
                if (!tc_wait_warp(&a_full[ss], (s / C::NSS) & 1)) { ok = false; break; }
                tmem_fence_after();
                const uint64_t bdesc = umma_desc_sw128(__shfl_sync(0xffffffffu, umma_smem_u32(bst), 0));
                const uint32_t dm = __shfl_sync(0xffffffffu, tmem + 128 * db, 0);
                const uint32_t ta0 = __shfl_sync(0xffffffffu, tmem + TC_TM_A + C::A_COLS * 4 * ss, 0);
                tc_mma_step<C::Q6, C::A_COLS>(dm, dm + 64, ta0, dm + 96, bdesc, idesc64, idescn);
                umma_commit_warp(&a_empty[ss]);
                umma_commit_warp(&b_empty[st]);
                umma_commit_warp(&d_full[db]);
                __syncwarp();
                if (lane == 0) tc_arrive(&d_full[db]);
            }
        }
        // teardown: every MMA issued has completed before tensor memory is freed
        umma_commit_warp(&fin);
        if (!ok && lane == 0) atomicExch(plan.error, TC_ERR_TIMEOUT);
        tc_wait_warp(&fin, 0);
    } else if (warp < TC_DQ_WARP0 + TC_DQ_WARPS) {
        // dequantization: warp (q, gp) owns tensor-memory lanes 32 q .. + 31
        // (A rows; lane = row; a warp reaches the lanes of its own index mod 4
        // only) and atoms 2 gp, 2 gp + 1 of every super-block
        const int q = warp & 3, gp = (warp - TC_DQ_WARP0) >> 2, row = 32 * q + lane;
        int rraw = row;  // raw tile row holding A row `row`
        if (MODE == 0) {
            const int h = (row >> 4) & 1, i = row & 15;  // row = 32 q + 16 h + i
            rraw = h * 64 + 16 * q + i;                   // gate rows first, then up rows
        }
        const uint32_t tlane = (uint32_t)(32 * q) << 16;
        int s = 0;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            TcItem it;
            if (!tc_item<MODE>(d, L, plan, n_rb, item, it)) continue;
            for (int sbk = 0; sbk < NB; sbk++, s++) {
                const int rs = s % TC_RNS;
                if (!tc_wait_warp(&raw_full[rs], (s / TC_RNS) & 1)) { ok = false; break; }
                const uint8_t *r = raw_ring + (size_t)rs * RAW;
                if constexpr (C::Q6) {
                    // atoms 2 gp, 2 gp + 1 lie in half gp of every 48-byte lane chunk
                    uint32_t w[24];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        const uint8_t *cp = r + rraw * TC_Q6_ROW + 48 * t;
                        if (gp == 0) {
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
                    const uint2 sc8 = *reinterpret_cast<const uint2 *>(r + TC_RAW_Q6Q + rraw * 16 + 8 * gp);
                    const float d6 =
                        __half2float(reinterpret_cast<const __half *>(r + TC_RAW_Q6Q + TC_RAW_Q6S)[rraw * nbp + sbk]);
                    // the stage's reads are done (their values are in registers); the
                    // arrive orders them before the producer's next TMA write into it
                    __syncwarp();
                    if (lane == 0) tc_arrive(&raw_empty[rs]);
                    const int ss = s % C::NSS;
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        uint32_t vp[32], vr[32];
                        if (gp == 0) {
                            if (half == 0) tc_deq_q6<0>(w, sc8.x, vp, vr);
                            else tc_deq_q6<1>(w, sc8.y, vp, vr);
                        } else {
                            if (half == 0) tc_deq_q6<2>(w, sc8.x, vp, vr);
                            else tc_deq_q6<3>(w, sc8.y, vp, vr);
                        }
                        if (half == 0) {
                            if (!tc_wait_warp(&a_empty[ss], ((s / C::NSS) & 1) ^ 1)) { ok = false; break; }
                            // (a_empty of step s: the MMAs of step s - 1 were issued, so
                            // read-back s - 3 is done with this dbuf slot)
                            if (gp == 0) dbuf[s & 3][row] = make_float2(d6, 0.0f);
                            tmem_fence_after();
                        }
                        const uint32_t ta = tmem + tlane + TC_TM_A + C::A_COLS * (4 * ss + 2 * gp + half);
                        tmem_st32(ta, vp);
                        tmem_st32(ta + 32, vr);
                        tmem_wait_st();
                    }
                    if (!ok) break;
                    tmem_fence_before();
                    __syncwarp();
                    if (lane == 0) tc_arrive(&a_full[ss]);
                } else {
                    const uint8_t *blk = r + rraw * MOE_Q4K_BYTES;
                    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
                    uint32_t w[2][8];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        // atoms 2 gp and 2 gp + 1: 16 consecutive bytes of lane chunk t
                        const uint4 x = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * t + 16 * gp);
                        w[0][2 * t] = x.x; w[0][2 * t + 1] = x.y;
                        w[1][2 * t] = x.z; w[1][2 * t + 1] = x.w;
                    }
                    __syncwarp();
                    if (lane == 0) tc_arrive(&raw_empty[rs]);
                    // 6-bit scales of the 8 sub-blocks, one per byte (get_scale_min_k4,
                    // quant.c:26-34): sub-blocks 4 gp + 0..3 are bytes 0..3 of
                    // sc_lo (gp 0) or sc_hi (gp 1)
                    const uint32_t scw = gp == 0 ? (hd.y & 0x3F3F3F3Fu)
                                                 : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
                    const int ss = s % C::NSS;
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        uint32_t v[32];
                        if (half == 0) tc_deq_q4(w[0], byte_h2<0>(scw, H2_1024), byte_h2<1>(scw, H2_1024), v);
                        else tc_deq_q4(w[1], byte_h2<2>(scw, H2_1024), byte_h2<3>(scw, H2_1024), v);
                        if (half == 0) {
                            if (!tc_wait_warp(&a_empty[ss], ((s / C::NSS) & 1) ^ 1)) { ok = false; break; }
                            tmem_fence_after();
                        }
                        tmem_st32(tmem + tlane + TC_TM_A + C::A_COLS * (4 * ss + 2 * gp + half), v);
                        if (gp == 0 && half == 0) {
                            // d and 32 dmin (the sums are stored / 32); a_empty of step s
                            // means the MMAs of step s - 2 were issued, so read-back
                            // s - 4 is done with this dbuf slot
                            dbuf[s & 3][row] = make_float2(h2f_bits((uint16_t)(hd.x & 0xFFFFu)),
                                                           32.0f * h2f_bits((uint16_t)(hd.x >> 16)));
                            // the min-term A: (m_j, m_j) for j = 0..7, 16 fp16 = 8 columns
                            const uint32_t mn_lo = hd.z & 0x3F3F3F3Fu;
                            const uint32_t mn_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
                            uint32_t vm[8];
                            vm[0] = vm[4] = hsub2u(prmt(mn_lo, 0x64u, 0x4140u), H2_1024);
                            vm[1] = vm[5] = hsub2u(prmt(mn_lo, 0x64u, 0x4342u), H2_1024);
                            vm[2] = vm[6] = hsub2u(prmt(mn_hi, 0x64u, 0x4140u), H2_1024);
                            vm[3] = vm[7] = hsub2u(prmt(mn_hi, 0x64u, 0x4342u), H2_1024);
                            tmem_st8(tmem + tlane + 128 * (s & 1) + 96, vm);
                        }
                        tmem_wait_st();
                    }
                    if (!ok) break;
                    tmem_fence_before();
                    __syncwarp();
                    if (lane == 0) tc_arrive(&a_full[ss]);
                }
            }
        }
        if (!ok && lane == 0) atomicExch(plan.error, TC_ERR_TIMEOUT);
    } else {
        // read-back: warp q reads tensor-memory lanes 32 q .. + 31 (its own
        // index mod 4), all token columns, after each super-block's MMAs
        const int q = warp & 3, row = 32 * q + lane;
        const uint32_t tlane = (uint32_t)(32 * q) << 16;
        float acc[TC_BOX_ROWS];
#pragma unroll
        for (int j = 0; j < TC_BOX_ROWS; j++) acc[j] = 0.0f;
        int s = 0;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            TcItem it;
            if (!tc_item<MODE>(d, L, plan, n_rb, item, it)) continue;
            const int ncols = (it.ntok + 15) & ~15;
            for (int sbk = 0; sbk < NB; sbk++, s++) {
                const int db = s & 1;
                if (!tc_wait_warp(&d_full[db], (s >> 1) & 1)) { ok = false; break; }
                tmem_fence_after();
                const float2 sc = dbuf[s & 3][row];
#pragma unroll
                for (int hc = 0; hc < TC_BOX_ROWS; hc += 16) {  // 16 token columns at a time
                    if (hc >= ncols) break;
                    float dv[16], nv[16];
                    float lv[16];
                    tmem_ld16(tmem + tlane + 128 * db + hc, dv);
                    tmem_ld16(tmem + tlane + 128 * db + 32 + hc, lv);
                    if (!C::Q6) tmem_ld16(tmem + tlane + 128 * db + 64 + hc, nv);
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        const float4 iv = *reinterpret_cast<const float4 *>(&inv_buf[db][hc + j]);
                        const float ivs[4] = {iv.x, iv.y, iv.z, iv.w};
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            const float dd = dv[j + u] + lv[j + u];
                            const float v = C::Q6 ? sc.x * dd : fmaf(-sc.y, nv[j + u], sc.x * dd);
                            acc[hc + j + u] = fmaf(ivs[u], v, acc[hc + j + u]);
                        }
                    }
                }
                tmem_fence_before();
                __syncwarp();
                if (lane == 0) tc_arrive(&d_empty[db]);
                if (sbk == NB - 1) {
                    // the item's outputs (columns past the chunk's tokens hold
                    // other rows' or stale values and are dropped)
#pragma unroll
                    for (int j = 0; j < TC_BOX_ROWS; j++) {
                        if (MODE == 0) {
                            // lanes 0-15: gate rows, 16-31: the matching up rows
                            const float u = __shfl_xor_sync(0xffffffffu, acc[j], 16);
                            if (lane < 16 && j < it.ntok)
                                out[(size_t)(it.p0 + j) * d.I + it.rb * 64 + 16 * q + lane] =
                                    (acc[j] / (1.0f + expf(-acc[j]))) * u;
                        } else if (j < it.ntok) {
                            out[(size_t)(it.p0 + j) * d.H + it.rb * TC_M + row] = acc[j];
                        }
                        acc[j] = 0.0f;
                    }
                }
            }
        }
        if (!ok && lane == 0) atomicExch(plan.error, TC_ERR_TIMEOUT);
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 1) tmem_free(tmem, TC_TM_COLS);
}

// ===========================================================================
// Operand rows of the tcgen05 chunks' pairs for gate/up: the fp16 part of the
// token's row of xop, copied to row `pair` of xtc (so that a chunk's pairs
// are consecutive rows a TMA box can load).  Block (token slot j, chunk c).
// ===========================================================================
__global__ void __launch_bounds__(256) k_tc_gather(MoeDims d, MoePlan plan, const uint8_t *__restrict__ xop,
                                                   uint8_t *__restrict__ xtc) {
    moe_pdl_wait();
    moe_pdl_trigger();
    const int ci = blockIdx.y, j = blockIdx.x;
    if (ci >= plan.counts[3]) return;
    const int c = plan.chunk_order[ci];
    if (j >= plan.chunk_ntok[c]) return;
    const int p = plan.chunk_pair0[c] + j;
    const size_t n16 = opw_bytes(d.H) / 16;
    const uint4 *src = reinterpret_cast<const uint4 *>(xop + (size_t)plan.pair_token[p] * opx_row(d.H) + op_bytes(d.H));
    uint4 *dst = reinterpret_cast<uint4 *>(xtc + (size_t)p * opw_bytes(d.H));
    for (size_t i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldg(src + i);
}

// ===========================================================================
// host side
// ===========================================================================
static int tc_num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

static size_t tc_smem(int mode, int nbp) {
    const size_t raw = mode == 2 ? (size_t)TC_RAW_Q6Q + TC_RAW_Q6S + (size_t)TC_M * 2 * nbp : (size_t)TC_RAW_Q4;
    return (size_t)(mode == 2 ? 3 : 4) * TC_BSTAGE + (size_t)TC_RNS * raw + 1024;
}

// at most max_pairs / (MOE_TC + 1) chunks of more than MOE_TC pairs
static int tc_grid(int max_pairs, int n_rb) {
    const long items = (long)(max_pairs / (MOE_TC + 1)) * n_rb;
    int grid = tc_num_sms();
    if (grid > items) grid = (int)items;
    return grid;
}

template <int MODE>
static void tc_launch(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const CUtensorMap &tm, float *out,
                      int max_pairs, cudaStream_t s, uint64_t *launches) {
    const int n_rb = MODE == 0 ? d.I / 64 : d.H / TC_M;
    const int grid = tc_grid(max_pairs, n_rb);
    if (grid < 1) return;
    const size_t smem = tc_smem(MODE, q6r_nb_pad((MODE == 0 ? d.H : d.I) / MOE_QK));
    static size_t attr[MOE_MAX_DEVICES];
    moe_smem_limit(k_experts_tc<MODE>, smem, attr);
    moe_launch_pdl(k_experts_tc<MODE>, dim3(grid), dim3(TC_THREADS), smem, s, d, L, plan, tm, out);
    if (launches) (*launches)++;
}

void moe_launch_tc_gather(const MoeDims &d, const MoePlan &plan, const uint8_t *xop, uint8_t *xtc, int max_pairs,
                          cudaStream_t s, uint64_t *launches) {
    const int chunks = max_pairs / (MOE_TC + 1);
    if (chunks < 1) return;
    moe_launch_pdl(k_tc_gather, dim3(MOE_CHUNK_MAX, chunks), dim3(256), 0, s, d, plan, xop, xtc);
    if (launches) (*launches)++;
}

void moe_launch_gateup_tc(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const CUtensorMap &tm_xtc,
                          float *act, int max_pairs, cudaStream_t s, uint64_t *launches) {
    tc_launch<0>(d, L, plan, tm_xtc, act, max_pairs, s, launches);
}

void moe_launch_down_tc(const MoeDims &d, const MoeLayerDev &L, const MoePlan &plan, const CUtensorMap &tm_dop,
                        float *eo, int max_pairs, cudaStream_t s, uint64_t *launches) {
    if (L.down_type == MOE_TYPE_Q6_K || L.sh_down_type == MOE_TYPE_Q6_K)
        tc_launch<2>(d, L, plan, tm_dop, eo, max_pairs, s, launches);
    if (L.down_type == MOE_TYPE_Q4_K || L.sh_down_type == MOE_TYPE_Q4_K)
        tc_launch<1>(d, L, plan, tm_dop, eo, max_pairs, s, launches);
}

int moe_make_map_opw(CUtensorMap *m, const void *base, int K, uint64_t rows) {
    return moe_make_map_f16_sw128(m, base, opw_bytes(K) / 2, rows, 64, TC_BOX_ROWS);
}
