// moe_umma.cuh -- the fifth-generation tensor-core (tcgen05) pieces used by
// the prefill GEMMs and the busy-expert kernels: tensor-memory allocation,
// shared-memory matrix descriptors for K-major 128-byte-swizzled tiles, the
// instruction descriptor of kind::f16, the MMA, its commit to an mbarrier,
// the tensor-memory loads and stores, and the mbarrier / TMA hand-offs of
// their pipelines.  Field layouts follow the PTX ISA for sm_100a (the same
// encodings CUTLASS writes in cute/arch/mma_sm100_desc.hpp).
#pragma once
#include <cuda.h>
#include <stdint.h>

// ---------------------------------------------------------------------------
// Shared-memory tiles.  A K-major operand tile of R rows x 64 fp16 (one
// 128-byte line per row) is stored as R/8 atoms of 8 rows x 128 B (1024 B
// apart); inside an atom the 16-byte chunk c of row r sits at chunk
// c ^ (r % 8) (the 128-byte swizzle, which TMA's SWIZZLE_128B writes too).
// Tiles start on a 1024-byte boundary.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
    const int chunk = (k >> 3) ^ (row & 7);
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + chunk * 16 + (k & 7) * 2);
}

// Matrix descriptor: start address >> 4 in [0,14), leading byte offset >> 4
// in [16,30) (unused by swizzled K-major tiles: 1), stride byte offset >> 4
// in [32,46) (1024 B between 8-row atoms), version 1 in [46,48), layout type
// in [61,64) (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    uint64_t d = (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor of kind::f16: D fp32 (bits 4-5 = 1), A and B fp16
// (formats 0), both K-major, N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t umma_smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one elected thread.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// Arrives on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     umma_smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// Whole warp: allocate / free `ncols` tensor-memory columns (power of two,
// >= 32); the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(umma_smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(ncols) : "memory");
}

// 16 consecutive fp32 columns of this thread's lane (warp w reads lanes
// 32 (w % 4) .. + 31; addr = base + (lane0 << 16) + column).
__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (the tensor core reading an operand tile).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T (A from tensor memory: row m in lane m,
// K elements packed two fp16 per 32-bit column, k = 2c in the low half of
// column c), one elected thread.
__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's lane (warp w writes lanes
// 32 (w % 4) .. + 31; addr = base + (lane0 << 16) + column); asynchronous
// until tmem_wait_st.
__device__ __forceinline__ void tmem_st32(uint32_t addr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(addr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
// 8 consecutive 32-bit columns of this thread's lane (see tmem_st32)
__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(addr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// Warp-wide forms: every lane of the warp executes them with the same
// operands (so the operands stay in uniform registers) and one elected lane
// issues the instruction.  An MMA loop written this way issues at the tensor
// core's rate; the same loop run by one lane inside a divergent branch pays
// ~90 cycles per MMA.
__device__ __forceinline__ void umma_f16_ta_warp(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// The elected lane (the same one as for the MMAs) commits: `bar` receives
// one arrival when every MMA issued so far has completed.
__device__ __forceinline__ void umma_commit_warp(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(
            umma_smem_u32(bar))
        : "memory");
}
// 1 in exactly one lane of the (converged) warp
__device__ __forceinline__ uint32_t elect_one() {
    uint32_t e;
    asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}\n" : "=r"(e));
    return e;
}

// A and B both from shared memory, warp-wide form (see umma_f16_ta_warp).
__device__ __forceinline__ void umma_f16_warp(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// ---------------------------------------------------------------------------
// Pipeline hand-offs of the tcgen05 kernels: mbarriers whose waits give up
// after about a second (the caller records an error instead of hanging), and
// TMA tile loads that complete on an mbarrier.
// ---------------------------------------------------------------------------
#define TC_WAIT_CYCLES (1ll << 31)
#define TC_SUSPEND_NS 1000000u  // a waiting thread sleeps up to 1 ms per try (woken when the phase completes)

__device__ __forceinline__ void tc_mbar_init(uint64_t *b, int n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(umma_smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void tc_expect(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(umma_smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void tc_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(umma_smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool tc_wait(uint64_t *b, uint32_t parity) {
    {
        // completed phases (the common case in a pipeline that keeps up) cost
        // one non-blocking test, without the suspend hint and the clock read
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(umma_smem_u32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(umma_smem_u32(b)), "r"(parity), "r"(TC_SUSPEND_NS)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > TC_WAIT_CYCLES) return false;
    }
}
// after a producer gave up: wait (bounded) for the copies it issued into
// the last `ns` stages of a ring, so that none lands after the CTA exits
__device__ __forceinline__ void tc_drain(uint64_t *full, int issued, int ns) {
    for (int k = issued > ns ? issued - ns : 0; k < issued; k++) tc_wait(&full[k % ns], (k / ns) & 1);
}
// the same, agreed by the whole warp (a lane that gave up fails them all)
__device__ __forceinline__ bool tc_wait_warp(uint64_t *b, uint32_t parity) {
    return __all_sync(0xffffffffu, tc_wait(b, parity));
}
__device__ __forceinline__ void tc_tma3(void *dst, const CUtensorMap *m, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];\n" ::"r"(umma_smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(umma_smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_tma2(void *dst, const CUtensorMap *m, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
            "r"(umma_smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(umma_smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cta_group::2).  Two CTAs of a 2-CTA cluster run on the two SMs
// of one TPC; one tcgen05.mma.cta_group::2 issued by the even CTA (the
// leader) computes M = 256 rows: A rows 0-127 from the leader's tensor
// memory and 128-255 from the peer's (the same column address in both), B
// columns 0 .. N/2 - 1 from the leader's shared memory and N/2 .. N - 1 from
// the peer's (the same shared address in both), and D rows 0-127 / 128-255
// into the leader's / the peer's tensor memory, all N columns in each.  Every
// tcgen05 instruction of such a kernel uses cta_group::2.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
// every thread of both CTAs; orders the mbarrier inits and the tensor-memory
// allocation of each CTA before any access from the other one
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// the shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_map(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(umma_smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t cluster_ld_u32(uint32_t cluster_addr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];\n" : "=r"(v) : "r"(cluster_addr) : "memory");
    return v;
}
// one arrival on an mbarrier of either CTA of the pair (cluster address).  The
// default (CTA-scope) semantics: a cluster-scope release here costs a memory
// barrier per arrival.  Tensor-memory stores are ordered for the MMA that the
// other CTA issues by tcgen05.wait::st + tcgen05.fence::before_thread_sync
// before the arrival and tcgen05.fence::after_thread_sync after the wait.
__device__ __forceinline__ void tc_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_addr) : "memory");
}
// 2D tile load into this CTA's shared memory whose completion (complete_tx)
// is signalled on an mbarrier of either CTA of the pair (cluster address)
__device__ __forceinline__ void tc_tma2_pair(void *dst, const CUtensorMap *m, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(umma_smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
// tensor memory of the pair: the same warp index in both CTAs allocates / frees
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(umma_smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_free_pair(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(ncols) : "memory");
}
// leader only, warp-wide form (see umma_f16_ta_warp): D (+)= A[tmem] * B[smem]^T over the pair
__device__ __forceinline__ void umma_f16_ta_pair_warp(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b,
                                                      uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}\n" ::"r"(
            tmem_d),
        "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// leader only, elected lane: one arrival on `bar` (the same shared address)
// in both CTAs once every pair MMA issued so far has completed
__device__ __forceinline__ void umma_commit_pair_warp(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}\n" ::
            "r"(umma_smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}
