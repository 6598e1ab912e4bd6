// GPU self-test of the tcgen05 building blocks of moe_umma.cuh (built into a
// throw-away shared library by tests/test_gpu_prefill.py): one CTA computes
// C[128 x N] = A[128 x K] * B[N x K]^T in fp16 with fp32 accumulation in
// tensor memory.  A is written into 128-byte-swizzled shared memory by the
// threads (the path the prefill dequantizer takes), B arrives by TMA with
// SWIZZLE_128B.  A second kernel runs the same kind of product on a CTA pair
// (cta_group::2, M = 256).  Every wait is bounded; a timeout sets *err.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../flash_deepseek_b200/csrc/moe_umma.cuh"

#define ST_N 128
#define ST_K 256

__device__ __forceinline__ bool st_wait(uint64_t *b, uint32_t parity) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(umma_smem_u32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > (1ll << 31)) return false;
    }
}

__global__ void __launch_bounds__(128, 1)
    k_umma_selftest(const __grid_constant__ CUtensorMap tmb, const __half *__restrict__ A, float *__restrict__ C,
                    int *err) {
    extern __shared__ uint8_t raw[];
    uint8_t *sm = raw + ((1024u - (umma_smem_u32(raw) & 1023u)) & 1023u);
    uint8_t *sa = sm;                      // 4 atoms x 16 KB
    uint8_t *sb = sm + 4 * 16384;          // 4 atoms x 16 KB
    __shared__ __align__(8) uint64_t bar_b, bar_mma;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(umma_smem_u32(&bar_b)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(umma_smem_u32(&bar_mma)));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    if (warp == 0) tmem_alloc(&tmem_base, 128);
    __syncthreads();
    if (tid == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(umma_smem_u32(&bar_b)),
                     "r"(4 * 16384)
                     : "memory");
        for (int a = 0; a < 4; a++)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
                "[%4];\n" ::"r"(umma_smem_u32(sb + a * 16384)),
                "l"(reinterpret_cast<uint64_t>(&tmb)), "r"(64 * a), "r"(0), "r"(umma_smem_u32(&bar_b))
                : "memory");
    }
    // A: thread = row, 256 fp16 -> 4 atoms
    for (int k = 0; k < ST_K; k += 8) {
        const uint4 v = *reinterpret_cast<const uint4 *>(A + (size_t)tid * ST_K + k);
        *reinterpret_cast<uint4 *>(sa + (k >> 6) * 16384 + sw128_offset(tid, k & 63)) = v;
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
        if (!st_wait(&bar_b, 0)) { atomicExch(err, 1); }
        else {
            tmem_fence_after();
            const uint32_t idesc = umma_idesc_f16(128, ST_N);
            for (int a = 0; a < 4; a++)
                for (int kk = 0; kk < 4; kk++) {
                    const uint64_t da = umma_desc_sw128(umma_smem_u32(sa + a * 16384 + kk * 32));
                    const uint64_t db = umma_desc_sw128(umma_smem_u32(sb + a * 16384 + kk * 32));
                    umma_f16(tmem_base, da, db, idesc, (a | kk) != 0);
                }
            umma_commit(&bar_mma);
        }
    }
    __syncthreads();
    const bool ok = st_wait(&bar_mma, 0);
    if (!ok && tid == 0) atomicExch(err, 2);
    tmem_fence_after();
    if (ok) {
        for (int c = 0; c < ST_N; c += 16) {
            float v[16];
            tmem_ld16(tmem_base + ((uint32_t)(32 * warp) << 16) + c, v);
            for (int i = 0; i < 16; i++) C[(size_t)tid * ST_N + c + i] = v[i];
        }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 0) tmem_free(tmem_base, 128);
}

// The same product with A written into tensor memory by the threads
// (tcgen05.st, thread = row) and read from there by the MMA.
__global__ void __launch_bounds__(128, 1)
    k_umma_selftest_ta(const __grid_constant__ CUtensorMap tmb, const __half *__restrict__ A, float *__restrict__ C,
                       int *err) {
    extern __shared__ uint8_t raw[];
    uint8_t *sb = raw + ((1024u - (umma_smem_u32(raw) & 1023u)) & 1023u);  // 4 atoms x 16 KB
    __shared__ __align__(8) uint64_t bar_b, bar_a, bar_mma;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(umma_smem_u32(&bar_b)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;\n" ::"r"(umma_smem_u32(&bar_a)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(umma_smem_u32(&bar_mma)));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    if (warp == 0) tmem_alloc(&tmem_base, 256);  // D: columns 0-127, A: 128-255
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tm = tmem_base;
    if (tid == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(umma_smem_u32(&bar_b)),
                     "r"(4 * 16384)
                     : "memory");
        for (int a = 0; a < 4; a++)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
                "[%4];\n" ::"r"(umma_smem_u32(sb + a * 16384)),
                "l"(reinterpret_cast<uint64_t>(&tmb)), "r"(64 * a), "r"(0), "r"(umma_smem_u32(&bar_b))
                : "memory");
    }
    // A row `tid` (lane tid of tensor memory): 256 fp16 = 128 columns, 4 stores of 32
    for (int c = 0; c < 4; c++) {
        uint32_t v[32];
        for (int j = 0; j < 32; j++) v[j] = reinterpret_cast<const uint32_t *>(A + (size_t)tid * ST_K)[32 * c + j];
        tmem_st32(tm + ((uint32_t)(32 * warp) << 16) + 128 + 32 * c, v);
    }
    tmem_wait_st();
    tmem_fence_before();
    __syncwarp();
    if ((tid & 31) == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(umma_smem_u32(&bar_a)) : "memory");
    if (tid == 0) {
        if (!st_wait(&bar_b, 0) || !st_wait(&bar_a, 0)) { atomicExch(err, 1); }
        else {
            tmem_fence_after();
            const uint32_t idesc = umma_idesc_f16(128, ST_N);
            for (int a = 0; a < 4; a++)
                for (int kk = 0; kk < 4; kk++) {
                    const uint64_t db = umma_desc_sw128(umma_smem_u32(sb + a * 16384 + kk * 32));
                    umma_f16_ta(tm, tm + 128 + 32 * a + 8 * kk, db, idesc, (a | kk) != 0);
                }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                         umma_smem_u32(&bar_mma))
                     : "memory");
    }
    __syncthreads();
    const bool ok = st_wait(&bar_mma, 0);
    if (!ok && tid == 0) atomicExch(err, 2);
    tmem_fence_after();
    if (ok) {
        for (int c = 0; c < ST_N; c += 16) {
            float v[16];
            tmem_ld16(tm + ((uint32_t)(32 * warp) << 16) + c, v);
            for (int i = 0; i < 16; i++) C[(size_t)tid * ST_N + c + i] = v[i];
        }
    }
    tmem_fence_before();
    __syncthreads();
    if (warp == 0) tmem_free(tm, 256);
}

// CTA pair (cta_group::2): C[256 x N] = A[256 x 256] * B[N x 256]^T.  CTA r
// (cluster rank) writes A rows 128 r .. + 127 into its tensor memory at
// column acol and loads B rows r N / 2 .. + N / 2 - 1 by TMA (16-row boxes,
// completing on the leader's barrier); the leader issues the M = 256 pair
// MMAs into columns dcol .. dcol + N - 1 of both CTAs and commits to both;
// each CTA reads back its own 128 rows of C.  The same hand-offs as the
// prefill GEMM: remote arrivals on the leader's barrier for A, the pair
// form of the B copies, commits that arrive in both CTAs.
#define SP_ATOM 10240  // one K atom of B in a CTA: up to 80 rows x 128 B
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    k_umma_selftest_pair(const __grid_constant__ CUtensorMap tmb, const __half *__restrict__ A,
                         float *__restrict__ C, int N, int dcol, int acol, int *err) {
    extern __shared__ uint8_t raw[];
    uint8_t *sb = raw + ((1024u - (umma_smem_u32(raw) & 1023u)) & 1023u);  // 4 atoms x SP_ATOM
    __shared__ __align__(8) uint64_t bar_b, bar_a, bar_mma;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t rank = cluster_ctarank();
    if (tid == 0) {
        tc_mbar_init(&bar_b, 1);
        tc_mbar_init(&bar_a, 8);
        tc_mbar_init(&bar_mma, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    if (warp == 0) tmem_alloc_pair(&tmem_base, 512);
    tmem_fence_before();
    cluster_sync_all();
    tmem_fence_after();
    const uint32_t tm = tmem_base;
    const bool same = cluster_ld_u32(cluster_map(&tmem_base, rank ^ 1u)) == tm;
    if (!same && tid == 0) atomicExch(err, 3);
    const int half = N / 2;
    if (same) {
        if (tid == 0) {
            if (rank == 0) tc_expect(&bar_b, (uint32_t)(4 * 2 * half * 128));
            const uint32_t bar = cluster_map(&bar_b, 0);
            for (int a = 0; a < 4; a++)
                for (int bx = 0; bx < half / 16; bx++)
                    tc_tma2_pair(sb + a * SP_ATOM + bx * 2048, &tmb, 64 * a, (int)rank * half + 16 * bx, bar);
        }
        // A row 128 rank + tid in lane tid: 256 fp16 = 128 columns, 4 stores of 32
        const uint32_t *arow = reinterpret_cast<const uint32_t *>(A + (size_t)(128 * rank + tid) * 256);
        for (int c = 0; c < 4; c++) {
            uint32_t v[32];
            for (int j = 0; j < 32; j++) v[j] = arow[32 * c + j];
            tmem_st32(tm + ((uint32_t)(32 * warp) << 16) + acol + 32 * c, v);
        }
        tmem_wait_st();
        tmem_fence_before();
        __syncwarp();
        if ((tid & 31) == 0) tc_arrive_cluster(cluster_map(&bar_a, 0));
        if (rank == 0 && warp == 0) {
            const bool ok = tc_wait_warp(&bar_b, 0) && tc_wait_warp(&bar_a, 0);
            if (!ok) {
                if ((tid & 31) == 0) atomicExch(err, 1);
            } else {
                tmem_fence_after();
                const uint32_t idesc = umma_idesc_f16(256, N);
                for (int a = 0; a < 4; a++)
                    for (int kk = 0; kk < 4; kk++)
                        umma_f16_ta_pair_warp(tm + dcol, tm + acol + 32 * a + 8 * kk,
                                              umma_desc_sw128(umma_smem_u32(sb + a * SP_ATOM + 32 * kk)), idesc,
                                              (a | kk) != 0);
            }
            umma_commit_pair_warp(&bar_mma);
        }
        const bool ok = tc_wait(&bar_mma, 0);
        if (!ok) atomicExch(err, 2);
        tmem_fence_after();
        if (ok) {
            for (int c = 0; c < N; c += 16) {
                float v[16];
                tmem_ld16(tm + ((uint32_t)(32 * warp) << 16) + dcol + c, v);
                for (int i = 0; i < 16; i++) C[(size_t)(128 * rank + tid) * N + c + i] = v[i];
            }
        }
    }
    tmem_fence_before();
    __syncwarp();
    cluster_sync_all();
    if (warp == 0) tmem_free_pair(tm, 512);
}

typedef CUresult (*st_encode_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// A [128 x 256] fp16, B [128 x 256] fp16, C [128 x 128] fp32, all device;
// a_in_tmem selects the kernel that keeps A in tensor memory.  Returns 0 on
// success.
extern "C" int umma_selftest(const void *A, const void *B, void *C, int a_in_tmem) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || !p) return -1;
    CUtensorMap m;
    const cuuint64_t dims[2] = {ST_K, ST_N};
    const cuuint64_t strides[1] = {ST_K * 2};
    const cuuint32_t box[2] = {64, ST_N};
    const cuuint32_t es[2] = {1, 1};
    if (((st_encode_fn)p)(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(B), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -2;
    int *err = nullptr;
    if (cudaMalloc(&err, sizeof(int)) != cudaSuccess) return -3;
    cudaMemset(err, 0, sizeof(int));
    const size_t smem = 8 * 16384 + 1024;
    if (a_in_tmem) {
        cudaFuncSetAttribute(k_umma_selftest_ta, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k_umma_selftest_ta<<<1, 128, smem>>>(m, (const __half *)A, (float *)C, err);
    } else {
        cudaFuncSetAttribute(k_umma_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k_umma_selftest<<<1, 128, smem>>>(m, (const __half *)A, (float *)C, err);
    }
    cudaError_t e = cudaDeviceSynchronize();
    int h = 0;
    cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(err);
    if (e != cudaSuccess) {
        fprintf(stderr, "umma_selftest: %s\n", cudaGetErrorString(e));
        return -4;
    }
    return h ? 10 + h : 0;
}

// A [256 x 256] fp16, B [N x 256] fp16, C [256 x N] fp32, all device; N a
// multiple of 32 up to 160; D at column dcol, A at column acol of tensor
// memory.  Returns 0 on success.
extern "C" int umma_selftest_pair(const void *A, const void *B, void *C, int N, int dcol, int acol) {
    if (N < 32 || N > 160 || N % 32 || dcol < 0 || acol < 0 || dcol + N > acol || acol + 128 > 512) return -5;
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || !p) return -1;
    CUtensorMap m;
    const cuuint64_t dims[2] = {256, (cuuint64_t)N};
    const cuuint64_t strides[1] = {256 * 2};
    const cuuint32_t box[2] = {64, 16};
    const cuuint32_t es[2] = {1, 1};
    if (((st_encode_fn)p)(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(B), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -2;
    int *err = nullptr;
    if (cudaMalloc(&err, sizeof(int)) != cudaSuccess) return -3;
    cudaMemset(err, 0, sizeof(int));
    const size_t smem = 4 * SP_ATOM + 1024;
    cudaFuncSetAttribute(k_umma_selftest_pair, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_umma_selftest_pair<<<2, 128, smem>>>(m, (const __half *)A, (float *)C, N, dcol, acol, err);
    cudaError_t e = cudaDeviceSynchronize();
    int h = 0;
    cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(err);
    if (e != cudaSuccess) {
        fprintf(stderr, "umma_selftest_pair: %s\n", cudaGetErrorString(e));
        return -4;
    }
    return h ? 10 + h : 0;
}
