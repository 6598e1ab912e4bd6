// GPU self-test of the tcgen05 building blocks of moe_umma.cuh (built into a
// throw-away shared library by tests/test_gpu_prefill.py): one CTA computes
// C[128 x N] = A[128 x K] * B[N x K]^T in fp16 with fp32 accumulation in
// tensor memory.  A is written into 128-byte-swizzled shared memory by the
// threads (the path the prefill dequantizer takes), B arrives by TMA with
// SWIZZLE_128B.  Every wait is bounded; a timeout sets *err.
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
