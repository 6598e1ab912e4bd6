// moe_noalloc.cu -- routing from hidden states without any allocation.
//
// Some callers cannot allocate device memory: a host engine that owns a fixed
// memory pool and forbids allocation after start-up, or one that runs decode
// under hard latency limits where a cudaMalloc (which may synchronize the
// device) is not allowed.  moe_route_hidden_noalloc() gives them the router
// logits GEMV + grouped top-k of the MoE block with all of its scratch (the
// split partial logits, the final logits and the completion counters) in a
// fixed array compiled into this library.  The caller passes only inputs and
// outputs.
#include <stdio.h>

#include "../../include/moe_cuda.h"
#include "moe_common.cuh"
#include "moe_internal.h"

// Scratch limits (floats): the router kernel keeps n_split * T * E partial
// sums (n_split = hidden / 256) and T * E final logits, plus one counter per
// 32 experts.  The partial sums cover DeepSeek-V3 at its largest decode batch
// (28 splits x 64 tokens x 256 experts): 1.75 MiB + 256 KiB + 256 bytes, held
// by every GPU that loads the library until the process exits.
#define NOALLOC_MAX_PART (28 * 64 * 256)
#define NOALLOC_MAX_LOGITS (64 * 1024)
#define NOALLOC_MAX_GROUPS 64
#define NOALLOC_MAX_DEVICES 64

static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_MAX_PART + NOALLOC_MAX_LOGITS + NOALLOC_MAX_GROUPS];

// Device address of g_noalloc_scratch, looked up once per device.  In host
// code the symbol itself is only a stand-in and must never be passed to a
// kernel.
static float *g_noalloc_ptr[NOALLOC_MAX_DEVICES];

static int noalloc_fail(const char *msg) {
    fprintf(stderr, "[moe_cuda] ERROR: moe_route_hidden_noalloc: %s\n", msg);
    return MOE_ERR_ARG;
}

extern "C" int moe_route_hidden_noalloc(const moe_config *cfg, const float *d_router_w, const float *d_bias,
                                        const float *d_h, int n_tokens, int *d_idx, float *d_w, void *stream) {
    if (!cfg || !d_router_w || !d_h || !d_idx || !d_w) return noalloc_fail("null pointer");
    const int H = cfg->hidden, E = cfg->n_experts, T = n_tokens;
    if (H <= 0 || H % 256 || H > 32768) return noalloc_fail("hidden must be a multiple of 256 in 256..32768");
    if (E <= 0 || E > 1024 || cfg->n_group <= 0 || cfg->n_group > 64 || E % cfg->n_group)
        return noalloc_fail("n_group must divide n_experts (n_experts <= 1024, n_group <= 64)");
    if (cfg->topk_group <= 0 || cfg->topk_group > cfg->n_group) return noalloc_fail("bad topk_group");
    if (cfg->top_k <= 0 || cfg->top_k > MOE_MAX_K || cfg->top_k > cfg->topk_group * (E / cfg->n_group))
        return noalloc_fail("bad top_k");
    if (T <= 0 || T > 64) return noalloc_fail("n_tokens must be in 1..64");
    const int n_split = H / 256;
    if ((size_t)n_split * T * E > NOALLOC_MAX_PART)
        return noalloc_fail("hidden/256 * n_tokens * n_experts exceeds the 458752-float scratch");
    if ((size_t)T * E > NOALLOC_MAX_LOGITS) return noalloc_fail("n_tokens * n_experts exceeds 65536");
    if ((E + 31) / 32 > NOALLOC_MAX_GROUPS) return noalloc_fail("too many expert groups");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NOALLOC_MAX_DEVICES)
        return noalloc_fail("no usable current CUDA device");
    if (!g_noalloc_ptr[dev]) {  // first call on this device: look up the array's device address
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            fprintf(stderr, "[moe_cuda] ERROR: moe_route_hidden_noalloc: cudaGetSymbolAddress: %s\n",
                    cudaGetErrorString(e));
            return MOE_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = (float *)p;
    }
    float *part = g_noalloc_ptr[dev];
    float *logits = part + NOALLOC_MAX_PART;
    int *counters = reinterpret_cast<int *>(logits + NOALLOC_MAX_LOGITS);
    cudaStream_t s = (cudaStream_t)stream;
    // the counters must start at zero (the kernel also resets them when done)
    if (cudaMemsetAsync(counters, 0, sizeof(int) * NOALLOC_MAX_GROUPS, s) != cudaSuccess)
        return noalloc_fail("clearing the counters failed");
    const MoeDims d{H, cfg->intermediate, E, cfg->n_group, cfg->topk_group, cfg->top_k, cfg->routed_scale};
    moe_launch_router_logits(d_router_w, d_h, T, H, E, part, n_split, logits, counters, s, nullptr);
    MoePlan none{};
    moe_launch_route_and_plan(d, nullptr, 0, logits, d_bias, nullptr, 0, nullptr, nullptr, T, d_idx, d_w, nullptr,
                              nullptr, 0, 0, none, nullptr, s, nullptr);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "[moe_cuda] ERROR: moe_route_hidden_noalloc: %s\n", cudaGetErrorString(e));
        return MOE_ERR_CUDA;
    }
    return MOE_OK;
}
