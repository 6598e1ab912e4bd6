// moe_common.cuh -- layouts, fragment maps and device helpers shared by the
// MoE kernels of libmoe_cuda.so (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MOE_QK 256
#define MOE_Q4K_BYTES 144  // quant.h:7
#define MOE_Q6K_BYTES 210  // quant.h:8
#define MOE_MAX_K 16       // infer.m:80
#define MOE_MAX_TOK_ROUTE 64
#define MOE_WARPS_GU 8     // gate/up CTA: 4 row tiles x 2 K halves
#define MOE_ROWS_GU 64     // rows of one gate/up CTA item
#define MOE_WARPS_DN 8     // down CTA: 8 independent warps

// ---------------------------------------------------------------------------
// Activation-operand layouts.  The decode GEMVs use the tensor core as an
// exact reducer: the K order inside an MMA is free, so each activation
// operand is stored pre-permuted to match the order in which a lane naturally
// decodes its weight bytes, and laid out so that a lane reads its fragments
// with 16-byte vector loads.
//
// Q4_K operand (fp16 MMA; gate/up and Q4_K down).  x*s = hi + lo (two fp16,
// s a power of two per vector).  Per vector and super-block (256 weights):
//   [part (hi, lo)][lane t][step 0..17][4 halves]      = 576 halves
//   step m < 16, slot j: weight q4k_k(m, t, j)
//   step 16: (X_a, X_b, 0, 0), X = sub-block sums of x*s for sub-blocks
//            q4k_min_sub(t), q4k_min_sub(t)+1;  step 17: zero padding
// Q6_K operand (int8 MMA; Q6_K down).  x*2^e rounded to a 21-bit integer
// split into three int8 planes x = p0 + 2^7 p1 + 2^14 p2 (p0, p1 in [0,127],
// p2 signed).  Per vector: [plane][super-block][lane t][step 0..15][4 bytes]
// = 3 * 256 bytes per super-block; step s, byte i: weight 16 s + 4 t + i.
// ---------------------------------------------------------------------------
#define Q4OP_STEPS 18
#define Q4OP_LANE_HALVES (Q4OP_STEPS * 4)            // 72 halves = 144 B per lane
#define Q4OP_HALVES_PER_SB (2 * 4 * Q4OP_LANE_HALVES) // 576
#define Q6I_BYTES_PER_SB 256                          // per plane
__host__ __device__ __forceinline__ size_t q4op_halves(int K) { return (size_t)(K / 256) * Q4OP_HALVES_PER_SB; }
__host__ __device__ __forceinline__ size_t q6i_bytes(int K) { return (size_t)3 * (K / 256) * Q6I_BYTES_PER_SB; }
// bytes reserved per vector in a buffer that may hold either operand
__host__ __device__ __forceinline__ size_t dop_bytes(int K) {
    const size_t a = q4op_halves(K) * 2, b = q6i_bytes(K);
    return a > b ? a : b;
}

__host__ __device__ __forceinline__ int perm_j(int j) { return (j == 1) ? 2 : ((j == 2) ? 1 : j); }

// Weight index (0..255) inside a Q4_K super-block for MMA step m, lane t, slot
// j.  Lane t loads qs bytes [64r + 16t, +16) (r = m/8); word i = (m/2)%4 of
// that load; m odd = high nibbles.  Low nibble of qs byte b of chunk c is
// weight 64c + b, the high nibble weight 64c + 32 + b (quant.c:49-58).
__host__ __device__ __forceinline__ int q4k_k(int m, int t, int j) {
    const int r = m >> 3, i = (m >> 1) & 3, hi = m & 1;
    const int c = 2 * r + (t >> 1);
    return 64 * c + 32 * hi + 16 * (t & 1) + 4 * i + perm_j(j);
}
// First of the two sub-blocks whose min-term lane t supplies (0, 4, 2, 6).
__host__ __device__ __forceinline__ int q4k_min_sub(int t) { return 2 * (t >> 1) + 4 * (t & 1); }

// Weight index inside a Q6_K super-block for sub-block step s (0..15), lane t,
// byte i of the lane's int8 fragment.
__host__ __device__ __forceinline__ int q6k_k(int s, int t, int i) { return 16 * s + 4 * t + i; }

// ---------------------------------------------------------------------------
// Repacked Q6_K matrix (lossless permutation of the GGUF bytes, done once at
// load so that every lane reads 16-byte aligned vectors):
//   plane Q [rows][nb][4 lanes][12 words]: lane t of block b holds, per half
//           h: ql words at byte offsets 4t, 16+4t, 32+4t, 48+4t of ql[64h..]
//           then qh words at 4t, 16+4t of qh[32h..]          (192 B / block)
//   plane S [rows][nb][16] int8 scales                        ( 16 B / block)
//   plane D [rows][nb_pad8] fp16 d                            (  2 B / block)
// Total = rows * nb * 210 bytes when nb % 8 == 0.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ size_t q6r_plane_s_off(int rows, int nb) { return (size_t)rows * nb * 192; }
__host__ __device__ __forceinline__ size_t q6r_plane_d_off(int rows, int nb) { return (size_t)rows * nb * 208; }
__host__ __device__ __forceinline__ int q6r_nb_pad(int nb) { return (nb + 7) & ~7; }
__host__ __device__ __forceinline__ size_t q6r_bytes(int rows, int nb) {
    return (size_t)rows * nb * 208 + (size_t)rows * q6r_nb_pad(nb) * 2;
}
// source byte (inside a 210-byte GGUF block) of repacked byte p (0..191) of
// the Q plane of one block.
__host__ __device__ __forceinline__ int q6r_src_byte(int p) {
    const int t = p / 48, rem = p % 48, h = rem / 24, w = (rem % 24) / 4, b = rem % 4;
    if (w < 4) return 64 * h + 16 * w + 4 * t + b;       // ql
    return 128 + 32 * h + 16 * (w - 4) + 4 * t + b;     // qh
}

// ---------------------------------------------------------------------------
// fp16 <-> fp32 (bit exact with quant.c:4-24 and with the test oracle).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// float -> half, round to nearest even (the quantizer's conversion; same
// integer algorithm as the oracle so both sides agree bit for bit).
__host__ __device__ __forceinline__ uint16_t f2h_rne_bits(float f) {
#ifdef __CUDA_ARCH__
    uint32_t x = __float_as_uint(f);
#else
    union { float f; uint32_t u; } cv; cv.f = f; uint32_t x = cv.u;
#endif
    uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (ax >= 0x38800000u) {
        uint32_t mant = ax & 0x7FFFFFu;
        uint32_t h = (((ax >> 23) - 112u) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    int e = (int)(ax >> 23);
    int shift = 126 - e;
    if (shift > 24) return (uint16_t)sign;
    uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t hm = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) hm++;
    return (uint16_t)(sign | hm);
}

// ---------------------------------------------------------------------------
// Tensor-core step: D = A(16x16 f16, row) * B(16x8 f16, col) + C (fp32).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1, float c0, float c1, float c2, float c3) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

// Integer tensor-core step: D = A(16x16 u8 / s8, row) * B(16x8 s8, col) + C (s32).
__device__ __forceinline__ void mma_u8s8_16816(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0, int c0, int c1,
                                               int c2, int c3) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}
__device__ __forceinline__ void mma_s8s8_16816(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0, int c0, int c1,
                                               int c2, int c3) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}
// sign-extended byte `i` (compile-time) of w
template <int I>
__device__ __forceinline__ int sext_byte(uint32_t w) {
    int r;
    asm("prmt.b32 %0, %1, 0, %2;\n" : "=r"(r) : "r"(w), "n"(I | ((8 | I) << 4) | ((8 | I) << 8) | ((8 | I) << 12)));
    return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Streaming 16-byte load of weight bytes: read-only path, no L1 allocation
// (each weight byte is used once per launch).
__device__ __forceinline__ uint4 ldg_stream16(const void *p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
// Activation-operand load (16 bytes, cached in L1: shared by many warps).
__device__ __forceinline__ uint4 ldg_op16(const void *p) {
    uint4 r;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Asynchronous 16-byte global -> shared copy (L2 only), completed with
// cp.async.wait_group.  Each lane later reads back only what it copied, so
// no barrier is needed between the copy and its use.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
#define MOE_STAGES 3        // per-warp weight pipeline depth
#define MOE_Q4_WORDS 6      // 16-byte words per lane per Q4_K super-block (2 rows)
#define MOE_Q6_WORDS 8      // 16-byte words per lane per Q6_K super-block (2 rows)

// ---------------------------------------------------------------------------
// Counter-based N(0, sigma) generator, bit-identical to the test oracle:
// splitmix64 keyed by (seed, stream, element) -> Marsaglia polar method with
// a log built from IEEE +,-,*,/ only (explicit _rn ops: no contraction).
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
__host__ __device__ __forceinline__ uint64_t synth_stream(int layer, int expert, int kind) {
    return ((uint64_t)(uint32_t)layer << 32) | ((uint64_t)(uint32_t)expert << 8) | (uint64_t)(uint32_t)kind;
}
enum { SYN_GATE = 0, SYN_UP = 1, SYN_DOWN = 2, SYN_ROUTER = 3, SYN_BIAS = 4, SYN_NORM = 5, SYN_ACT = 6 };

__device__ __forceinline__ double det_log(double s) {
    uint64_t b = (uint64_t)__double_as_longlong(s);
    int e = (int)((b >> 52) & 0x7FF) - 1023;
    double m = __longlong_as_double((long long)((b & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull));
    if (m > 1.4142135623730951) { m = __dmul_rn(m, 0.5); e += 1; }
    double t = __ddiv_rn(__dadd_rn(m, -1.0), __dadd_rn(m, 1.0));
    double t2 = __dmul_rn(t, t);
    double acc = __ddiv_rn(1.0, 25.0);
    for (int k = 11; k >= 0; k--) acc = __dadd_rn(__dmul_rn(acc, t2), __ddiv_rn(1.0, (double)(2 * k + 1)));
    return __dadd_rn(__dmul_rn((double)e, 0.6931471805599453), __dmul_rn(__dmul_rn(2.0, t), acc));
}

__device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
}
__device__ __forceinline__ float synth_normal(uint64_t key, uint64_t index, double sigma) {
    for (uint64_t a = 0; a < 64; a++) {
        uint64_t r = splitmix64(key + (index << 6) + a);
        double u = __dmul_rn((double)(int32_t)(uint32_t)(r >> 32), 1.0 / 2147483648.0);
        double v = __dmul_rn((double)(int32_t)(uint32_t)(r & 0xFFFFFFFFu), 1.0 / 2147483648.0);
        double s = __dadd_rn(__dmul_rn(u, u), __dmul_rn(v, v));
        if (s < 1.0 && s > 0.0) {
            double z = __dmul_rn(u, __dsqrt_rn(__ddiv_rn(__dmul_rn(-2.0, det_log(s)), s)));
            return __double2float_rn(__dmul_rn(z, sigma));
        }
    }
    return __double2float_rn(__dmul_rn(0.0, sigma));
}

// round half away from zero on a clamped float (the quantizer's rounding)
__device__ __forceinline__ int q_rnd(float v) {
    v = fminf(fmaxf(v, -1.0e6f), 1.0e6f);
    return v >= 0.0f ? (int)__fadd_rn(v, 0.5f) : -(int)__fadd_rn(-v, 0.5f);
}
