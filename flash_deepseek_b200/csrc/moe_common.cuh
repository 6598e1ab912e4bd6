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
// Activation operand (int8 planes).  The decode GEMVs use the tensor core as
// an exact reducer: x * s (s a power of two per super-block) is rounded to an
// integer v with |v| <= 2^20 and split into three int8 planes
//     v = p0 + 2^7 p1 + 2^14 p2,   p0, p1 in [0, 127], p2 in [-64, 64],
// so that every product with a weight is exact in int32.  The K order inside
// one MMA is free, so the planes are stored pre-permuted to the order in
// which a lane naturally decodes its weight bytes.  Per vector and 256-weight
// super-block, OPB_SB = 960 bytes: three plane blocks of 320 bytes
//   [0, 256)   int8 values in lane order (style Q4 or Q6, below)
//   [256, 288) style Q4 only: fp16 sums of 16 consecutive plane values,
//              lane t: sums 2t, 2t+1, 2t+8, 2t+9 (exact: |sum| <= 2032)
//   [288, 292) plane 0 only: 1/s of this super-block (fp32); s is a power
//              of two per vector and super-block, from the super-block's
//              max |x|
//   [292, 320) padding: plane blocks 80 words apart keep the 16-byte
//              fragment loads of one quarter-warp on distinct banks
// Style Q4 (Q4_K weights, m16n8k32 u8 x s8): weight k = 32 s + 8 t + i of
// sub-block s = 2 j + h sits at 64 j + 16 t + 8 h + i.
// Style Q6 (Q6_K weights, m16n8k16 s8 x s8): weight k = 16 s + 4 t + i of
// sub-block s = 4 q + u sits at 64 q + 16 t + 4 u + i.
// ---------------------------------------------------------------------------
#define OPB_PLANE 320
#define OPB_SB (3 * OPB_PLANE)
#define OPB_XSUM 256
#define OPB_SCALE 288
__host__ __device__ __forceinline__ size_t op_bytes(int K) { return (size_t)(K / 256) * OPB_SB; }
__host__ __device__ __forceinline__ int opq4_off(int k) {
    const int s = k >> 5, t = (k >> 3) & 3, i = k & 7;
    return 64 * (s >> 1) + 16 * t + 8 * (s & 1) + i;
}
__host__ __device__ __forceinline__ int opq6_off(int k) {
    const int s = k >> 4, t = (k >> 2) & 3, i = k & 3;
    return 64 * (s >> 2) + 16 * t + 4 * (s & 3) + i;
}
// byte offset (inside a plane block) of the fp16 sum of plane values
// [16 jj, 16 jj + 16) of a super-block
__host__ __device__ __forceinline__ int opq4_xsum_off(int jj) {
    const int t = (jj & 7) >> 1, u = 2 * (jj >> 3) + (jj & 1);
    return OPB_XSUM + 8 * t + 2 * u;
}

// ---------------------------------------------------------------------------
// Wide activation operand (fp16 planes), for the expert GEMVs' fp16 path: x
// times a power of two s per super-block (max |x s| in [2^14, 2^15)) is split
// into x_hi = fp16(x s) and x_lo = fp16(x s - x_hi) (22 significant bits
// together).  Per vector and super-block, OPW_SB = 1104 bytes:
//   [0, 512)     x_hi, 256 fp16 in lane order (style Q4 or Q6, below)
//   [512, 528)   style Q4: fp16 hi parts of the 8 sub-block sums / 32
//   [528, 544)   style Q4: fp16 lo parts of the same
//   [544, 548)   1/s (fp32)
//   [576, 1088)  x_lo in the same order (576: the two planes' 16-byte
//                fragment loads of one quarter-warp fall on distinct banks)
//   [1088, 1104) padding: vectors 4 apart differ by 64 mod 128 bytes, so the
//                x_hi loads of tokens k and k + 4 by one quarter-warp (the
//                Q6_K residual tiles) fall on distinct banks too
// Style Q4 (m16n8k16 fp16, Q4_K weights): element 8 t + i of sub-block j
// (32 weights) sits at fp16 index 32 j + 8 t + perm(i), perm = 0 2 1 3 4 6 5 7,
// so that one 16-byte load gives lane t the B fragments of both k16 steps.
// Style Q6 (Q6_K weights, one sub-block of 16 per k16 step): element 4 t + i
// of sub-block s sits at fp16 index 32 (s / 2) + 8 t + 4 (s % 2) + i.
// ---------------------------------------------------------------------------
#define OPW_SB 1104
#define OPW_XSUM 512
#define OPW_SCALE 544
#define OPW_LO 576
#define OPW_TOP 15  // max |x s| in [2^14, 2^15)
__host__ __device__ __forceinline__ size_t opw_bytes(int K) { return (size_t)(K / 256) * OPW_SB; }
// one decode activation row: the int8 planes, then the fp16 planes
__host__ __device__ __forceinline__ size_t opx_row(int K) { return op_bytes(K) + opw_bytes(K); }
__host__ __device__ __forceinline__ int opw4_idx(int k) {
    const int j = k >> 5, t = (k >> 3) & 3, i = k & 7;
    return 32 * j + 8 * t + ((i & 4) | ((i & 1) << 1) | ((i >> 1) & 1));
}
__host__ __device__ __forceinline__ int opw6_idx(int k) {
    const int s = k >> 4, t = (k >> 2) & 3, i = k & 3;
    return 32 * (s >> 1) + 8 * t + 4 * (s & 1) + i;
}

// ---------------------------------------------------------------------------
// Repacked Q4_K block (lossless, done once at load): the 16-byte header
// (d, dmin, 12 scale bytes) stays, the 128 qs bytes are transposed as a 4x4
// grid of 8-byte chunks, new chunk 4 t + j = old chunk 4 j + t, so that lane
// t of an MMA finds its 32 bytes (old bytes 32 j + 8 t + [0, 8), j = 0..3)
// contiguous.  The transpose is its own inverse.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int q4r_src_qs(int p) {
    const int c = p >> 3, i = p & 7;
    return 8 * (4 * (c & 3) + (c >> 2)) + i;
}

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

// sign-extended byte `i` (compile-time) of w
template <int I>
__device__ __forceinline__ int sext_byte(uint32_t w) {
    int r;
    asm("prmt.b32 %0, %1, 0, %2;\n" : "=r"(r) : "r"(w), "n"(I | ((8 | I) << 4) | ((8 | I) << 8) | ((8 | I) << 12)));
    return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
// fp16 pair arithmetic on raw 32-bit words (sm_53 and later; the layout
// tools that include this header on the host compile without them)
#if !defined(__CUDA_ARCH__) || __CUDA_ARCH__ >= 530
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    return h2_as_u32(__hfma2(u32_as_h2(a), u32_as_h2(b), u32_as_h2(c)));
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
    return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    return h2_as_u32(__hsub2(u32_as_h2(a), u32_as_h2(b)));
}
// fp16 pair constants
#define H2_1024 0x64006400u
#define H2_M1024 0xE400E400u
#define H2_1056 0x64206420u
#define H2_1152 0x64806480u
#define H2_16TH 0x2C002C00u
#define H2_M64 0xD400D400u
// (v, v) for byte B of w (an integer v < 1024): bytes (v, 0x64) are 1024 + v
template <int B>
__device__ __forceinline__ uint32_t byte_h2(uint32_t w, uint32_t minus) {
    return hsub2u(prmt(w, 0x64u, (uint32_t)(B | (4 << 4) | (B << 8) | (4 << 12))), minus);
}
#endif

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

// ---------------------------------------------------------------------------
// Activation operands (built by the route / prep kernels of moe_kernels.cu
// and the expert-parallel row kernel of moe_ep.cu)
// ---------------------------------------------------------------------------
// power-of-two scale s with max|x| * s in [2^(top-1), 2^top); returns s, sets
// *inv = 1/s.  The int8-plane operand uses top = 20 (|rint(x * s)| <= 2^20).
__device__ __forceinline__ float op_scale(float amax, float *inv, int top) {
    if (!(amax > 0.0f) || !isfinite(amax)) { *inv = 1.0f; return 1.0f; }
    int ex;
    frexpf(amax, &ex);  // amax = m 2^ex, m in [0.5, 1)
    int e = top - ex;
    if (e > 120) e = 120;
    if (e < -120) e = -120;
    *inv = ldexpf(1.0f, -e);
    return ldexpf(1.0f, e);
}

// One 256-weight super-block of one vector, built by one warp: s = power of
// two from the super-block's max |x| (|rint(x s)| <= 2^20), int8 planes in
// the lane order of `style` (4: Q4_K weights, with the fp16 sums of 16
// consecutive plane values; 6: Q6_K weights) and 1/s.  Layout in
// moe_common.cuh.  x must be 16-byte aligned.
__device__ __forceinline__ void build_op_sb(const float *__restrict__ x, uint8_t *__restrict__ op, int style,
                                            int lane) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(x) + 2 * lane);
    const float4 b = __ldg(reinterpret_cast<const float4 *>(x) + 2 * lane + 1);
    const float v8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(v8[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float inv;
    const float s = op_scale(m, &inv, 20);
    uint32_t w[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
    int ps[3] = {0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int v = __float2int_rn(__fmul_rn(v8[i], s));
        const int p0 = v & 127, p1 = (v >> 7) & 127, p2 = v >> 14;
        w[0][i >> 2] |= (uint32_t)p0 << (8 * (i & 3));
        w[1][i >> 2] |= (uint32_t)p1 << (8 * (i & 3));
        w[2][i >> 2] |= (uint32_t)(p2 & 255) << (8 * (i & 3));
        ps[0] += p0;
        ps[1] += p1;
        ps[2] += p2;
    }
    const int k = 8 * lane;
    const int off0 = style == 4 ? opq4_off(k) : opq6_off(k), off1 = style == 4 ? opq4_off(k + 4) : opq6_off(k + 4);
#pragma unroll
    for (int p = 0; p < 3; p++) {
        *reinterpret_cast<uint32_t *>(op + p * OPB_PLANE + off0) = w[p][0];
        *reinterpret_cast<uint32_t *>(op + p * OPB_PLANE + off1) = w[p][1];
    }
    if (style == 4) {  // lanes 2j, 2j + 1 hold the 16 values [16 j, 16 j + 16)
        int tot[3];
#pragma unroll
        for (int p = 0; p < 3; p++) tot[p] = ps[p] + __shfl_xor_sync(0xffffffffu, ps[p], 1);
        if ((lane & 1) == 0) {
#pragma unroll
            for (int p = 0; p < 3; p++)
                *reinterpret_cast<__half *>(op + p * OPB_PLANE + opq4_xsum_off(lane >> 1)) = __int2half_rn(tot[p]);
        }
    }
    if (lane == 0) *reinterpret_cast<float *>(op + OPB_SCALE) = inv;
}

// One 256-weight super-block of one vector in the wide (fp16 hi/lo) form,
// built by one warp (layout in moe_common.cuh): s = power of two from the
// super-block's max |x| (max |x s| in [2^14, 2^15)), x_hi = fp16(x s),
// x_lo = fp16(x s - x_hi), both planes in the lane order of `style`; style 4
// adds the sub-block sums of x_hi + x_lo (divided by 32, as fp16 hi/lo) for
// the Q4_K min term.  x must be 16-byte aligned.
__device__ __forceinline__ void build_opw_sb(const float *__restrict__ x, uint8_t *__restrict__ op, int style,
                                             int lane) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(x) + 2 * lane);
    const float4 b = __ldg(reinterpret_cast<const float4 *>(x) + 2 * lane + 1);
    const float v8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(v8[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float inv;
    const float sc = op_scale(m, &inv, OPW_TOP);
    __half hi[8], lo[8];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float xs = __fmul_rn(v8[i], sc);  // exact: sc is a power of two
        hi[i] = __float2half_rn(xs);
        const float hv = __half2float(hi[i]);
        lo[i] = __float2half_rn(__fsub_rn(xs, hv));  // xs - hv is exact in fp32
        sum = __fadd_rn(sum, __fadd_rn(hv, __half2float(lo[i])));  // hv + lo exact (22 bits)
    }
    __half *H = reinterpret_cast<__half *>(op), *L = reinterpret_cast<__half *>(op + OPW_LO);
    if (style == 4) {
        // elements 8 lane + i: sub-block lane / 4, t = lane % 4 -> 16 contiguous bytes
        const int base = 8 * lane;  // opw4_idx(8 lane + i) = 8 lane + perm(i)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int ix = base + ((i & 4) | ((i & 1) << 1) | ((i >> 1) & 1));
            H[ix] = hi[i];
            L[ix] = lo[i];
        }
        // sub-block j = lane / 4: sum over its four lanes in a fixed order
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
        if ((lane & 3) == 0) {
            const float s32 = __fmul_rn(sum, 0.03125f);  // exact
            const __half sh = __float2half_rn(s32);
            const __half sl = __float2half_rn(__fsub_rn(s32, __half2float(sh)));
            reinterpret_cast<__half *>(op + OPW_XSUM)[lane >> 2] = sh;
            reinterpret_cast<__half *>(op + OPW_XSUM + 16)[lane >> 2] = sl;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int ix = opw6_idx(8 * lane + i);
            H[ix] = hi[i];
            L[ix] = lo[i];
        }
    }
    if (lane == 0) *reinterpret_cast<float *>(op + OPW_SCALE) = inv;
}

// Operand of a K-vector by the warps of the block, one super-block per warp:
// the int8 planes into op8 and, when opw is set, the fp16 planes into opw.
__device__ __forceinline__ void build_op_rows(const float *__restrict__ x, int K, uint8_t *__restrict__ op8,
                                              uint8_t *__restrict__ opw, int style) {
    const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int sb = threadIdx.x >> 5; sb < K / MOE_QK; sb += nw) {
        if (op8) build_op_sb(x + (size_t)sb * MOE_QK, op8 + (size_t)sb * OPB_SB, style, lane);
        if (opw) build_opw_sb(x + (size_t)sb * MOE_QK, opw + (size_t)sb * OPW_SB, style, lane);
    }
}

// scale and min of sub-block J of a Q4_K block (get_scale_min_k4,
// quant.c:26-34); h.y, h.z, h.w = the 12 scale bytes
template <int J>
__device__ __forceinline__ void q4_scale_min(uint4 h, int &sc, int &m) {
    const uint32_t s[3] = {h.y, h.z, h.w};
#define PF_B(k) ((int)((s[(k) >> 2] >> (8 * ((k) & 3))) & 0xFFu))
    if (J < 4) {
        sc = PF_B(J) & 63;
        m = PF_B(J + 4) & 63;
    } else {
        sc = (PF_B(J + 4) & 0xF) | ((PF_B(J - 4) >> 6) << 4);
        m = (PF_B(J + 4) >> 4) | ((PF_B(J) >> 6) << 4);
    }
#undef PF_B
}
