// ffn_common.cuh -- shared device helpers of the fused NeRF step.
//
// Exactness policy.  Everything that decides *which* samples, cells and occupancy nibbles are
// touched (sampler, compositing transmittance, occupancy proposals, decay) is computed with
// explicit round-to-nearest single/double operations (__fmul_rn, __fadd_rn, ...) so nvcc cannot
// contract them into FMAs, and with the exp/pow below instead of the CUDA math library.  The same
// operation sequence, compiled for the CPU with contraction disabled, is the parity oracle; the
// two agree bit for bit.  The MLP, its backward and the hash-grid interpolation are ordinary
// fp32 code and are compared within tolerance.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/ffnerf.h"

namespace ffn {

constexpr int L = FFN_N_LEVELS;   // hash levels (reference N_LEVELS, ffnerf_OG.cl:166)
constexpr int M = 64;             // hidden width (ffnerf_OG.cl:45)
constexpr int D_OUT = 16;         // density head (ffnerf_OG.cl:42)
constexpr int L_DIR = 16;         // SH coefficients (ffnerf_OG.cl:41)
constexpr int C_IN = 32;          // color input (ffnerf_OG.cl:43)
constexpr int C_OUT = 3;          // rgb (ffnerf_OG.cl:44)
constexpr int S_MAX = 64;         // samples per ray (ffnerf_OG.cl:47)

// Parameter indices in the canonical blob order (reference kernel argument order).
enum { P_WD_IN, P_WD_01, P_WD_12, P_WD_OUT, P_WC_IN, P_WC_01, P_WC_12, P_WC_23, P_WC_OUT,
       P_BD_0, P_BD_1, P_BD_2, P_BD_OUT, P_BC_0, P_BC_1, P_BC_2, P_BC_3, P_BC_OUT, P_COUNT };

struct ParamLayout {
    int off[P_COUNT];
    int size[P_COUNT];
    int total;
};

__host__ __device__ inline ParamLayout make_param_layout(int F, int ND, int NC) {
    ParamLayout lo{};
    const int lpos = L * F;
    const int sz[P_COUNT] = {M * lpos, ND >= 2 ? M * M : 0, ND >= 3 ? M * M : 0, D_OUT * M,
                             M * C_IN, NC >= 2 ? M * M : 0, NC >= 3 ? M * M : 0, NC >= 4 ? M * M : 0,
                             C_OUT * M,
                             M, ND >= 2 ? M : 0, ND >= 3 ? M : 0, D_OUT,
                             M, NC >= 2 ? M : 0, NC >= 3 ? M : 0, NC >= 4 ? M : 0, C_OUT};
    int o = 0;
    for (int i = 0; i < P_COUNT; ++i) {
        lo.off[i] = o;
        lo.size[i] = sz[i];
        o += (sz[i] + 3) & ~3;
    }
    lo.total = o;
    return lo;
}

// Kernel-side copy of the configuration (passed by value).
struct DevConfig {
    int F, ND, NC, spr, G, background;
    uint32_t level_log2[L];
    uint32_t level_offset[L];
    int level_res[L];
    float hash_lr_scale[L];
    float bmin[3], bmax[3];
    float rho_min, rho_max, dt_min, dt_max, t_near, t_far;
    int transfer;   // format of the weight-gradient operands: 32 fp32, 16 fp16, 8 the reference's fp8
};

// The reference's transfer formats (ffnerf_OG.cl:85-156): the weight update reads the staged
// activations and deltas as stored in the format.  fp16: saturate to +-65504 (non-finite to
// +-65504), round to nearest even.  fp8 (e4m3-like minifloat): saturate to +-15.5 (non-finite to
// +-15.5), flush |x| < 1e-8 and exponents below the bias to zero, 3 mantissa bits rounded to
// nearest even (a carry bumps the exponent), exponents above 14 stored as 2^3 * 1.875.
__device__ __forceinline__ float transfer_fp16(float x) {
    if (!isfinite(x)) x = copysignf(65504.0f, x);
    return __half2float(__float2half_rn(fminf(fmaxf(x, -65504.0f), 65504.0f)));
}
__device__ __forceinline__ float transfer_fp8(float x) {
    x = isfinite(x) ? fminf(fmaxf(x, -15.5f), 15.5f) : copysignf(15.5f, x);
    const bool neg = x < 0.0f;
    const float ax = fabsf(x);
    if (ax < 1.0e-8f) return neg ? -0.0f : 0.0f;
    int e = 0;
    const float m = frexpf(ax, &e);
    int ef = e - 1 + 7;
    if (ef <= 0) return neg ? -0.0f : 0.0f;
    int mant;
    if (ef > 14) {
        ef = 10; mant = 7;
    } else {
        mant = (int)rintf(__fmul_rn(__fsub_rn(__fmul_rn(m, 2.0f), 1.0f), 8.0f));
        if (mant >= 8) { mant = 0; ef += 1; }
        if (ef > 14) { ef = 10; mant = 7; }
    }
    const float v = ldexpf(1.0f + (float)mant * 0.125f, ef - 7);
    return neg ? -v : v;
}
__device__ __forceinline__ float transfer_q(float x, int fmt) {
    return fmt == 16 ? transfer_fp16(x) : (fmt == 8 ? transfer_fp8(x) : x);
}

// ------------------------------------------------------------------------- integer RNG
// hash_u32 / rand01 (ffnerf_OG.cl:293-311)
__host__ __device__ __forceinline__ uint32_t hash_u32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352du; x ^= x >> 15; x *= 0x846ca68bu; x ^= x >> 16;
    return x;
}
__device__ __forceinline__ float rand01(uint32_t* s) {
    uint32_t x = *s;
    x ^= x << 13; x ^= x >> 17; x ^= x << 5;
    *s = x;
    return __fmul_rn((float)(x & 0x00FFFFFFu), 1.0f / 16777216.0f);
}

// ------------------------------------------------------------------------- exact fp32 ops
__device__ __forceinline__ float fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fa(float a, float b) { return __fadd_rn(a, b); }

// Barrier over the threads of one 128-sample tile.  Kernels of at most 128 threads hold one tile:
// the whole block.  The tensor-core kernel runs two tiles side by side in a 256-thread block, one
// per 128-thread group, and each group synchronises on its own named barrier (1 + group), so the
// groups never wait for each other.
__device__ __forceinline__ void tile_sync() {
    if (blockDim.x <= 128) __syncthreads();
    else asm volatile("bar.sync %0, 128;" :: "r"(1 + (threadIdx.x >> 7)) : "memory");
}
__device__ __forceinline__ float fs(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fd(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fclamp(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }
__device__ __forceinline__ int iclamp(int x, int lo, int hi) { return min(max(x, lo), hi); }
// OpenCL mix(a,b,t) = a + (b-a)*t
__device__ __forceinline__ float fmix(float a, float b, float t) { return fa(a, fm(fs(b, a), t)); }

struct V3 { float x, y, z; };
__device__ __forceinline__ V3 v3(float x, float y, float z) { return V3{x, y, z}; }
__device__ __forceinline__ V3 vadd(V3 a, V3 b) { return v3(fa(a.x, b.x), fa(a.y, b.y), fa(a.z, b.z)); }
__device__ __forceinline__ V3 vsub(V3 a, V3 b) { return v3(fs(a.x, b.x), fs(a.y, b.y), fs(a.z, b.z)); }
__device__ __forceinline__ V3 vmul(V3 a, V3 b) { return v3(fm(a.x, b.x), fm(a.y, b.y), fm(a.z, b.z)); }
__device__ __forceinline__ V3 vdiv(V3 a, V3 b) { return v3(fd(a.x, b.x), fd(a.y, b.y), fd(a.z, b.z)); }
__device__ __forceinline__ V3 vscale(float s, V3 a) { return v3(fm(s, a.x), fm(s, a.y), fm(s, a.z)); }
// o + t*d with separate rounding of the product and the sum
__device__ __forceinline__ V3 ray_point(V3 o, V3 d, float t) { return vadd(o, vscale(t, d)); }
__device__ __forceinline__ float vlength(V3 v) {
    return __fsqrt_rn(fa(fa(fm(v.x, v.x), fm(v.y, v.y)), fm(v.z, v.z)));
}

// ------------------------------------------------------------------------- own exp / pow
// exp(z) in double: Cody-Waite reduction z = k*ln2 + r (ln2 split into a 24-bit head and a
// tail, both from the decimal expansion of ln 2), e^r by its degree-17 Taylor polynomial in
// Horner form, then scaling by 2^k.  log(x): x = m*2^e with m in (sqrt(1/2), sqrt(2)],
// log m = 2*atanh(s), s = (m-1)/(m+1), by the odd series in s (12 terms).
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }

__device__ __forceinline__ double own_exp_d(double z) {
    const double kLn2Hi = 0x1.62e43p-1;
    const double kLn2Lo = -0x1.05c610ca86c39p-29;
    const double kInvLn2 = 0x1.71547652b82fep+0;
    const double c[18] = {
        0x1p+0, 0x1p+0, 0x1p-1, 0x1.5555555555555p-3, 0x1.5555555555555p-5,
        0x1.1111111111111p-7, 0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13,
        0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22,
        0x1.ae64567f544e4p-26, 0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33,
        0x1.93974a8c07c9dp-37, 0x1.ae7f3e733b81fp-41, 0x1.ae7f3e733b81fp-45,
        0x1.952c77030ad4ap-49};
    double kd = rint(dmul(z, kInvLn2));
    double r = dsub(dsub(z, dmul(kd, kLn2Hi)), dmul(kd, kLn2Lo));
    double p = c[17];
#pragma unroll
    for (int n = 16; n >= 0; --n) p = dadd(dmul(p, r), c[n]);
    return ldexp(p, (int)kd);
}

__device__ __forceinline__ double own_log_d(double x) {
    const double kLn2Hi = 0x1.62e43p-1;
    const double kLn2Lo = -0x1.05c610ca86c39p-29;
    const double kSqrt2 = 0x1.6a09e667f3bcdp+0;
    const double q[13] = {
        0x1p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
        0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4,
        0x1.1111111111111p-4, 0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5,
        0x1.8618618618618p-5, 0x1.642c8590b2164p-5, 0x1.47ae147ae147bp-5};
    int e;
    double m = frexp(x, &e);
    m = dmul(m, 2.0);
    e = e - 1;
    if (m > kSqrt2) { m = dmul(m, 0.5); e = e + 1; }
    double s = __ddiv_rn(dsub(m, 1.0), dadd(m, 1.0));
    double z = dmul(s, s);
    double acc = q[12];
#pragma unroll
    for (int n = 11; n >= 0; --n) acc = dadd(dmul(acc, z), q[n]);
    double lm = dmul(dmul(2.0, s), acc);
    return dadd(dadd(dmul((double)e, kLn2Hi), lm), dmul((double)e, kLn2Lo));
}

__device__ __forceinline__ float own_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return __int_as_float(0x7f800000);
    if (x < -104.0f) return 0.0f;
    return __double2float_rn(own_exp_d((double)x));
}

// powr(x, y) for x >= 0 (OpenCL powr domain); x <= 0 gives 0 (the reference's safe_pow_pos).
__device__ __forceinline__ float own_powr(float x, float y) {
    if (!(x > 0.0f)) return 0.0f;
    double t = dmul((double)y, own_log_d((double)x));
    if (t > 710.0) return __int_as_float(0x7f800000);
    if (t < -745.0) return 0.0f;
    return __double2float_rn(own_exp_d(t));
}

// ------------------------------------------------------------------------- error word
// Bits set by kernels in the context's device status word (read asynchronously by the host).
// Vector float adds to global memory without a returned value (red, not atom): nothing waits for
// the old value, and the issuing thread's registers are free at once.
__device__ __forceinline__ void red_add2(float* p, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// device status word bits (ffn_status)
enum { ST_NONFINITE = 1, ST_TC_TIMEOUT = 4, ST_DP_TIMEOUT = 8 };

}  // namespace ffn
