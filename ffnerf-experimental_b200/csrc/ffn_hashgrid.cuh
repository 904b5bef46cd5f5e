// ffn_hashgrid.cuh -- multiresolution hash-grid encoding and its gradient scatter, plus the
// per-sample activation functions shared by the fused kernels.
#pragma once
#include "ffn_common.cuh"

namespace ffn {

// directional_encode, degrees 0..3 (ffnerf_OG.cl:572-602)
__device__ __forceinline__ void sh16(float x, float y, float z, float* sh) {
    sh[0] = 0.28209479177387814f;
    sh[1] = 0.4886025119029199f * y;
    sh[2] = 0.4886025119029199f * z;
    sh[3] = 0.4886025119029199f * x;
    sh[4] = 1.0925484305920792f * x * y;
    sh[5] = 1.0925484305920792f * y * z;
    sh[6] = 0.31539156525252005f * (3.0f * z * z - 1.0f);
    sh[7] = 1.0925484305920792f * x * z;
    sh[8] = 0.5462742152960396f * (x * x - y * y);
    sh[9] = 0.5900435899266435f * y * (3.0f * x * x - y * y);
    sh[10] = 2.890611442640554f * x * y * z;
    sh[11] = 0.4570457994644658f * y * (5.0f * z * z - 1.0f);
    sh[12] = 0.3731763325901154f * (5.0f * z * z * z - 3.0f * z);
    sh[13] = 0.4570457994644658f * x * (5.0f * z * z - 1.0f);
    sh[14] = 1.445305721320277f * z * (x * x - y * y);
    sh[15] = 0.5900435899266435f * x * (x * x - 3.0f * y * y);
}

// softplus / derivative / soft sigmoid (ffnerf_OG.cl:218-244)
__device__ __forceinline__ float softplus(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return expf(x);
    return log1pf(expf(x));
}
__device__ __forceinline__ float softplus_prime(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    float e = expf(x);
    return e / (1.0f + e);
}
__device__ __forceinline__ float sigmoid_soft(float x) {
    x *= 0.5f;
    x = fclamp(x, -18.0f, 18.0f);
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    float e = expf(x);
    return e / (1.0f + e);
}

// Per-level trilinear corners (ffnerf_OG.cl:1308-1338)
struct Corner8 { float w[8]; uint32_t base[8]; };
template <int F>
__device__ __forceinline__ void level_corners(const DevConfig& c, V3 p, int lvl, Corner8& k, uint64_t* cell_key = nullptr) {
    const int R = c.level_res[lvl];
    const float Rf = (float)R;
    const float ux = fm(p.x, Rf), uy = fm(p.y, Rf), uz = fm(p.z, Rf);
    const int ix0 = iclamp((int)floorf(ux), 0, R - 2);
    const int iy0 = iclamp((int)floorf(uy), 0, R - 2);
    const int iz0 = iclamp((int)floorf(uz), 0, R - 2);
    if (cell_key) *cell_key = (uint64_t)ix0 | ((uint64_t)iy0 << 21) | ((uint64_t)iz0 << 42);   // exact: R < 2^21
    const float fx = fs(ux, (float)ix0), fy = fs(uy, (float)iy0), fz = fs(uz, (float)iz0);
    const float wx[2] = {fs(1.0f, fx), fx}, wy[2] = {fs(1.0f, fy), fy}, wz[2] = {fs(1.0f, fz), fz};
    const uint32_t mask = (1u << c.level_log2[lvl]) - 1u;
    const uint32_t off = c.level_offset[lvl];
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
        const int dx = cc & 1, dy = (cc >> 1) & 1, dz = (cc >> 2) & 1;
        k.w[cc] = fm(fm(wx[dx], wy[dy]), wz[dz]);
        const uint32_t h = hash_u32((uint32_t)(ix0 + dx) * 73856093u ^ (uint32_t)(iy0 + dy) * 19349663u ^
                                    (uint32_t)(iz0 + dz) * 83492791u ^ (uint32_t)lvl * 2654435761u);
        k.base[cc] = (off + (h & mask)) * (uint32_t)F;
    }
}

// ffnerf_OG.cl:1291-1296
__device__ __forceinline__ V3 normalize_pos(const DevConfig& c, V3 x) {
    const V3 bmin = v3(c.bmin[0], c.bmin[1], c.bmin[2]);
    const V3 bsz = vsub(v3(c.bmax[0], c.bmax[1], c.bmax[2]), bmin);
    V3 p = vdiv(vsub(x, bmin), bsz);
    const float hi = 1.0f - 1.0e-6f;
    return v3(fclamp(p.x, 0.0f, hi), fclamp(p.y, 0.0f, hi), fclamp(p.z, 0.0f, hi));
}

// Reads one table entry: through L2 only (COHERENT, for tables updated during the kernel) or
// through the read-only cache.
template <bool COHERENT>
__device__ __forceinline__ float2 table_ld2(const float* p) {
    if constexpr (COHERENT) return __ldcg(reinterpret_cast<const float2*>(p));
    else return __ldg(reinterpret_cast<const float2*>(p));
}
template <bool COHERENT>
__device__ __forceinline__ float4 table_ld4(const float* p) {
    if constexpr (COHERENT) return __ldcg(reinterpret_cast<const float4*>(p));
    else return __ldg(reinterpret_cast<const float4*>(p));
}

// Writes the 16*F features of point p to a0 (a shared-memory row or a global output row).
template <int F, bool COHERENT = false>
__device__ __forceinline__ void encode(const DevConfig& c, const float* __restrict__ table, V3 p,
                                       float* a0) {
#pragma unroll 2
    for (int lvl = 0; lvl < L; ++lvl) {
        Corner8 k;
        level_corners<F>(c, p, lvl, k);
        float acc[F];
#pragma unroll
        for (int f = 0; f < F; ++f) acc[f] = 0.0f;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            if constexpr (F == 2) {
                const float2 t = table_ld2<COHERENT>(table + k.base[cc]);
                acc[0] = fmaf(k.w[cc], t.x, acc[0]);
                acc[1] = fmaf(k.w[cc], t.y, acc[1]);
            } else {
                const float4 t = table_ld4<COHERENT>(table + k.base[cc]);
                acc[0] = fmaf(k.w[cc], t.x, acc[0]);
                acc[1] = fmaf(k.w[cc], t.y, acc[1]);
                acc[2] = fmaf(k.w[cc], t.z, acc[2]);
                acc[3] = fmaf(k.w[cc], t.w, acc[3]);
            }
        }
        if constexpr (F == 2) *reinterpret_cast<float2*>(a0 + lvl * F) = make_float2(acc[0], acc[1]);
        else *reinterpret_cast<float4*>(a0 + lvl * F) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
}

template <int F>
__device__ __forceinline__ void scatter_grad(const DevConfig& c, float* __restrict__ grad, V3 p,
                                             const float* g /* 16*F */, const float* coef) {
#pragma unroll 1
    for (int lvl = 0; lvl < L; ++lvl) {
        float gf[F];
        bool any = false;
        float gv[4];
        if constexpr (F == 2) { const float2 t = *reinterpret_cast<const float2*>(g + lvl * F); gv[0] = t.x; gv[1] = t.y; }
        else { const float4 t = *reinterpret_cast<const float4*>(g + lvl * F); gv[0] = t.x; gv[1] = t.y; gv[2] = t.z; gv[3] = t.w; }
#pragma unroll
        for (int f = 0; f < F; ++f) {
            float v = gv[f];
            gf[f] = isfinite(v) ? coef[lvl] * v : 0.0f;   // non-finite features are skipped (ffnerf_OG.cl:2162)
            any |= gf[f] != 0.0f;
        }
        if (!any) continue;
        Corner8 k;
        level_corners<F>(c, p, lvl, k);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const float w = k.w[cc];
            if constexpr (F == 2) {
                red_add2(grad + k.base[cc], gf[0] * w, gf[1] * w);
            } else {
                red_add4(grad + k.base[cc], gf[0] * w, gf[1] * w, gf[2] * w, gf[3] * w);
            }
        }
    }
}

// Register-resident variants (fully unrolled over the levels): the 16 x 8 corner loads of a sample
// are independent, so the compiler can keep several levels' gathers in flight at once.
template <int F>
__device__ __forceinline__ void encode_regs(const DevConfig& c, const float* __restrict__ table, V3 p,
                                            float (&a0)[L * F]) {
#pragma unroll
    for (int lvl = 0; lvl < L; ++lvl) {
        Corner8 k;
        level_corners<F>(c, p, lvl, k);
        float acc[F];
#pragma unroll
        for (int f = 0; f < F; ++f) acc[f] = 0.0f;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            if constexpr (F == 2) {
                const float2 t = __ldg(reinterpret_cast<const float2*>(table + k.base[cc]));
                acc[0] = fmaf(k.w[cc], t.x, acc[0]);
                acc[1] = fmaf(k.w[cc], t.y, acc[1]);
            } else {
                const float4 t = __ldg(reinterpret_cast<const float4*>(table + k.base[cc]));
                acc[0] = fmaf(k.w[cc], t.x, acc[0]);
                acc[1] = fmaf(k.w[cc], t.y, acc[1]);
                acc[2] = fmaf(k.w[cc], t.z, acc[2]);
                acc[3] = fmaf(k.w[cc], t.w, acc[3]);
            }
        }
#pragma unroll
        for (int f = 0; f < F; ++f) a0[lvl * F + f] = acc[f];
    }
}

template <int F>
__device__ __forceinline__ void scatter_grad_regs(const DevConfig& c, float* __restrict__ grad, V3 p,
                                                  const float (&g)[L * F]) {
#pragma unroll
    for (int lvl = 0; lvl < L; ++lvl) {
        float gf[F];
        bool any = false;
#pragma unroll
        for (int f = 0; f < F; ++f) {
            const float v = g[lvl * F + f];
            gf[f] = isfinite(v) ? v : 0.0f;   // non-finite features are skipped (ffnerf_OG.cl:2162)
            any |= gf[f] != 0.0f;
        }
        if (!any) continue;
        Corner8 k;
        level_corners<F>(c, p, lvl, k);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const float w = k.w[cc];
            if constexpr (F == 2) {
                red_add2(grad + k.base[cc], gf[0] * w, gf[1] * w);
            } else {
                red_add4(grad + k.base[cc], gf[0] * w, gf[1] * w, gf[2] * w, gf[3] * w);
            }
        }
    }
}

}  // namespace ffn
