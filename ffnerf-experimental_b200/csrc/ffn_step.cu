// ffn_step.cu -- device kernels of the fused NeRF training step for B200 (sm_100a).
//
// Kernel map (reference file:line in MolSzabi/ffnerf-experimental):
//   fused_step_kernel    ffnerf_train_step (ffnerf_OG.cl:838-2174) + the per-sample half of
//                        update_ffnerf_oneWG's reduction (weight_update.cl:210-314)
//   reduce_partials      the cross-CTA half of that reduction
//   mlp_adam_kernel      adam_update_1_i32 (weight_update.cl:177-201) for every MLP parameter
//   table_sgd_kernel     the hash-table SGD update (ffnerf_OG.cl:2155-2169), applied from the
//                        accumulated gradient instead of in-kernel Hogwild adds
//   table_adam_kernel    opt-in Adam for the table (no reference counterpart)
//   occ_decay_kernel     occ_nibble_decay_write_both_q24 (decay_occ_grid_in-st.cl:13-113)
//   hash_fwd/bwd_kernel  the hash-grid encode (ffnerf_OG.cl:1286-1364) and its scatter
//                        (ffnerf_OG.cl:2090-2173) on their own, for the encode microbenchmark
//
// Layout of one tile in the fused kernel: ROWS samples (ROWS/spr rays), one thread per sample.
// The activations every layer produces are kept in shared memory as fp32 rows (padded by 4 floats
// so a row read by its own thread is bank-conflict free); the backward overwrites them in place
// with the deltas, so nothing per-sample is written to HBM except the ray colour.  The weight
// gradient of a layer is the outer product of its delta and input tiles summed over the tile's
// rows, computed cooperatively in 4x4 register blocks and accumulated into a per-CTA partial in
// global memory (L2-resident); a second kernel sums the partials in a fixed order.
#include "ffn_common.cuh"

#include <cfloat>

namespace ffn {

struct StepArgs {
    DevConfig c;
    ParamLayout lo;
    const float* params;
    const float* table;
    const uint32_t* occ_in;
    uint32_t* occ_st;
    const float4* rays;        // [n][2]: o, d
    const float4* targets;     // [n]
    float4* out;               // [n]
    float* grad_table;         // table gradient accumulator (sum of g*w)
    float* partials;           // [gridDim.x][P] per-CTA weight-gradient partials
    uint32_t n_rays;
    uint32_t ray_offset;
    float sh_mult, occ_strength;
    uint32_t seed;
    int do_train;
    int probe;                 // ffn_probe: forward with training rules, no backward
    // diagnostics (ffn_probe); all optional
    const float4* bypass;
    float* dbg_t; float* dbg_dt; int* dbg_idx; uint32_t* dbg_flags;
    float* dbg_sigma; float* dbg_rgb; float* dbg_trans;
};

// ---------------------------------------------------------------------------- small helpers
template <int N>
__device__ __forceinline__ void load_row(float (&r)[N], const float* row) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
        float4 v = *reinterpret_cast<const float4*>(row + i);
        r[i] = v.x; r[i + 1] = v.y; r[i + 2] = v.z; r[i + 3] = v.w;
    }
}

// out_row[i] = act(b[i] + sum_j W[i*IN+j] * in[j]), i < OUT  (fc_relu_in / fc_relu_mm /
// fc_linear_out, ffnerf_OG.cl:754-806).  W, b in shared memory.
template <int IN, bool RELU>
__device__ __forceinline__ void dense_fwd(const float (&in)[IN], const float* W, const float* b,
                                          int OUT, float* out_row) {
    for (int i = 0; i < OUT; ++i) {
        float s = b[i];
        const float* w = W + i * IN;
#pragma unroll
        for (int j = 0; j < IN; j += 4) {
            float4 wv = *reinterpret_cast<const float4*>(w + j);
            s = fmaf(wv.x, in[j], s);
            s = fmaf(wv.y, in[j + 1], s);
            s = fmaf(wv.z, in[j + 2], s);
            s = fmaf(wv.w, in[j + 3], s);
        }
        out_row[i] = RELU ? (s > 0.0f ? s : 0.0f) : s;
    }
}

// out_row[k] = (sum_j W[j*IN+k] * d[j]) masked by act_row[k] > 0, k < IN (bwd_linear_to_M /
// bwd_mm_to_M + relu_mask_apply, ffnerf_OG.cl:741-748,811-835).  out_row may alias act_row.
template <int OUT, int IN, bool MASK>
__device__ __forceinline__ void dense_bwd(const float (&d)[OUT], const float* W, const float* act_row,
                                          float* out_row) {
    for (int k = 0; k < IN; k += 4) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int j = 0; j < OUT; ++j) {
            float4 wv = *reinterpret_cast<const float4*>(W + j * IN + k);
            s0 = fmaf(wv.x, d[j], s0);
            s1 = fmaf(wv.y, d[j], s1);
            s2 = fmaf(wv.z, d[j], s2);
            s3 = fmaf(wv.w, d[j], s3);
        }
        if (MASK) {
            float4 a = *reinterpret_cast<const float4*>(act_row + k);
            s0 = a.x > 0.f ? s0 : 0.f; s1 = a.y > 0.f ? s1 : 0.f;
            s2 = a.z > 0.f ? s2 : 0.f; s3 = a.w > 0.f ? s3 : 0.f;
        }
        *reinterpret_cast<float4*>(out_row + k) = make_float4(s0, s1, s2, s3);
    }
}

// Weight gradient of one layer over the tile: gW[o][i] += sum_r D[r][o] * A[r][i] and
// gb[o] += sum_r D[r][o]  (update_layer_tile_adam_i32's reduction, weight_update.cl:260-314).
// D may have a zero pad column (OUT = 3 is read as 4).
template <int ROWS>
__device__ __forceinline__ void coop_wgrad(const float* D, int ldd, int OUT, const float* A, int lda,
                                           int IN, float* gW, float* gb) {
    const int nib = IN >> 2, nob = (OUT + 3) >> 2;
    for (int b = threadIdx.x; b < nib * nob; b += ROWS) {
        const int ob = b / nib, ib = b - ob * nib;
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
        for (int r = 0; r < ROWS; ++r) {
            const float4 dv = *reinterpret_cast<const float4*>(D + r * ldd + ob * 4);
            const float4 av = *reinterpret_cast<const float4*>(A + r * lda + ib * 4);
            const float dd[4] = {dv.x, dv.y, dv.z, dv.w};
            const float aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(dd[i], aa[j], acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int o = ob * 4 + i;
            if (o < OUT) {
                float4* g = reinterpret_cast<float4*>(gW + o * IN + ib * 4);
                float4 v = *g;
                v.x += acc[i][0]; v.y += acc[i][1]; v.z += acc[i][2]; v.w += acc[i][3];
                *g = v;
            }
        }
    }
    for (int o = threadIdx.x; o < OUT; o += ROWS) {
        float s = 0.f;
        for (int r = 0; r < ROWS; ++r) s += D[r * ldd + o];
        gb[o] += s;
    }
}

// ---------------------------------------------------------------------------- exact scans
// Blelloch exclusive scan of one ray's slice (ffnerf_OG.cl:619-637); every thread of the CTA
// calls it (one lane of one ray), levels separated by __syncthreads.
__device__ __forceinline__ void scan_excl(float* a, int lid, int n) {
    for (int stride = 1; stride < n; stride <<= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) a[idx] = fa(a[idx], a[idx - stride]);
        __syncthreads();
    }
    if (lid == 0) a[n - 1] = 0.0f;
    __syncthreads();
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) {
            float t = a[idx - stride];
            a[idx - stride] = a[idx];
            a[idx] = fa(a[idx], t);
        }
        __syncthreads();
    }
}
// ffnerf_OG.cl:639-646
__device__ __forceinline__ float reduce_sum(float* a, int lid, int n) {
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        if (lid < stride) a[lid] = fa(a[lid], a[lid + stride]);
        __syncthreads();
    }
    return a[0];
}
// ffnerf_OG.cl:648-656
__device__ __forceinline__ int lower_bound_cdf(const float* cdf, int n, float u) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (cdf[mid] >= u) hi = mid; else lo = mid + 1;
    }
    return lo;
}
// Seg = {a, v.xyz} in a float4; seg_combine(L,R) = {L.a*R.a, L.v + L.a*R.v} (ffnerf_OG.cl:686-687)
__device__ __forceinline__ float4 seg_combine(float4 l, float4 r) {
    return make_float4(fm(l.x, r.x), fa(l.y, fm(l.x, r.y)), fa(l.z, fm(l.x, r.z)), fa(l.w, fm(l.x, r.w)));
}
// scan_excl_seg (ffnerf_OG.cl:693-713); returns the ray's total to every lane.
__device__ __forceinline__ float4 scan_excl_seg(float4* s, int lid, int n) {
    for (int stride = 1; stride < n; stride <<= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) s[idx] = seg_combine(s[idx - stride], s[idx]);
        __syncthreads();
    }
    float4 total = s[n - 1];
    __syncthreads();
    if (lid == 0) s[n - 1] = make_float4(1.0f, 0.0f, 0.0f, 0.0f);
    __syncthreads();
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) {
            float4 t = s[idx - stride];
            s[idx - stride] = s[idx];
            s[idx] = seg_combine(t, s[idx]);
        }
        __syncthreads();
    }
    return total;
}
// aff_combine_rev(L,R) = {R.a*L.a, R.a*L.b + R.b} (ffnerf_OG.cl:689-691)
__device__ __forceinline__ float2 aff_combine_rev(float2 l, float2 r) {
    return make_float2(fm(r.x, l.x), fa(fm(r.x, l.y), r.y));
}
// scan_excl_aff_rev (ffnerf_OG.cl:715-735)
__device__ __forceinline__ void scan_excl_aff_rev(float2* s, int lid, int n) {
    for (int stride = 1; stride < n; stride <<= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) s[idx] = aff_combine_rev(s[idx - stride], s[idx]);
        __syncthreads();
    }
    if (lid == 0) s[n - 1] = make_float2(1.0f, 0.0f);
    __syncthreads();
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) {
            float2 t = s[idx - stride];
            s[idx - stride] = s[idx];
            s[idx] = aff_combine_rev(t, s[idx]);
        }
        __syncthreads();
    }
}

// ray_aabb_intersect (ffnerf_OG.cl:322-343)
__device__ __forceinline__ bool ray_aabb(V3 o, V3 d, V3 bmin, V3 bmax, float* t0, float* t1) {
    const float inf = __int_as_float(0x7f800000);
    V3 invd = v3(d.x != 0.0f ? fd(1.0f, d.x) : inf, d.y != 0.0f ? fd(1.0f, d.y) : inf,
                 d.z != 0.0f ? fd(1.0f, d.z) : inf);
    V3 tb = vmul(vsub(bmin, o), invd);
    V3 tt = vmul(vsub(bmax, o), invd);
    float tmin = fmaxf(fminf(tb.x, tt.x), fmaxf(fminf(tb.y, tt.y), fminf(tb.z, tt.z)));
    float tmax = fminf(fmaxf(tb.x, tt.x), fminf(fmaxf(tb.y, tt.y), fmaxf(tb.z, tt.z)));
    if (tmax < tmin) return false;
    *t0 = tmin;
    *t1 = tmax;
    return true;
}

// atomic nibble max (ffnerf_OG.cl:486-512)
__device__ __forceinline__ void occ_nibble_max(uint32_t* grid, int cell, uint32_t sub, uint32_t q) {
    const uint32_t shift = 4u * sub, mask = 0xFu << shift;
    uint32_t old = grid[cell];
    for (int it = 0; it < 64; ++it) {   // bounded: 8 nibbles can each rise at most 15 times
        uint32_t old_q = ((old >> shift) & 0xFu) + 1u;
        if (q <= old_q) return;
        uint32_t nw = (old & ~mask) | (((q - 1u) & 0xFu) << shift);
        uint32_t prev = atomicCAS(grid + cell, old, nw);
        if (prev == old) return;
        old = prev;
    }
}

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
__device__ __forceinline__ void level_corners(const DevConfig& c, V3 p, int lvl, Corner8& k) {
    const int R = c.level_res[lvl];
    const float Rf = (float)R;
    const float ux = fm(p.x, Rf), uy = fm(p.y, Rf), uz = fm(p.z, Rf);
    const int ix0 = iclamp((int)floorf(ux), 0, R - 2);
    const int iy0 = iclamp((int)floorf(uy), 0, R - 2);
    const int iz0 = iclamp((int)floorf(uz), 0, R - 2);
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

// Writes the 16*F features of point p to a0 (a shared-memory row or a global output row).
template <int F>
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
        if constexpr (F == 2) *reinterpret_cast<float2*>(a0 + lvl * F) = make_float2(acc[0], acc[1]);
        else *reinterpret_cast<float4*>(a0 + lvl * F) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
}

template <int F>
__device__ __forceinline__ void scatter_grad(const DevConfig& c, float* __restrict__ grad, V3 p,
                                             const float* g /* 16*F */) {
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
                atomicAdd(reinterpret_cast<float2*>(grad + k.base[cc]), make_float2(gf[0] * w, gf[1] * w));
            } else {
                atomicAdd(reinterpret_cast<float4*>(grad + k.base[cc]),
                          make_float4(gf[0] * w, gf[1] * w, gf[2] * w, gf[3] * w));
            }
        }
    }
}

// ---------------------------------------------------------------------------- fused kernel
template <int F, int ND, int NC, int ROWS>
struct Smem {
    static constexpr int LPOS = L * F;
    static constexpr int LDA0 = LPOS + 4;
    static constexpr int LDH = M + 4;
    static constexpr int LDC = C_IN + 4;
    static constexpr int MAX_RAYS = ROWS / 16;
    __host__ __device__ static int floats(int P) {
        int pw = (P + 3) & ~3;
        return pw + ROWS * (LDA0 + ND * LDH + LDC + NC * LDH + 4)  // weights + activation tiles
               + ROWS * 6          // cand, cdf, Ts, DTs, Tr, key
               + ROWS * 4          // segs (float4)
               + ROWS * 4          // aff scan + elem (float2 each)
               + MAX_RAYS * 2      // run-start bits
               + MAX_RAYS * 16;    // per-ray scalars
    }
};

enum { RS_T0, RS_T1, RS_DTB, RS_U0, RS_HIT, RS_TFIN, RS_GRX, RS_GRY, RS_GRZ, RS_GTEND };

template <int F, int ND, int NC, int ROWS>
__global__ void __launch_bounds__(ROWS, 1) fused_step_kernel(const StepArgs a) {
    using S = Smem<F, ND, NC, ROWS>;
    constexpr int LPOS = S::LPOS, LDA0 = S::LDA0, LDH = S::LDH, LDC = S::LDC;
    extern __shared__ __align__(16) float smem[];
    const DevConfig& c = a.c;
    const int P = a.lo.total;
    const int Pw = (P + 3) & ~3;
    float* sW = smem;
    float* sA0 = sW + Pw;
    float* sHd = sA0 + ROWS * LDA0;
    float* sAc = sHd + ND * ROWS * LDH;
    float* sHc = sAc + ROWS * LDC;
    float* sDC = sHc + NC * ROWS * LDH;
    float* sCand = sDC + ROWS * 4;
    float* sCdf = sCand + ROWS;
    float* sTs = sCdf + ROWS;
    float* sDTs = sTs + ROWS;
    float* sTr = sDTs + ROWS;
    uint32_t* sKey = reinterpret_cast<uint32_t*>(sTr + ROWS);
    float4* sSeg = reinterpret_cast<float4*>(sKey + ROWS);
    float2* sAffS = reinterpret_cast<float2*>(sSeg + ROWS);
    float2* sAffE = sAffS + ROWS;
    uint32_t* sChg = reinterpret_cast<uint32_t*>(sAffE + ROWS);
    float* sRay = reinterpret_cast<float*>(sChg + S::MAX_RAYS * 2);

    const int tid = threadIdx.x;
    const int spr = c.spr;
    const int rl = tid / spr, lid = tid - rl * spr, rbase = rl * spr;
    const int rays_per_tile = ROWS / spr;
    const bool train = a.do_train != 0;
    const bool probe = a.probe != 0;
    const int n_tiles = (int)((a.n_rays + rays_per_tile - 1) / rays_per_tile);

    // weights -> shared memory (fp32, the parameter blob as is)
    for (int i = tid * 4; i < Pw; i += ROWS * 4)
        *reinterpret_cast<float4*>(sW + i) = *reinterpret_cast<const float4*>(a.params + i);
    float* part = a.partials ? a.partials + (size_t)blockIdx.x * Pw : nullptr;
    if (train && !probe && part)
        for (int i = tid * 4; i < Pw; i += ROWS * 4) *reinterpret_cast<float4*>(part + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();

    const float* Wd_in = sW + a.lo.off[P_WD_IN];
    const float* Wd_out = sW + a.lo.off[P_WD_OUT];
    const float* bd_out = sW + a.lo.off[P_BD_OUT];
    const float* Wc_in = sW + a.lo.off[P_WC_IN];
    const float* Wc_out = sW + a.lo.off[P_WC_OUT];
    const float* bc_out = sW + a.lo.off[P_BC_OUT];

    const V3 bmin = v3(c.bmin[0], c.bmin[1], c.bmin[2]);
    const V3 bmax = v3(c.bmax[0], c.bmax[1], c.bmax[2]);
    const V3 bsize = vsub(bmax, bmin);
    const V3 inv_box = v3(fd(1.0f, bsize.x), fd(1.0f, bsize.y), fd(1.0f, bsize.z));
    const float Gf = (float)c.G;
    const float inv_n = 1.0f / (float)spr;

    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const uint32_t ray_idx = (uint32_t)tile * rays_per_tile + rl;   // index in this launch
        const bool valid = ray_idx < a.n_rays;
        const uint32_t ray_id = a.ray_offset + ray_idx;                  // global id (RNG key)
        float4 ro = make_float4(0.f, 0.f, 0.f, 0.f), rd = make_float4(0.f, 0.f, 1.f, 0.f);
        if (valid) { ro = a.rays[2 * ray_idx]; rd = a.rays[2 * ray_idx + 1]; }
        const V3 o = v3(ro.x, ro.y, ro.z), d = v3(rd.x, rd.y, rd.z);

        // ------------------------------------------------ sampler (ffnerf_OG.cl:1002-1250)
        if (lid == 0) {
            float t0 = 0.f, t1 = 0.f, dtb = 0.f, u0 = 0.f;
            bool hit = false;
            if (valid) {
                float ta, tb;
                hit = ray_aabb(o, d, bmin, bmax, &ta, &tb);
                if (hit) {
                    ta = fmaxf(ta, c.t_near);
                    tb = fminf(tb, c.t_far);
                    if (tb <= ta) hit = false; else { t0 = fa(ta, 1.0e-6f); t1 = tb; }
                }
                float x = hit ? fm(fs(t1, t0), inv_n) : 0.0f;
                x = fminf(c.dt_max, fmaxf(c.dt_min, x));
                dtb = hit ? x : 0.0f;
                if (hit) {
                    uint32_t r0 = hash_u32(a.seed ^ ray_id * 1597334677u);
                    u0 = fm(rand01(&r0), inv_n);
                }
            }
            float* rs = sRay + rl * 16;
            rs[RS_T0] = t0; rs[RS_T1] = t1; rs[RS_DTB] = dtb; rs[RS_U0] = u0; rs[RS_HIT] = hit ? 1.f : 0.f;
        }
        if (lid < 2) sChg[rl * 2 + lid] = 0u;
        __syncthreads();
        const float* rs = sRay + rl * 16;
        const bool hit = rs[RS_HIT] != 0.0f;
        const float t0 = rs[RS_T0], t1 = rs[RS_T1], dtb = rs[RS_DTB], u0 = rs[RS_U0];
        int idx_sel = 0;
        {
            float wp = 0.0f, active = 0.0f, tk = 0.0f;
            if (hit) {
                uint32_t rng = hash_u32(a.seed ^ ray_id * 747796405u ^ (uint32_t)lid * 2891336453u);
                const float u = fm(fa((float)lid, rand01(&rng)), inv_n);
                tk = fa(t0, fm(fs(t1, t0), u));
                const V3 xk = ray_point(o, d, tk);
                const V3 gm = v3(fm(fm(fs(xk.x, bmin.x), inv_box.x), Gf), fm(fm(fs(xk.y, bmin.y), inv_box.y), Gf),
                                 fm(fm(fs(xk.z, bmin.z), inv_box.z), Gf));
                float occ = 0.0f;
                if (gm.x >= 0.0f && gm.x < Gf && gm.y >= 0.0f && gm.y < Gf && gm.z >= 0.0f && gm.z < Gf) {
                    const int G = c.G;
                    const int ix = iclamp((int)floorf(gm.x), 0, G - 1);
                    const int iy = iclamp((int)floorf(gm.y), 0, G - 1);
                    const int iz = iclamp((int)floorf(gm.z), 0, G - 1);
                    const uint32_t packed = __ldg(a.occ_in + (ix + G * (iy + G * iz)));
                    const float fx = fclamp(fs(gm.x, floorf(gm.x)), 0.0f, 1.0f - 1e-7f);
                    const float fy = fclamp(fs(gm.y, floorf(gm.y)), 0.0f, 1.0f - 1e-7f);
                    const float fz = fclamp(fs(gm.z, floorf(gm.z)), 0.0f, 1.0f - 1e-7f);
                    const uint32_t sub = (uint32_t)(fx > 0.5f) + 2u * (uint32_t)(fy > 0.5f) + 4u * (uint32_t)(fz > 0.5f);
                    const uint32_t occ4 = (packed >> (4u * sub)) & 0xFu;
                    const uint32_t q = train ? occ4 + 1u : (occ4 > 2u ? occ4 - 2u : 0u);
                    occ = fm((float)q, 1.0f / 16.0f);
                }
                const float infer_f = train ? 0.0f : 1.0f;
                active = occ > 0.0f ? 1.0f : 0.0f;
                const float rho_base = fa(c.rho_min, fm(fs(c.rho_max, c.rho_min), occ));
                const float rho = fm(rho_base, fa(fs(1.0f, infer_f), fm(infer_f, active)));
                const float w_raw = fmaxf(fm(rho, dtb), 0.0f);
                wp = w_raw <= 0.0f ? 0.0f : own_powr(w_raw, 1.3f);       // GAMMA_W
            }
            sCand[tid] = tk;
            float* cdf = sCdf + rbase;
            sCdf[tid] = wp;
            __syncthreads();
            scan_excl(cdf, lid, spr);
            const float pref = sCdf[tid];
            sCdf[tid] = wp;
            __syncthreads();
            const float Wtot = fmaxf(reduce_sum(cdf, lid, spr), 1.0e-12f);
            __syncthreads();
            const float pi = fclamp(fd(pref, Wtot), 0.0f, 1.0f);
            const float g = fm(wp, own_expf(fm(-0.0f, pi)));        // LAMBDA_FOCUS = 0
            sCdf[tid] = g;
            __syncthreads();
            const float gtot = fmaxf(reduce_sum(cdf, lid, spr), 1.0e-12f);
            __syncthreads();
            sCdf[tid] = active;
            __syncthreads();
            const float active_count = reduce_sum(cdf, lid, spr);
            __syncthreads();
            const float any_active = active_count > 0.5f ? 1.0f : 0.0f;
            const float inv_active = fd(1.0f, fmaxf(active_count, 1.0f));
            const float ut = fmix(inv_n, fm(active, inv_active), any_active);
            const float pt = fm(any_active, fd(g, gtot));
            const float p = fa(fm(0.3f, ut), fm(1.0f - 0.3f, pt));  // UNIFORM_PART
            sCdf[tid] = p;
            __syncthreads();
            scan_excl(cdf, lid, spr);
            sCdf[tid] = fa(sCdf[tid], p);
            __syncthreads();
            float t_out = 0.0f;
            uint32_t key = 0xFFFFFFFEu;
            if (hit) {
                const float uk = fminf(fa(u0, fm((float)lid, inv_n)), 0.99999994f);
                idx_sel = lower_bound_cdf(cdf, spr, uk);
                t_out = sCand[rbase + idx_sel];
                const V3 xo = ray_point(o, d, t_out);
                const V3 go = v3(fm(fm(fs(xo.x, bmin.x), inv_box.x), Gf), fm(fm(fs(xo.y, bmin.y), inv_box.y), Gf),
                                 fm(fm(fs(xo.z, bmin.z), inv_box.z), Gf));
                const int ix = (int)floorf(go.x), iy = (int)floorf(go.y), iz = (int)floorf(go.z);
                const uint32_t G = (uint32_t)c.G;
                if ((uint32_t)ix < G && (uint32_t)iy < G && (uint32_t)iz < G) {
                    const float fx = fclamp(fs(go.x, floorf(go.x)), 0.0f, 1.0f - 1e-7f);
                    const float fy = fclamp(fs(go.y, floorf(go.y)), 0.0f, 1.0f - 1e-7f);
                    const float fz = fclamp(fs(go.z, floorf(go.z)), 0.0f, 1.0f - 1e-7f);
                    const uint32_t sub = (uint32_t)(fx >= 0.5f) + 2u * (uint32_t)(fy >= 0.5f) + 4u * (uint32_t)(fz >= 0.5f);
                    const uint32_t cell = (uint32_t)ix + G * ((uint32_t)iy + G * (uint32_t)iz);
                    key = (cell << 3) | (sub & 7u);
                }
            }
            __syncthreads();   // every lane has read cand/cdf
            sTs[tid] = t_out;
            sDTs[tid] = hit ? dtb : 0.0f;
            sKey[tid] = key;
            __syncthreads();
            if (hit) {
                if (lid == 0 || sKey[tid] != sKey[tid - 1]) atomicOr(sChg + rl * 2 + (lid >> 5), 1u << (lid & 31));
            } else if (lid < 2) {
                // no hit: every sample starts a run (ffnerf_OG.cl:1058-1063)
                const int lo_bit = lid * 32;
                const int nb = min(32, max(0, spr - lo_bit));
                sChg[rl * 2 + lid] = nb == 32 ? 0xFFFFFFFFu : ((1u << nb) - 1u);
            }
            __syncthreads();
        }

        // ------------------------------------------------ per-sample forward (:1257-1496)
        const float t_s = sTs[tid];
        const float dt_s = sDTs[tid];
        const V3 xs = ray_point(o, d, t_s);
        const V3 pn = normalize_pos(c, xs);
        float sigma, rgb[3], dout0 = 0.0f;
        if (probe && a.bypass) {
            float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
            if (valid) b = a.bypass[(size_t)ray_idx * spr + lid];
            sigma = b.x; rgb[0] = b.y; rgb[1] = b.z; rgb[2] = b.w;
        } else {
            float* a0row = sA0 + tid * LDA0;
            if (hit) encode<F>(c, a.table, pn, a0row);   // rays that miss the box contribute nothing
            else {
#pragma unroll
                for (int i = 0; i < LPOS; i += 4) *reinterpret_cast<float4*>(a0row + i) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            // density MLP
            {
                float in[LPOS];
                load_row<LPOS>(in, a0row);
                dense_fwd<LPOS, true>(in, Wd_in, sW + a.lo.off[P_BD_0], M, sHd + tid * LDH);
            }
#pragma unroll
            for (int l = 1; l < ND; ++l) {
                float in[M];
                load_row<M>(in, sHd + (l - 1) * ROWS * LDH + tid * LDH);
                dense_fwd<M, true>(in, sW + a.lo.off[P_WD_IN + l], sW + a.lo.off[P_BD_0 + l], M,
                                   sHd + l * ROWS * LDH + tid * LDH);
            }
            float* acrow = sAc + tid * LDC;
            {
                float in[M];
                load_row<M>(in, sHd + (ND - 1) * ROWS * LDH + tid * LDH);
                dense_fwd<M, false>(in, Wd_out, bd_out, D_OUT, acrow);
            }
            dout0 = acrow[0];
            sigma = softplus(fclamp(dout0, -10.0f, 10.0f));
            {
                float sh[L_DIR];
                sh16(d.x, d.y, d.z, sh);
#pragma unroll
                for (int i = 0; i < L_DIR; ++i) acrow[D_OUT + i] = sh[i] * a.sh_mult;
            }
            // color MLP
            {
                float in[C_IN];
                load_row<C_IN>(in, acrow);
                dense_fwd<C_IN, true>(in, Wc_in, sW + a.lo.off[P_BC_0], M, sHc + tid * LDH);
            }
#pragma unroll
            for (int l = 1; l < NC; ++l) {
                float in[M];
                load_row<M>(in, sHc + (l - 1) * ROWS * LDH + tid * LDH);
                dense_fwd<M, true>(in, sW + a.lo.off[P_WC_IN + l], sW + a.lo.off[P_BC_0 + l], M,
                                   sHc + l * ROWS * LDH + tid * LDH);
            }
            {
                float in[M];
                load_row<M>(in, sHc + (NC - 1) * ROWS * LDH + tid * LDH);
                float co[4];
                dense_fwd<M, false>(in, Wc_out, bc_out, C_OUT, co);
#pragma unroll
                for (int k = 0; k < 3; ++k) rgb[k] = sigmoid_soft(co[k]);
            }
        }
        if (dt_s <= 0.0f) sigma = 0.0f;

        // ------------------------------------------------ compositing (:1505-1634)
        float alpha = 0.0f;
        if (dt_s > 0.0f) alpha = fs(1.0f, own_expf(fclamp(fm(-sigma, dt_s), -5.0f, 18.0f)));
        const float oma = fs(1.0f, alpha);
        sSeg[tid] = make_float4(oma, fm(alpha, rgb[0]), fm(alpha, rgb[1]), fm(alpha, rgb[2]));
        __syncthreads();
        const float4 total = scan_excl_seg(sSeg + rbase, lid, spr);
        const float T_s = sSeg[tid].x;
        sTr[tid] = T_s;
        const float T_final = total.x;
        if (lid == 0) {
            float bg[3] = {0.f, 0.f, 0.f};
            if (train) {
                if (c.background == 1) { bg[0] = bg[1] = bg[2] = 1.0f; }
                else if (c.background == 2) {
                    uint32_t rb = hash_u32(a.seed ^ ray_id * 747796405u ^ 0xA511E9B3u);
                    bg[0] = rand01(&rb); bg[1] = rand01(&rb); bg[2] = rand01(&rb);
                }
            }
            const float cf[3] = {fa(total.y, fm(T_final, bg[0])), fa(total.z, fm(T_final, bg[1])),
                                 fa(total.w, fm(T_final, bg[2]))};
            float4 tg = make_float4(0.f, 0.f, 0.f, 0.f);
            if (valid && a.targets) tg = a.targets[ray_idx];
            const float tv[3] = {tg.x, tg.y, tg.z};
            float gr[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const float df = fs(cf[k], tv[k]);
                gr[k] = fm(df, fd(1.0f, __fsqrt_rn(fa(fm(df, df), 1.0e-3f * 1.0e-3f))));  // charbonnier'
            }
            float* rw = sRay + rl * 16;
            rw[RS_TFIN] = T_final;
            rw[RS_GRX] = gr[0]; rw[RS_GRY] = gr[1]; rw[RS_GRZ] = gr[2];
            rw[RS_GTEND] = fa(fa(fm(gr[0], bg[0]), fm(gr[1], bg[1])), fm(gr[2], bg[2]));
            if (valid)
                a.out[ray_idx] = make_float4(fclamp(cf[0], 0.f, 1.f), fclamp(cf[1], 0.f, 1.f),
                                             fclamp(cf[2], 0.f, 1.f), (train && !probe) ? 4.0f : 0.0f);
        }
        __syncthreads();
        const float gr0 = rs[RS_GRX], gr1 = rs[RS_GRY], gr2 = rs[RS_GRZ], gT_end = rs[RS_GTEND];
        const float w_s = fm(T_s, alpha);
        const float dLdc[3] = {fm(w_s, gr0), fm(w_s, gr1), fm(w_s, gr2)};
        {
            const float B_s = fa(fa(fm(gr0, fm(alpha, rgb[0])), fm(gr1, fm(alpha, rgb[1]))), fm(gr2, fm(alpha, rgb[2])));
            const int k = spr - 1 - lid;
            sAffE[rbase + k] = make_float2(oma, B_s);
            sAffS[rbase + k] = make_float2(oma, B_s);
        }
        __syncthreads();
        scan_excl_aff_rev(sAffS + rbase, lid, spr);
        float dLds;
        {
            const int k = spr - 1 - lid;
            float gT_next = gT_end;
            if (k >= 1) {
                const float2 incl = aff_combine_rev(sAffS[rbase + k - 1], sAffE[rbase + k - 1]);
                gT_next = fa(fm(incl.x, gT_end), incl.y);
            }
            const float gAC = fa(fa(fm(gr0, fm(T_s, rgb[0])), fm(gr1, fm(T_s, rgb[1]))), fm(gr2, fm(T_s, rgb[2])));
            const float gAlpha = fs(gAC, fm(gT_next, T_s));
            const float dad = dt_s > 0.0f ? fm(dt_s, oma) : 0.0f;
            const float regu = dt_s > 0.0f ? fd(fm(5e-3f, dt_s), (float)(uint32_t)spr) : 0.0f;  // DENSITY_PENALTY_LMD
            dLds = fa(fm(gAlpha, dad), regu);
        }

        // ------------------------------------------------ occupancy proposals (:1640-1821)
        const uint32_t chg0 = sChg[rl * 2], chg1 = sChg[rl * 2 + 1];
        if (train && a.occ_strength > 0.0f && dt_s > 0.0f && valid) {
            const bool is_rep = (((lid < 32 ? chg0 : chg1) >> (lid & 31)) & 1u) != 0u;
            const int G = c.G;
            const V3 gp = v3(fm(fm(fs(xs.x, bmin.x), inv_box.x), Gf), fm(fm(fs(xs.y, bmin.y), inv_box.y), Gf),
                             fm(fm(fs(xs.z, bmin.z), inv_box.z), Gf));
            const int ix = (int)floorf(gp.x), iy = (int)floorf(gp.y), iz = (int)floorf(gp.z);
            if (is_rep && (uint32_t)ix < (uint32_t)G && (uint32_t)iy < (uint32_t)G && (uint32_t)iz < (uint32_t)G) {
                const float fx = fs(gp.x, floorf(gp.x)), fy = fs(gp.y, floorf(gp.y)), fz = fs(gp.z, floorf(gp.z));
                const uint32_t sub = (uint32_t)(fx >= 0.5f) + 2u * (uint32_t)(fy >= 0.5f) + 4u * (uint32_t)(fz >= 0.5f);
                const int cell = ix + G * (iy + G * iz);
                // next run start after lid (chg_find_next, ffnerf_OG.cl:446-469)
                int next = spr;
                {
                    const uint64_t bits = ((uint64_t)chg1 << 32) | chg0;
                    const uint64_t rest = (lid + 1 < 64) ? (bits >> (lid + 1)) : 0ull;
                    if (rest) next = min(spr, lid + 1 + __ffsll((long long)rest) - 1);
                }
                float pred = 0.0f;
                {
                    const V3 csz = vscale(1.0f / Gf, bsize);   // box_size * (1/G)
                    const V3 cmin = vadd(bmin, vmul(v3((float)ix, (float)iy, (float)iz), csz));
                    const V3 cmax = vadd(cmin, csz);
                    float te, tx;
                    if (ray_aabb(o, d, cmin, cmax, &te, &tx)) {
                        te = fmaxf(te, c.t_near);
                        tx = fminf(tx, c.t_far);
                        if (tx > te) {
                            const int pe = lid > 0 ? lid - 1 : 0;
                            const float t_prev = sTs[rbase + pe], T_prev = sTr[rbase + pe];
                            const float t_cur = sTs[tid], T_cur = sTr[tid];
                            const float den0 = fs(t_cur, t_prev);
                            float uu0 = fabsf(den0) > 1.0e-8f ? fd(fs(te, t_prev), den0) : 0.0f;
                            uu0 = fclamp(uu0, 0.0f, 1.0f);
                            const float T_enter = fmix(T_prev, T_cur, uu0);
                            const int last = next < spr ? next - 1 : spr - 1;
                            const float t_last = sTs[rbase + last], T_last = sTr[rbase + last];
                            const float t_next = next < spr ? sTs[rbase + next] : tx;
                            const float T_next = next < spr ? sTr[rbase + next] : T_final;
                            const float den1 = fs(t_next, t_last);
                            float uu1 = fabsf(den1) > 1.0e-8f ? fd(fs(tx, t_last), den1) : 1.0f;
                            uu1 = fclamp(uu1, 0.0f, 1.0f);
                            const float T_exit = fmix(T_last, T_next, uu1);
                            pred = fclamp(fd(fs(T_enter, T_exit), fmaxf(T_enter, 1.0e-12f)), 0.0f, 1.0f);
                        }
                    }
                }
                const uint32_t old_q = ((__ldg(a.occ_in + cell) >> (4u * sub)) & 0xFu) + 1u;
                uint32_t proposed = old_q;
                const float pred16 = fm(pred, 16.0f);
                const uint32_t rkey = hash_u32(a.seed ^ ray_id * 747796405u ^ (uint32_t)lid * 2891336453u ^
                                               (uint32_t)cell * 9781u ^ sub * 6271u);
                if (pred16 > (float)old_q && old_q < 16u) {
                    const float f0 = floorf(pred16);
                    const float frac = fs(pred16, f0);
                    const uint32_t q0 = (uint32_t)f0;
                    const uint32_t thresh = (uint32_t)fm(frac, 16777216.0f);
                    uint32_t qs = (rkey & 0x00FFFFFFu) < thresh ? q0 + 1u : q0;
                    proposed = qs > 16u ? 16u : qs;
                }
                const float lat = fm(fs(bmax.x, bmin.x), 1.0f / Gf);
                const float Dh = fm(0.5f, vlength(bsize));
                const float tl = fd(t_s, fmaxf(lat, 1.0e-12f));
                const float Dl = fd(Dh, fmaxf(lat, 1.0e-12f));
                const float num = fa(fa(fm(tl, tl), tl), 1.0f / 3.0f);
                const float den = fa(fa(fm(Dl, Dl), Dl), 1.0f / 3.0f);
                const float keep_p = fminf(fd(num, fmaxf(den, 1.0e-12f)), 1.0f);
                bool send = keep_p >= 1.0f;
                if (!send) {
                    uint32_t rk = rkey;
                    send = rand01(&rk) <= keep_p;
                }
                if (send) occ_nibble_max(a.occ_st, cell, sub, proposed);
            }
        }

        if (probe) {
            if (valid) {
                const size_t s = (size_t)ray_idx * spr + lid;
                if (a.dbg_t) a.dbg_t[s] = t_s;
                if (a.dbg_dt) a.dbg_dt[s] = dt_s;
                if (a.dbg_idx) a.dbg_idx[s] = idx_sel;
                if (a.dbg_sigma) a.dbg_sigma[s] = sigma;
                if (a.dbg_rgb) { a.dbg_rgb[3 * s] = rgb[0]; a.dbg_rgb[3 * s + 1] = rgb[1]; a.dbg_rgb[3 * s + 2] = rgb[2]; }
                if (a.dbg_trans) a.dbg_trans[s] = T_s;
                if (a.dbg_flags && lid == 0) { a.dbg_flags[2 * ray_idx] = chg0; a.dbg_flags[2 * ray_idx + 1] = chg1; }
            }
            __syncthreads();
            continue;
        }
        if (!train) {
            __syncthreads();
            continue;
        }

        // ------------------------------------------------ output deltas (:1858-1891)
        float dcout[3];
        float ddout0;
        {
            const float Dh = 0.5f * vlength(bsize);
            const float t = t_s, dtl = dt_s;
            const float num = t * t + t * dtl + (dtl * dtl / 3.0f);
            const float den = Dh * Dh + Dh * dtl + (dtl * dtl / 3.0f);
            const float xr = t / fmaxf(Dh, 1.0e-12f);
            const float sflag = xr >= 1.0f ? 0.0f : 1.0f;
            const float gate = (1.0f - sflag) * 1.0f + sflag * powf(fmaxf(xr, 1.0e-12f), 0.2f);
            float f_vol = gate * num / fmaxf(den, 1.0e-12f);
            if (!valid || !hit) f_vol = 0.0f;
            const float d_sigma = f_vol * dLds;
#pragma unroll
            for (int k = 0; k < 3; ++k) dcout[k] = (f_vol * dLdc[k]) * ((rgb[k] * (1.0f - rgb[k])) * 0.5f);
            ddout0 = 1.0f * d_sigma * softplus_prime(fclamp(dout0, -18.0f, 18.0f));
        }
        *reinterpret_cast<float4*>(sDC + tid * 4) = make_float4(dcout[0], dcout[1], dcout[2], 0.0f);
        __syncthreads();

        // ------------------------------------------------ backward (:1930-2082) + weight grads
        float* gpart = part;
        const ParamLayout& lo = a.lo;
        // color head
        coop_wgrad<ROWS>(sDC, 4, C_OUT, sHc + (NC - 1) * ROWS * LDH, LDH, M, gpart + lo.off[P_WC_OUT], gpart + lo.off[P_BC_OUT]);
        __syncthreads();
        {
            float dv[C_OUT] = {dcout[0], dcout[1], dcout[2]};
            float* row = sHc + (NC - 1) * ROWS * LDH + tid * LDH;
            dense_bwd<C_OUT, M, true>(dv, Wc_out, row, row);
        }
#pragma unroll
        for (int l = NC - 1; l >= 1; --l) {
            __syncthreads();
            coop_wgrad<ROWS>(sHc + l * ROWS * LDH, LDH, M, sHc + (l - 1) * ROWS * LDH, LDH, M,
                             gpart + lo.off[P_WC_IN + l], gpart + lo.off[P_BC_0 + l]);
            __syncthreads();
            float dv[M];
            load_row<M>(dv, sHc + l * ROWS * LDH + tid * LDH);
            float* row = sHc + (l - 1) * ROWS * LDH + tid * LDH;
            dense_bwd<M, M, true>(dv, sW + lo.off[P_WC_IN + l], row, row);
        }
        __syncthreads();
        coop_wgrad<ROWS>(sHc, LDH, M, sAc, LDC, C_IN, gpart + lo.off[P_WC_IN], gpart + lo.off[P_BC_0]);
        __syncthreads();
        {
            // delta at the density output: color contribution through Wc_in[:, :16] (:2016-2020)
            float dv[M];
            load_row<M>(dv, sHc + tid * LDH);
            float* row = sAc + tid * LDC;
            for (int i = 0; i < D_OUT; i += 4) {
                float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
                for (int j = 0; j < M; ++j) {
                    const float4 w = *reinterpret_cast<const float4*>(Wc_in + j * C_IN + i);
                    s0 = fmaf(w.x, dv[j], s0); s1 = fmaf(w.y, dv[j], s1);
                    s2 = fmaf(w.z, dv[j], s2); s3 = fmaf(w.w, dv[j], s3);
                }
                const float base0 = i == 0 ? ddout0 : 0.0f;
                *reinterpret_cast<float4*>(row + i) = make_float4(base0 + s0, s1, s2, s3);
            }
        }
        __syncthreads();
        coop_wgrad<ROWS>(sAc, LDC, D_OUT, sHd + (ND - 1) * ROWS * LDH, LDH, M, gpart + lo.off[P_WD_OUT], gpart + lo.off[P_BD_OUT]);
        __syncthreads();
        {
            float dv[D_OUT];
            load_row<D_OUT>(dv, sAc + tid * LDC);
            float* row = sHd + (ND - 1) * ROWS * LDH + tid * LDH;
            dense_bwd<D_OUT, M, true>(dv, Wd_out, row, row);
        }
#pragma unroll
        for (int l = ND - 1; l >= 1; --l) {
            __syncthreads();
            coop_wgrad<ROWS>(sHd + l * ROWS * LDH, LDH, M, sHd + (l - 1) * ROWS * LDH, LDH, M,
                             gpart + lo.off[P_WD_IN + l], gpart + lo.off[P_BD_0 + l]);
            __syncthreads();
            float dv[M];
            load_row<M>(dv, sHd + l * ROWS * LDH + tid * LDH);
            float* row = sHd + (l - 1) * ROWS * LDH + tid * LDH;
            dense_bwd<M, M, true>(dv, sW + lo.off[P_WD_IN + l], row, row);
        }
        __syncthreads();
        coop_wgrad<ROWS>(sHd, LDH, M, sA0, LDA0, LPOS, gpart + lo.off[P_WD_IN], gpart + lo.off[P_BD_0]);
        __syncthreads();
        // ------------------------------------------------ hash-grid gradient (:2090-2173)
        {
            float dv[M];
            load_row<M>(dv, sHd + tid * LDH);
            float* grow = sA0 + tid * LDA0;   // A0 is no longer needed: reuse for g
            dense_bwd<M, LPOS, false>(dv, Wd_in, nullptr, grow);
            if (hit && valid) scatter_grad<F>(c, a.grad_table, pn, grow);
        }
        __syncthreads();
    }
}

// Fixed-order sum of the per-CTA weight-gradient partials into the MLP gradient.
__global__ void reduce_partials(const float* __restrict__ partials, int n_parts, int Pw, float* __restrict__ grad) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= Pw) return;
    float s = 0.0f;
    for (int p = 0; p < n_parts; ++p) s += partials[(size_t)p * Pw + i];
    grad[i] += s;
}

// adam_update_1_i32 (weight_update.cl:177-201); the gradient is cleared after use.
__device__ __forceinline__ void adam1(float& p, float g, float& m, float& v, float lr, float b1, float b2, float eps) {
    const float mi = fmaf(1.0f - b1, g, fm(b1, m));
    const float vi = fmaf(1.0f - b2, fm(g, g), fm(b2, v));
    const float denom = fa(__fsqrt_rn(vi), eps);
    p = fs(p, fm(lr, fd(mi, denom)));
    m = mi;
    v = vi;
}

// Color parameters are the ranges [c0, c1) and [c2, Pw) of the blob.
__global__ void mlp_adam_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m,
                                float* __restrict__ v, int Pw, int c0, int c1, int c2, float lr_t,
                                float color_rel_lr, float b1, float b2, float eps) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= Pw) return;
    const bool color = (i >= c0 && i < c1) || i >= c2;
    const float lr = color ? fm(lr_t, color_rel_lr) : lr_t;
    float pp = p[i], mm = m[i], vv = v[i];
    adam1(pp, g[i], mm, vv, lr, b1, b2, eps);
    p[i] = pp; m[i] = mm; v[i] = vv;
    g[i] = 0.0f;
}

__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, int64_t n, float lr_t, float b1, float b2, float eps) {
    const int64_t n4 = n >> 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 pp = reinterpret_cast<float4*>(p)[i];
        const float4 gg = reinterpret_cast<const float4*>(g)[i];
        float4 mm = reinterpret_cast<float4*>(m)[i];
        float4 vv = reinterpret_cast<float4*>(v)[i];
        adam1(pp.x, gg.x, mm.x, vv.x, lr_t, b1, b2, eps);
        adam1(pp.y, gg.y, mm.y, vv.y, lr_t, b1, b2, eps);
        adam1(pp.z, gg.z, mm.z, vv.z, lr_t, b1, b2, eps);
        adam1(pp.w, gg.w, mm.w, vv.w, lr_t, b1, b2, eps);
        reinterpret_cast<float4*>(p)[i] = pp;
        reinterpret_cast<float4*>(m)[i] = mm;
        reinterpret_cast<float4*>(v)[i] = vv;
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
        const int64_t i = (n4 << 2) + threadIdx.x;
        float pp = p[i], mm = m[i], vv = v[i];
        adam1(pp, g[i], mm, vv, lr_t, b1, b2, eps);
        p[i] = pp; m[i] = mm; v[i] = vv;
    }
}

struct LevelCoef {
    uint32_t start[L + 1];   // first element (float index) of each level, then the end
    float coef[L];
};

__device__ __forceinline__ int level_of(const LevelCoef& lc, uint32_t e) {
    int l = 0;
#pragma unroll
    for (int k = 1; k < L; ++k) l += e >= lc.start[k] ? 1 : 0;
    return l;
}

// table += coef_level * grad; grad = 0.  coef = -(lr * 2^(-0.1 l)) * HASH_LR_RATE.
__global__ void table_sgd_kernel(float* __restrict__ table, float* __restrict__ grad, uint32_t n4, const LevelCoef lc) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const float cf = lc.coef[level_of(lc, i * 4u)];
        float4 t = reinterpret_cast<float4*>(table)[i];
        const float4 g = reinterpret_cast<const float4*>(grad)[i];
        t.x = fa(t.x, fm(cf, g.x)); t.y = fa(t.y, fm(cf, g.y));
        t.z = fa(t.z, fm(cf, g.z)); t.w = fa(t.w, fm(cf, g.w));
        reinterpret_cast<float4*>(table)[i] = t;
        reinterpret_cast<float4*>(grad)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Opt-in Adam for the table (no reference counterpart): step size lr_t * 2^(-0.1 l) per level.
__global__ void table_adam_kernel(float* __restrict__ table, float* __restrict__ grad, float* __restrict__ m,
                                  float* __restrict__ v, uint32_t n4, const LevelCoef lc,
                                  float b1, float b2, float eps) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const float lr = lc.coef[level_of(lc, i * 4u)];
        float4 t = reinterpret_cast<float4*>(table)[i];
        const float4 g = reinterpret_cast<const float4*>(grad)[i];
        float4 mm = reinterpret_cast<float4*>(m)[i];
        float4 vv = reinterpret_cast<float4*>(v)[i];
        adam1(t.x, g.x, mm.x, vv.x, lr, b1, b2, eps);
        adam1(t.y, g.y, mm.y, vv.y, lr, b1, b2, eps);
        adam1(t.z, g.z, mm.z, vv.z, lr, b1, b2, eps);
        adam1(t.w, g.w, mm.w, vv.w, lr, b1, b2, eps);
        reinterpret_cast<float4*>(table)[i] = t;
        reinterpret_cast<float4*>(m)[i] = mm;
        reinterpret_cast<float4*>(v)[i] = vv;
        reinterpret_cast<float4*>(grad)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// occ_nibble_decay_write_both_q24 (decay_occ_grid_in-st.cl:13-113)
__global__ void occ_decay_kernel(uint32_t* __restrict__ occ_in, uint32_t* __restrict__ occ_st, uint32_t n,
                                 uint32_t dq, uint32_t seed) {
    for (uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x; gid < n; gid += gridDim.x * blockDim.x) {
        const uint32_t win = occ_in[gid], wst = occ_st[gid];
        const uint32_t x = wst ^ win;
        uint32_t outw = wst;
#pragma unroll
        for (uint32_t s = 0; s < 8; ++s) {
            const uint32_t shift = s * 4u;
            if (((x >> shift) & 0xFu) != 0u) continue;
            const uint32_t q = ((wst >> shift) & 0xFu) + 1u;
            if (q <= 1u) continue;
            const uint32_t qd = q * dq;
            uint32_t cand = (qd >> 24) + 1u;
            const uint32_t thresh = 0x01000000u - (qd & 0x00FFFFFFu);
            const uint32_t key = win == wst ? (seed ^ (gid * 9781u) ^ (s * 6271u) ^ wst)
                                            : (seed ^ (gid * 9781u) ^ (s * 6271u) ^ wst ^ (win * 1597u));
            const uint32_t r24 = hash_u32(key) & 0x00FFFFFFu;
            if (cand > 1u && r24 < thresh) cand -= 1u;
            cand = cand < 1u ? 1u : (cand > 16u ? 16u : cand);
            const uint32_t mask = 0xFu << shift;
            outw = (outw & ~mask) | (((cand - 1u) & 0xFu) << shift);
        }
        occ_st[gid] = outw;
        occ_in[gid] = outw;
    }
}

// One byte per nibble: expand (to_bytes = 1) or pack back (to_bytes = 0); 8 bytes per word.
__global__ void occ_bytes_kernel(uint32_t* __restrict__ grid, uint8_t* __restrict__ bytes, uint32_t n, int to_bytes) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        uint2* b = reinterpret_cast<uint2*>(bytes) + i;
        if (to_bytes) {
            const uint32_t w = grid[i];
            uint2 v;
            v.x = (w & 0xFu) | ((w >> 4) & 0xFu) << 8 | ((w >> 8) & 0xFu) << 16 | ((w >> 12) & 0xFu) << 24;
            v.y = ((w >> 16) & 0xFu) | ((w >> 20) & 0xFu) << 8 | ((w >> 24) & 0xFu) << 16 | ((w >> 28) & 0xFu) << 24;
            *b = v;
        } else {
            const uint2 v = *b;
            uint32_t w = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                w |= ((v.x >> (8 * k)) & 0xFu) << (4 * k);
                w |= ((v.y >> (8 * k)) & 0xFu) << (4 * (k + 4));
            }
            grid[i] = w;
        }
    }
}

template <int F>
__global__ void hash_fwd_kernel(const DevConfig c, const float* __restrict__ table, const float* __restrict__ pts,
                                int64_t n, float* __restrict__ enc) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float hi = 1.0f - 1.0e-6f;
        const V3 p = v3(fclamp(pts[3 * i], 0.f, hi), fclamp(pts[3 * i + 1], 0.f, hi), fclamp(pts[3 * i + 2], 0.f, hi));
        encode<F>(c, table, p, enc + i * (L * F));
    }
}

template <int F>
__global__ void hash_bwd_kernel(const DevConfig c, float* __restrict__ grad, const float* __restrict__ pts,
                                const float* __restrict__ denc, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float hi = 1.0f - 1.0e-6f;
        const V3 p = v3(fclamp(pts[3 * i], 0.f, hi), fclamp(pts[3 * i + 1], 0.f, hi), fclamp(pts[3 * i + 2], 0.f, hi));
        scatter_grad<F>(c, grad, p, denc + i * (L * F));
    }
}

}  // namespace ffn
