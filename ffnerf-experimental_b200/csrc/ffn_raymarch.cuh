// ffn_raymarch.cuh -- the per-ray phases of the fused step shared by the fp32 and the tensor-core
// kernels: occupancy-guided sampling, front-to-back compositing with the loss gradient, the
// reverse-mode scan and the occupancy proposals.  Everything here follows the exactness policy
// of ffn_common.cuh (explicit round-to-nearest operations, own exp/pow), so both kernels produce
// bit-identical sample positions, transmittances and proposals.
//
// Both functions are called by every thread of a 128-sample tile (one thread per sample, rays of
// spr consecutive threads) and synchronise the tile's threads internally (tile_sync).
#pragma once
#include "ffn_common.cuh"

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
    float* grad_table;         // destination of the hash scatter: gradient buffer or the table itself
    float hash_coef[L];        // scatter value = (hash_coef[l] * g) * w: 1 (gradient) or -lr*2^(-0.1l)*0.5
    float* partials;           // [gridDim.x][P] per-CTA weight-gradient partials
    uint32_t n_rays;
    uint32_t ray_offset;
    float sh_mult, occ_strength;
    uint32_t seed;
    int do_train;
    int* status;               // device status word (ST_* bits), may be null
    int probe;                 // ffn_probe: forward with training rules, no backward
    // split tensor-core step: sampling and encoding staged by sample_stage_kernel and
    // encode_stage_kernel (null when the fused kernel samples and encodes itself)
    const unsigned char* x0_stage;   // [tiles][128 x 16F fp16 operand tile]
    const float2* tdt_stage;         // [n_rays * spr]: sample time, step
    const uint4* ray_stage;          // [n_rays]: run-start bits (2 words), hit
    // diagnostics (ffn_probe); all optional
    const float4* bypass;
    float* dbg_t; float* dbg_dt; int* dbg_idx; uint32_t* dbg_flags;
    float* dbg_sigma; float* dbg_rgb; float* dbg_trans;
};

// ---------------------------------------------------------------------------- exact scans
// Blelloch exclusive scan of one ray's slice (ffnerf_OG.cl:619-637); every thread of the CTA
// calls it (one lane of one ray), levels separated by tile barriers.
__device__ __forceinline__ void scan_excl(float* a, int lid, int n) {
    for (int stride = 1; stride < n; stride <<= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) a[idx] = fa(a[idx], a[idx - stride]);
        tile_sync();
    }
    if (lid == 0) a[n - 1] = 0.0f;
    tile_sync();
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) {
            float t = a[idx - stride];
            a[idx - stride] = a[idx];
            a[idx] = fa(a[idx], t);
        }
        tile_sync();
    }
}
// ffnerf_OG.cl:639-646
__device__ __forceinline__ float reduce_sum(float* a, int lid, int n) {
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        if (lid < stride) a[lid] = fa(a[lid], a[lid + stride]);
        tile_sync();
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
        tile_sync();
    }
    float4 total = s[n - 1];
    tile_sync();
    if (lid == 0) s[n - 1] = make_float4(1.0f, 0.0f, 0.0f, 0.0f);
    tile_sync();
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) {
            float4 t = s[idx - stride];
            s[idx - stride] = s[idx];
            s[idx] = seg_combine(t, s[idx]);
        }
        tile_sync();
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
        tile_sync();
    }
    if (lid == 0) s[n - 1] = make_float2(1.0f, 0.0f);
    tile_sync();
    for (int stride = n >> 1; stride >= 1; stride >>= 1) {
        int idx = (lid + 1) * (stride << 1) - 1;
        if (idx < n) {
            float2 t = s[idx - stride];
            s[idx - stride] = s[idx];
            s[idx] = aff_combine_rev(t, s[idx]);
        }
        tile_sync();
    }
}

// The two scans above with warp shuffles, for rays of n = 2^k samples (2 <= n <= 64): the same
// up-sweep / down-sweep tree, so every combine sees the same operands in the same order and the
// results are bit-identical to the shared-memory form, with one exchange through shared memory for
// the stride that crosses two warps (n = 64) instead of a block barrier at every stride.  The element
// at position p of the ray is held by this thread; dir = +1 when positions ascend with the lanes,
// -1 when they descend (the reversed scan).  xchg: 2 slots of shared memory per ray.  All threads of
// the block call it (it contains block barriers when n = 64).
__device__ __forceinline__ float4 shfl_up4(float4 v, int s) {
    return make_float4(__shfl_up_sync(0xffffffffu, v.x, s), __shfl_up_sync(0xffffffffu, v.y, s),
                       __shfl_up_sync(0xffffffffu, v.z, s), __shfl_up_sync(0xffffffffu, v.w, s));
}
__device__ __forceinline__ float4 shfl_down4(float4 v, int s) {
    return make_float4(__shfl_down_sync(0xffffffffu, v.x, s), __shfl_down_sync(0xffffffffu, v.y, s),
                       __shfl_down_sync(0xffffffffu, v.z, s), __shfl_down_sync(0xffffffffu, v.w, s));
}
__device__ __forceinline__ float4 shfl_idx4(float4 v, int l) {
    return make_float4(__shfl_sync(0xffffffffu, v.x, l), __shfl_sync(0xffffffffu, v.y, l),
                       __shfl_sync(0xffffffffu, v.z, l), __shfl_sync(0xffffffffu, v.w, l));
}
__device__ __forceinline__ float2 shfl_up2(float2 v, int s) {
    return make_float2(__shfl_up_sync(0xffffffffu, v.x, s), __shfl_up_sync(0xffffffffu, v.y, s));
}
__device__ __forceinline__ float2 shfl_down2(float2 v, int s) {
    return make_float2(__shfl_down_sync(0xffffffffu, v.x, s), __shfl_down_sync(0xffffffffu, v.y, s));
}
__device__ __forceinline__ float2 shfl_idx2(float2 v, int l) {
    return make_float2(__shfl_sync(0xffffffffu, v.x, l), __shfl_sync(0xffffffffu, v.y, l));
}
__device__ __forceinline__ float4 shfl_up_t(float4 v, int s) { return shfl_up4(v, s); }
__device__ __forceinline__ float4 shfl_down_t(float4 v, int s) { return shfl_down4(v, s); }
__device__ __forceinline__ float4 shfl_idx_t(float4 v, int l) { return shfl_idx4(v, l); }
__device__ __forceinline__ float2 shfl_up_t(float2 v, int s) { return shfl_up2(v, s); }
__device__ __forceinline__ float2 shfl_down_t(float2 v, int s) { return shfl_down2(v, s); }
__device__ __forceinline__ float2 shfl_idx_t(float2 v, int l) { return shfl_idx2(v, l); }

__device__ __forceinline__ float shfl_up_t(float v, int s) { return __shfl_up_sync(0xffffffffu, v, s); }
__device__ __forceinline__ float shfl_down_t(float v, int s) { return __shfl_down_sync(0xffffffffu, v, s); }
__device__ __forceinline__ float shfl_idx_t(float v, int l) { return __shfl_sync(0xffffffffu, v, l); }

template <typename T, typename Comb>
__device__ __forceinline__ T scan_excl_warp(T v, int p, int n, int dir, T ident, T* xchg, T& total, Comb comb) {
    const int lim = n < 32 ? n : 32;
    for (int s = 1; s < lim; s <<= 1) {                        // up-sweep, strides inside a warp
        const T lo = dir > 0 ? shfl_up_t(v, s) : shfl_down_t(v, s);   // the element at p - s
        if (((p + 1) & (2 * s - 1)) == 0) v = comb(lo, v);
    }
    if (n == 64) {                                             // stride 32: across the two warps
        if (p == 31) xchg[0] = v;
        tile_sync();
        if (p == 63) { v = comb(xchg[0], v); xchg[1] = v; }
        tile_sync();
        total = xchg[1];
        // down-sweep stride 32: position 31 takes position 63's value (the identity), position 63
        // takes comb(position 31, identity)
        if (p == 63) v = comb(xchg[0], ident);
        else if (p == 31) v = ident;
    } else {
        const int lane = threadIdx.x & 31;
        total = shfl_idx_t(v, dir > 0 ? lane - p + (n - 1) : lane + p - (n - 1));
        if (p == n - 1) v = ident;
    }
    for (int s = lim >> 1; s >= 1; s >>= 1) {                  // down-sweep, strides inside a warp
        const T lo = dir > 0 ? shfl_up_t(v, s) : shfl_down_t(v, s);   // the element at p - s
        const T hi = dir > 0 ? shfl_down_t(v, s) : shfl_up_t(v, s);   // the element at p + s
        if (((p + 1) & (2 * s - 1)) == 0) v = comb(lo, v);
        else if (((p + 1 + s) & (2 * s - 1)) == 0) v = hi;
    }
    return v;
}
// scan_excl's combine: a[idx] = a[idx] + a[idx - stride]
struct AddCombine {
    __device__ __forceinline__ float operator()(float lo, float v) const { return fa(v, lo); }
};
// reduce_sum with warp shuffles for rays of n = 2^k samples (2 <= n <= 64): the same tree
// (a[p] += a[p + stride], stride n/2 .. 1), the stride 32 of n = 64 through shared memory (xchg: 33
// floats per ray); every lane of the ray gets the sum.  All threads of the block call it.
__device__ __forceinline__ float reduce_sum_warp(float v, int p, int n, float* xchg) {
    int s = n >> 1;
    if (n == 64) {
        if (p >= 32) xchg[p - 32] = v;
        tile_sync();
        if (p < 32) v = fa(v, xchg[p]);
        s = 16;
    }
    for (; s >= 1; s >>= 1) {
        const float t = __shfl_down_sync(0xffffffffu, v, s);
        if (p < s) v = fa(v, t);
    }
    if (n == 64) {
        if (p == 0) xchg[32] = v;
        tile_sync();
        return xchg[32];
    }
    return __shfl_sync(0xffffffffu, v, (int)(threadIdx.x & 31) - p);
}
struct SegCombine {
    __device__ __forceinline__ float4 operator()(float4 l, float4 r) const { return seg_combine(l, r); }
};
struct AffCombineRev {
    __device__ __forceinline__ float2 operator()(float2 l, float2 r) const { return aff_combine_rev(l, r); }
};

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

enum { RS_T0, RS_T1, RS_DTB, RS_U0, RS_HIT, RS_TFIN, RS_GRX, RS_GRY, RS_GRZ, RS_GTEND };

// Shared arrays of one tile and this thread's view of it.
struct RayTile {
    float* cand; float* cdf; float* Ts; float* DTs; float* Tr; uint32_t* key;
    float4* seg; float2* affS; float2* affE; uint32_t* chg; float* ray;   // ray: [rays][16] scalars
    int tid, spr, rl, lid, rbase;
    uint32_t ray_idx, ray_id;
    bool valid, train, probe;
    V3 o, d, bmin, bmax, bsize, inv_box;
    float Gf, inv_n;
    bool has_target;                 // `target` holds this ray's target (loaded ahead by the caller)
    float4 target;
};

// Sampler (ffnerf_OG.cl:1002-1250): stratified candidates, occupancy weights, exact Blelloch
// scans, systematic resampling, (cell, sub-cell) run starts.  Leaves Ts/DTs/chg of the tile in
// shared memory; returns whether the ray hits the box and this lane's candidate index.
__device__ __forceinline__ void ray_sampler(const StepArgs& a, const RayTile& R, bool& hit_out, int& idx_out) {
    float* sRay = R.ray; uint32_t* sChg = R.chg; float* sCand = R.cand; float* sCdf = R.cdf; float* sTs = R.Ts;
    float* sDTs = R.DTs; float* sTr = R.Tr; uint32_t* sKey = R.key; float4* sSeg = R.seg; float2* sAffS = R.affS;
    float2* sAffE = R.affE;
    const int tid = R.tid, spr = R.spr, rl = R.rl, lid = R.lid, rbase = R.rbase;
    const uint32_t ray_idx = R.ray_idx, ray_id = R.ray_id;
    const bool valid = R.valid, train = R.train, probe = R.probe;
    const V3 o = R.o, d = R.d, bmin = R.bmin, bmax = R.bmax, bsize = R.bsize, inv_box = R.inv_box;
    const float Gf = R.Gf, inv_n = R.inv_n;
    const DevConfig& c = a.c;
    (void)sRay; (void)sChg; (void)sCand; (void)sCdf; (void)sTs; (void)sDTs; (void)sTr; (void)sKey; (void)sSeg;
    (void)sAffS; (void)sAffE; (void)ray_idx; (void)valid; (void)probe; (void)bsize; (void)train;
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
    tile_sync();
    const float* rs = sRay + rl * 16;
    const bool hit = rs[RS_HIT] != 0.0f;
    hit_out = hit;
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
        // scans and sums by warp shuffles for power-of-two rays (the same trees, bit-identical),
        // else through shared memory with a barrier per stride
        const bool warp_scan = spr >= 2 && spr <= 64 && (spr & (spr - 1)) == 0;   // uniform over the block
        float* xs = reinterpret_cast<float*>(sSeg + rbase);   // exchange slots: scans [0, 2), sums [4, 37)
        float pref, Wtot, g, gtot, active_count;
        if (warp_scan) {
            float unused;
            pref = scan_excl_warp(wp, lid, spr, 1, 0.0f, xs, unused, AddCombine());
            Wtot = fmaxf(reduce_sum_warp(wp, lid, spr, xs + 4), 1.0e-12f);
            const float pi = fclamp(fd(pref, Wtot), 0.0f, 1.0f);
            g = fm(wp, own_expf(fm(-0.0f, pi)));        // LAMBDA_FOCUS = 0
            gtot = fmaxf(reduce_sum_warp(g, lid, spr, xs + 4), 1.0e-12f);
            active_count = reduce_sum_warp(active, lid, spr, xs + 4);
        } else {
            sCdf[tid] = wp;
            tile_sync();
            scan_excl(cdf, lid, spr);
            pref = sCdf[tid];
            sCdf[tid] = wp;
            tile_sync();
            Wtot = fmaxf(reduce_sum(cdf, lid, spr), 1.0e-12f);
            tile_sync();
            const float pi = fclamp(fd(pref, Wtot), 0.0f, 1.0f);
            g = fm(wp, own_expf(fm(-0.0f, pi)));        // LAMBDA_FOCUS = 0
            sCdf[tid] = g;
            tile_sync();
            gtot = fmaxf(reduce_sum(cdf, lid, spr), 1.0e-12f);
            tile_sync();
            sCdf[tid] = active;
            tile_sync();
            active_count = reduce_sum(cdf, lid, spr);
            tile_sync();
        }
        const float any_active = active_count > 0.5f ? 1.0f : 0.0f;
        const float inv_active = fd(1.0f, fmaxf(active_count, 1.0f));
        const float ut = fmix(inv_n, fm(active, inv_active), any_active);
        const float pt = fm(any_active, fd(g, gtot));
        const float p = fa(fm(0.3f, ut), fm(1.0f - 0.3f, pt));  // UNIFORM_PART
        if (warp_scan) {
            float unused;
            const float ex = scan_excl_warp(p, lid, spr, 1, 0.0f, xs, unused, AddCombine());
            sCdf[tid] = fa(ex, p);
        } else {
            sCdf[tid] = p;
            tile_sync();
            scan_excl(cdf, lid, spr);
            sCdf[tid] = fa(sCdf[tid], p);
        }
        tile_sync();
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
        tile_sync();   // every lane has read cand/cdf
        sTs[tid] = t_out;
        sDTs[tid] = hit ? dtb : 0.0f;
        sKey[tid] = key;
        tile_sync();
        const bool pow2 = spr <= 64 && (spr & (spr - 1)) == 0;   // uniform over the block
        if (pow2) {
            // run starts as a warp ballot: a warp holds 32 lanes of one ray, or whole rays when spr < 32
            const bool start = hit && (lid == 0 || sKey[tid] != sKey[tid - 1]);
            const unsigned m = __ballot_sync(0xffffffffu, start);
            if (hit) {
                if (spr >= 32) {
                    if ((lid & 31) == 0) sChg[rl * 2 + (lid >> 5)] = m;
                } else if (lid == 0) {
                    sChg[rl * 2] = (m >> (tid & 31)) & ((1u << spr) - 1u);
                }
            }
        } else if (hit) {
            if (lid == 0 || sKey[tid] != sKey[tid - 1]) atomicOr(sChg + rl * 2 + (lid >> 5), 1u << (lid & 31));
        }
        if (!hit && lid < 2) {
            // no hit: every sample starts a run (ffnerf_OG.cl:1058-1063)
            const int lo_bit = lid * 32;
            const int nb = min(32, max(0, spr - lo_bit));
            sChg[rl * 2 + lid] = nb == 32 ? 0xFFFFFFFFu : ((1u << nb) - 1u);
        }
        tile_sync();
    }

    idx_out = idx_sel;
}

// Compositing, loss gradient, reverse scan (ffnerf_OG.cl:1505-1634) and occupancy proposals
// (ffnerf_OG.cl:1640-1821) for one sample with density sigma and colour rgb.  Lane 0 of every
// ray writes the ray colour.  Returns the transmittance before the sample, dL/dsigma, dL/dc and
// the ray's run-start bits.
__device__ __forceinline__ void ray_composite(const StepArgs& a, const RayTile& R, const float* rs, float sigma,
                                              const float (&rgb)[3], V3 xs, float t_s, float dt_s, float& T_s_out,
                                              float& dLds_out, float (&dLdc_out)[3], uint32_t& chg0_out,
                                              uint32_t& chg1_out) {
    float* sRay = R.ray; uint32_t* sChg = R.chg; float* sCand = R.cand; float* sCdf = R.cdf; float* sTs = R.Ts;
    float* sDTs = R.DTs; float* sTr = R.Tr; uint32_t* sKey = R.key; float4* sSeg = R.seg; float2* sAffS = R.affS;
    float2* sAffE = R.affE;
    const int tid = R.tid, spr = R.spr, rl = R.rl, lid = R.lid, rbase = R.rbase;
    const uint32_t ray_idx = R.ray_idx, ray_id = R.ray_id;
    const bool valid = R.valid, train = R.train, probe = R.probe;
    const V3 o = R.o, d = R.d, bmin = R.bmin, bmax = R.bmax, bsize = R.bsize, inv_box = R.inv_box;
    const float Gf = R.Gf, inv_n = R.inv_n;
    const DevConfig& c = a.c;
    (void)sRay; (void)sChg; (void)sCand; (void)sCdf; (void)sTs; (void)sDTs; (void)sTr; (void)sKey; (void)sSeg;
    (void)sAffS; (void)sAffE; (void)ray_idx; (void)valid; (void)probe; (void)bsize; (void)train;
    // ------------------------------------------------ compositing (:1505-1634)
    float alpha = 0.0f;
    if (dt_s > 0.0f) alpha = fs(1.0f, own_expf(fclamp(fm(-sigma, dt_s), -5.0f, 18.0f)));
    const float oma = fs(1.0f, alpha);
    const bool warp_scan = spr >= 2 && spr <= 64 && (spr & (spr - 1)) == 0;   // uniform over the block
    float4 total;
    float T_s;
    if (warp_scan) {
        const float4 ex = scan_excl_warp(make_float4(oma, fm(alpha, rgb[0]), fm(alpha, rgb[1]), fm(alpha, rgb[2])),
                                         lid, spr, 1, make_float4(1.0f, 0.0f, 0.0f, 0.0f), sSeg + rbase, total,
                                         SegCombine());
        T_s = ex.x;
    } else {
        sSeg[tid] = make_float4(oma, fm(alpha, rgb[0]), fm(alpha, rgb[1]), fm(alpha, rgb[2]));
        tile_sync();
        total = scan_excl_seg(sSeg + rbase, lid, spr);
        T_s = sSeg[tid].x;
    }
    T_s_out = T_s;
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
        if (R.has_target) tg = R.target;
        else if (valid && a.targets) tg = a.targets[ray_idx];
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
        if (valid) {
            a.out[ray_idx] = make_float4(fclamp(cf[0], 0.f, 1.f), fclamp(cf[1], 0.f, 1.f),
                                         fclamp(cf[2], 0.f, 1.f), (train && !probe) ? 4.0f : 0.0f);
            // a NaN / Inf colour means the model diverged: flag it for the host (ffn_status)
            if (a.status && !(isfinite(cf[0]) && isfinite(cf[1]) && isfinite(cf[2]))) atomicOr(a.status, ST_NONFINITE);
        }
    }
    tile_sync();
    const float gr0 = rs[RS_GRX], gr1 = rs[RS_GRY], gr2 = rs[RS_GRZ], gT_end = rs[RS_GTEND];
    const float w_s = fm(T_s, alpha);
    const float dLdc[3] = {fm(w_s, gr0), fm(w_s, gr1), fm(w_s, gr2)};
    dLdc_out[0] = dLdc[0]; dLdc_out[1] = dLdc[1]; dLdc_out[2] = dLdc[2];
    {
        const float B_s = fa(fa(fm(gr0, fm(alpha, rgb[0])), fm(gr1, fm(alpha, rgb[1]))), fm(gr2, fm(alpha, rgb[2])));
        const int k = spr - 1 - lid;
        sAffE[rbase + k] = make_float2(oma, B_s);
        if (warp_scan) {
            float2 unused;
            sAffS[rbase + k] = scan_excl_warp(make_float2(oma, B_s), k, spr, -1, make_float2(1.0f, 0.0f),
                                              reinterpret_cast<float2*>(sSeg + rbase), unused, AffCombineRev());
        } else {
            sAffS[rbase + k] = make_float2(oma, B_s);
        }
    }
    tile_sync();
    if (!warp_scan) scan_excl_aff_rev(sAffS + rbase, lid, spr);
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
    chg0_out = chg0; chg1_out = chg1;
    dLds_out = dLds;
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
}

}  // namespace ffn
