// ffn_oracle.cpp -- TEST INFRASTRUCTURE ONLY: the CPU parity checker for the fused NeRF step.
//
// A restatement of the reference's OpenCL kernels in plain C++, phase by phase, with every
// work-group barrier turned into a loop over the lanes of one ray.  Floating-point expressions
// keep the reference's operation order and are compiled with -ffp-contract=off, so the float
// results are the IEEE-literal reading of the reference source.  Each function cites the
// reference file:line it restates (paths relative to the reference repository root).
//
// Two math modes:
//   math_mode 0: exp/pow come from orc_expf/orc_powr below (double-precision range reduction +
//                Taylor/atanh series, plain + and *), written to be bit-identical to the device
//                implementation in the product; this is the mode the GPU is compared against.
//   math_mode 1: exp/pow/log1p from the C library, to match the reference compiled from its own
//                sources for the CPU (oracle/ref_build.py) bit for bit.
//
// Parity status: pinned against the reference kernels compiled from their own sources (same
// binary semantics, libm math) and against fixtures from the reference's Python host module.
#include "ffn_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

constexpr int L = ORC_N_LEVELS;   // ffnerf_OG.cl:166 N_LEVELS
constexpr int M = 64;             // ffnerf_OG.cl:45  hidden width
constexpr int D_OUT = 16;         // ffnerf_OG.cl:42
constexpr int L_DIR = 16;         // ffnerf_OG.cl:41
constexpr int C_IN = 32;          // ffnerf_OG.cl:43
constexpr int C_OUT = 3;          // ffnerf_OG.cl:44
constexpr int S_MAX = 64;         // ffnerf_OG.cl:47

// ---------------------------------------------------------------- own exp / pow (math_mode 0)
// exp(z) in double: Cody-Waite reduction z = k*ln2 + r (ln2 split into a 24-bit head and a
// tail, both derived from the decimal expansion of ln 2), e^r by its Taylor series (degree 17,
// Horner form), then scaling by 2^k.  Plain multiplies and adds only (no contraction).
const double kLn2Hi = 0x1.62e43p-1;
const double kLn2Lo = -0x1.05c610ca86c39p-29;
const double kInvLn2 = 0x1.71547652b82fep+0;
const double kInvFact[18] = {
    0x1p+0, 0x1p+0, 0x1p-1, 0x1.5555555555555p-3, 0x1.5555555555555p-5,
    0x1.1111111111111p-7, 0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13,
    0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22,
    0x1.ae64567f544e4p-26, 0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33,
    0x1.93974a8c07c9dp-37, 0x1.ae7f3e733b81fp-41, 0x1.ae7f3e733b81fp-45,
    0x1.952c77030ad4ap-49};
// 1/(2n+1) for the atanh series of log.
const double kInvOdd[13] = {
    0x1p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
    0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4,
    0x1.1111111111111p-4, 0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5,
    0x1.8618618618618p-5, 0x1.642c8590b2164p-5, 0x1.47ae147ae147bp-5};
const double kSqrt2 = 0x1.6a09e667f3bcdp+0;

double own_exp_d(double z) {
    double kd = std::rint(z * kInvLn2);
    double r = (z - kd * kLn2Hi) - kd * kLn2Lo;
    double p = kInvFact[17];
    for (int n = 16; n >= 0; --n) p = p * r + kInvFact[n];
    return std::ldexp(p, (int)kd);
}

double own_log_d(double x) {  // x > 0, finite
    int e;
    double m = std::frexp(x, &e);   // x = m * 2^e, m in [0.5, 1)
    m = m * 2.0;
    e = e - 1;                      // m in [1, 2)
    if (m > kSqrt2) { m = m * 0.5; e = e + 1; }
    double s = (m - 1.0) / (m + 1.0);
    double z = s * s;
    double q = kInvOdd[12];
    for (int n = 11; n >= 0; --n) q = q * z + kInvOdd[n];
    double lm = 2.0 * s * q;
    return ((double)e * kLn2Hi + lm) + (double)e * kLn2Lo;
}

float own_expf(float x) {
    if (x != x) return x;
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    return (float)own_exp_d((double)x);
}

float own_powr(float x, float y) {  // x >= 0 (OpenCL powr domain)
    if (!(x > 0.0f)) return 0.0f;
    double t = (double)y * own_log_d((double)x);
    if (t > 710.0) return INFINITY;
    if (t < -745.0) return 0.0f;
    return (float)own_exp_d(t);
}

// ---------------------------------------------------------------- small helpers
struct V3 { float x, y, z; };
inline V3 v3(float x, float y, float z) { return V3{x, y, z}; }
inline V3 operator+(V3 a, V3 b) { return V3{a.x + b.x, a.y + b.y, a.z + b.z}; }
inline V3 operator-(V3 a, V3 b) { return V3{a.x - b.x, a.y - b.y, a.z - b.z}; }
inline V3 operator*(V3 a, V3 b) { return V3{a.x * b.x, a.y * b.y, a.z * b.z}; }
inline V3 operator/(V3 a, V3 b) { return V3{a.x / b.x, a.y / b.y, a.z / b.z}; }
inline V3 operator*(float s, V3 a) { return V3{s * a.x, s * a.y, s * a.z}; }
inline V3 operator*(V3 a, float s) { return V3{a.x * s, a.y * s, a.z * s}; }

inline float fclampf(float x, float lo, float hi) { return std::fmin(std::fmax(x, lo), hi); }
inline int iclamp(int x, int lo, int hi) { return std::min(std::max(x, lo), hi); }
inline float mixf(float a, float b, float t) { return a + (b - a) * t; }  // OpenCL mix
inline float length3(V3 v) { return std::sqrt(v.x * v.x + v.y * v.y + v.z * v.z); }

// ffnerf_OG.cl:293-301
inline uint32_t hash_u32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352du; x ^= x >> 15; x *= 0x846ca68bu; x ^= x >> 16;
    return x;
}
// ffnerf_OG.cl:303-311
inline float rand01(uint32_t* s) {
    uint32_t x = *s;
    x ^= x << 13; x ^= x >> 17; x ^= x << 5;
    *s = x;
    return (float)(x & 0x00FFFFFFu) * (1.0f / 16777216.0f);
}

struct Math {
    int mode;
    float exp(float x) const { return mode ? std::exp(x) : own_expf(x); }
    float powr(float x, float y) const { return mode ? std::pow(x, y) : own_powr(x, y); }
    float pow(float x, float y) const { return std::pow(x, y); }
};

// ffnerf_OG.cl:218-222
inline float softplus(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return std::exp(x);
    return std::log1p(std::exp(x));
}
// ffnerf_OG.cl:223-226
inline float softplus_prime_from_pre(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + std::exp(-x));
    return std::exp(x) / (1.0f + std::exp(x));
}
// ffnerf_OG.cl:234-239 (RGB_SIGMOID_SCALE = 0.5)
inline float sigmoid_soft(float x) {
    x *= 0.5f;
    x = fclampf(x, -18.0f, 18.0f);
    if (x >= 0.0f) return 1.0f / (1.0f + std::exp(-x));
    return std::exp(x) / (1.0f + std::exp(x));
}
// ffnerf_OG.cl:251-253 (RGB_CHARB_EPS = 1e-3); rsqrt written as 1/sqrt
inline float charbonnier_prime(float x) {
    return x * (1.0f / std::sqrt(x * x + 1.0e-3f * 1.0e-3f));
}

// ffnerf_OG.cl:322-343
inline int ray_aabb(V3 o, V3 d, V3 bmin, V3 bmax, float* t0, float* t1) {
    V3 invd = v3(d.x != 0.0f ? 1.0f / d.x : INFINITY, d.y != 0.0f ? 1.0f / d.y : INFINITY,
                 d.z != 0.0f ? 1.0f / d.z : INFINITY);
    V3 tbot = (bmin - o) * invd;
    V3 ttop = (bmax - o) * invd;
    V3 tmin3 = v3(std::fmin(tbot.x, ttop.x), std::fmin(tbot.y, ttop.y), std::fmin(tbot.z, ttop.z));
    V3 tmax3 = v3(std::fmax(tbot.x, ttop.x), std::fmax(tbot.y, ttop.y), std::fmax(tbot.z, ttop.z));
    float tmin = std::fmax(tmin3.x, std::fmax(tmin3.y, tmin3.z));
    float tmax = std::fmin(tmax3.x, std::fmin(tmax3.y, tmax3.z));
    if (tmax < tmin) return 0;
    *t0 = tmin; *t1 = tmax;
    return 1;
}

// ffnerf_OG.cl:619-637 Blelloch exclusive scan, lanes executed level by level.
void scan_excl(float* a, int n) {
    for (int stride = 1; stride < n; stride <<= 1)
        for (int lid = 0; lid < n; ++lid) {
            int idx = (lid + 1) * (stride << 1) - 1;
            if (idx < n) a[idx] += a[idx - stride];
        }
    a[n - 1] = 0.0f;
    for (int stride = n >> 1; stride >= 1; stride >>= 1)
        for (int lid = 0; lid < n; ++lid) {
            int idx = (lid + 1) * (stride << 1) - 1;
            if (idx < n) { float t = a[idx - stride]; a[idx - stride] = a[idx]; a[idx] += t; }
        }
}
// ffnerf_OG.cl:639-646
float reduce_sum(float* a, int n) {
    for (int stride = n >> 1; stride >= 1; stride >>= 1)
        for (int lid = 0; lid < stride; ++lid) a[lid] += a[lid + stride];
    return a[0];
}
// ffnerf_OG.cl:648-656
int lower_bound_cdf(const float* cdf, int n, float u) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (cdf[mid] >= u) hi = mid; else lo = mid + 1;
    }
    return lo;
}

// ffnerf_OG.cl:686-713  (Seg = {a, v}; seg_combine(L,R) = {L.a*R.a, L.v + L.a*R.v})
struct Seg { float a; V3 v; };
inline Seg seg_combine(Seg l, Seg r) { return Seg{l.a * r.a, l.v + l.a * r.v}; }
Seg scan_excl_seg(Seg* s, int n) {
    for (int stride = 1; stride < n; stride <<= 1)
        for (int lid = 0; lid < n; ++lid) {
            int idx = (lid + 1) * (stride << 1) - 1;
            if (idx < n) s[idx] = seg_combine(s[idx - stride], s[idx]);
        }
    Seg total = s[n - 1];
    s[n - 1] = Seg{1.0f, v3(0.0f, 0.0f, 0.0f)};
    for (int stride = n >> 1; stride >= 1; stride >>= 1)
        for (int lid = 0; lid < n; ++lid) {
            int idx = (lid + 1) * (stride << 1) - 1;
            if (idx < n) { Seg t = s[idx - stride]; s[idx - stride] = s[idx]; s[idx] = seg_combine(t, s[idx]); }
        }
    return total;
}
// ffnerf_OG.cl:689-691,715-735  (aff_combine_rev(L,R) = {R.a*L.a, R.a*L.b + R.b})
struct Aff { float a, b; };
inline Aff aff_combine_rev(Aff l, Aff r) { return Aff{r.a * l.a, r.a * l.b + r.b}; }
void scan_excl_aff_rev(Aff* s, int n) {
    for (int stride = 1; stride < n; stride <<= 1)
        for (int lid = 0; lid < n; ++lid) {
            int idx = (lid + 1) * (stride << 1) - 1;
            if (idx < n) s[idx] = aff_combine_rev(s[idx - stride], s[idx]);
        }
    s[n - 1] = Aff{1.0f, 0.0f};
    for (int stride = n >> 1; stride >= 1; stride >>= 1)
        for (int lid = 0; lid < n; ++lid) {
            int idx = (lid + 1) * (stride << 1) - 1;
            if (idx < n) { Aff t = s[idx - stride]; s[idx - stride] = s[idx]; s[idx] = aff_combine_rev(t, s[idx]); }
        }
}

// ffnerf_OG.cl:446-469 (next set bit strictly after idx, or n)
int chg_find_next(const uint32_t* f, int idx, int n) {
    int i = idx + 1;
    if (i >= n) return n;
    int w = i >> 5, b = i & 31;
    uint32_t mask = f[w] & (~0u << b);
    for (;;) {
        if (mask) {
            int res = (w << 5) + __builtin_ctz(mask);
            return res < n ? res : n;
        }
        ++w;
        if ((w << 5) >= n) break;
        mask = f[w];
    }
    return n;
}

// ffnerf_OG.cl:486-512 atomic nibble max (sequential here)
void occ_nibble_max(uint32_t* grid, int cell, uint32_t sub, uint32_t q) {
    uint32_t shift = 4u * sub, mask = 0xFu << shift;
    uint32_t old = grid[cell];
    uint32_t old_q = ((old >> shift) & 0xFu) + 1u;
    if (q <= old_q) return;
    grid[cell] = (old & ~mask) | (((q - 1u) & 0xFu) << shift);
}

// ffnerf_OG.cl:572-602 SH degree 0..3
void sh16(V3 d, float* sh) {
    float x = d.x, y = d.y, z = d.z;
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

// ---------------------------------------------------------------- parameter blob layout
// Canonical order (reference kernel argument order, ffnerf_OG.cl:843-861):
enum { P_WD_IN, P_WD_01, P_WD_12, P_WD_OUT, P_WC_IN, P_WC_01, P_WC_12, P_WC_23, P_WC_OUT,
       P_BD_0, P_BD_1, P_BD_2, P_BD_OUT, P_BC_0, P_BC_1, P_BC_2, P_BC_3, P_BC_OUT };

struct Layout { int off[ORC_N_PARAMS]; int size[ORC_N_PARAMS]; int total; };

Layout make_layout(int F, int ND, int NC) {
    Layout lo{};
    int lpos = L * F;
    int sz[ORC_N_PARAMS] = {
        M * lpos, ND >= 2 ? M * M : 0, ND >= 3 ? M * M : 0, D_OUT * M,
        M * C_IN, NC >= 2 ? M * M : 0, NC >= 3 ? M * M : 0, NC >= 4 ? M * M : 0, C_OUT * M,
        M, ND >= 2 ? M : 0, ND >= 3 ? M : 0, D_OUT,
        M, NC >= 2 ? M : 0, NC >= 3 ? M : 0, NC >= 4 ? M : 0, C_OUT};
    int o = 0;
    for (int i = 0; i < ORC_N_PARAMS; ++i) {
        lo.off[i] = o;
        lo.size[i] = sz[i];
        o += (sz[i] + 3) & ~3;   // 16-byte aligned segments
    }
    lo.total = o;
    return lo;
}

// ---------------------------------------------------------------- hash-grid helpers
// ffnerf_OG.cl:1299-1304 HASH_ENTRY, :187-211 level tables
inline uint32_t hash_entry(const orc_config* c, int ix, int iy, int iz, int lvl) {
    uint32_t h = hash_u32((uint32_t)ix * 73856093u ^ (uint32_t)iy * 19349663u ^
                          (uint32_t)iz * 83492791u ^ (uint32_t)lvl * 2654435761u);
    return h & ((1u << c->level_log2[lvl]) - 1u);
}

struct Corners { float w[8]; int base[8]; };

// ffnerf_OG.cl:1308-1338 (per-level corner weights and base feature indices)
inline void level_corners(const orc_config* c, V3 p, int lvl, Corners* k) {
    int R = c->level_res[lvl];
    if (R < 2) R = 2;
    V3 u = p * (float)R;
    int ix0 = (int)std::floor(u.x), iy0 = (int)std::floor(u.y), iz0 = (int)std::floor(u.z);
    ix0 = iclamp(ix0, 0, R - 2); iy0 = iclamp(iy0, 0, R - 2); iz0 = iclamp(iz0, 0, R - 2);
    float fx = u.x - (float)ix0, fy = u.y - (float)iy0, fz = u.z - (float)iz0;
    float wx0 = 1.0f - fx, wx1 = fx, wy0 = 1.0f - fy, wy1 = fy, wz0 = 1.0f - fz, wz1 = fz;
    for (int cc = 0; cc < 8; ++cc) {
        int dx = cc & 1, dy = (cc >> 1) & 1, dz = (cc >> 2) & 1;
        k->w[cc] = (dx ? wx1 : wx0) * (dy ? wy1 : wy0) * (dz ? wz1 : wz0);
        uint32_t entry = hash_entry(c, ix0 + dx, iy0 + dy, iz0 + dz, lvl);
        k->base[cc] = (int)((c->level_offset[lvl] + entry) * (uint32_t)c->F);
    }
}

// ffnerf_OG.cl:1291-1296 normalized, clamped position
inline V3 normalize_pos(const orc_config* c, V3 x) {
    V3 bmin = v3(c->box_min[0], c->box_min[1], c->box_min[2]);
    V3 bmax = v3(c->box_max[0], c->box_max[1], c->box_max[2]);
    V3 p = (x - bmin) / (bmax - bmin);
    const float hi = 1.0f - 1.0e-6f;
    return v3(fclampf(p.x, 0.0f, hi), fclampf(p.y, 0.0f, hi), fclampf(p.z, 0.0f, hi));
}

// ffnerf_OG.cl:1340-1357
void encode(const orc_config* c, const float* table, V3 p, float* a0) {
    for (int lvl = 0; lvl < L; ++lvl) {
        Corners k;
        level_corners(c, p, lvl, &k);
        float acc[4] = {0, 0, 0, 0};
        for (int cc = 0; cc < 8; ++cc)
            for (int f = 0; f < c->F; ++f) acc[f] += k.w[cc] * table[k.base[cc] + f];
        for (int f = 0; f < c->F; ++f) a0[lvl * c->F + f] = acc[f];
    }
}

// ffnerf_OG.cl:754-806 forward layers, :811-835 backward layers
inline float relu(float x) { return x > 0.0f ? x : 0.0f; }
void fc_relu(float* out, const float* in, int in_dim, const float* W, const float* b) {
    for (int i = 0; i < M; ++i) {
        float s = b[i];
        for (int j = 0; j < in_dim; ++j) s += W[i * in_dim + j] * in[j];
        out[i] = relu(s);
    }
}
void fc_linear(float* out, int out_dim, const float* in, const float* W, const float* b) {
    for (int i = 0; i < out_dim; ++i) {
        float s = b[i];
        for (int j = 0; j < M; ++j) s += W[i * M + j] * in[j];
        out[i] = s;
    }
}
void bwd_to_M(float* din, const float* dout, int out_dim, const float* W) {
    for (int j = 0; j < M; ++j) {
        float s = 0.0f;
        for (int i = 0; i < out_dim; ++i) s += W[i * M + j] * dout[i];
        din[j] = s;
    }
}
inline void relu_mask(float* d, const float* act) {
    for (int j = 0; j < M; ++j) d[j] = act[j] > 0.0f ? d[j] : 0.0f;
}

// Per-sample record of the staged activations and deltas (ffnerf_OG.cl:873-894): what the
// reference writes to global scratch for update_ffnerf_oneWG.
struct Stage {
    float apos[64];
    float ad[3][M];
    float acin[C_IN];
    float ac[4][M];
    float dd[3][M];
    float dd_out[D_OUT];
    float dc[4][M];
    float dc_out[C_OUT];
};

// Transfer formats of the staged activations and deltas (ffnerf_OG.cl:85-156, read back by
// weight_update.cl's tload): the weight update sees each staged value as stored in the format.
// fp16: saturate to +-65504 (non-finite -> +-65504), round to nearest even.
inline float transfer_fp16(float x) {
    if (!std::isfinite(x)) x = std::copysign(65504.0f, x);
    x = fclampf(x, -65504.0f, 65504.0f);
    return (float)(_Float16)x;
}
// fp8: the reference's e4m3-like minifloat -- saturate to +-15.5 (non-finite -> +-15.5), flush
// |x| < 1e-8 and exponents below the bias to zero, 3 mantissa bits rounded to nearest even (a
// carry bumps the exponent), exponents above 14 stored as 2^3 * 1.875.
inline float transfer_fp8(float x) {
    x = std::isfinite(x) ? fclampf(x, -15.5f, 15.5f) : std::copysign(15.5f, x);
    const bool neg = x < 0.0f;
    const float ax = std::fabs(x);
    if (ax < 1.0e-8f) return neg ? -0.0f : 0.0f;
    int e = 0;
    const float m = std::frexp(ax, &e);
    int ef = e - 1 + 7;
    if (ef <= 0) return neg ? -0.0f : 0.0f;
    int mant;
    if (ef > 14) {
        ef = 10; mant = 7;
    } else {
        mant = (int)std::rint((m * 2.0f - 1.0f) * 8.0f);
        if (mant >= 8) { mant = 0; ef += 1; }
        if (ef > 14) { ef = 10; mant = 7; }
    }
    const float v = std::ldexp(1.0f + (float)mant * (1.0f / 8.0f), ef - 7);
    return neg ? -v : v;
}
void quantize_stage(Stage& s, int fmt) {
    if (fmt != 16 && fmt != 8) return;
    float* f = reinterpret_cast<float*>(&s);
    for (size_t i = 0; i < sizeof(Stage) / sizeof(float); ++i) f[i] = fmt == 16 ? transfer_fp16(f[i]) : transfer_fp8(f[i]);
}

}  // namespace

// ============================================================================ public API
extern "C" int32_t orc_param_layout(int32_t F, int32_t ND, int32_t NC, int32_t* offsets,
                                     int32_t* sizes) {
    Layout lo = make_layout(F, ND, NC);
    for (int i = 0; i < ORC_N_PARAMS; ++i) {
        if (offsets) offsets[i] = lo.off[i];
        if (sizes) sizes[i] = lo.size[i];
    }
    return lo.total;
}

extern "C" float orc_expf(float x) { return own_expf(x); }
extern "C" float orc_powr(float x, float y) { return own_powr(x, y); }
extern "C" uint32_t orc_hash_u32(uint32_t x) { return hash_u32(x); }

// Restates ffnerf_train_step (ffnerf_OG.cl:838-2174) for all rays; the weight-gradient part of
// update_ffnerf_oneWG (weight_update.cl:210-314) is applied to the staged records at the end.
extern "C" int32_t orc_forward_backward(const orc_config* c, const orc_step* st,
                                        const float* params, float* table,
                                        const uint32_t* occ_in, uint32_t* occ_st,
                                        const float* rays, const float* targets, float* out,
                                        int32_t n_rays, float* table_grad, float* mlp_grad,
                                        const orc_debug* dbg, const float* bypass) {
    const int WG = c->spr;
    if (WG > S_MAX || WG < 1 || (WG & (WG - 1))) return -1;
    if (c->F != 2 && c->F != 4) return -2;
    if (c->ND < 1 || c->ND > 3 || c->NC < 1 || c->NC > 4) return -3;
    const Math mth{c->math_mode};
    const int F = c->F, LPOS = L * F, ND = c->ND, NC = c->NC, G = c->G;
    const Layout lo = make_layout(F, ND, NC);
    const float* P = params;
    const float* Wd[3] = {P + lo.off[P_WD_IN], P + lo.off[P_WD_01], P + lo.off[P_WD_12]};
    const float* bd[3] = {P + lo.off[P_BD_0], P + lo.off[P_BD_1], P + lo.off[P_BD_2]};
    const float* Wd_out = P + lo.off[P_WD_OUT];
    const float* bd_out = P + lo.off[P_BD_OUT];
    const float* Wc[4] = {P + lo.off[P_WC_IN], P + lo.off[P_WC_01], P + lo.off[P_WC_12], P + lo.off[P_WC_23]};
    const float* bc[4] = {P + lo.off[P_BC_0], P + lo.off[P_BC_1], P + lo.off[P_BC_2], P + lo.off[P_BC_3]};
    const float* Wc_out = P + lo.off[P_WC_OUT];
    const float* bc_out = P + lo.off[P_BC_OUT];

    const V3 bmin = v3(c->box_min[0], c->box_min[1], c->box_min[2]);
    const V3 bmax = v3(c->box_max[0], c->box_max[1], c->box_max[2]);
    const uint32_t seed = st->rng_seed;
    const bool train = st->do_train != 0;
    const bool sequential = c->table_mode == 1;

    std::vector<Stage> stage;
    if (train && mlp_grad && !bypass) stage.resize((size_t)n_rays * WG);

    for (int r = 0; r < n_rays; ++r) {
        const uint32_t ray_id = st->ray_offset + (uint32_t)r;
        const float* rr = rays + (size_t)r * 8;
        const V3 o = v3(rr[0], rr[1], rr[2]);
        const V3 d = v3(rr[4], rr[5], rr[6]);

        float Ts[S_MAX], DTs[S_MAX], Tr[S_MAX];
        uint32_t chg[2] = {0u, 0u};
        int idx_dbg[S_MAX];
        for (int i = 0; i < WG; ++i) idx_dbg[i] = 0;

        // ------------------------------------------------ sampler (ffnerf_OG.cl:1002-1250)
        {
            float t0 = 0.0f, t1 = 0.0f, dt_base = 0.0f, u0 = 0.0f;
            int hit;
            {
                float a, b;
                hit = ray_aabb(o, d, bmin, bmax, &a, &b);
                if (hit) {
                    a = std::fmax(a, c->t_near);
                    b = std::fmin(b, c->t_far);
                    if (b <= a) hit = 0; else { t0 = a + 1.0e-6f; t1 = b; }
                }
                float dtb = hit ? (t1 - t0) * (1.0f / (float)WG) : 0.0f;
                dtb = std::fmin(c->dt_max, std::fmax(c->dt_min, dtb));
                dt_base = hit ? dtb : 0.0f;
                if (hit) {
                    uint32_t rng0 = hash_u32(seed ^ ray_id * 1597334677u);
                    u0 = rand01(&rng0) * (1.0f / (float)WG);
                }
            }
            if (!hit) {
                for (int i = 0; i < WG; ++i) { Ts[i] = 0.0f; DTs[i] = 0.0f; chg[i >> 5] |= 1u << (i & 31); }
            } else {
                float cand_t[S_MAX], wp[S_MAX], active[S_MAX], cdf[S_MAX];
                const V3 bsize = bmax - bmin;
                const V3 inv_box = v3(1.0f / bsize.x, 1.0f / bsize.y, 1.0f / bsize.z);
                for (int lid = 0; lid < WG; ++lid) {
                    uint32_t rng = hash_u32(seed ^ ray_id * 747796405u ^ (uint32_t)lid * 2891336453u);
                    float u = ((float)lid + rand01(&rng)) * (1.0f / (float)WG);
                    float tk = t0 + (t1 - t0) * u;
                    cand_t[lid] = tk;
                    V3 xk = o + tk * d;
                    V3 gm = (xk - bmin) * inv_box * (float)G;
                    float occ = 0.0f;
                    if (gm.x >= 0.0f && gm.x < (float)G && gm.y >= 0.0f && gm.y < (float)G &&
                        gm.z >= 0.0f && gm.z < (float)G) {
                        int ixm = iclamp((int)std::floor(gm.x), 0, G - 1);
                        int iym = iclamp((int)std::floor(gm.y), 0, G - 1);
                        int izm = iclamp((int)std::floor(gm.z), 0, G - 1);
                        int cell = ixm + G * (iym + G * izm);
                        uint32_t packed = occ_in[cell];
                        float fx = fclampf(gm.x - std::floor(gm.x), 0.0f, 1.0f - 1e-7f);
                        float fy = fclampf(gm.y - std::floor(gm.y), 0.0f, 1.0f - 1e-7f);
                        float fz = fclampf(gm.z - std::floor(gm.z), 0.0f, 1.0f - 1e-7f);
                        uint32_t sub = (uint32_t)(fx > 0.5f) + 2u * (uint32_t)(fy > 0.5f) + 4u * (uint32_t)(fz > 0.5f);
                        uint32_t occ4 = (packed >> (4u * sub)) & 0xFu;
                        uint32_t q_train = occ4 + 1u;
                        uint32_t q_infer = occ4 > 2u ? occ4 - 2u : 0u;
                        uint32_t q_eff = train ? q_train : q_infer;
                        occ = (float)q_eff * (1.0f / 16.0f);
                    }
                    float infer_f = train ? 0.0f : 1.0f;
                    active[lid] = occ > 0.0f ? 1.0f : 0.0f;
                    float rho_base = c->rho_min + (c->rho_max - c->rho_min) * occ;
                    float rho = rho_base * (1.0f - infer_f + infer_f * active[lid]);
                    float w_raw = rho * dt_base;
                    float x = std::fmax(w_raw, 0.0f);                   // safe_pow_pos :665-671
                    wp[lid] = (x <= 0.0f) ? 0.0f : mth.powr(x, 1.3f);   // GAMMA_W
                }
                for (int i = 0; i < WG; ++i) cdf[i] = wp[i];
                scan_excl(cdf, WG);
                float pref[S_MAX];
                for (int i = 0; i < WG; ++i) pref[i] = cdf[i];
                for (int i = 0; i < WG; ++i) cdf[i] = wp[i];
                float Wtot = std::fmax(reduce_sum(cdf, WG), 1.0e-12f);
                float g[S_MAX];
                for (int i = 0; i < WG; ++i) {
                    float pi = pref[i] / Wtot;
                    pi = fclampf(pi, 0.0f, 1.0f);                 // focus_gain_unitprefix :672-677
                    g[i] = wp[i] * mth.exp(-0.0f * pi);            // LAMBDA_FOCUS = 0
                }
                for (int i = 0; i < WG; ++i) cdf[i] = g[i];
                float gtot = std::fmax(reduce_sum(cdf, WG), 1.0e-12f);
                for (int i = 0; i < WG; ++i) cdf[i] = active[i];
                float active_count = reduce_sum(cdf, WG);
                float any_active = active_count > 0.5f ? 1.0f : 0.0f;
                float inv_active = 1.0f / std::fmax(active_count, 1.0f);
                float pr[S_MAX];
                for (int i = 0; i < WG; ++i) {
                    float uta = active[i] * inv_active;
                    float ut = mixf(1.0f / (float)WG, uta, any_active);
                    float pt = any_active * (g[i] / gtot);
                    pr[i] = 0.3f * ut + (1.0f - 0.3f) * pt;      // UNIFORM_PART
                }
                for (int i = 0; i < WG; ++i) cdf[i] = pr[i];
                scan_excl(cdf, WG);
                for (int i = 0; i < WG; ++i) cdf[i] = cdf[i] + pr[i];
                uint32_t key[S_MAX];
                for (int lid = 0; lid < WG; ++lid) {
                    float uk = u0 + (float)lid * (1.0f / (float)WG);
                    uk = std::fmin(uk, 0.99999994f);
                    int idx = lower_bound_cdf(cdf, WG, uk);
                    idx_dbg[lid] = idx;
                    float t_out = cand_t[idx];
                    Ts[lid] = t_out;
                    DTs[lid] = dt_base;
                    V3 xo = o + t_out * d;
                    V3 go = (xo - bmin) * inv_box * (float)G;
                    uint32_t kk = 0xFFFFFFFEu;
                    int ixo = (int)std::floor(go.x), iyo = (int)std::floor(go.y), izo = (int)std::floor(go.z);
                    if ((uint32_t)ixo < (uint32_t)G && (uint32_t)iyo < (uint32_t)G && (uint32_t)izo < (uint32_t)G) {
                        float fx = fclampf(go.x - std::floor(go.x), 0.0f, 1.0f - 1e-7f);
                        float fy = fclampf(go.y - std::floor(go.y), 0.0f, 1.0f - 1e-7f);
                        float fz = fclampf(go.z - std::floor(go.z), 0.0f, 1.0f - 1e-7f);
                        uint32_t sub = (uint32_t)(fx >= 0.5f) + 2u * (uint32_t)(fy >= 0.5f) + 4u * (uint32_t)(fz >= 0.5f);
                        int cell = ixo + G * (iyo + G * izo);
                        kk = ((uint32_t)cell << 3) | (sub & 7u);
                    }
                    key[lid] = kk;
                }
                for (int lid = 0; lid < WG; ++lid)
                    if (lid == 0 || key[lid] != key[lid - 1]) chg[lid >> 5] |= 1u << (lid & 31);
            }
        }

        // ------------------------------------------------ per-sample forward (:1257-1496)
        float sigma_s[S_MAX], rgb_s[S_MAX][3];
        std::vector<Stage> lane_st((size_t)WG);
        float a0s[S_MAX][64], dout0[S_MAX];
        for (int lid = 0; lid < WG; ++lid) {
            float t = Ts[lid];
            V3 x = o + t * d;
            Stage& S = lane_st[lid];
            float sigma;
            float rgb[3];
            V3 p = normalize_pos(c, x);
            encode(c, table, p, a0s[lid]);
            if (bypass) {
                const float* bp = bypass + ((size_t)r * WG + lid) * 4;
                sigma = bp[0]; rgb[0] = bp[1]; rgb[1] = bp[2]; rgb[2] = bp[3];
                dout0[lid] = 0.0f;
            } else {
                for (int i = 0; i < LPOS; ++i) S.apos[i] = a0s[lid][i];
                const float* cur = S.apos;
                int in_dim = LPOS;
                for (int l = 0; l < ND; ++l) {
                    fc_relu(S.ad[l], cur, in_dim, Wd[l], bd[l]);
                    cur = S.ad[l];
                    in_dim = M;
                }
                float dout[D_OUT];
                fc_linear(dout, D_OUT, cur, Wd_out, bd_out);
                for (int i = 0; i < D_OUT; ++i) S.acin[i] = dout[i];
                sigma = softplus(fclampf(dout[0], -10.0f, 10.0f));
                dout0[lid] = dout[0];
                sh16(d, S.acin + D_OUT);
                for (int i = 0; i < L_DIR; ++i) S.acin[D_OUT + i] *= st->sh_mult;
                cur = S.acin;
                in_dim = C_IN;
                for (int l = 0; l < NC; ++l) {
                    fc_relu(S.ac[l], cur, in_dim, Wc[l], bc[l]);
                    cur = S.ac[l];
                    in_dim = M;
                }
                float cout[C_OUT];
                fc_linear(cout, C_OUT, cur, Wc_out, bc_out);
                for (int k = 0; k < 3; ++k) rgb[k] = sigmoid_soft(cout[k]);
            }
            if (DTs[lid] <= 0.0f) sigma = 0.0f;
            sigma_s[lid] = sigma;
            for (int k = 0; k < 3; ++k) rgb_s[lid][k] = rgb[k];
        }

        // ------------------------------------------------ compositing (:1505-1634)
        float alpha[S_MAX];
        Seg segs[S_MAX];
        for (int lid = 0; lid < WG; ++lid) {
            float a = 0.0f;
            if (DTs[lid] > 0.0f) {
                float xx = fclampf(-sigma_s[lid] * DTs[lid], -5.0f, 18.0f);  // SxDT_CAP_FOR_ALPHA
                a = 1.0f - mth.exp(xx);
            }
            alpha[lid] = a;
            segs[lid] = Seg{1.0f - a, a * v3(rgb_s[lid][0], rgb_s[lid][1], rgb_s[lid][2])};
        }
        // The reference stores the scan total in a private variable of lane 0 only
        // (ffnerf_OG.cl:699,1531); every lane here sees the total, which is what lane 0 holds.
        Seg total = scan_excl_seg(segs, WG);
        for (int lid = 0; lid < WG; ++lid) Tr[lid] = segs[lid].a;
        const float T_final = total.a;
        V3 gr = v3(0, 0, 0);
        float gT_end = 0.0f;
        {
            V3 bg = v3(0, 0, 0);
            if (train) {
                if (c->background == 1) bg = v3(1, 1, 1);
                else if (c->background == 2) {
                    uint32_t rb = hash_u32(seed ^ ray_id * 747796405u ^ 0xA511E9B3u);
                    float bx = rand01(&rb), by = rand01(&rb), bz = rand01(&rb);
                    bg = v3(bx, by, bz);
                }
            }
            V3 C_final = total.v + T_final * bg;
            float* op = out + (size_t)r * 4;
            op[0] = fclampf(C_final.x, 0.0f, 1.0f);
            op[1] = fclampf(C_final.y, 0.0f, 1.0f);
            op[2] = fclampf(C_final.z, 0.0f, 1.0f);
            op[3] = 0.0f;
            const float* tg = targets + (size_t)r * 4;
            V3 diff = C_final - v3(tg[0], tg[1], tg[2]);
            gr = v3(charbonnier_prime(diff.x), charbonnier_prime(diff.y), charbonnier_prime(diff.z));
            gT_end = gr.x * bg.x + gr.y * bg.y + gr.z * bg.z;
        }
        float dL_dsigma[S_MAX], dL_dc[S_MAX][3];
        {
            Aff elem[S_MAX], scan[S_MAX];
            for (int lid = 0; lid < WG; ++lid) {
                float a = alpha[lid], T_s = Tr[lid];
                float w_s = T_s * a;
                dL_dc[lid][0] = w_s * gr.x; dL_dc[lid][1] = w_s * gr.y; dL_dc[lid][2] = w_s * gr.z;
                const float* cs = rgb_s[lid];
                float B_s = gr.x * (a * cs[0]) + gr.y * (a * cs[1]) + gr.z * (a * cs[2]);
                int k = WG - 1 - lid;
                elem[k] = Aff{1.0f - a, B_s};
                scan[k] = elem[k];
            }
            scan_excl_aff_rev(scan, WG);
            for (int lid = 0; lid < WG; ++lid) {
                float a = alpha[lid], T_s = Tr[lid], dt_s = DTs[lid];
                int k = WG - 1 - lid;
                float gT_next = gT_end;
                if (k >= 1) {
                    Aff incl = aff_combine_rev(scan[k - 1], elem[k - 1]);
                    gT_next = incl.a * gT_end + incl.b;
                }
                const float* cs = rgb_s[lid];
                float gA_C = gr.x * (T_s * cs[0]) + gr.y * (T_s * cs[1]) + gr.z * (T_s * cs[2]);
                float gAlpha = gA_C - gT_next * T_s;
                float dad = dt_s > 0.0f ? dt_s * (1.0f - a) : 0.0f;
                float regu = dt_s > 0.0f ? 5e-3f * dt_s / (float)(uint32_t)WG : 0.0f;  // DENSITY_PENALTY_LMD
                dL_dsigma[lid] = gAlpha * dad + regu;
            }
        }

        // ------------------------------------------------ occupancy proposals (:1640-1821)
        if (st->occ_strength > 0.0f && train) {
            const V3 bsize = bmax - bmin;
            const V3 inv_box = v3(1.0f / bsize.x, 1.0f / bsize.y, 1.0f / bsize.z);
            for (int lid = 0; lid < WG; ++lid) {
                if (!(DTs[lid] > 0.0f)) continue;
                if (!((chg[lid >> 5] >> (lid & 31)) & 1u)) continue;
                float t = Ts[lid];
                V3 x = o + t * d;
                V3 gp = (x - bmin) * inv_box * (float)G;
                int ix = (int)std::floor(gp.x), iy = (int)std::floor(gp.y), iz = (int)std::floor(gp.z);
                if (!((uint32_t)ix < (uint32_t)G && (uint32_t)iy < (uint32_t)G && (uint32_t)iz < (uint32_t)G)) continue;
                float fx = gp.x - std::floor(gp.x), fy = gp.y - std::floor(gp.y), fz = gp.z - std::floor(gp.z);
                uint32_t sub = (uint32_t)(fx >= 0.5f) + 2u * (uint32_t)(fy >= 0.5f) + 4u * (uint32_t)(fz >= 0.5f);
                int cell = ix + G * (iy + G * iz);
                int next = chg_find_next(chg, lid, WG);
                float pred = 0.0f;
                {
                    V3 cell_size = bsize * (1.0f / (float)G);
                    V3 cmin = bmin + v3((float)ix, (float)iy, (float)iz) * cell_size;
                    V3 cmax = cmin + cell_size;
                    float te, tx;
                    if (ray_aabb(o, d, cmin, cmax, &te, &tx)) {
                        te = std::fmax(te, c->t_near);
                        tx = std::fmin(tx, c->t_far);
                        if (tx > te) {
                            int prev_end = lid > 0 ? lid - 1 : 0;
                            float t_prev = Ts[prev_end], T_prev = Tr[prev_end];
                            float t_cur = Ts[lid], T_cur = Tr[lid];
                            float den0 = t_cur - t_prev;
                            float u0 = std::fabs(den0) > 1.0e-8f ? (te - t_prev) / den0 : 0.0f;
                            u0 = fclampf(u0, 0.0f, 1.0f);
                            float T_enter = mixf(T_prev, T_cur, u0);
                            int last = next < WG ? next - 1 : WG - 1;
                            float t_last = Ts[last], T_last = Tr[last];
                            float t_next = next < WG ? Ts[next] : tx;
                            float T_next = next < WG ? Tr[next] : T_final;
                            float den1 = t_next - t_last;
                            float u1 = std::fabs(den1) > 1.0e-8f ? (tx - t_last) / den1 : 1.0f;
                            u1 = fclampf(u1, 0.0f, 1.0f);
                            float T_exit = mixf(T_last, T_next, u1);
                            pred = fclampf((T_enter - T_exit) / std::fmax(T_enter, 1.0e-12f), 0.0f, 1.0f);
                        }
                    }
                }
                uint32_t old_q = ((occ_in[cell] >> (4u * sub)) & 0xFu) + 1u;
                uint32_t proposed = old_q;
                float pred16 = pred * 16.0f;
                if (pred16 > (float)old_q && old_q < 16u) {
                    float f0 = std::floor(pred16);
                    float frac = pred16 - f0;
                    uint32_t q0 = (uint32_t)f0;
                    uint32_t rh = hash_u32(seed ^ ray_id * 747796405u ^ (uint32_t)lid * 2891336453u ^
                                           (uint32_t)cell * 9781u ^ sub * 6271u);
                    uint32_t thresh = (uint32_t)(frac * 16777216.0f);
                    uint32_t qs = (rh & 0x00FFFFFFu) < thresh ? q0 + 1u : q0;
                    if (qs > 16u) qs = 16u;
                    proposed = qs;
                }
                float lat = (bmax.x - bmin.x) * (1.0f / (float)G);
                float D = 0.5f * length3(bmax - bmin);
                float tl = t / std::fmax(lat, 1.0e-12f);
                float Dl = D / std::fmax(lat, 1.0e-12f);
                float num = tl * tl + tl + (1.0f / 3.0f);
                float den = Dl * Dl + Dl + (1.0f / 3.0f);
                float keep_p = std::fmin(num / std::fmax(den, 1.0e-12f), 1.0f);
                if (keep_p >= 1.0f) {
                    occ_nibble_max(occ_st, cell, sub, proposed);
                } else {
                    uint32_t rk = hash_u32(seed ^ ray_id * 747796405u ^ (uint32_t)lid * 2891336453u ^
                                           (uint32_t)cell * 9781u ^ sub * 6271u);
                    if (rand01(&rk) <= keep_p) occ_nibble_max(occ_st, cell, sub, proposed);
                }
            }
        }

        if (dbg) {
            for (int lid = 0; lid < WG; ++lid) {
                size_t s = (size_t)r * WG + lid;
                if (dbg->t) dbg->t[s] = Ts[lid];
                if (dbg->dt) dbg->dt[s] = DTs[lid];
                if (dbg->idx) dbg->idx[s] = idx_dbg[lid];
                if (dbg->sigma) dbg->sigma[s] = sigma_s[lid];
                if (dbg->rgb) for (int k = 0; k < 3; ++k) dbg->rgb[s * 3 + k] = rgb_s[lid][k];
                if (dbg->trans) dbg->trans[s] = Tr[lid];
                if (dbg->dsigma) dbg->dsigma[s] = dL_dsigma[lid];
                if (dbg->enc) for (int k = 0; k < LPOS; ++k) dbg->enc[s * LPOS + k] = a0s[lid][k];
            }
            if (dbg->flags) { dbg->flags[(size_t)r * 2] = chg[0]; dbg->flags[(size_t)r * 2 + 1] = chg[1]; }
        }
        if (!train || bypass) continue;
        out[(size_t)r * 4 + 3] += 4.0f;   // ffnerf_OG.cl:2091 debug marker

        // ------------------------------------------------ backward (:1858-2082)
        const float Dhalf = 0.5f * length3(bmax - bmin);
        float dh1[S_MAX][M];
        for (int lid = 0; lid < WG; ++lid) {
            Stage& S = lane_st[lid];
            float t = Ts[lid], dtl = DTs[lid];
            float num = t * t + t * dtl + (dtl * dtl / 3.0f);
            float den = Dhalf * Dhalf + Dhalf * dtl + (dtl * dtl / 3.0f);
            float xr = t / std::fmax(Dhalf, 1.0e-12f);
            float s = xr >= 1.0f ? 0.0f : 1.0f;
            float gate = (1.0f - s) * 1.0f + s * mth.pow(std::fmax(xr, 1.0e-12f), 0.2f);
            float f_vol = gate * num / std::fmax(den, 1.0e-12f);
            float d_sigma = f_vol * dL_dsigma[lid];
            float dcol[3] = {f_vol * dL_dc[lid][0], f_vol * dL_dc[lid][1], f_vol * dL_dc[lid][2]};
            for (int k = 0; k < 3; ++k) {
                float sv = rgb_s[lid][k];
                S.dc_out[k] = dcol[k] * ((sv * (1.0f - sv)) * 0.5f);
            }
            float ddo[D_OUT];
            ddo[0] = 1.0f * d_sigma * softplus_prime_from_pre(fclampf(S.acin[0], -18.0f, 18.0f));
            for (int i = 1; i < D_OUT; ++i) ddo[i] = 0.0f;
            // color backprop (:1932-2020)
            float cur[M], nxt[M];
            bwd_to_M(cur, S.dc_out, C_OUT, Wc_out);
            relu_mask(cur, S.ac[NC - 1]);
            for (int j = 0; j < M; ++j) S.dc[NC - 1][j] = cur[j];
            for (int l = NC - 1; l >= 1; --l) {
                bwd_to_M(nxt, cur, M, Wc[l]);
                relu_mask(nxt, S.ac[l - 1]);
                for (int j = 0; j < M; ++j) { cur[j] = nxt[j]; S.dc[l - 1][j] = cur[j]; }
            }
            for (int i = 0; i < D_OUT; ++i) {
                float sacc = 0.0f;
                for (int j = 0; j < M; ++j) sacc += Wc[0][j * C_IN + i] * cur[j];
                ddo[i] += sacc;
            }
            // density backprop (:2034-2078)
            for (int i = 0; i < D_OUT; ++i) S.dd_out[i] = ddo[i];
            bwd_to_M(cur, ddo, D_OUT, Wd_out);
            relu_mask(cur, S.ad[ND - 1]);
            for (int j = 0; j < M; ++j) S.dd[ND - 1][j] = cur[j];
            for (int l = ND - 1; l >= 1; --l) {
                bwd_to_M(nxt, cur, M, Wd[l]);
                relu_mask(nxt, S.ad[l - 1]);
                for (int j = 0; j < M; ++j) { cur[j] = nxt[j]; S.dd[l - 1][j] = cur[j]; }
            }
            for (int j = 0; j < M; ++j) dh1[lid][j] = cur[j];
        }
        // ------------------------------------------------ hash-grid gradient (:2090-2173)
        for (int lid = 0; lid < WG; ++lid) {
            V3 x = o + Ts[lid] * d;
            V3 p = normalize_pos(c, x);
            for (int lvl = 0; lvl < L; ++lvl) {
                float lr_lvl = st->lr_f * c->hash_lr_scale[lvl];
                Corners k;
                level_corners(c, p, lvl, &k);
                for (int f = 0; f < F; ++f) {
                    int kk = lvl * F + f;
                    float gf = 0.0f;
                    for (int j = 0; j < M; ++j) gf += Wd[0][j * LPOS + kk] * dh1[lid][j];
                    if (!std::isfinite(gf)) continue;
                    for (int cc = 0; cc < 8; ++cc) {
                        int i = k.base[cc] + f;
                        if (sequential) table[i] += -lr_lvl * 0.5f * gf * k.w[cc];   // HASH_LR_RATE
                        else if (table_grad) table_grad[i] += gf * k.w[cc];
                    }
                }
            }
        }
        if (!stage.empty())
            for (int lid = 0; lid < WG; ++lid) {
                stage[(size_t)r * WG + lid] = lane_st[lid];
                quantize_stage(stage[(size_t)r * WG + lid], c->transfer_fmt);
            }
    }

    // ---------------------------------------------------- weight gradients (weight_update.cl:210-314)
    if (!stage.empty()) {
        const int B = (int)stage.size();
        const int TK = c->tilek > 0 ? c->tilek : 236;
        std::memset(mlp_grad, 0, sizeof(float) * (size_t)lo.total);
        // Per weight (oo, ii): acc over each TILEK chunk of samples in sample order, chunk sums
        // added in chunk order; per bias: one running sum in sample order.  All weights of a layer
        // advance together so each staged sample is read once per layer (same sums, same order).
        std::vector<float> tot, acc, bacc;
        auto layer = [&](int wi, int bi, int OUT, int IN, auto dsel, auto asel) {
            float* gW = mlp_grad + lo.off[wi];
            float* gb = mlp_grad + lo.off[bi];
            tot.assign((size_t)OUT * IN, 0.0f);
            acc.resize((size_t)OUT * IN);
            bacc.assign((size_t)OUT, 0.0f);
            for (int kb = 0; kb < B; kb += TK) {
                std::fill(acc.begin(), acc.end(), 0.0f);
                const int ke = std::min(B, kb + TK);
                for (int k = kb; k < ke; ++k) {
                    const float* d = dsel(stage[k]);
                    const float* a = asel(stage[k]);
                    for (int oo = 0; oo < OUT; ++oo) {
                        float* row = acc.data() + (size_t)oo * IN;
                        const float dv = d[oo];
                        for (int ii = 0; ii < IN; ++ii) row[ii] += dv * a[ii];
                        bacc[oo] += dv;
                    }
                }
                for (size_t i = 0; i < tot.size(); ++i) tot[i] += acc[i];
            }
            for (size_t i = 0; i < tot.size(); ++i) gW[i] = tot[i];
            for (int oo = 0; oo < OUT; ++oo) gb[oo] = bacc[oo];
        };
        const int LP = LPOS;
        // color head and hidden layers (weight_update.cl:487-533)
        layer(P_WC_OUT, P_BC_OUT, C_OUT, M, [](const Stage& s) { return s.dc_out; },
              [NC](const Stage& s) { return s.ac[NC - 1]; });
        for (int l = NC - 1; l >= 1; --l)
            layer(P_WC_IN + l, P_BC_0 + l, M, M, [l](const Stage& s) { return s.dc[l]; },
                  [l](const Stage& s) { return s.ac[l - 1]; });
        layer(P_WC_IN, P_BC_0, M, C_IN, [](const Stage& s) { return s.dc[0]; },
              [](const Stage& s) { return s.acin; });
        // density (weight_update.cl:537-573)
        layer(P_WD_OUT, P_BD_OUT, D_OUT, M, [](const Stage& s) { return s.dd_out; },
              [ND](const Stage& s) { return s.ad[ND - 1]; });
        for (int l = ND - 1; l >= 1; --l)
            layer(P_WD_IN + l, P_BD_0 + l, M, M, [l](const Stage& s) { return s.dd[l]; },
                  [l](const Stage& s) { return s.ad[l - 1]; });
        layer(P_WD_IN, P_BD_0, M, LP, [](const Stage& s) { return s.dd[0]; },
              [](const Stage& s) { return s.apos; });
    }
    return 0;
}

// weight_update.cl:177-201 (native_sqrt written as sqrt)
extern "C" void orc_adam(float* p, const float* g, float* m, float* v, int64_t n, float lr_t,
                         float b1, float b2, float eps) {
    for (int64_t i = 0; i < n; ++i) {
        float gi = g[i];
        float mi = std::fma(1.0f - b1, gi, b1 * m[i]);
        float vi = std::fma(1.0f - b2, gi * gi, b2 * v[i]);
        float denom = std::sqrt(vi) + eps;
        p[i] -= lr_t * (mi / denom);
        m[i] = mi;
        v[i] = vi;
    }
}

// update_ffnerf_oneWG (weight_update.cl:487-573): color layers use lr_t*color_MLP_rel_lr.
extern "C" void orc_mlp_adam(const orc_config* c, float* params, const float* grad, float* m,
                             float* v, float lr_t, float color_rel_lr, float b1, float b2,
                             float eps) {
    Layout lo = make_layout(c->F, c->ND, c->NC);
    const float lr_c = lr_t * color_rel_lr;
    for (int i = 0; i < ORC_N_PARAMS; ++i) {
        bool color = (i >= P_WC_IN && i <= P_WC_OUT) || (i >= P_BC_0 && i <= P_BC_OUT);
        int o = lo.off[i];
        orc_adam(params + o, grad + o, m + o, v + o, lo.size[i], color ? lr_c : lr_t, b1, b2, eps);
    }
}

// Opt-in Adam for the hash table (no reference counterpart: the reference trains the table with
// the in-kernel SGD step, ffnerf_OG.cl:2155-2168).  The reference's Adam update
// (weight_update.cl:177-201, orc_adam above) per level, with step size lr_t * 2^(-0.1 l) -- the
// reference's per-level SGD roll-off (ffnerf_OG.cl:2110-2111) applied to Adam's step.
extern "C" void orc_table_adam(const orc_config* c, float* table, const float* tg, float* m, float* v,
                               float lr_t, float b1, float b2, float eps) {
    for (int lvl = 0; lvl < L; ++lvl) {
        const float lr = lr_t * c->hash_lr_scale[lvl];
        const int64_t b = (int64_t)c->level_offset[lvl] * c->F;
        const int64_t n = ((int64_t)1 << c->level_log2[lvl]) * c->F;
        orc_adam(table + b, tg + b, m + b, v + b, n, lr, b1, b2, eps);
    }
}

// Deferred application of the hash SGD step: table += (-lr_lvl * HASH_LR_RATE) * sum(g*w).
extern "C" void orc_table_apply(const orc_config* c, float* table, const float* tg, float lr_f) {
    for (int lvl = 0; lvl < L; ++lvl) {
        float coef = -(lr_f * c->hash_lr_scale[lvl]) * 0.5f;
        int64_t b = (int64_t)c->level_offset[lvl] * c->F;
        int64_t e = b + ((int64_t)1 << c->level_log2[lvl]) * c->F;
        for (int64_t i = b; i < e; ++i) table[i] = table[i] + coef * tg[i];
    }
}

// decay_occ_grid_in-st.cl:13-113
extern "C" void orc_decay(uint32_t* occ_in, uint32_t* occ_st, uint32_t n, uint32_t dq,
                          uint32_t seed) {
    for (uint32_t gid = 0; gid < n; ++gid) {
        uint32_t win = occ_in[gid], wst = occ_st[gid];
        uint32_t x = wst ^ win;
        uint32_t outw = wst;
        for (uint32_t s = 0; s < 8; ++s) {
            uint32_t shift = s * 4u;
            if (((x >> shift) & 0xFu) != 0u) continue;
            uint32_t q = ((wst >> shift) & 0xFu) + 1u;
            if (q <= 1u) continue;
            uint32_t qd = q * dq;
            uint32_t cand = (qd >> 24) + 1u;
            uint32_t thresh = 0x01000000u - (qd & 0x00FFFFFFu);
            uint32_t key = (win == wst) ? (seed ^ (gid * 9781u) ^ (s * 6271u) ^ wst)
                                        : (seed ^ (gid * 9781u) ^ (s * 6271u) ^ wst ^ (win * 1597u));
            uint32_t r24 = hash_u32(key) & 0x00FFFFFFu;
            if (cand > 1u && r24 < thresh) cand -= 1u;
            if (cand < 1u) cand = 1u;
            if (cand > 16u) cand = 16u;
            uint32_t mask = 0xFu << shift;
            outw = (outw & ~mask) | (((cand - 1u) & 0xFu) << shift);
        }
        occ_st[gid] = outw;
        occ_in[gid] = outw;
    }
}

extern "C" void orc_hash_fwd(const orc_config* c, const float* table, const float* pts,
                             int64_t n, float* enc) {
    const int LP = L * c->F;
    for (int64_t i = 0; i < n; ++i) {
        const float hi = 1.0f - 1.0e-6f;
        V3 p = v3(fclampf(pts[i * 3], 0.0f, hi), fclampf(pts[i * 3 + 1], 0.0f, hi),
                  fclampf(pts[i * 3 + 2], 0.0f, hi));
        encode(c, table, p, enc + i * LP);
    }
}

extern "C" void orc_hash_bwd(const orc_config* c, const float* pts, const float* denc,
                             int64_t n, float* tg) {
    const int F = c->F, LP = L * F;
    for (int64_t i = 0; i < n; ++i) {
        const float hi = 1.0f - 1.0e-6f;
        V3 p = v3(fclampf(pts[i * 3], 0.0f, hi), fclampf(pts[i * 3 + 1], 0.0f, hi),
                  fclampf(pts[i * 3 + 2], 0.0f, hi));
        for (int lvl = 0; lvl < L; ++lvl) {
            Corners k;
            level_corners(c, p, lvl, &k);
            for (int f = 0; f < F; ++f) {
                float g = denc[i * LP + lvl * F + f];
                for (int cc = 0; cc < 8; ++cc) tg[k.base[cc] + f] += g * k.w[cc];
            }
        }
    }
}
