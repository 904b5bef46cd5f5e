// ffn_batch.cu -- training batches generated on the device from images resident in HBM.
// Included into ffn_capi.cu's translation unit.
//
// The reference's trainer draws each batch on the host (run_ffnerf_OG.py:585-685): an image per
// ray uniformly, then per image a pixel either uniformly (a fifth of the draws) or by rejection
// against a per-image uint8 weight map (propose a uniform pixel, accept when a uniform byte is
// <= its weight, run_ffnerf_OG.py:493-519), then the pinhole ray and the 8-bit colour of that pixel
// (ffnerf_tools.py:175-234).  Periodically the per-ray colour error feeds back into the weight maps
// through an EMA towards a median-normalised target weight, capped for background pixels
// (run_ffnerf_OG.py:459-490).  Here both run as kernels: one thread per ray, a counter-based hash
// RNG keyed by (seed, ray), so a batch depends only on its seed, the weight maps and the images.
#include <cuda_runtime.h>

namespace ffn {

struct BatchGen {
    const void* images;      // [n_img][H][W][C]: uint8 (colour / 255) or float32 in [0, 1]
    int img_f32;
    const uint8_t* weights;  // [n_img][H][W] uint8 in 1..255
    const float* c2w;        // [n_img][4][4] row-major camera-to-world
    const float* K;          // [3][3] or [n_img][3][3]; null = the reference's fallback focal sqrt(H*W)
    int k_per_image;
    int n_img, W, H, C;
    uint32_t n;              // rays
    float uniform_frac;      // share of uniformly drawn pixels
    uint32_t seed;
    uint32_t max_tries;      // rejection proposals before the last proposal is taken
};

__device__ __forceinline__ uint32_t rng_next(uint32_t& s) {
    s = hash_u32(s + 0x9E3779B9u);
    return s;
}
// uniform integer in [0, m) from 32 random bits (multiply-high)
__device__ __forceinline__ uint32_t rng_below(uint32_t& s, uint32_t m) {
    return (uint32_t)(((uint64_t)rng_next(s) * (uint64_t)m) >> 32);
}

__global__ void __launch_bounds__(256) batch_generate_kernel(const BatchGen g, float4* __restrict__ rays,
                                                             float4* __restrict__ targets, int32_t* __restrict__ im_out,
                                                             int32_t* __restrict__ x_out, int32_t* __restrict__ y_out) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < g.n; i += gridDim.x * blockDim.x) {
        uint32_t s = hash_u32(g.seed ^ (i * 0x85EBCA6Bu) ^ 0x5BD1E995u);
        const int im = (int)rng_below(s, (uint32_t)g.n_img);
        const bool uniform = (float)(rng_next(s) >> 8) * (1.0f / 16777216.0f) < g.uniform_frac;
        int x = (int)rng_below(s, (uint32_t)g.W), y = (int)rng_below(s, (uint32_t)g.H);
        if (!uniform) {
            const uint8_t* wm = g.weights + (size_t)im * g.W * g.H;
            for (uint32_t t = 0; t < g.max_tries; ++t) {
                if ((rng_next(s) & 255u) <= (uint32_t)wm[(size_t)y * g.W + x]) break;
                x = (int)rng_below(s, (uint32_t)g.W);
                y = (int)rng_below(s, (uint32_t)g.H);
            }
        }
        // pinhole ray, OpenCV camera axes (x right, y down, z forward)
        float cx_, cy_, cz_;
        if (g.K) {
            const float* k = g.K + (g.k_per_image ? (size_t)im * 9 : 0);
            cx_ = __fdiv_rn(__fsub_rn(__fadd_rn((float)x, 0.5f), k[2]), k[0]);
            cy_ = __fdiv_rn(__fsub_rn(__fadd_rn((float)y, 0.5f), k[5]), k[4]);
            cz_ = 1.0f;
        } else {
            cx_ = __fadd_rn(__fsub_rn((float)x, (float)g.W * 0.5f), 0.5f);
            cy_ = __fadd_rn(__fsub_rn((float)y, (float)g.H * 0.5f), 0.5f);
            cz_ = __fsqrt_rn((float)g.H * (float)g.W);
        }
        const float* m = g.c2w + (size_t)im * 16;
        float d[3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
            d[r] = __fadd_rn(__fadd_rn(__fmul_rn(m[4 * r], cx_), __fmul_rn(m[4 * r + 1], cy_)), __fmul_rn(m[4 * r + 2], cz_));
        const float nrm = __fadd_rn(__fsqrt_rn(__fadd_rn(__fadd_rn(__fmul_rn(d[0], d[0]), __fmul_rn(d[1], d[1])),
                                                         __fmul_rn(d[2], d[2]))), 1e-12f);
        rays[2 * (size_t)i] = make_float4(m[3], m[7], m[11], 1.0f);
        rays[2 * (size_t)i + 1] = make_float4(__fdiv_rn(d[0], nrm), __fdiv_rn(d[1], nrm), __fdiv_rn(d[2], nrm), 0.0f);
        const size_t px = (((size_t)im * g.H + y) * g.W + x) * g.C;
        if (g.img_f32) {
            const float* f = static_cast<const float*>(g.images) + px;
            targets[i] = make_float4(f[0], f[1], f[2], 0.0f);
        } else {
            const uint8_t* b = static_cast<const uint8_t*>(g.images) + px;
            targets[i] = make_float4(__fdiv_rn((float)b[0], 255.0f), __fdiv_rn((float)b[1], 255.0f),
                                     __fdiv_rn((float)b[2], 255.0f), 0.0f);
        }
        if (im_out) { im_out[i] = im; x_out[i] = x; y_out[i] = y; }
    }
}

// Rays through pixels first .. first + n - 1 of a W x H view in row-major order (x fastest): the
// view rays of the reference's renderer (rays_from_rt_indices, ffnerf_tools.py:237-272) with the
// same pinhole arithmetic as batch_generate_kernel.
struct ViewCam {
    float c2w[16];
    float k[9];
    int has_k;
    int W, H;
};

__global__ void __launch_bounds__(256) camera_rays_kernel(const ViewCam v, uint32_t first, uint32_t n,
                                                          float4* __restrict__ rays) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const uint32_t p = first + i;
        const int x = (int)(p % (uint32_t)v.W), y = (int)(p / (uint32_t)v.W);
        float cx_, cy_, cz_;
        if (v.has_k) {
            cx_ = __fdiv_rn(__fsub_rn(__fadd_rn((float)x, 0.5f), v.k[2]), v.k[0]);
            cy_ = __fdiv_rn(__fsub_rn(__fadd_rn((float)y, 0.5f), v.k[5]), v.k[4]);
            cz_ = 1.0f;
        } else {
            cx_ = __fadd_rn(__fsub_rn((float)x, (float)v.W * 0.5f), 0.5f);
            cy_ = __fadd_rn(__fsub_rn((float)y, (float)v.H * 0.5f), 0.5f);
            cz_ = __fsqrt_rn((float)v.H * (float)v.W);
        }
        float d[3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
            d[r] = __fadd_rn(__fadd_rn(__fmul_rn(v.c2w[4 * r], cx_), __fmul_rn(v.c2w[4 * r + 1], cy_)),
                             __fmul_rn(v.c2w[4 * r + 2], cz_));
        const float nrm = __fadd_rn(__fsqrt_rn(__fadd_rn(__fadd_rn(__fmul_rn(d[0], d[0]), __fmul_rn(d[1], d[1])),
                                                         __fmul_rn(d[2], d[2]))), 1e-12f);
        rays[2 * (size_t)i] = make_float4(v.c2w[3], v.c2w[7], v.c2w[11], 1.0f);
        rays[2 * (size_t)i + 1] = make_float4(__fdiv_rn(d[0], nrm), __fdiv_rn(d[1], nrm), __fdiv_rn(d[2], nrm), 0.0f);
    }
}

// Per-ray colour error sqrt(mean_rgb((out - target)^2)) clipped to [0, 1] (run_ffnerf_OG.py:1383),
// and optionally the batch's sum of squared colour differences (double, one atomic add per block),
// from which the trainer's periodic metrics follow: mse = S / (3 n), rmse = sqrt(mse),
// l2 = sqrt(S / n) (run_ffnerf_OG.py:1389-1391).
__global__ void __launch_bounds__(256) batch_error_kernel(const float4* __restrict__ out,
                                                          const float4* __restrict__ targets, uint32_t n,
                                                          float* __restrict__ err, double* __restrict__ sum_sq) {
    __shared__ double part[8];
    double acc = 0.0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float4 o = out[i], t = targets[i];
        const float a = __fsub_rn(o.x, t.x), b = __fsub_rn(o.y, t.y), c = __fsub_rn(o.z, t.z);
        const float ss = __fadd_rn(__fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)), __fmul_rn(c, c));
        if (err) err[i] = fminf(fmaxf(__fsqrt_rn(__fdiv_rn(ss, 3.0f)), 0.0f), 1.0f);
        acc += (double)ss;
    }
    if (!sum_sq) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += part[w];
        atomicAdd(sum_sq, s);
    }
}

// EMA of the weight maps towards the error-derived target weight (run_ffnerf_OG.py:459-490), in the
// reference's precisions: scale = (median + 1e-6) * 2 in double, rounded to float; score =
// clip(err / scale, 0, 8) and target = 1 + 254 * (score / 8) in float; the target is capped at
// bg_cap for background pixels (max colour <= fg_tau out of 255, run_ffnerf_OG.py:402-421); the EMA
// (1 - ema) * w + ema * target and the rounding int(w + 0.5) in double; w clipped to 1..255.
// Rays that hit the same pixel race; one of their updates lands (the reference applies them in
// order, each on the previous value).
__global__ void batch_feedback_kernel(uint8_t* __restrict__ weights, const void* __restrict__ images, int img_f32,
                                      int C, int W, int H, const int32_t* __restrict__ im,
                                      const int32_t* __restrict__ xs, const int32_t* __restrict__ ys,
                                      const float* __restrict__ err, uint32_t n, const float* __restrict__ median,
                                      double ema, int bg_cap, int fg_tau) {
    const float scale = (float)(((double)median[0] + 1e-6) * 2.0);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const size_t pix = ((size_t)im[i] * H + ys[i]) * W + xs[i];
        const float score = fminf(fmaxf(__fdiv_rn(err[i], scale), 0.0f), 8.0f);
        float wt = __fadd_rn(1.0f, __fmul_rn(254.0f, __fdiv_rn(score, 8.0f)));
        bool fg;
        if (img_f32) {
            const float* f = static_cast<const float*>(images) + pix * C;
            fg = fmaxf(fmaxf(f[0], f[1]), f[2]) > (float)((double)fg_tau / 255.0);
        } else {
            const uint8_t* b = static_cast<const uint8_t*>(images) + pix * C;
            fg = max(max((int)b[0], (int)b[1]), (int)b[2]) > fg_tau;
        }
        if (!fg && bg_cap < 255) wt = fminf(wt, (float)bg_cap);
        const double w_new = (1.0 - ema) * (double)weights[pix] + ema * (double)wt;
        const int q = (int)(w_new + 0.5);
        weights[pix] = (uint8_t)min(max(q, 1), 255);
    }
}

}  // namespace ffn
