// ffn_step_tc.cu -- the fused training step with the MLPs on the 5th-generation tensor cores.
//
// Same tile structure as fused_step_kernel (one tile = 128 samples, thread t = sample t), with
// every dense layer of ffnerf_train_step (ffnerf_OG.cl:1378-1466, 1930-2082) and every per-layer
// reduction of update_ffnerf_oneWG (weight_update.cl:210-314) issued as tcgen05.mma:
//
//   forward       ACC[128 x N] = X[128 x K] * W^T         X K-major, W K-major (fp32 accumulate),
//                 each operand as a compensated fp16 pair: hi*hi + hi*lo + lo*hi (three MMAs)
//   backward      ACC[128 x N] = D[128 x K] * W           D K-major, W read MN-major (fp16 hi)
//   weight grad   dW[64 x N]  += D^T[64 x 128] * X[128 x N]   both read MN-major, accumulated in
//                 TMEM over every tile the group processes; bias grads as D^T * e_0 with a constant
//                 one-hot tile.
//
// Why the forward is compensated: the backward masks every hidden delta with the sign of the
// forward activation (ReLU), so a forward that is off by fp16 rounding flips masks of activations
// near zero and moves whole delta entries; that, not the backward's own rounding, dominated the
// gradient error of a plain fp16 forward.  With the hi/lo pairs the forward is as close to fp32 as
// the accumulation, and the remaining error is the backward's fp16 operand rounding.
//
// Accumulators live in tensor memory; the epilogues (bias, ReLU, masks, fp16 packing) run in the
// thread that owns the row (TMEM lane t = sample t).  Deltas are stored scaled by DELTA_SCALE in
// fp16 and unscaled on the way out.  All operand tiles use the core-matrix interleaved layout
// of ffn_tcgen05.cuh.  With F=2, ND=1 one CTA of 256 threads runs two tiles side by side (two
// groups of 4 warps, each with its own operand tiles, mbarrier, named barrier and 256 TMEM columns)
// and the groups share one copy of the weights; other geometries run one group per CTA.  Every
// mbarrier wait is bounded; on a timeout the group flags the status word, stops issuing work, and
// the CTA releases its tensor memory.
#include "ffn_common.cuh"
#include "ffn_hashgrid.cuh"
#include "ffn_raymarch.cuh"
#include "ffn_tcgen05.cuh"

namespace ffn {

constexpr float DELTA_SCALE = 1024.0f;
// The hash encoding is stored as X0 * INPUT_SCALE: freshly initialised tables give features of
// ~1e-4, at the bottom of fp16's normal range; the first layer's accumulator and dWd_in are
// divided by the same factor.
constexpr float INPUT_SCALE = 256.0f;
constexpr uint32_t WAIT_LIMIT = 1u << 22;   // polls of an mbarrier before a wait is declared failed

constexpr int round_up_1k(int x) { return (x + 1023) & ~1023; }

template <int F, int ND>
struct TcPlan {
    static constexpr int ROWS = 128;
    static constexpr int LPOS = 16 * F;
    // tiles side by side per CTA: two where both groups' tiles and tensor memory fit one SM
    static constexpr int GROUPS = (F == 2 && ND == 1) ? 2 : 1;
    static constexpr int THREADS = ROWS * GROUPS;
    // ---- per CTA, shared by the groups: fp16 weights (rows = outputs, columns = inputs).  The
    // 64-row weights have their hi copy at W_HI and their lo copy at W_LO (same offsets in both sets);
    // each 16-row weight has its hi copy at W_DOUT / W_COUT (offsets from W_HI = 0) and its lo copy
    // right behind it, W16_LO bytes on, so that the pair is one [32 x 64] operand and hi*Wh + hi*Wl is
    // one N = 32 MMA per K step.  Then the one-hot tile and the fp32 biases.
    static constexpr int W_DIN = 0;                           // [64 x LPOS]
    static constexpr int W_D01 = W_DIN + 64 * LPOS * 2;       // [64 x 64] (ND = 2)
    static constexpr int W_CIN = W_D01 + (ND >= 2 ? 64 * 64 * 2 : 0);   // [64 x 32]
    static constexpr int W_C01 = W_CIN + 64 * 32 * 2;         // [64 x 64]
    static constexpr int W_SET = W_C01 + 64 * 64 * 2;         // bytes of one set
    static constexpr int W_HI = 0;
    static constexpr int W_LO = W_SET;
    static constexpr int W16_LO = 16 * 64 * 2;
    static constexpr int W_DOUT = 2 * W_SET;                  // [16 x 64], then its lo copy
    static constexpr int W_COUT = W_DOUT + 2 * W16_LO;        // [16 x 64], rows 3..15 zero, then its lo copy
    static constexpr int ONES = W_COUT + 2 * W16_LO;          // one-hot [128 x 8]
    static constexpr int BIAS = ONES + ROWS * 8 * 2;          // bd_0[64] bd_1[64] bd_out[16] bc_0[64] bc_1[64] bc_out[16]
    static constexpr int SHARED_BYTES = round_up_1k(BIAS + (64 * 2 + 16 + 64 * 2 + 16) * 4);
    // ---- per group, at SHARED_BYTES + group * GROUP_BYTES: fp16 operand tiles
    static constexpr int X0 = 0;                              // encoding hi [128 x LPOS]
    static constexpr int LO = X0 + ROWS * LPOS * 2;           // the lo tile of the operand being multiplied
                                                              // (16 KB: any [128 x 64] or X0); the
                                                              // output-delta tile in the backward
    static constexpr int DC = LO;                             // output delta [128 x 16], its lo at DC + DC_LO
    static constexpr int DC_LO = ROWS * 16 * 2;
    static constexpr int HD = LO + ROWS * 64 * 2;             // ND density hidden tiles [128 x 64]
    static constexpr int XC = HD + ND * ROWS * 64 * 2;        // colour input [128 x 32]
    static constexpr int C1 = XC + ROWS * 32 * 2;             // colour hidden 1 [128 x 64]
    static constexpr int C2 = C1 + ROWS * 64 * 2;             // colour hidden 2 [128 x 64]
    static constexpr int BGRAD = C2 + ROWS * 64 * 2;          // bd_out[16], bc_out[16] gradient sums
    static constexpr int RAY = BGRAD + 32 * 4;                // ray-phase arrays
    static constexpr int RAY_BYTES = ROWS * 6 * 4 + ROWS * 16 + ROWS * 16 + 8 * 2 * 4 + 8 * 16 * 4;
    static constexpr int MISC = RAY + RAY_BYTES;              // mbarrier (8), tmem base (4), abort (4)
    static constexpr int GROUP_BYTES = round_up_1k(MISC + 64);
    static constexpr int BYTES = SHARED_BYTES + GROUPS * GROUP_BYTES;
    // staged operand tile in global memory: hi tile then lo tile
    static constexpr int X0_STAGE_BYTES = 2 * ROWS * LPOS * 2;
    // tensor-memory columns of one group
    static constexpr uint32_t ACC = 0;                         // per-tile accumulator (64 cols)
    static constexpr uint32_t DW_C01 = 64;
    static constexpr uint32_t DW_DIN = 128;
    static constexpr uint32_t DW_CIN = DW_DIN + LPOS;
    static constexpr uint32_t DW_COUT_T = DW_CIN + 32;         // [64 in x 16 out]
    static constexpr uint32_t DW_DOUT_T = DW_COUT_T + 16;      // [64 in x 16 out]
    static constexpr uint32_t B_D0 = DW_DOUT_T + 16;
    static constexpr uint32_t B_C0 = B_D0 + 8;
    static constexpr uint32_t B_C1 = B_C0 + 8;
    static constexpr uint32_t DW_D01 = B_C1 + 8;               // ND = 2
    static constexpr uint32_t B_D1 = DW_D01 + 64;
    static constexpr uint32_t USED = ND >= 2 ? B_D1 + 8 : B_C1 + 8;
    static constexpr uint32_t TMEM_GROUP = USED <= 256 ? 256 : 512;
    static constexpr uint32_t TMEM_COLS = TMEM_GROUP * GROUPS;
    static constexpr int CTAS_PER_SM = 1;
    static_assert(TMEM_COLS <= 512, "tensor memory of one SM");
    static_assert(BYTES <= 227 * 1024, "shared memory of one CTA");
};

// This thread's row of its group's tile, and the TMEM lane base of its warp within the group.
__device__ __forceinline__ int trow() { return (int)(threadIdx.x & 127u); }
__device__ __forceinline__ uint32_t tlane() { return (threadIdx.x & 96u) << 16; }

// Converts one fp32 weight matrix [rows x cols] (row-major, from the parameter blob) into the
// interleaved fp16 pair (hi tile, lo tile); rows beyond `rows` up to `pad_rows` are zero.
__device__ __forceinline__ void stage_weight(unsigned char* hi, unsigned char* lo, const float* W, int rows, int pad_rows,
                                             int cols) {
    for (int e = threadIdx.x; e < pad_rows * (cols / 8); e += blockDim.x) {
        const int r = e / (cols / 8), c0 = (e - r * (cols / 8)) * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = r < rows ? W[r * cols + c0 + i] : 0.0f;
        tc::st_chunk8_hilo(hi, lo, r, c0, cols, v);
    }
}

// Issues ACC (+)= A * B for a K range in steps of 16 (one thread).  The descriptors are formed once:
// the descriptor of the tile advanced by k steps is the first one plus (k * step) >> 4 in its start
// field, which cannot carry out of its 14 bits (shared-memory addresses are below 2^18).
__device__ __forceinline__ void gemm(uint32_t d, uint32_t a, int a_cols, bool a_mn, uint32_t b, int b_cols, bool b_mn,
                                     int M, int N, int K, uint32_t accumulate) {
    const uint32_t idesc = tc::idesc_f16(M, N, a_mn, b_mn);
    const uint32_t a_step = a_mn ? 2u * (uint32_t)(a_cols / 8) * 128u : 256u;
    const uint32_t b_step = b_mn ? 2u * (uint32_t)(b_cols / 8) * 128u : 256u;
    const uint64_t ad0 = a_mn ? tc::desc_mnmajor(a, a_cols) : tc::desc_kmajor(a, a_cols);
    const uint64_t bd0 = b_mn ? tc::desc_mnmajor(b, b_cols) : tc::desc_kmajor(b, b_cols);
#pragma unroll
    for (int k = 0; k < K / 16; ++k)
        tc::mma_f16(d, ad0 + (uint64_t)((k * a_step) >> 4), bd0 + (uint64_t)((k * b_step) >> 4), idesc,
                    (k > 0 || accumulate) ? 1u : 0u);
}

// The helpers below take CP (compensated): true forms every product from fp16 operand pairs, the
// training step's form; false multiplies the hi tiles alone and stores no lo tiles (plain fp16
// operands, fp32 accumulation: the MLP microbenchmark's plain form).
//
// Forward layer with compensated operands: ACC = Ah*Wh^T + Ah*Wl^T + Al*Wh^T (both K-major; one
// thread).  The large term first, then the two corrections into the same fp32 accumulator.
template <bool CP = true>
__device__ __forceinline__ void gemm_fwd3(uint32_t d, uint32_t a_hi, uint32_t a_lo, int a_cols, uint32_t w_hi,
                                         uint32_t w_lo, int N, int K) {
    gemm(d, a_hi, a_cols, false, w_hi, a_cols, false, 128, N, K, 0);
    if constexpr (CP) {
        gemm(d, a_hi, a_cols, false, w_lo, a_cols, false, 128, N, K, 1);
        gemm(d, a_lo, a_cols, false, w_hi, a_cols, false, 128, N, K, 1);
    }
}

// Forward layer with 16 outputs and compensated operands, its weight pair stored as one [32 x 64]
// tile (hi rows, then lo rows): ACC[:, 0:16] = Ah*Wh^T + Al*Wh^T and ACC[:, 16:32] = Ah*Wl^T, two MMAs
// per K step instead of three (the issuing thread's time per MMA, not the tensor pipe, sets the
// pace of these small GEMMs); acc_row16_pair adds the halves.  Plain operands: ACC = Ah*Wh^T.
template <bool CP = true>
__device__ __forceinline__ void gemm_fwd16(uint32_t d, uint32_t a_hi, uint32_t a_lo, int a_cols, uint32_t w_pair, int K) {
    gemm(d, a_hi, a_cols, false, w_pair, a_cols, false, 128, CP ? 32 : 16, K, 0);
    if constexpr (CP) gemm(d, a_lo, a_cols, false, w_pair, a_cols, false, 128, 16, K, 1);
}

// Backward-data layer with compensated operands: ACC = Dh*Wh + Dl*Wh + Dh*Wl, D [128 x K] K-major
// (d_cols columns), W [K x N] read MN-major (w_cols columns).  One thread.
template <bool CP = true>
__device__ __forceinline__ void gemm_bwd3(uint32_t d, uint32_t d_hi, uint32_t d_lo, int d_cols, uint32_t w_hi,
                                         uint32_t w_lo, int w_cols, int N, int K) {
    gemm(d, d_hi, d_cols, false, w_hi, w_cols, true, 128, N, K, 0);
    if constexpr (CP) {
        gemm(d, d_lo, d_cols, false, w_hi, w_cols, true, 128, N, K, 1);
        gemm(d, d_hi, d_cols, false, w_lo, w_cols, true, 128, N, K, 1);
    }
}

// Weight (or bias, with the one-hot tile) gradient with a compensated delta: ACC (+)= Dh^T X + Dl^T X,
// D [128 x 64] and X [128 x N] both read MN-major (the activation X stays a single fp16 tile).
template <bool CP = true>
__device__ __forceinline__ void gemm_wgrad2(uint32_t d, uint32_t d_hi, uint32_t d_lo, uint32_t x, int x_cols, int N,
                                           uint32_t accumulate) {
    gemm(d, d_hi, 64, true, x, x_cols, true, 64, N, 128, accumulate);
    if constexpr (CP) gemm(d, d_lo, 64, true, x, x_cols, true, 64, N, 128, 1);
}

// One 8-value chunk as the operand pair (CP) or as the hi tile alone.
template <bool CP = true>
__device__ __forceinline__ void st_pair8(unsigned char* hi, unsigned char* lo, int r, int c0, int cols, const float* v) {
    if constexpr (CP) tc::st_chunk8_hilo(hi, lo, r, c0, cols, v);
    else tc::st_chunk8(hi, r, c0, cols, v);
}

// One row (this thread's sample) of an ACC region into registers.
template <int N>
__device__ __forceinline__ void acc_row(uint32_t tmem, uint32_t col, float (&v)[N]) {
    const uint32_t lane = tlane();
#pragma unroll
    for (int j = 0; j < N; j += 16) {
        float t[16];
        tc::tmem_ld16(tmem + lane + col + j, t);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[j + i] = t[i];
    }
    tc::tmem_wait_ld();
}

// The 16 outputs of a gemm_fwd16 layer: the two accumulator halves added (compensated form).
template <bool CP = true>
__device__ __forceinline__ void acc_row16_pair(uint32_t tmem, uint32_t col, float (&v)[16]) {
    if constexpr (CP) {
        float t[32];
        acc_row<32>(tmem, col, t);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = t[j] + t[16 + j];
    } else {
        acc_row<16>(tmem, col, v);
    }
}

template <int N>
__device__ __forceinline__ void store_row(unsigned char* tile, int cols, const float (&v)[N]) {
#pragma unroll
    for (int c = 0; c < N; c += 8) tc::st_chunk8(tile, trow(), c, cols, v + c);
}
template <int N, bool CP = true>
__device__ __forceinline__ void store_row_hilo(unsigned char* hi, unsigned char* lo, int cols, const float (&v)[N]) {
#pragma unroll
    for (int c = 0; c < N; c += 8) st_pair8<CP>(hi, lo, trow(), c, cols, v + c);
}

// Epilogue of a forward layer: row = relu(ACC * in_scale + bias) for N columns, 32 at a time (two
// TMEM loads per wait; one copy of the loop body, to keep the kernel's code small), stored as the
// (hi, lo) pair that the next forward layer multiplies.
template <bool CP = true>
__device__ __forceinline__ void epi_bias_relu(uint32_t tmem, uint32_t col, int N, const float* bias, unsigned char* tile,
                                              unsigned char* lo_tile, int cols, float in_scale = 1.0f) {
    const uint32_t lane = tlane();
    const int r = trow();
#pragma unroll 1
    for (int j = 0; j < N; j += 32) {
        float v[32];
        tc::tmem_ld16(tmem + lane + col + j, *reinterpret_cast<float(*)[16]>(v));
        tc::tmem_ld16(tmem + lane + col + j + 16, *reinterpret_cast<float(*)[16]>(v + 16));
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = fmaxf(fmaf(v[i], in_scale, bias[j + i]), 0.0f);
#pragma unroll
        for (int q = 0; q < 32; q += 8) st_pair8<CP>(tile, lo_tile, r, j + q, cols, v + q);
    }
}

// Epilogue of a backward layer: row = ACC masked by (activation in `tile` > 0), written in place,
// 32 columns at a time.  The mask reads the hi copy of the activation, which is > 0 whenever the
// activation is, except below fp16's smallest subnormal (2^-24), where the delta's share is negligible.
template <bool CP = true>
__device__ __forceinline__ void epi_relu_mask(uint32_t tmem, uint32_t col, int N, unsigned char* tile,
                                              unsigned char* lo_tile, int cols) {
    const uint32_t lane = tlane();
    const int r = trow();
#pragma unroll 1
    for (int j = 0; j < N; j += 32) {
        float v[32], act[32];
        tc::tmem_ld16(tmem + lane + col + j, *reinterpret_cast<float(*)[16]>(v));
        tc::tmem_ld16(tmem + lane + col + j + 16, *reinterpret_cast<float(*)[16]>(v + 16));
#pragma unroll
        for (int q = 0; q < 32; q += 8) tc::ld_chunk8(tile, r, j + q, cols, act + q);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = act[i] > 0.0f ? v[i] : 0.0f;
#pragma unroll
        for (int q = 0; q < 32; q += 8) st_pair8<CP>(tile, lo_tile, r, j + q, cols, v + q);
    }
}

// Hash encoding of this thread's sample straight into its row of the X0 tile pair (hi, lo), one
// 8-feature chunk (8/F levels, 64/F independent gathers) at a time.
template <int F>
__device__ __forceinline__ void encode_rows(const DevConfig& c, const float* __restrict__ table, V3 p, bool hit,
                                            unsigned char* tile, unsigned char* lo_tile) {
    constexpr int LPOS = L * F, LV = 8 / F;
    const int r = trow();
#pragma unroll 1
    for (int q = 0; q < LPOS / 8; ++q) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        if (hit) {
#pragma unroll
            for (int li = 0; li < LV; ++li) {
                const int lvl = q * LV + li;
                Corner8 k;
                level_corners<F>(c, p, lvl, k);
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    if constexpr (F == 2) {
                        const float2 t = table_ld2<true>(table + k.base[cc]);
                        v[li * 2] = fmaf(k.w[cc], t.x, v[li * 2]);
                        v[li * 2 + 1] = fmaf(k.w[cc], t.y, v[li * 2 + 1]);
                    } else {
                        const float4 t = table_ld4<true>(table + k.base[cc]);
                        v[li * 4] = fmaf(k.w[cc], t.x, v[li * 4]);
                        v[li * 4 + 1] = fmaf(k.w[cc], t.y, v[li * 4 + 1]);
                        v[li * 4 + 2] = fmaf(k.w[cc], t.z, v[li * 4 + 2]);
                        v[li * 4 + 3] = fmaf(k.w[cc], t.w, v[li * 4 + 3]);
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] *= INPUT_SCALE;
        tc::st_chunk8_hilo(tile, lo_tile, r, q * 8, LPOS, v);
    }
}


// Scatter of one level's hash-grid gradient (ffnerf_OG.cl:2090-2173): the thread's F raw feature
// gradients `gl` become (coef_l * g) * w_c at the 8 trilinear corners, added with vector atomics.
// The lanes of a warp -- consecutive samples of a ray, in ray order (of two or more rays below 32
// samples per ray) -- often sit in the same grid cell and would add to the same 8 table entries (on
// the coarse levels nearly always; on the fine ones where the occupancy-guided sampler packs samples
// densely).  A ray leaves a (convex) cell only once, so a ray's lanes in one cell form a run: a lane starts a run when the lane before it is not scattering this
// level or holds another cell (one shuffle of the 64-bit cell key, one ballot).  A segmented suffix
// sum by shuffles leaves each run's total in its first lane, in log2(longest run) steps, and that lane
// adds the run's sums with one set of atomics.  Merging on all 16 levels measured fastest (cfg3 step
// 1.80 ms with the 10 coarsest, 1.74 ms with all 16, 1.86 ms with none, when the runs were found by
// a match on the key; finding them from the neighbour's key took the step from 1.729 to 1.711 ms):
// the reductions themselves are the scatter's cost.
template <int F>
__device__ __forceinline__ void scatter_level(const DevConfig& c, float* __restrict__ grad, V3 p, int lvl,
                                              const float* gl, const float* coef) {
    const int lid = threadIdx.x & 31;
    float gf[F];
    bool any = false;
#pragma unroll
    for (int f = 0; f < F; ++f) {
        const float v = gl[f];
        gf[f] = isfinite(v) ? coef[lvl] * v : 0.0f;   // non-finite features are skipped (ffnerf_OG.cl:2162)
        any |= gf[f] != 0.0f;
    }
    if (!any) return;
    Corner8 k;
    uint64_t key;
    level_corners<F>(c, p, lvl, k, &key);
    const unsigned act = __activemask();
    const unsigned klo = (unsigned)key, khi = (unsigned)(key >> 32);
    const unsigned plo = __shfl_up_sync(act, klo, 1), phi = __shfl_up_sync(act, khi, 1);
    const bool prev_in = lid > 0 && ((act >> (lid - 1)) & 1u);
    const unsigned heads = __ballot_sync(act, !prev_in || plo != klo || phi != khi);
    const unsigned upto = (2u << lid) - 1u;                 // lanes 0..lid (all 32 for lane 31)
    const unsigned after = (heads | ~act) & ~upto;         // later lanes that end this lane's run
    const int last = after ? __ffs(after) - 2 : 31;         // the run's last lane
    const int first = 31 - __clz(heads & upto);             // the run's first lane
    const int span = (int)__reduce_max_sync(act, (unsigned)(last - first + 1));
    if (span == 1) {
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const float w = k.w[cc];
            if constexpr (F == 2)
                red_add2(grad + k.base[cc], gf[0] * w, gf[1] * w);
            else
                red_add4(grad + k.base[cc], gf[0] * w, gf[1] * w, gf[2] * w, gf[3] * w);
        }
        return;
    }
    float v[8 * F];
#pragma unroll
    for (int cc = 0; cc < 8; ++cc)
#pragma unroll
        for (int f = 0; f < F; ++f) v[cc * F + f] = gf[f] * k.w[cc];
    // every lane of [first, last] is active, so the shuffles below read live values only
    for (int off = 1; off < span; off <<= 1) {
#pragma unroll
        for (int q = 0; q < 8 * F; ++q) {
            const float t = __shfl_down_sync(act, v[q], off);
            if (lid + off <= last) v[q] += t;
        }
    }
    if (lid == first) {
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            if constexpr (F == 2) red_add2(grad + k.base[cc], v[2 * cc], v[2 * cc + 1]);
            else red_add4(grad + k.base[cc], v[4 * cc], v[4 * cc + 1], v[4 * cc + 2], v[4 * cc + 3]);
        }
    }
}

// Hash-grid gradient from the ACC region (scaled deltas times Wd_in).  F = 2: the thread's 32 values are
// first parked in its row of `gbuf` (shared memory, 32 floats per thread, float4 slots XOR-swizzled
// by the row so that a warp's stores and loads spread over the banks), then the levels are scattered
// one at a time by a single (not unrolled) copy of the level code: the kernel is large and its
// instruction cache is a limit.
// Every lane of the warp executes the TMEM loads (tcgen05.ld is warp-aligned: with fewer than 32
// samples per ray a warp holds two or more rays, which may differ in hitting the box); only `live`
// lanes (a sample of a hitting ray) scatter.
template <int F>
__device__ __forceinline__ void scatter_from_tmem(const DevConfig& c, uint32_t tmem, uint32_t col, float* __restrict__ grad,
                                                  V3 p, float unscale, const float* coef, float* gbuf,
                                                  bool live) {
    constexpr int LPOS = L * F;
    const uint32_t lane = tlane();
    if constexpr (F != 2) {
        // F = 4: the parked rows would not fit the free C2 tile; levels straight from the TMEM loads
#pragma unroll 1
        for (int j = 0; j < LPOS; j += 16) {
            float g[16];
            tc::tmem_ld16(tmem + lane + col + j, g);
            tc::tmem_wait_ld();
            if (!live) continue;
#pragma unroll
            for (int li = 0; li < 16 / F; ++li) {
                float gl[F];
#pragma unroll
                for (int f = 0; f < F; ++f) gl[f] = g[li * F + f] * unscale;
                scatter_level<F>(c, grad, p, j / F + li, gl, coef);
            }
        }
        return;
    }
    const int row = trow(), sw = row & 7;
    float4* grow = reinterpret_cast<float4*>(gbuf + row * LPOS);
#pragma unroll
    for (int j = 0; j < LPOS; j += 16) {
        float g[16];
        tc::tmem_ld16(tmem + lane + col + j, g);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 16; q += 4)
            grow[((j + q) / 4) ^ (sw % (LPOS / 4))] =
                make_float4(g[q] * unscale, g[q + 1] * unscale, g[q + 2] * unscale, g[q + 3] * unscale);
    }
    if (!live) return;
#pragma unroll 1
    for (int lvl = 0; lvl < L; ++lvl) {
        const float4 t = grow[((lvl * F) / 4) ^ (sw % (LPOS / 4))];
        float gl[F];
        if constexpr (F == 2) {
            const bool hi = (lvl & 1) != 0;
            gl[0] = hi ? t.z : t.x;
            gl[1] = hi ? t.w : t.y;
        } else {
            gl[0] = t.x; gl[1] = t.y; gl[2] = t.z; gl[3] = t.w;
        }
        scatter_level<F>(c, grad, p, lvl, gl, coef);
    }
}

// Sums v[0..15] over the warp's 32 lanes by a transposed butterfly (16 shuffles instead of 80): lane
// l ends with the sum for index (l >> 1) & 15 (lanes l and l ^ 1 hold the same sum).
__device__ __forceinline__ float warp_sum16(const float (&v)[16]) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    float a[8], b[4], e[2];
    const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0, h4 = (lane & 4) != 0, h2 = (lane & 2) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = (h16 ? v[i + 8] : v[i]) + __shfl_xor_sync(full, h16 ? v[i] : v[i + 8], 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = (h8 ? a[i + 4] : a[i]) + __shfl_xor_sync(full, h8 ? a[i] : a[i + 4], 8);
#pragma unroll
    for (int i = 0; i < 2; ++i) e[i] = (h4 ? b[i + 2] : b[i]) + __shfl_xor_sync(full, h4 ? b[i] : b[i + 2], 4);
    float d = (h2 ? e[1] : e[0]) + __shfl_xor_sync(full, h2 ? e[0] : e[1], 2);
    return d + __shfl_xor_sync(full, d, 1);
}

// Sums v[0..3] over the warp's 32 lanes (6 shuffles instead of 20): lane l ends with the sum for
// index (l >> 3) & 3.
__device__ __forceinline__ float warp_sum4(const float (&v)[4]) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
    float a[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) a[i] = (h16 ? v[i + 2] : v[i]) + __shfl_xor_sync(full, h16 ? v[i] : v[i + 2], 16);
    float b = (h8 ? a[1] : a[0]) + __shfl_xor_sync(full, h8 ? a[0] : a[1], 8);
    b += __shfl_xor_sync(full, b, 4);
    b += __shfl_xor_sync(full, b, 2);
    return b + __shfl_xor_sync(full, b, 1);
}

// 16-byte global -> shared copies that complete in the background (cp.async, L2 only).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// MLPB (the MLP microbenchmark, staged form only): the tiles hold given inputs instead of hash
// encodings; every sample is live, the view direction is fixed at (0.36, 0.48, 0.8), and the
// compositing is replaced by the loss sum_k 0.5 (rgb_k - 0.5)^2 per sample (no density term), so
// the step is the two MLPs forward and backward with their weight gradients; no table scatter.
//
// Work split: tile g of the CTA's groups takes tiles blockIdx.x * GROUPS + g, advancing by
// gridDim.x * GROUPS; each group writes its own row of weight-gradient partials
// (a.partials[(blockIdx.x * GROUPS + g) * P]).
template <int F, int ND, bool STAGED = false, bool MLPB = false, bool PLAIN = false>
__global__ void __launch_bounds__(TcPlan<F, ND>::THREADS, 1) fused_step_tc_kernel(const StepArgs a) {
    static_assert(!MLPB || STAGED, "the MLP microbenchmark runs the staged form");
    static_assert(!PLAIN || MLPB, "plain fp16 operands are the MLP microbenchmark's form only");
    constexpr bool CP = !PLAIN;     // compensated operand pairs
    using PL = TcPlan<F, ND>;
    constexpr int LPOS = PL::LPOS;
    extern __shared__ __align__(1024) unsigned char smem_tc[];
    // The group index and the tensor-memory base are broadcast from lane 0 (every lane holds the same
    // value): the compiler then treats them, and every shared-memory and tensor-memory address and MMA
    // descriptor formed from them, as warp-uniform, and the issuing thread forms its descriptors in
    // uniform registers instead of converting each one (cfg3 step 1.723 -> 1.652 ms).
    const int grp = PL::GROUPS == 1 ? 0 : __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 7), 0);
    unsigned char* gsm = smem_tc + PL::SHARED_BYTES + grp * PL::GROUP_BYTES;   // this group's tiles
    const DevConfig& c = a.c;
    const ParamLayout& lo = a.lo;
    const int tid = trow();            // this thread's row of the group's tile
    const int warp = tid >> 5;         // warp within the group
    unsigned char* tX0 = gsm + PL::X0;
    unsigned char* tLO = gsm + PL::LO;
    unsigned char* tXC = gsm + PL::XC;
    unsigned char* tC1 = gsm + PL::C1;
    unsigned char* tC2 = gsm + PL::C2;
    unsigned char* tDC = gsm + PL::DC;
    const float* bias = reinterpret_cast<const float*>(smem_tc + PL::BIAS);
    float* bgrad = reinterpret_cast<float*>(gsm + PL::BGRAD);
    float* rayb = reinterpret_cast<float*>(gsm + PL::RAY);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(gsm + PL::MISC);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_tc + PL::SHARED_BYTES + PL::MISC + 8);   // group 0's slot
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gsm + PL::MISC + 12);
    const uint32_t sbase = tc::smem_u32(smem_tc);
    const uint32_t gbase = tc::smem_u32(gsm);
    auto S = [&](int off) { return sbase + (uint32_t)off; };        // shared region (weights, one-hot)
    auto G = [&](int off) { return gbase + (uint32_t)off; };        // this group's tiles
    auto tH = [&](int l) { return gsm + PL::HD + l * 128 * 64 * 2; };

    const bool train = a.do_train != 0;
    const bool probe = a.probe != 0;
    const bool backward = train && !probe;

    // ---- one-time set-up: barriers, tensor memory, fp16 weight pairs, biases, one-hot tile
    if (tid == 0) {
        tc::mbar_init(mbar, 1);
        *abort_flag = 0;
    }
    if (threadIdx.x < 32) tc::tmem_alloc(tmem_slot, PL::TMEM_COLS);
    const float* P = a.params;
    unsigned char* wh = smem_tc + PL::W_HI;
    unsigned char* wl = smem_tc + PL::W_LO;
    stage_weight(wh + PL::W_DIN, wl + PL::W_DIN, P + lo.off[P_WD_IN], 64, 64, LPOS);
    if (ND >= 2) stage_weight(wh + PL::W_D01, wl + PL::W_D01, P + lo.off[P_WD_01], 64, 64, 64);
    stage_weight(wh + PL::W_DOUT, wh + PL::W_DOUT + PL::W16_LO, P + lo.off[P_WD_OUT], 16, 16, 64);
    stage_weight(wh + PL::W_CIN, wl + PL::W_CIN, P + lo.off[P_WC_IN], 64, 64, 32);
    stage_weight(wh + PL::W_C01, wl + PL::W_C01, P + lo.off[P_WC_01], 64, 64, 64);
    stage_weight(wh + PL::W_COUT, wh + PL::W_COUT + PL::W16_LO, P + lo.off[P_WC_OUT], 3, 16, 64);
    {
        float* sb = reinterpret_cast<float*>(smem_tc + PL::BIAS);
        for (int i = threadIdx.x; i < 64; i += blockDim.x) {
            sb[i] = P[lo.off[P_BD_0] + i];
            sb[64 + i] = ND >= 2 ? P[lo.off[P_BD_1] + i] : 0.0f;
            sb[144 + i] = P[lo.off[P_BC_0] + i];
            sb[208 + i] = P[lo.off[P_BC_1] + i];
        }
        if (threadIdx.x < 16) {
            sb[128 + threadIdx.x] = P[lo.off[P_BD_OUT] + threadIdx.x];
            sb[272 + threadIdx.x] = threadIdx.x < 3 ? P[lo.off[P_BC_OUT] + threadIdx.x] : 0.0f;
        }
    }
    if (tid < 32) bgrad[tid] = 0.0f;
    if (threadIdx.x < 128) {
        float v[8] = {1.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        tc::st_chunk8(smem_tc + PL::ONES, threadIdx.x, 0, 8, v);
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem_base = __shfl_sync(0xffffffffu, *tmem_slot, 0);
    const uint32_t tmem = tmem_base + (uint32_t)grp * PL::TMEM_GROUP;   // this group's columns
    uint32_t phase = 0;
    bool dw_started = false;

    // Commit the MMAs this group issued so far and wait for them (the group's threads).
    auto sync_mma = [&]() {
        if (tid == 0) tc::commit(mbar);
        if (!*abort_flag) {
            if (!tc::mbar_wait(mbar, phase, WAIT_LIMIT)) {
                *abort_flag = 1;
                if (a.status) atomicOr(a.status, ST_TC_TIMEOUT);
            }
        }
        phase ^= 1u;
        tc::fence_after_sync();
    };
    // The group's threads have finished reading TMEM and writing shared operands: MMAs may be issued.
    auto handoff = [&]() {
        tc::fence_proxy_async();
        tc::fence_before_sync();
        tile_sync();
        tc::fence_after_sync();
    };

    const V3 bmin = v3(c.bmin[0], c.bmin[1], c.bmin[2]);
    const V3 bmax = v3(c.bmax[0], c.bmax[1], c.bmax[2]);
    const V3 bsize = vsub(bmax, bmin);
    const V3 inv_box = v3(fd(1.0f, bsize.x), fd(1.0f, bsize.y), fd(1.0f, bsize.z));
    const int spr = c.spr;
    const int rl = tid / spr, lid = tid - rl * spr, rbase = rl * spr;
    const int rays_per_tile = 128 / spr;
    const int n_tiles = (int)((a.n_rays + rays_per_tile - 1) / rays_per_tile);
    float* sCand = rayb;
    float* sCdf = sCand + 128;
    float* sTs = sCdf + 128;
    float* sDTs = sTs + 128;
    float* sTr = sDTs + 128;
    uint32_t* sKey = reinterpret_cast<uint32_t*>(sTr + 128);
    float4* sSeg = reinterpret_cast<float4*>(sKey + 128);
    float2* sAffS = reinterpret_cast<float2*>(sSeg + 128);
    float2* sAffE = sAffS + 128;
    uint32_t* sChg = reinterpret_cast<uint32_t*>(sAffE + 128);
    float* sRay = reinterpret_cast<float*>(sChg + 16);

    const int first_tile = (int)blockIdx.x * PL::GROUPS + grp;
    const int tile_step = (int)gridDim.x * PL::GROUPS;

    // Staged form: the next tile's X0 pair is copied (cp.async) into X0 / LO as soon as the current
    // tile's last MMA that reads them has completed -- before the table scatter, which it overlaps
    // -- and its per-sample inputs are loaded into registers.
    float2 nx_tdt = make_float2(0.f, 0.f);
    uint4 nx_rst = make_uint4(0u, 0u, 0u, 0u);
    float4 nx_ro = make_float4(0.f, 0.f, 0.f, 0.f), nx_rd = make_float4(0.f, 0.f, 1.f, 0.f);
    float4 nx_tg = make_float4(0.f, 0.f, 0.f, 0.f);
    auto prefetch = [&](int t) {
        const uint32_t ri = (uint32_t)t * rays_per_tile + rl;
        nx_tdt = make_float2(0.f, 0.f);
        nx_rst = make_uint4(0u, 0u, 0u, 0u);
        nx_ro = make_float4(0.f, 0.f, 0.f, 0.f);
        nx_rd = make_float4(0.f, 0.f, 1.f, 0.f);
        nx_tg = make_float4(0.f, 0.f, 0.f, 0.f);
        if (!MLPB && ri < a.n_rays) {
            nx_tdt = a.tdt_stage[(size_t)t * 128 + tid];
            nx_rst = a.ray_stage[ri];
            nx_ro = a.rays[2 * ri];
            nx_rd = a.rays[2 * ri + 1];
            if (lid == 0 && a.targets) nx_tg = a.targets[ri];   // read by the ray's lane 0 in the compositing
        }
        constexpr int HALF = 128 * LPOS * 2;   // bytes of the hi (and of the lo) tile
        const unsigned char* src = a.x0_stage + (size_t)t * PL::X0_STAGE_BYTES;
#pragma unroll
        for (int k = tid; k < HALF / 16; k += 128) {
            cp_async16(G(PL::X0) + 16u * (uint32_t)k, src + 16 * k);
            cp_async16(G(PL::LO) + 16u * (uint32_t)k, src + HALF + 16 * k);
        }
        cp_async_commit();
    };
    if constexpr (STAGED) {
        if (first_tile < n_tiles) prefetch(first_tile);
    }

    for (int tile = first_tile; tile < n_tiles && !*abort_flag; tile += tile_step) {
        const uint32_t ray_idx = (uint32_t)tile * rays_per_tile + rl;
        const bool valid = ray_idx < a.n_rays;
        const uint32_t ray_id = a.ray_offset + ray_idx;
        const bool more = tile + tile_step < n_tiles;
        float4 ro = make_float4(0.f, 0.f, 0.f, 0.f), rd = make_float4(0.f, 0.f, 1.f, 0.f);
        if constexpr (MLPB) {
            rd = make_float4(0.36f, 0.48f, 0.8f, 0.f);
        } else if constexpr (STAGED) {
            ro = nx_ro;
            rd = nx_rd;
        } else if (valid) {
            ro = a.rays[2 * ray_idx];
            rd = a.rays[2 * ray_idx + 1];
        }
        const V3 o = v3(ro.x, ro.y, ro.z), d = v3(rd.x, rd.y, rd.z);
        RayTile R{sCand, sCdf, sTs, sDTs, sTr, sKey, sSeg, sAffS, sAffE, sChg, sRay, tid, spr, rl, lid, rbase,
                  ray_idx, ray_id, valid, train, probe, o, d, bmin, bmax, bsize, inv_box, (float)c.G, 1.0f / (float)spr,
                  STAGED, nx_tg};
        bool hit;
        int idx_sel = 0;
        if constexpr (STAGED) {
            // sampling and encoding were done by the stage kernels: their results were prefetched
            const float2 tdt = nx_tdt;
            const uint4 rst = nx_rst;
            sTs[tid] = tdt.x;
            sDTs[tid] = tdt.y;
            if (lid == 0) { sChg[rl * 2] = rst.x; sChg[rl * 2 + 1] = rst.y; }
            hit = MLPB || rst.z != 0u;
            cp_async_wait_all();
            tile_sync();
        } else {
            ray_sampler(a, R, hit, idx_sel);
        }
        bool prefetched = false;
        auto prefetch_next = [&]() {
            if constexpr (STAGED) {
                if (more && !prefetched) prefetch(tile + tile_step);
            }
            prefetched = true;
        };
        const float* rs = sRay + rl * 16;
        const float t_s = sTs[tid];
        const float dt_s = sDTs[tid];
        const V3 xs = ray_point(o, d, t_s);
        const V3 pn = normalize_pos(c, xs);

        // ---------------- forward MLP on the tensor cores (compensated operand pairs)
        float sigma = 0.0f, rgb[3] = {0.f, 0.f, 0.f}, dout0 = 0.0f;
        if (probe && a.bypass) {
            float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
            if (valid) b = a.bypass[(size_t)ray_idx * spr + lid];
            sigma = b.x; rgb[0] = b.y; rgb[1] = b.z; rgb[2] = b.w;
        } else {
            if constexpr (!STAGED) encode_rows<F>(c, a.table, pn, hit, tX0, tLO);
            handoff();
            if (tid == 0) gemm_fwd3<CP>(tmem + PL::ACC, G(PL::X0), G(PL::LO), LPOS, S(PL::W_HI + PL::W_DIN), S(PL::W_LO + PL::W_DIN), 64, LPOS);
            sync_mma();
            epi_bias_relu<CP>(tmem, PL::ACC, 64, bias, tH(0), tLO, 64, 1.0f / INPUT_SCALE);
            if (ND >= 2) {
                handoff();
                if (tid == 0) gemm_fwd3<CP>(tmem + PL::ACC, G(PL::HD), G(PL::LO), 64, S(PL::W_HI + PL::W_D01), S(PL::W_LO + PL::W_D01), 64, 64);
                sync_mma();
                epi_bias_relu<CP>(tmem, PL::ACC, 64, bias + 64, tH(ND - 1), tLO, 64);
            }
            handoff();
            if (tid == 0)
                gemm_fwd16<CP>(tmem + PL::ACC, G(PL::HD + (ND - 1) * 128 * 64 * 2), G(PL::LO), 64, S(PL::W_HI + PL::W_DOUT), 64);
            sync_mma();
            {
                float v[32];
                float dv[16];
                acc_row16_pair<CP>(tmem, PL::ACC, dv);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = dv[j] + bias[128 + j];
                dout0 = v[0];
                sigma = softplus(fclamp(dout0, -10.0f, 10.0f));
                float sh[L_DIR];
                sh16(d.x, d.y, d.z, sh);
#pragma unroll
                for (int j = 0; j < 16; ++j) v[16 + j] = sh[j] * a.sh_mult;
                store_row_hilo<32, CP>(tXC, tLO, 32, v);
            }
            handoff();
            if (tid == 0) gemm_fwd3<CP>(tmem + PL::ACC, G(PL::XC), G(PL::LO), 32, S(PL::W_HI + PL::W_CIN), S(PL::W_LO + PL::W_CIN), 64, 32);
            sync_mma();
            epi_bias_relu<CP>(tmem, PL::ACC, 64, bias + 144, tC1, tLO, 64);
            handoff();
            if (tid == 0) gemm_fwd3<CP>(tmem + PL::ACC, G(PL::C1), G(PL::LO), 64, S(PL::W_HI + PL::W_C01), S(PL::W_LO + PL::W_C01), 64, 64);
            sync_mma();
            epi_bias_relu<CP>(tmem, PL::ACC, 64, bias + 208, tC2, tLO, 64);
            handoff();
            if (tid == 0) gemm_fwd16<CP>(tmem + PL::ACC, G(PL::C2), G(PL::LO), 64, S(PL::W_HI + PL::W_COUT), 64);
            sync_mma();
            {
                float v[16];
                acc_row16_pair<CP>(tmem, PL::ACC, v);
#pragma unroll
                for (int k = 0; k < 3; ++k) rgb[k] = sigmoid_soft(v[k] + bias[272 + k]);
            }
        }
        if (!MLPB && dt_s <= 0.0f) sigma = 0.0f;

        // ---------------- compositing, loss gradient, occupancy proposals
        float T_s, dLds, dLdc[3];
        uint32_t chg0, chg1;
        if constexpr (MLPB) {
            T_s = 1.0f;
            dLds = 0.0f;
#pragma unroll
            for (int k = 0; k < 3; ++k) dLdc[k] = rgb[k] - 0.5f;
            chg0 = chg1 = 0u;
        } else {
            ray_composite(a, R, rs, sigma, rgb, xs, t_s, dt_s, T_s, dLds, dLdc, chg0, chg1);
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
        }
        if (!backward) {
            tc::fence_before_sync();
            tile_sync();          // every thread is past its reads of X0 / LO / the ray arrays
            prefetch_next();
            continue;
        }

        // ---------------- output deltas (ffnerf_OG.cl:1858-1891)
        float dcout[3], ddout0;
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
            if constexpr (MLPB) f_vol = valid ? 1.0f : 0.0f;
            const float d_sigma = f_vol * dLds;
#pragma unroll
            for (int k = 0; k < 3; ++k) dcout[k] = (f_vol * dLdc[k]) * ((rgb[k] * (1.0f - rgb[k])) * 0.5f);
            ddout0 = 1.0f * d_sigma * softplus_prime(fclamp(dout0, -18.0f, 18.0f));
        }
        {
            // the forward's last MMA (which read the lo tile) has completed: DC takes its place
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = 0.0f;
            v[0] = dcout[0] * DELTA_SCALE; v[1] = dcout[1] * DELTA_SCALE; v[2] = dcout[2] * DELTA_SCALE;
            store_row_hilo<16, CP>(tDC, tDC + PL::DC_LO, 16, v);
            // colour-head bias gradient: a transposed warp butterfly, then three lanes add at once
            {
                const float v4[4] = {v[0], v[1], v[2], 0.0f};
                const float sum = warp_sum4(v4);
                const int k = (tid >> 3) & 3;
                if ((tid & 7) == 0 && k < 3) atomicAdd(bgrad + 16 + k, sum);
            }
        }
        // every tile runs the backward: the weight-gradient accumulators start on the group's first tile
        const uint32_t acc0 = tile != first_tile ? 1u : 0u;
        handoff();
        if (tid == 0) {
            gemm(tmem + PL::DW_COUT_T, G(PL::C2), 64, true, G(PL::DC), 16, true, 64, 16, 128, acc0);            // dWc_out^T
            if constexpr (CP) gemm(tmem + PL::DW_COUT_T, G(PL::C2), 64, true, G(PL::DC) + PL::DC_LO, 16, true, 64, 16, 128, 1);
            gemm_bwd3<CP>(tmem + PL::ACC, G(PL::DC), G(PL::DC) + PL::DC_LO, 16, S(PL::W_HI + PL::W_COUT),
                      S(PL::W_HI + PL::W_COUT + PL::W16_LO), 64, 64, 16);                                                       // dC2
        }
        sync_mma();
        {
            epi_relu_mask<CP>(tmem, PL::ACC, 64, tC2, tLO, 64);
        }
        handoff();
        if (tid == 0) {
            gemm_wgrad2<CP>(tmem + PL::DW_C01, G(PL::C2), G(PL::LO), G(PL::C1), 64, 64, acc0);                      // dWc_01
            gemm_wgrad2<CP>(tmem + PL::B_C1, G(PL::C2), G(PL::LO), S(PL::ONES), 8, 8, acc0);                        // dbc_1
            gemm_bwd3<CP>(tmem + PL::ACC, G(PL::C2), G(PL::LO), 64, S(PL::W_HI + PL::W_C01), S(PL::W_LO + PL::W_C01),
                      64, 64, 64);                                                                                // dC1
        }
        sync_mma();
        {
            epi_relu_mask<CP>(tmem, PL::ACC, 64, tC1, tLO, 64);
        }
        handoff();
        if (tid == 0) {
            gemm_wgrad2<CP>(tmem + PL::DW_CIN, G(PL::C1), G(PL::LO), G(PL::XC), 32, 32, acc0);                      // dWc_in
            gemm_wgrad2<CP>(tmem + PL::B_C0, G(PL::C1), G(PL::LO), S(PL::ONES), 8, 8, acc0);                        // dbc_0
            gemm_bwd3<CP>(tmem + PL::ACC, G(PL::C1), G(PL::LO), 64, S(PL::W_HI + PL::W_CIN), S(PL::W_LO + PL::W_CIN),
                      32, 16, 64);                                                                                // dDout
        }
        sync_mma();
        {
            float v[16];
            acc_row<16>(tmem, PL::ACC, v);
            v[0] += ddout0 * DELTA_SCALE;
            // delta at the density output replaces the colour input's first 16 columns
#pragma unroll
            for (int cc = 0; cc < 16; cc += 8) st_pair8<CP>(tXC, tLO, tid, cc, 32, v + cc);
            {
                const float sum = warp_sum16(v);
                if ((tid & 1) == 0) atomicAdd(bgrad + ((tid >> 1) & 15), sum);
            }
        }
        const uint32_t hlast = G(PL::HD + (ND - 1) * 128 * 64 * 2);
        handoff();
        if (tid == 0) {
            gemm(tmem + PL::DW_DOUT_T, hlast, 64, true, G(PL::XC), 32, true, 64, 16, 128, acc0);               // dWd_out^T
            if constexpr (CP) gemm(tmem + PL::DW_DOUT_T, hlast, 64, true, G(PL::LO), 32, true, 64, 16, 128, 1);
            gemm_bwd3<CP>(tmem + PL::ACC, G(PL::XC), G(PL::LO), 32, S(PL::W_HI + PL::W_DOUT), S(PL::W_HI + PL::W_DOUT + PL::W16_LO),
                      64, 64, 16);                                                                                // dH_last
        }
        sync_mma();
        {
            epi_relu_mask<CP>(tmem, PL::ACC, 64, tH(ND - 1), tLO, 64);
        }
        if (ND >= 2) {
            handoff();
            if (tid == 0) {
                gemm_wgrad2<CP>(tmem + PL::DW_D01, hlast, G(PL::LO), G(PL::HD), 64, 64, acc0);                      // dWd_01
                gemm_wgrad2<CP>(tmem + PL::B_D1, hlast, G(PL::LO), S(PL::ONES), 8, 8, acc0);                        // dbd_1
                gemm_bwd3<CP>(tmem + PL::ACC, hlast, G(PL::LO), 64, S(PL::W_HI + PL::W_D01), S(PL::W_LO + PL::W_D01),
                          64, 64, 64);                                                                            // dH_0
            }
            sync_mma();
            epi_relu_mask<CP>(tmem, PL::ACC, 64, tH(0), tLO, 64);
        }
        handoff();
        if (tid == 0) {
            gemm_wgrad2<CP>(tmem + PL::DW_DIN, G(PL::HD), G(PL::LO), G(PL::X0), LPOS, LPOS, acc0);                  // dWd_in
            gemm_wgrad2<CP>(tmem + PL::B_D0, G(PL::HD), G(PL::LO), S(PL::ONES), 8, 8, acc0);                        // dbd_0
            gemm_bwd3<CP>(tmem + PL::ACC, G(PL::HD), G(PL::LO), 64, S(PL::W_HI + PL::W_DIN), S(PL::W_LO + PL::W_DIN),
                      LPOS, LPOS, 64);                                                                            // hash grads
        }
        sync_mma();
        dw_started = true;
        // X0 and LO are dead: the next tile's pair lands while this tile scatters
        prefetch_next();
        // the activation tiles are dead once the last MMAs completed: C2 holds the parked gradients
        if (!MLPB)
            scatter_from_tmem<F>(c, tmem, PL::ACC, a.grad_table, pn, 1.0f / DELTA_SCALE, a.hash_coef,
                                 reinterpret_cast<float*>(tC2), hit && valid);
        tc::fence_before_sync();
        tile_sync();
    }

    if constexpr (STAGED) cp_async_wait_all();      // a prefetch left by an early exit
    // ---- weight-gradient partials of this group: TMEM (M = 64 layout) -> global, unscaled
    if (backward && a.partials) {
        float* part = a.partials + ((size_t)blockIdx.x * PL::GROUPS + grp) * lo.total;
        const int lane = tid & 31;
        const int row = warp * 16 + lane;              // M = 64: rows 16w..16w+15 live in lanes 32w..32w+15
        const bool live = dw_started && !*abort_flag;
        auto dump = [&](uint32_t col, int ncols, int dst_off, bool transposed, int out_rows, int in_cols,
                        float extra = 1.0f) {
            for (int j = 0; j < ncols; j += 16) {
                float v[16];
                tc::tmem_ld16(tmem + tlane() + col + j, v);
                tc::tmem_wait_ld();
                if (lane < 16) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int n = j + i;
                        const float g = live ? v[i] * (extra / DELTA_SCALE) : 0.0f;
                        if (!transposed) { if (row < out_rows && n < in_cols) part[dst_off + row * in_cols + n] = g; }
                        else { if (n < out_rows && row < in_cols) part[dst_off + n * in_cols + row] = g; }
                    }
                }
            }
        };
        dump(PL::DW_DIN, LPOS, lo.off[P_WD_IN], false, 64, LPOS, 1.0f / INPUT_SCALE);
        if (ND >= 2) dump(PL::DW_D01, 64, lo.off[P_WD_01], false, 64, 64);
        dump(PL::DW_DOUT_T, 16, lo.off[P_WD_OUT], true, 16, 64);
        dump(PL::DW_CIN, 32, lo.off[P_WC_IN], false, 64, 32);
        dump(PL::DW_C01, 64, lo.off[P_WC_01], false, 64, 64);
        dump(PL::DW_COUT_T, 16, lo.off[P_WC_OUT], true, 3, 64);
        auto dump_bias = [&](uint32_t col, int dst_off) {
            float v[16];
            tc::tmem_ld16(tmem + tlane() + col, v);
            tc::tmem_wait_ld();
            if (lane < 16) part[dst_off + row] = live ? v[0] * (1.0f / DELTA_SCALE) : 0.0f;
        };
        // bias accumulators are 8 columns wide; a 16-column load spans the next one, which is fine
        dump_bias(PL::B_D0, lo.off[P_BD_0]);
        if (ND >= 2) dump_bias(PL::B_D1, lo.off[P_BD_1]);
        dump_bias(PL::B_C0, lo.off[P_BC_0]);
        dump_bias(PL::B_C1, lo.off[P_BC_1]);
        if (tid < 16) part[lo.off[P_BD_OUT] + tid] = live ? bgrad[tid] * (1.0f / DELTA_SCALE) : 0.0f;
        if (tid < 4) part[lo.off[P_BC_OUT] + tid] = (live && tid < 3) ? bgrad[16 + tid] * (1.0f / DELTA_SCALE) : 0.0f;
    }
    tc::fence_before_sync();
    __syncthreads();
    if (threadIdx.x < 32) tc::tmem_dealloc(tmem_base, PL::TMEM_COLS);
}




// ---------------------------------------------------------------- split step: stage kernels
// The tensor-core step as three launches: the sampler of every tile, the hash encoding of every
// (sample, level) straight into the fp16 operand tiles, then fused_step_tc_kernel<..., true>, which
// loads both and runs the MLPs, compositing, backward and scatter.  The first two carry no tensor
// memory and little shared memory, so many more warps per SM keep the gathers in flight than the
// fused kernel's two CTAs can.  Arithmetic is the fused kernel's, operation for operation.

// Sampler of 128-sample tiles (ray_sampler unchanged); writes (t, dt) per sample, the normalised
// position with a hit flag per sample, and (run-start bits, hit) per ray.
__global__ void __launch_bounds__(128) sample_stage_kernel(const StepArgs a, float4* __restrict__ pn_out,
                                                           float2* __restrict__ tdt_out, uint4* __restrict__ ray_out) {
    constexpr int RAY_BYTES = 128 * 6 * 4 + 128 * 16 + 128 * 16 + 8 * 2 * 4 + 8 * 16 * 4;
    __shared__ __align__(16) unsigned char sm[RAY_BYTES];
    const DevConfig& c = a.c;
    const int tid = threadIdx.x;
    float* rayb = reinterpret_cast<float*>(sm);
    float* sCand = rayb;
    float* sCdf = sCand + 128;
    float* sTs = sCdf + 128;
    float* sDTs = sTs + 128;
    float* sTr = sDTs + 128;
    uint32_t* sKey = reinterpret_cast<uint32_t*>(sTr + 128);
    float4* sSeg = reinterpret_cast<float4*>(sKey + 128);
    float2* sAffS = reinterpret_cast<float2*>(sSeg + 128);
    float2* sAffE = sAffS + 128;
    uint32_t* sChg = reinterpret_cast<uint32_t*>(sAffE + 128);
    float* sRay = reinterpret_cast<float*>(sChg + 16);
    const V3 bmin = v3(c.bmin[0], c.bmin[1], c.bmin[2]);
    const V3 bmax = v3(c.bmax[0], c.bmax[1], c.bmax[2]);
    const V3 bsize = vsub(bmax, bmin);
    const V3 inv_box = v3(fd(1.0f, bsize.x), fd(1.0f, bsize.y), fd(1.0f, bsize.z));
    const int spr = c.spr;
    const int rl = tid / spr, lid = tid - rl * spr, rbase = rl * spr;
    const int rays_per_tile = 128 / spr;
    const int n_tiles = (int)((a.n_rays + rays_per_tile - 1) / rays_per_tile);
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const uint32_t ray_idx = (uint32_t)tile * rays_per_tile + rl;
        const bool valid = ray_idx < a.n_rays;
        const uint32_t ray_id = a.ray_offset + ray_idx;
        float4 ro = make_float4(0.f, 0.f, 0.f, 0.f), rd = make_float4(0.f, 0.f, 1.f, 0.f);
        if (valid) { ro = a.rays[2 * ray_idx]; rd = a.rays[2 * ray_idx + 1]; }
        const V3 o = v3(ro.x, ro.y, ro.z), d = v3(rd.x, rd.y, rd.z);
        RayTile R{sCand, sCdf, sTs, sDTs, sTr, sKey, sSeg, sAffS, sAffE, sChg, sRay, tid, spr, rl, lid, rbase,
                  ray_idx, ray_id, valid, a.do_train != 0, false, o, d, bmin, bmax, bsize, inv_box, (float)c.G,
                  1.0f / (float)spr};
        bool hit;
        int idx_sel;
        ray_sampler(a, R, hit, idx_sel);
        if (valid) {
            const size_t s = (size_t)tile * 128 + tid;
            const float t_s = sTs[tid];
            tdt_out[s] = make_float2(t_s, sDTs[tid]);
            const V3 pn = normalize_pos(c, ray_point(o, d, t_s));
            pn_out[s] = make_float4(pn.x, pn.y, pn.z, hit ? 1.0f : 0.0f);
            if (lid == 0) ray_out[ray_idx] = make_uint4(sChg[rl * 2], sChg[rl * 2 + 1], hit ? 1u : 0u, 0u);
        }
        __syncthreads();
    }
}

// Hash encoding into the staged X0 operand tiles (x INPUT_SCALE, as the compensated fp16 pair: the
// hi tile, then the lo tile, TcPlan::X0_STAGE_BYTES per 128-row tile), the same accumulation order as
// encode_rows.  Work is level-major: block-sized chunks of 256 consecutive samples for one level,
// all chunks of level 0 first, so the whole grid gathers from one level's table at a time (an L2
// working set of one level), and the 32 lanes of a warp -- consecutive samples of one ray -- read
// the same corner slot, so samples that share a cell share the sector request.  Rows of samples
// that are not staged (past the last ray) or whose ray misses the box are zero.  The table is only
// read during this launch.
template <int F>
__global__ void __launch_bounds__(256) encode_stage_kernel(const DevConfig c, const float* __restrict__ table,
                                                           const float4* __restrict__ pn_in, int64_t n_valid,
                                                           int64_t n_rows, unsigned char* __restrict__ x0_out) {
    constexpr int LPOS = L * F;
    constexpr int HALF = 128 * LPOS * 2;   // bytes of one fp16 tile
    const int n_chunks = (int)((n_rows + 255) / 256);
    const int items = n_chunks * L;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int lvl = item / n_chunks;
        const int64_t i = (int64_t)(item - lvl * n_chunks) * 256 + threadIdx.x;
        if (i >= n_rows) continue;
        float v[F];
#pragma unroll
        for (int f = 0; f < F; ++f) v[f] = 0.0f;
        if (i < n_valid) {
            const float4 q = pn_in[i];
            if (q.w != 0.0f) {
                Corner8 k;
                level_corners<F>(c, v3(q.x, q.y, q.z), lvl, k);
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    if constexpr (F == 2) {
                        const float2 t = __ldg(reinterpret_cast<const float2*>(table + k.base[cc]));
                        v[0] = fmaf(k.w[cc], t.x, v[0]);
                        v[1] = fmaf(k.w[cc], t.y, v[1]);
                    } else {
                        const float4 t = __ldg(reinterpret_cast<const float4*>(table + k.base[cc]));
                        v[0] = fmaf(k.w[cc], t.x, v[0]);
                        v[1] = fmaf(k.w[cc], t.y, v[1]);
                        v[2] = fmaf(k.w[cc], t.z, v[2]);
                        v[3] = fmaf(k.w[cc], t.w, v[3]);
                    }
                }
            }
        }
        unsigned char* tile = x0_out + (i >> 7) * (int64_t)(2 * HALF);
        const int r = (int)(i & 127);
        uint32_t hi[F / 2], lo[F / 2];
#pragma unroll
        for (int f = 0; f < F; f += 2) {
            const float x0 = v[f] * INPUT_SCALE, x1 = v[f + 1] * INPUT_SCALE;
            hi[f / 2] = tc::pack_half2_sat(x0, x1);
            const float2 b = tc::unpack_half2(hi[f / 2]);
            lo[f / 2] = tc::pack_half2_sat(x0 - b.x, x1 - b.y);
        }
        const uint32_t off = tc::tile_off(r, lvl * F, LPOS);
        if constexpr (F == 2) {
            *reinterpret_cast<uint32_t*>(tile + off) = hi[0];
            *reinterpret_cast<uint32_t*>(tile + HALF + off) = lo[0];
        } else {
            *reinterpret_cast<uint2*>(tile + off) = make_uint2(hi[0], hi[1]);
            *reinterpret_cast<uint2*>(tile + HALF + off) = make_uint2(lo[0], lo[1]);
        }
    }
}

// Packs row-major fp16 rows [n][16F] into the staged operand tiles of the MLP kernels (x INPUT_SCALE,
// the encoder's convention; a power-of-two scale of an fp16 value is exact, so every lo tile is
// zero); one thread per (row, 8-column chunk).
template <int F>
__global__ void pack_x0_kernel(const __half* __restrict__ x, int64_t n, unsigned char* __restrict__ tiles) {
    constexpr int LPOS = L * F, CH = LPOS / 8, HALF = 128 * LPOS * 2;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * CH) return;
    const int64_t row = i / CH;
    const int c0 = (int)(i - row * CH) * 8;
    const uint4 u = *reinterpret_cast<const uint4*>(x + row * LPOS + c0);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        v[2 * k] = f.x * INPUT_SCALE;
        v[2 * k + 1] = f.y * INPUT_SCALE;
    }
    unsigned char* tile = tiles + (row / 128) * (2 * HALF);
    tc::st_chunk8_hilo(tile, tile + HALF, (int)(row % 128), c0, LPOS, v);
}

}  // namespace ffn
