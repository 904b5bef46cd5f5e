/*
 * ffnerf.h -- C ABI of the B200 fused NeRF training step (libffnerf.so).
 *
 * Drop-in for the device side of the reference's PyOpenCL path (MolSzabi/ffnerf-experimental):
 * the host module ffnerf_tools.py binds these entry points with ctypes in place of the three
 * OpenCL programs it builds and launches.  Plain pointers and sizes only; device pointers are
 * CUDA global-memory addresses on the context's device, `stream` is a cudaStream_t (NULL = the
 * legacy default stream).  Every function returns 0 on success or a negative FFN_E* code; the
 * message of the last failure is available from ffn_last_error().
 *
 * Reference interfaces replaced (paths relative to the reference repository root):
 *   ffn_create / ffn_destroy      Nerf.from_kernels + Nerf.setup_buffers (ffnerf_tools.py:583-671,
 *                                 926-977): program build, parameter and scratch allocation
 *   ffn_buffer                    Nerf.buf / Nerf.tmp device buffers (ffnerf_tools.py:939-977),
 *                                 used for checkpoint I/O (Nerf.save/load_latest, :989-1189)
 *   ffn_forward_backward          enqueue of ffnerf_train_step with do_train=1
 *                                 (ffnerf_tools.py:1410-1445; kernel ffnerf_OG.cl:838-2174)
 *   ffn_apply_updates             enqueue of update_ffnerf_oneWG (ffnerf_tools.py:1478-1518;
 *                                 kernel weight_update.cl:346-577) plus the hash-table SGD step
 *                                 that the reference applies inside ffnerf_train_step
 *                                 (ffnerf_OG.cl:2090-2173)
 *   ffn_train_step                Nerf.step(do_train=True) device work (ffnerf_tools.py:1357-1544)
 *   ffn_render                    Nerf.step(do_train=False) (ffnerf_tools.py:1357-1544 with
 *                                 do_train=0; kernel path ffnerf_OG.cl:1115-1134,1848)
 *   ffn_occ_maintenance           enqueue of occ_nibble_decay_write_both_q24
 *                                 (ffnerf_tools.py:1452-1476; decay_occ_grid_in-st.cl:13-113)
 *   ffn_grad_buffer,              (no reference counterpart: the reference has one device) the
 *   ffn_occ_st_bytes,             gradient buffer and the occupancy proposals merged across
 *   ffn_dp_*                      data-parallel ranks, and the fused NVLink exchange
 */
#ifndef FFNERF_H
#define FFNERF_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FFN_N_LEVELS 16
#define FFN_ABI_VERSION 6   /* 2: ffn_step_scalars.flags; 3: batch/exchange entry points;
                                   4: fp16-table hash and MLP microbenchmark entry points;
                                   5: ffn_dp_set_wait_limit, ffn_config.transfer_fmt,
                                      ffn_probe_random_access; 6: ffn_mlp_bench_f16 */

enum {
    FFN_OK = 0,
    FFN_E_CONFIG = -1,    /* invalid configuration or argument (reference: ValueError) */
    FFN_E_CUDA = -2,      /* CUDA runtime / launch failure                             */
    FFN_E_CAPACITY = -3,  /* more rays than the context was created for                */
    FFN_E_NAME = -4,      /* unknown buffer name                                        */
    FFN_E_STATE = -5      /* call order violated (e.g. apply without gradients)         */
};

/* Buffer ids for ffn_buffer(). */
enum {
    FFN_BUF_PARAMS = 0,     /* float32 MLP parameter blob (active layers, canonical order)      */
    FFN_BUF_ADAM_M = 1,     /* float32, same layout                                             */
    FFN_BUF_ADAM_V = 2,     /* float32, same layout                                             */
    FFN_BUF_TABLE = 3,      /* float32 [table_entries * F], index (level_offset[l]+entry)*F+f   */
    FFN_BUF_OCC_IN = 4,     /* uint32 [G^3], 8 nibbles per cell                                 */
    FFN_BUF_OCC_ST = 5,     /* uint32 [G^3]                                                     */
    FFN_BUF_GRADS = 6,      /* float32 [table_entries * F + params]: table grads, then MLP grads */
    FFN_BUF_TABLE_M = 7,    /* float32 table Adam state (table_optimizer = 1 only)              */
    FFN_BUF_TABLE_V = 8
};

typedef struct ffn_config {
    int32_t F;               /* features per hash level: 2 or 4                         */
    int32_t ND;              /* density hidden layers 1..3                              */
    int32_t NC;              /* color hidden layers 1..4                                */
    int32_t spr;             /* samples per ray: 16, 32 or 64                           */
    int32_t G;               /* occupancy grid side                                     */
    int32_t background;      /* 0 black, 1 white, 2 random per ray                      */
    int32_t table_optimizer; /* 0: reference SGD (hash lr roll-off), 1: Adam            */
    int32_t max_rays;        /* capacity: largest n_rays of any call                    */
    uint32_t level_log2[FFN_N_LEVELS];
    uint32_t level_offset[FFN_N_LEVELS];
    int32_t level_res[FFN_N_LEVELS];
    float hash_lr_scale[FFN_N_LEVELS];
    float box_min[4], box_max[4];
    float rho_min, rho_max, dt_min, dt_max, t_near, t_far;
    float adam_beta1, adam_beta2, adam_eps;   /* MLP (and table) Adam */
    float table_adam_eps;
    int32_t mlp_precision;   /* 0: fp32 on the CUDA cores (reference-exact arithmetic),
                                1: fp16 operands / fp32 accumulation on the tensor cores (tcgen05) */
    int32_t transfer_fmt;    /* the reference's TRANSFER_FMT (ffnerf_OG.cl:85-156): the format in which
                                the weight update reads the step's activations and deltas --
                                32 (or 0) fp32, 16 fp16 (saturating, round to nearest even), 8 the
                                reference's e4m3-like fp8 (saturating at +-15.5).  16 and 8 need
                                mlp_precision 0 (the tensor-core MLP keeps its own operand formats). */
} ffn_config;

typedef struct ffn_step_scalars {
    float lr_f;            /* base learning rate of the step (hash SGD lr, kernel arg `lr`) */
    float lr_t;            /* bias-corrected Adam step size for the MLP                     */
    float sh_mult;         /* spherical-harmonics multiplier                                */
    float color_rel_lr;    /* color-MLP learning-rate factor                                */
    float occ_strength;    /* occupancy update strength (0 disables proposals)              */
    uint32_t rng_u32;      /* per-step seed                                                 */
    uint32_t ray_offset;   /* global index of the first ray (data-parallel shards)          */
    float table_lr_t;      /* bias-corrected Adam step size for the table (optimizer 1)     */
    uint32_t spr;          /* samples per ray of this batch (16/32/64); 0 = ffn_config.spr  */
    uint32_t flags;        /* FFN_STEP_* bits                                               */
} ffn_step_scalars;

/* ffn_step_scalars.flags: apply the hash-table SGD step inside ffn_forward_backward, as atomic adds
 * of -lr_f * hash_lr_scale[l] * 0.5 * g * w into the table while other rays read it -- the
 * reference's own (Hogwild) semantics.  The table part of FFN_BUF_GRADS stays zero and
 * ffn_apply_updates skips the table pass.  Needs table_optimizer = 0; not for data-parallel runs,
 * whose table gradients must be all-reduced first. */
#define FFN_STEP_TABLE_IMMEDIATE 1u
/* ffn_step_scalars.flags: the table SGD step of this step was applied by ffn_dp_reduce_apply;
 * ffn_apply_updates skips its table pass (MLP Adam only). */
#define FFN_STEP_TABLE_APPLIED 2u

typedef struct ffn_ctx ffn_ctx;

int ffn_abi_version(void);
const char* ffn_last_error(const ffn_ctx* ctx);   /* ctx may be NULL (creation errors) */

int ffn_create(const ffn_config* cfg, int device, ffn_ctx** out);
int ffn_destroy(ffn_ctx* ctx);

/* Device pointer and size in bytes of one context buffer (FFN_BUF_*). */
int ffn_buffer(ffn_ctx* ctx, int id, void** dev_ptr, size_t* bytes);
/* Offset (floats) and size of each active parameter in FFN_BUF_PARAMS, canonical order
 * Wd_in Wd_01 Wd_12 Wd_out Wc_in Wc_01 Wc_12 Wc_23 Wc_out bd_0 bd_1 bd_2 bd_out bc_0 bc_1 bc_2
 * bc_3 bc_out; returns the blob length in floats. */
int ffn_param_layout(const ffn_config* cfg, int32_t* offsets18, int32_t* sizes18);

/* Forward + backward for n_rays rays (rays: [n][8] float o.xyzw d.xyzw, targets/out: [n][4]).
 * Accumulates into FFN_BUF_GRADS, proposes occupancy into FFN_BUF_OCC_ST, writes out. */
int ffn_forward_backward(ffn_ctx* ctx, const void* rays, const void* targets, void* out,
                         uint32_t n_rays, const ffn_step_scalars* s, void* stream);
/* Applies the accumulated gradients (table SGD or Adam, MLP Adam) and clears them. */
int ffn_apply_updates(ffn_ctx* ctx, const ffn_step_scalars* s, void* stream);
/* ffn_forward_backward + ffn_apply_updates. */
int ffn_train_step(ffn_ctx* ctx, const void* rays, const void* targets, void* out,
                   uint32_t n_rays, const ffn_step_scalars* s, void* stream);
/* Forward only (do_train = 0): occupancy-guided sampling with the inference rule, black
 * background, no gradients. */
int ffn_render(ffn_ctx* ctx, const void* rays, void* out, uint32_t n_rays,
               const ffn_step_scalars* s, void* stream);
/* Occupancy maintenance: decay unchanged nibbles, merge proposals, write both grids. */
int ffn_occ_maintenance(ffn_ctx* ctx, uint32_t decay_q24, uint32_t seed, void* stream);
/* The contiguous gradient buffer (table grads then MLP grads) for a data-parallel all-reduce. */
int ffn_grad_buffer(ffn_ctx* ctx, void** dev_ptr, size_t* n_floats);
/* Occupancy proposals as one byte per nibble ([G^3 * 8] uint8, value = nibble) so that ranks can
 * merge them with a byte-wise MAX all-reduce: to_bytes = 1 expands FFN_BUF_OCC_ST into bytes,
 * to_bytes = 0 packs bytes back into FFN_BUF_OCC_ST.  (No reference counterpart: one device.) */
int ffn_occ_st_bytes(ffn_ctx* ctx, uint8_t* bytes, int to_bytes, void* stream);

/* Diagnostics of one forward pass (any pointer may be NULL): per sample t, dt, resampled
 * candidate index, sigma, rgb[3], transmittance; per ray the 64-bit run-start set.  When
 * bypass is non-NULL ([n*spr][4] sigma,r,g,b) it replaces the MLP output, and sampling,
 * compositing and occupancy proposals run on it (do_train = 1 rules, no backward). */
int ffn_probe(ffn_ctx* ctx, const void* rays, const void* targets, void* out, uint32_t n_rays,
              const ffn_step_scalars* s, const void* bypass, float* t, float* dt, int32_t* idx,
              uint32_t* flags, float* sigma, float* rgb, float* trans, void* stream);

/* Hash-grid encoding on its own (microbenchmark of the encode/scatter kernels): points are
 * normalized coordinates [n][3] in [0,1]^3; enc is [n][16*F]; the backward scatter-adds
 * denc [n][16*F] weighted by the trilinear weights into FFN_BUF_GRADS (table part). */
int ffn_hash_encode(ffn_ctx* ctx, const float* pts, float* enc, int64_t n, void* stream);
int ffn_hash_encode_bwd(ffn_ctx* ctx, const float* pts, const float* denc, int64_t n,
                        void* stream);
/* The same two operations on an fp16 table owned by the caller (table16 / grad16: the context's
 * table layout, FFN_BUF_TABLE's element count, as IEEE half; enc16 is [n][16*F] half; denc stays
 * fp32).  The fp16-table case of the hash microbenchmark; no reference counterpart (the
 * reference's table is fp32).  Gathers accumulate in fp32; the scatter adds packed half2. */
int ffn_hash_encode_f16(ffn_ctx* ctx, const void* table16, const float* pts, void* enc16, int64_t n,
                        void* stream);
int ffn_hash_encode_bwd_f16(ffn_ctx* ctx, void* grad16, const float* pts, const float* denc, int64_t n,
                            void* stream);
/* The MLP microbenchmark (no reference counterpart; the MLP half of the "fused MLP + Adam"
 * microbenchmark).  ffn_pack_x0 packs row-major fp16 inputs x16 [n][16*F] into the tensor-core
 * operand tiles (tiles: n*16*F*4 bytes -- per 128 rows an fp16 hi tile and an fp16 lo tile -- n a
 * multiple of 128).  ffn_mlp_bench runs the density and
 * colour MLPs forward and backward over those inputs on the tensor cores (tensor-core MLP, F=2,
 * ND=1 contexts), with the view direction fixed at (0.36, 0.48, 0.8), sh multiplier 1 and the loss
 * sum_k 0.5 (rgb_k - 0.5)^2 per sample, and adds the summed MLP weight and bias gradients to the MLP
 * part of FFN_BUF_GRADS.  The table and its gradients are not touched. */
int ffn_pack_x0(ffn_ctx* ctx, const void* x16, void* tiles, int64_t n, void* stream);
int ffn_mlp_bench(ffn_ctx* ctx, const void* tiles, int64_t n, void* stream);
/* The same with plain fp16 operands: one MMA per product from the hi tiles, no lo tiles stored
 * (the training step forms every product from compensated fp16 pairs, as ffn_mlp_bench does). */
int ffn_mlp_bench_f16(ffn_ctx* ctx, const void* tiles, int64_t n, void* stream);
/* Ceiling probe (no reference counterpart): n_ops fully random 8-byte accesses (mode 0: float2
 * loads through the read-only path, as the hash encoders do; mode 1: red.global.add.v2.f32
 * reductions, as the gradient scatter does; both adding a negligible value) over the largest
 * power-of-two number of 8-byte entries in the caller's device buffer buf (bytes), eight
 * independent accesses in flight per thread.  Timed by the caller, it gives the achievable
 * random-access rate that bounds the encode and scatter kernels at that table size. */
int ffn_probe_random_access(void* buf, size_t bytes, int mode, uint64_t n_ops, uint32_t seed, void* stream);
/* Kernels this context has launched so far (all entry points; no reference counterpart). */
uint64_t ffn_kernel_launches(const ffn_ctx* ctx);
/* Reads and clears the context's device status word (waits for the device): 0 when every kernel
 * since the last call completed normally; bit 0 = a ray colour or an MLP gradient was not finite
 * (the model diverged: NaN/Inf weights); bit 2 = a tensor-core wait exceeded its bound; bit 3 = a cross-rank wait of the
 * data-parallel exchange ran out. */
int ffn_status(ffn_ctx* ctx, uint32_t* status);

/* Data-parallel exchange over NVLink peer memory (no reference counterpart: the reference runs on
 * one device).  One process per GPU, every rank with an identical context.  ffn_dp_ipc_handles
 * writes 3 CUDA IPC handles (3 x 64 bytes: gradient buffer, table, flag words) that the caller
 * exchanges between ranks (e.g. an all-gather), then ffn_dp_attach maps every peer's buffers
 * (handles: world x 3 x 64 bytes, rank order).  After ffn_forward_backward (deferred table update),
 * ffn_dp_reduce_apply sums every rank's gradients, applies the table SGD step to this rank's shard
 * and writes it into every rank's table, leaves the summed MLP gradient in every rank's gradient
 * buffer and clears the table gradients -- the all-reduce and the table pass in one kernel.  Then
 * ffn_apply_updates with FFN_STEP_TABLE_APPLIED runs the MLP Adam.  Every rank must call it in
 * the same steps; its cross-rank waits are bounded (status bit 8 on a timeout).  SGD table only. */
int ffn_dp_ipc_handles(ffn_ctx* ctx, void* handles_out);
int ffn_dp_attach(ffn_ctx* ctx, int rank, int world, const void* handles);
int ffn_dp_reduce_apply(ffn_ctx* ctx, const ffn_step_scalars* s, void* stream);
/* Polls (about 1 us each) that each cross-rank wait of ffn_dp_reduce_apply makes before it gives up
 * and sets status bit 8; default 2^24 (about 16 s).  Call after ffn_dp_ipc_handles.  No reference
 * counterpart (the reference has no multi-device path); it lets a caller bound how long a rank
 * waits for a peer that stopped calling the exchange. */
int ffn_dp_set_wait_limit(ffn_ctx* ctx, uint32_t polls);
/* NVSwitch (NVLS) variant of the exchange.  ffn_bind_external moves the context's table or
 * gradient buffer (FFN_BUF_TABLE / FFN_BUF_GRADS) into caller-owned device memory of at least the
 * same size -- here, memory bound to a multicast object on every rank -- copying the contents; the
 * caller keeps it alive until ffn_destroy.  Bind both before ffn_dp_attach (which then maps only
 * the peers' flag words), then ffn_dp_attach_multicast gives the two multicast addresses:
 * ffn_dp_reduce_apply then reads the cross-rank gradient sum with multimem.ld_reduce and writes
 * the updated table shard with multimem.st, moving each shard once through the switch. */
int ffn_bind_external(ffn_ctx* ctx, int buffer_id, void* dev_ptr, size_t bytes);
int ffn_dp_attach_multicast(ffn_ctx* ctx, void* mc_grads, void* mc_table);

/* Training batches on the device (replace the host batch producer, run_ffnerf_OG.py:585-685, and
 * rays_targets_from_indices, ffnerf_tools.py:175-234).  images: [n_img][H][W][channels] uint8
 * (img_f32 = 0) or float32 in [0,1]; weights: [n_img][H][W] uint8 pixel weights (1..255); c2w:
 * [n_img][4][4] camera-to-world; K: [3][3] (k_per_image = 0) or [n_img][3][3], or NULL for the
 * reference's fallback focal.  Each ray takes a uniform image and, with probability uniform_frac,
 * a uniform pixel, else a pixel by rejection against the weight map (at most max_tries proposals);
 * rays [n][2] float4 (o, d), targets [n] float4, and optionally the drawn (im, x, y).  Rays depend
 * only on seed and the inputs (counter-based RNG per ray). */
int ffn_batch_generate(const void* images, int img_f32, int channels, const uint8_t* weights, const float* c2w,
                       const float* K, int k_per_image, int n_img, int W, int H, uint32_t n_rays,
                       float uniform_frac, uint32_t seed, uint32_t max_tries, void* rays, void* targets,
                       int32_t* im, int32_t* x, int32_t* y, void* stream);
/* Rays of a view for pixels first .. first + n_rays - 1 (row-major, x fastest), written to device
 * memory [n_rays][2] float4: the renderer's rays_from_rt_indices (ffnerf_tools.py:237-272).  c2w
 * (4x4 row-major) and K (3x3, or NULL for the fallback focal) are HOST arrays. */
int ffn_camera_rays(const float* c2w, const float* K, int W, int H, uint32_t first, uint32_t n_rays, void* rays,
                    void* stream);
/* Per-ray colour error sqrt(mean_rgb((out - targets)^2)) clipped to [0, 1] (run_ffnerf_OG.py:1383)
 * into err (may be NULL), and, when sum_sq is given, adds the batch's sum S of squared colour
 * differences to *sum_sq (a device double): mse = S / (3 n), l2 = sqrt(S / n)
 * (run_ffnerf_OG.py:1389-1391). */
int ffn_batch_errors(const void* out, const void* targets, uint32_t n_rays, float* err, double* sum_sq,
                     void* stream);
/* Weight-map EMA from per-ray errors and their median (a device float), as the reference's
 * _update_weights_u8 (run_ffnerf_OG.py:459-490) with the RGB-threshold foreground of
 * make_fg_mask_from_rgb (run_ffnerf_OG.py:402-421, dilate = 0). */
int ffn_batch_feedback(uint8_t* weights, const void* images, int img_f32, int channels, int W, int H,
                       const int32_t* im, const int32_t* x, const int32_t* y, const float* err,
                       uint32_t n_rays, const float* median, double ema, int bg_cap, int fg_tau, void* stream);

/* Plain Adam over n float32 parameters (vectorised; beta/eps as given). */
int ffn_adam(float* p, const float* g, float* m, float* v, int64_t n, float lr_t, float beta1,
             float beta2, float eps, void* stream);

/* ffn_forward_backward for callers that cannot allocate device memory.  No reference
 * counterpart: the reference allocates its buffers through PyOpenCL.  It serves code that runs
 * inside another runtime's device-memory budget (an engine or serving process that owns every
 * allocation through its own pool), where the library may not call cudaMalloc: such a caller
 * holds the model's buffers itself and passes them in, with no ffn_ctx.
 *
 * Inputs: cfg (as for ffn_create), params (FFN_BUF_PARAMS layout), occ_in, rays, targets; in/out:
 * table (read; also updated when s->flags has FFN_STEP_TABLE_IMMEDIATE), occ_st (occupancy
 * proposals when s->occ_strength > 0); outputs: out [n][4], grads (FFN_BUF_GRADS layout,
 * table_entries*F + params floats, overwritten: cleared, then accumulated), status (device int,
 * ffn_status bits; may be NULL).  The device is the caller's current device.
 *
 * Allocates nothing: no cudaMalloc, cudaFree or allocating library call.  The per-CTA
 * weight-gradient partial sums live in a static device array of FFN_NOALLOC_SCRATCH_BYTES that
 * every GPU which loads the library holds until the process exits; a call whose partials
 * (CTAs x params floats, plus 256 bytes) exceed it fails with FFN_E_CAPACITY.  The first call on
 * each device also resolves that array's address and sets the kernels' shared-memory limits;
 * make that first call before any stream capture.  All calls on a device share the array, so
 * calls that overlap on the GPU (other streams, other threads) race and must be serialised by
 * the caller. */
#define FFN_NOALLOC_SCRATCH_BYTES (24u << 20)
int ffn_forward_backward_noalloc(const ffn_config* cfg, const float* params, float* table,
                                 const uint32_t* occ_in, uint32_t* occ_st, const void* rays,
                                 const void* targets, void* out, float* grads, int* status,
                                 uint32_t n_rays, const ffn_step_scalars* s, void* stream);

#ifdef __cplusplus
}
#endif
#endif
