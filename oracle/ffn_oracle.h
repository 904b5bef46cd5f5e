/*
 * ffn_oracle.h -- TEST INFRASTRUCTURE ONLY (the parity checker, never the product).
 *
 * CPU restatement of the reference's fused NeRF training step (MolSzabi/ffnerf-experimental):
 *   ffnerf_OG.cl              ffnerf_train_step          (sampler, hash encode, MLPs, compositing,
 *                                                          backward, occupancy proposals, hash SGD)
 *   weight_update.cl          update_ffnerf_oneWG        (per-layer dW/db reduction + Adam)
 *   decay_occ_grid_in-st.cl   occ_nibble_decay_write_both_q24
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load this library.
 * Its results are pinned against the reference kernels compiled from their own sources
 * (oracle/ref_build.py builds them into oracle/_ref/) and against golden fixtures generated
 * from the reference's Python host module (tests/golden/make_golden.py).
 */
#ifndef FFN_ORACLE_H
#define FFN_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_N_LEVELS 16
#define ORC_N_PARAMS 18   /* Wd_in Wd_01 Wd_12 Wd_out Wc_in Wc_01 Wc_12 Wc_23 Wc_out
                             bd_0 bd_1 bd_2 bd_out bc_0 bc_1 bc_2 bc_3 bc_out */

typedef struct {
    int32_t F;            /* features per level (reference F_PER_LEVEL)            */
    int32_t ND;           /* density hidden layers 1..3 (reference ND)              */
    int32_t NC;           /* color hidden layers 1..4 (reference NC)                */
    int32_t spr;          /* samples per ray = work-group size, power of two <= 64  */
    int32_t G;            /* occupancy grid side                                    */
    int32_t background;   /* 0 black, 1 white, 2 random per ray (BACKGROUND_COLOR)  */
    int32_t math_mode;    /* 0: own exp/pow (device-identical), 1: C libm          */
    int32_t table_mode;   /* 0: deferred (reads see step-start table, grads summed),
                             1: sequential (one legal Hogwild schedule: rays in order,
                                updates applied immediately)                        */
    int32_t tilek;        /* weight-update K chunk (reference TILEK)                */
    int32_t transfer_fmt; /* staged activations / deltas read by the weight update:
                             32 fp32, 16 fp16, 8 the reference's e4m3-like fp8     */
    uint32_t level_log2[ORC_N_LEVELS];   /* log2 entries per level                 */
    uint32_t level_offset[ORC_N_LEVELS]; /* first entry of each level              */
    int32_t  level_res[ORC_N_LEVELS];    /* grid resolution per level              */
    float    hash_lr_scale[ORC_N_LEVELS];/* 2^(-0.1*lvl)                           */
    float box_min[4], box_max[4];
    float rho_min, rho_max, dt_min, dt_max, t_near, t_far;
    float pad1, pad2;
} orc_config;

typedef struct {
    float lr_f;           /* hash SGD learning rate (kernel arg `lr`)               */
    float sh_mult;        /* SH multiplier                                          */
    float occ_strength;   /* occupancy update strength                              */
    uint32_t rng_seed;    /* per-step seed (kernel arg rng_seed_base)               */
    int32_t do_train;
    uint32_t ray_offset;  /* global id of the first ray (data-parallel shards)      */
} orc_step;

/* Optional per-sample / per-ray outputs (any field may be NULL). */
typedef struct {
    float*    t;          /* [n*spr] sample time                                     */
    float*    dt;         /* [n*spr] sample dt                                       */
    int32_t*  idx;        /* [n*spr] resampled candidate index                       */
    uint32_t* flags;      /* [n*2]   run-start bitset (64 bits per ray)              */
    float*    sigma;      /* [n*spr]                                                 */
    float*    rgb;        /* [n*spr*3]                                               */
    float*    trans;      /* [n*spr] transmittance before the sample                 */
    float*    dsigma;     /* [n*spr] dL/dsigma                                       */
    float*    enc;        /* [n*spr*L*F] hash encoding                               */
} orc_debug;

int32_t orc_param_layout(int32_t F, int32_t ND, int32_t NC, int32_t* offsets, int32_t* sizes);

/* Forward + backward over n_rays rays.  table_grad (deferred mode) receives sum(g*w) per
 * table element; mlp_grad receives dW/db (sums over samples) in the param-blob layout.
 * bypass (optional, [n*spr*4] sigma,r,g,b) replaces the MLP output: sampler, compositing and
 * occupancy proposals run, the backward does not. */
int32_t orc_forward_backward(const orc_config* cfg, const orc_step* st, const float* params,
                             float* table, const uint32_t* occ_in, uint32_t* occ_st,
                             const float* rays, const float* targets, float* out, int32_t n_rays,
                             float* table_grad, float* mlp_grad, const orc_debug* dbg,
                             const float* bypass);

void orc_adam(float* p, const float* g, float* m, float* v, int64_t n,
              float lr_t, float b1, float b2, float eps);
void orc_mlp_adam(const orc_config* cfg, float* params, const float* grad, float* m, float* v,
                  float lr_t, float color_rel_lr, float b1, float b2, float eps);
void orc_table_apply(const orc_config* cfg, float* table, const float* table_grad, float lr_f);
/* Opt-in table Adam: orc_adam per level with step lr_t * 2^(-0.1 l). */
void orc_table_adam(const orc_config* cfg, float* table, const float* table_grad, float* m, float* v,
                    float lr_t, float b1, float b2, float eps);
void orc_decay(uint32_t* occ_in, uint32_t* occ_st, uint32_t n_words, uint32_t decay_q24,
               uint32_t seed);

/* Hash-grid microbench restatement: points are normalized coordinates in [0,1]^3. */
void orc_hash_fwd(const orc_config* cfg, const float* table, const float* pts, int64_t n,
                  float* enc);
void orc_hash_bwd(const orc_config* cfg, const float* pts, const float* denc, int64_t n,
                  float* table_grad);

float orc_expf(float x);
float orc_powr(float x, float y);
uint32_t orc_hash_u32(uint32_t x);

#ifdef __cplusplus
}
#endif
#endif
