/*
 * ref_abi.h -- TEST INFRASTRUCTURE ONLY: C entry points of the reference kernels compiled for
 * the CPU by ref_build.py (library oracle/_ref/libffnref_<variant>.so).  Each launcher runs the
 * reference kernel unmodified over its NDRange, one fiber per work-item (clemu.h).
 */
#ifndef FFN_REF_ABI_H
#define FFN_REF_ABI_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int32_t* W[9];        /* Wd_in Wd_01 Wd_12 Wd_out Wc_in Wc_01 Wc_12 Wc_23 Wc_out (float bits) */
    int32_t* b[9];        /* bd_0 bd_1 bd_2 bd_out bc_0 bc_1 bc_2 bc_3 bc_out                     */
    int32_t* table;
    const float* rays;    /* [n][8] float4 o, float4 d */
    const float* targets; /* [n][4] */
    float* deltas[9];     /* gl_dd1 gl_dd2 gl_dd3 gl_dd_out gl_dc1 gl_dc2 gl_dc3 gl_dc4 gl_dc_out  */
    float* acts[9];       /* gl_apos gl_ad1 gl_ad2 gl_ad3 gl_ac_in gl_ac1 gl_ac2 gl_ac3 gl_ac4     */
    float* out;           /* [n][4] */
    float lr;
    uint32_t num_rays, spr;
    int32_t do_train;
    float sh_mult;
    uint32_t* occ_in;
    uint32_t* occ_st;
    float box_min[3], box_max[3];
    int32_t G;
    float rho_min, rho_max, dt_min, dt_max, t_near, t_far;
    uint32_t seed;
    float occ_strength;
    int32_t n_threads;    /* OS threads running work-groups (1 = sequential ray order) */
    int32_t lockstep;     /* 1: all rays' work-groups advance barrier interval by barrier interval
                             together (every table read of the step precedes every table update,
                             as on a GPU that holds the whole batch); 0: one work-group at a time
                             per OS thread */
} ffnref_train_args;

typedef struct {
    int32_t* W[9];
    int32_t* b[9];
    float* mW[9];
    float* vW[9];
    float* mb[9];
    float* vb[9];
    float* deltas[9];
    float* acts[9];
    int32_t B, L, M;
    float lr_t, color_rel_lr, beta1, beta2, eps;
    int32_t n_threads;
} ffnref_wu_args;

void ffnref_train(const ffnref_train_args* a);
void ffnref_weight_update(const ffnref_wu_args* a);
void ffnref_decay(uint32_t* occ_in, uint32_t* occ_st, uint32_t n_words, uint32_t decay_q24,
                  uint32_t seed);
/* compile-time geometry of this variant */
void ffnref_info(int32_t* f_per_level, int32_t* n_density, int32_t* n_color, int32_t* log2_entries,
                 float* finest_res);

#ifdef __cplusplus
}
#endif
#endif
