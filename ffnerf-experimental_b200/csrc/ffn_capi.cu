// ffn_capi.cu -- the extern "C" entry points declared in include/ffnerf.h.
//
// One ffn_ctx per device and model: it owns the parameter blob, the Adam moments, the hash
// table, both occupancy grids, the gradient buffer and the per-CTA weight-gradient partials.
// Callers own rays / targets / outputs (device pointers).  Every entry point is stream-ordered
// and returns a status code; nothing synchronises the device except ffn_create/ffn_destroy.
#include <cstdio>
#include <cstring>
#include <string>

#include "ffn_common.cuh"
#include "ffn_step.cu"
#include "ffn_step_tc.cu"
#include "ffn_dp.cu"
#include "ffn_batch.cu"

using namespace ffn;

struct ffn_ctx {
    ffn_config cfg;
    int device = 0;
    DevConfig dc{};
    ParamLayout lo{};
    size_t table_floats = 0;
    int Pw = 0;
    float* params = nullptr;
    float* adam_m = nullptr;
    float* adam_v = nullptr;
    float* table = nullptr;
    float* table_m = nullptr;
    float* table_v = nullptr;
    uint32_t* occ_in = nullptr;
    uint32_t* occ_st = nullptr;
    float* grads = nullptr;      // [table_floats + Pw]
    float* partials = nullptr;   // [max_grid * groups * Pw]
    int* status = nullptr;       // device status word
    int max_grid = 0;
    int rows = 0;                // samples per tile
    int threads = 0;             // threads per block of the fused kernel (tiles side by side x rows)
    int groups = 1;              // tiles side by side per block (one weight-gradient partial row each)
    int ctas_per_sm = 1;
    size_t smem = 0;
    void (*kernel)(StepArgs) = nullptr;
    // split tensor-core step (mlp_precision = 1): stage kernels and their buffers, sized for
    // STAGE_SAMPLES samples per launch group
    void (*kernel_staged)(StepArgs) = nullptr;
    void (*encoder)(DevConfig, const float*, const float4*, int64_t, int64_t, unsigned char*) = nullptr;
    unsigned char* x0_stage = nullptr;
    float2* tdt_stage = nullptr;
    float4* pn_stage = nullptr;
    uint4* ray_stage = nullptr;
    uint64_t launches = 0;         // kernels this context has launched (ffn_kernel_launches)
    DpState* dp = nullptr;       // data-parallel peer mappings (ffn_dp_attach)
    bool ext_table = false;      // table / gradient buffer bound from outside (ffn_bind_external)
    bool ext_grads = false;
    std::string err;
};

namespace {

thread_local std::string g_create_err;

constexpr int64_t STAGE_SAMPLES = 1 << 20;   // samples per group of the split tensor-core step

int fail(ffn_ctx* ctx, int code, const std::string& msg) {
    if (ctx) ctx->err = msg; else g_create_err = msg;
    return code;
}

int cuda_fail(ffn_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, FFN_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

template <int F, int ND, int NC, int ROWS>
void bind_kernel(ffn_ctx* c) {
    if (c->cfg.mlp_precision == 1) {
        using PL = TcPlan<F, ND>;
        c->kernel = fused_step_tc_kernel<F, ND>;
        c->kernel_staged = fused_step_tc_kernel<F, ND, true>;
        c->encoder = encode_stage_kernel<F>;
        c->rows = PL::ROWS;
        c->threads = PL::THREADS;
        c->groups = PL::GROUPS;
        c->smem = PL::BYTES;
        c->ctas_per_sm = PL::CTAS_PER_SM;
        return;
    }
    c->kernel = fused_step_kernel<F, ND, NC, ROWS>;
    c->kernel_staged = fused_step_kernel<F, ND, NC, ROWS, true>;
    c->encoder = encode_stage_f32_kernel<F>;
    c->rows = ROWS;
    c->threads = ROWS;
    c->groups = 1;
    c->smem = (size_t)Smem<F, ND, NC, ROWS>::floats(c->Pw) * sizeof(float);
    c->ctas_per_sm = 1;
}

// The (F, ND, NC) combinations compiled into this library; the tile height is the largest of
// 128 / 64 samples whose shared-memory footprint fits in one SM.
bool select_kernel(ffn_ctx* c) {
    const ffn_config& g = c->cfg;
    if (g.NC != 2) return false;
    if (g.F == 2 && g.ND == 1) { bind_kernel<2, 1, 2, 128>(c); return true; }
    if (g.F == 4 && g.ND == 1) { bind_kernel<4, 1, 2, 128>(c); return true; }
    if (g.F == 2 && g.ND == 2) { bind_kernel<2, 2, 2, 64>(c); return true; }
    if (g.F == 4 && g.ND == 2) { bind_kernel<4, 2, 2, 64>(c); return true; }
    return false;
}

int check_config(const ffn_config* g, std::string* why) {
    if (g->F != 2 && g->F != 4) { *why = "F (features per level) must be 2 or 4"; return FFN_E_CONFIG; }
    if (g->ND < 1 || g->ND > 3 || g->NC < 1 || g->NC > 4) { *why = "ND must be 1..3 and NC 1..4"; return FFN_E_CONFIG; }
    if (g->spr != 16 && g->spr != 32 && g->spr != 64) {
        *why = "samples_per_ray must be 16, 32 or 64 (power of two, <= S_MAX=64)";
        return FFN_E_CONFIG;
    }
    if (g->G < 1 || g->G > 1024) { *why = "occupancy grid side must be 1..1024"; return FFN_E_CONFIG; }
    if (g->background < 0 || g->background > 2) { *why = "background must be 0 (black), 1 (white) or 2 (random)"; return FFN_E_CONFIG; }
    if (g->mlp_precision != 0 && g->mlp_precision != 1) { *why = "mlp_precision must be 0 (fp32) or 1 (fp16 tensor cores)"; return FFN_E_CONFIG; }
    if (g->transfer_fmt != 0 && g->transfer_fmt != 32 && g->transfer_fmt != 16 && g->transfer_fmt != 8) {
        *why = "transfer_fmt must be 32 (fp32), 16 (fp16) or 8 (fp8)";
        return FFN_E_CONFIG;
    }
    if (g->mlp_precision == 1 && g->transfer_fmt != 0 && g->transfer_fmt != 32) {
        *why = "the fp16 / fp8 transfer formats are reproduced by the fp32 MLP (mlp_precision 0) only";
        return FFN_E_CONFIG;
    }
    uint64_t expect = 0;
    for (int l = 0; l < FFN_N_LEVELS; ++l) {
        if (g->level_log2[l] < 1 || g->level_log2[l] > 24) { *why = "per-level table size must be 2^1..2^24"; return FFN_E_CONFIG; }
        if (g->level_offset[l] != expect) { *why = "level offsets must be the running sum of the level sizes"; return FFN_E_CONFIG; }
        if (g->level_res[l] < 2 || g->level_res[l] > (1 << 20)) { *why = "level resolution must be 2..2^20"; return FFN_E_CONFIG; }
        expect += 1ull << g->level_log2[l];
    }
    if (expect * (uint64_t)g->F >= (1ull << 32)) { *why = "hash table too large (>= 2^32 floats)"; return FFN_E_CONFIG; }
    for (int i = 0; i < 3; ++i)
        if (!(g->box_max[i] > g->box_min[i])) { *why = "box_max must exceed box_min"; return FFN_E_CONFIG; }
    return FFN_OK;
}

void fill_dev_config(ffn_ctx* c) {
    DevConfig& d = c->dc;
    const ffn_config& g = c->cfg;
    d.F = g.F; d.ND = g.ND; d.NC = g.NC; d.spr = g.spr; d.G = g.G; d.background = g.background;
    for (int l = 0; l < L; ++l) {
        d.level_log2[l] = g.level_log2[l];
        d.level_offset[l] = g.level_offset[l];
        d.level_res[l] = g.level_res[l];
        d.hash_lr_scale[l] = g.hash_lr_scale[l];
    }
    for (int i = 0; i < 3; ++i) { d.bmin[i] = g.box_min[i]; d.bmax[i] = g.box_max[i]; }
    d.rho_min = g.rho_min; d.rho_max = g.rho_max; d.dt_min = g.dt_min; d.dt_max = g.dt_max;
    d.t_near = g.t_near; d.t_far = g.t_far;
    d.transfer = g.transfer_fmt ? g.transfer_fmt : 32;
}

StepArgs base_args(ffn_ctx* c, const void* rays, const void* targets, void* out, uint32_t n,
                   const ffn_step_scalars* s) {
    StepArgs a{};
    a.c = c->dc;
    if (s->spr) a.c.spr = (int)s->spr;
    a.lo = c->lo;
    a.params = c->params;
    a.table = c->table;
    a.occ_in = c->occ_in;
    a.occ_st = c->occ_st;
    a.rays = static_cast<const float4*>(rays);
    a.targets = static_cast<const float4*>(targets);
    a.out = static_cast<float4*>(out);
    a.grad_table = c->grads;
    for (int l = 0; l < L; ++l) a.hash_coef[l] = 1.0f;
    if (s->flags & FFN_STEP_TABLE_IMMEDIATE) {
        a.grad_table = c->table;
        for (int l = 0; l < L; ++l) a.hash_coef[l] = -(s->lr_f * c->cfg.hash_lr_scale[l]) * 0.5f;   // HASH_LR_RATE
    }
    a.partials = c->partials;
    a.status = c->status;
    a.n_rays = n;
    a.ray_offset = s->ray_offset;
    a.sh_mult = s->sh_mult;
    a.occ_strength = s->occ_strength;
    a.seed = s->rng_u32;
    return a;
}

// Blocks for n_tiles tiles at c->groups tiles per block, at most max_grid.
int fused_grid(const ffn_ctx* c, int n_tiles) {
    const int blocks = (n_tiles + c->groups - 1) / c->groups;
    return blocks < c->max_grid ? blocks : c->max_grid;
}

// Launches the fused kernel; *parts_out = weight-gradient partial rows it writes (blocks x groups).
int launch_fused(ffn_ctx* c, const StepArgs& a, cudaStream_t st, int* parts_out) {
    const int rpt = c->rows / a.c.spr;
    const int n_tiles = (int)((a.n_rays + (uint32_t)rpt - 1) / (uint32_t)rpt);
    const int grid = fused_grid(c, n_tiles);
    if (parts_out) *parts_out = grid * c->groups;
    if (grid == 0) return FFN_OK;
    c->kernel<<<grid, c->threads, c->smem, st>>>(a);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "fused step launch");
    return FFN_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Blocks for a grid-stride launch over `work` items of `per_block`: at most per_sm blocks per SM of
// the current device (SM count cached per device).
int grid_for(uint64_t work, int per_block, int per_sm) {
    static int sms_of[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = dev >= 0 && dev < 64 ? sms_of[dev] : 0;
    if (sms == 0) {
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
        if (dev >= 0 && dev < 64) sms_of[dev] = sms;
    }
    const uint64_t need = (work + (uint64_t)per_block - 1) / (uint64_t)per_block;
    const uint64_t cap = (uint64_t)sms * (uint64_t)per_sm;
    return (int)(need < cap ? (need ? need : 1) : cap);
}

// The split tensor-core step over groups of at most STAGE_SAMPLES samples: sampler, encoder,
// then the MLP/compositing/backward kernel and the fixed-order partial reduction per group.
// (Running the encoder of the next half-group on a second stream beside the MLP kernel was slower:
// its blocks hold SM resources the MLP kernel's CTAs need.)
int forward_backward_staged(ffn_ctx* c, const void* rays, const void* targets, void* out, uint32_t n,
                            const ffn_step_scalars* s, cudaStream_t st) {
    const int spr = s->spr ? (int)s->spr : c->cfg.spr;
    const uint32_t group_rays = (uint32_t)(STAGE_SAMPLES / spr);
    const int rpt = 128 / spr;
    const int sms = c->max_grid / c->ctas_per_sm;
    for (uint32_t r0 = 0; r0 < n; r0 += group_rays) {
        const uint32_t m = n - r0 < group_rays ? n - r0 : group_rays;
        StepArgs a = base_args(c, static_cast<const float4*>(rays) + 2 * (size_t)r0,
                               static_cast<const float4*>(targets) + r0, static_cast<float4*>(out) + r0, m, s);
        a.ray_offset = s->ray_offset + r0;
        a.do_train = 1;
        const int n_tiles = (int)((m + (uint32_t)rpt - 1) / (uint32_t)rpt);
        const int sgrid = n_tiles < sms * 8 ? n_tiles : sms * 8;
        sample_stage_kernel<<<sgrid, 128, 0, st>>>(a, c->pn_stage, c->tdt_stage, c->ray_stage);
        ++c->launches;
        const int64_t rows = (int64_t)n_tiles * 128;
        const int64_t chunks = (rows + 255) / 256 * L;
        const int eblocks = (int)(chunks < (int64_t)sms * 16 ? chunks : (int64_t)sms * 16);
        c->encoder<<<eblocks, 256, 0, st>>>(a.c, c->table, c->pn_stage, (int64_t)m * spr, rows, c->x0_stage);
        ++c->launches;
        a.x0_stage = c->x0_stage;
        a.tdt_stage = c->tdt_stage;
        a.ray_stage = c->ray_stage;
        const int mtiles = (int)((m + (uint32_t)(c->rows / spr) - 1) / (uint32_t)(c->rows / spr));   // MLP-kernel tiles
        const int grid = fused_grid(c, mtiles);
        c->kernel_staged<<<grid, c->threads, c->smem, st>>>(a);
        ++c->launches;
        reduce_partials<<<(c->Pw + 255) / 256, 256, 0, st>>>(c->partials, grid * c->groups, c->Pw,
                                                            c->grads + c->table_floats, c->status);
        ++c->launches;
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(c, e, "split step launch");
    }
    return FFN_OK;
}

// The MLP microbenchmark launch: compensated operand pairs (the step's form) or plain fp16.
template <bool PLAIN>
int mlp_bench(ffn_ctx* c, const void* tiles, int64_t n, void* stream) {
    if (!c || (n > 0 && !tiles)) return fail(c, FFN_E_CONFIG, "null argument");
    if (n <= 0) return FFN_OK;
    if (c->cfg.mlp_precision != 1 || c->cfg.F != 2 || c->cfg.ND != 1)
        return fail(c, FFN_E_CONFIG, "the MLP microbenchmark is compiled for the tensor-core MLP with F=2, ND=1");
    if (n % 128 != 0 || (uint64_t)n / (uint64_t)c->cfg.spr > 0xFFFFFFFFull || 128 % c->cfg.spr != 0)
        return fail(c, FFN_E_CONFIG, "n must be a multiple of 128 and the configured samples per ray divide 128");
    if (!aligned16(tiles)) return fail(c, FFN_E_CONFIG, "tiles must be 16-byte aligned");
    DeviceGuard guard(c->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    using PL = TcPlan<2, 1>;
    auto kfn = fused_step_tc_kernel<2, 1, true, true, PLAIN>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::BYTES);
    if (e != cudaSuccess) return cuda_fail(c, e, "MLP microbenchmark kernel attribute");
    ffn_step_scalars s{};
    s.sh_mult = 1.0f;
    s.spr = (uint32_t)c->cfg.spr;
    StepArgs a = base_args(c, nullptr, nullptr, nullptr, (uint32_t)(n / c->cfg.spr), &s);
    a.do_train = 1;
    a.x0_stage = static_cast<const unsigned char*>(tiles);
    const int grid = fused_grid(c, (int)(n / 128));
    kfn<<<grid, PL::THREADS, PL::BYTES, st>>>(a);
    ++c->launches;
    reduce_partials<<<(c->Pw + 255) / 256, 256, 0, st>>>(c->partials, grid * PL::GROUPS, c->Pw,
                                                        c->grads + c->table_floats, c->status);
    ++c->launches;
    e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "MLP microbenchmark launch");
}

}  // namespace

extern "C" {

int ffn_abi_version(void) { return FFN_ABI_VERSION; }

const char* ffn_last_error(const ffn_ctx* ctx) { return ctx ? ctx->err.c_str() : g_create_err.c_str(); }

int ffn_param_layout(const ffn_config* cfg, int32_t* offsets18, int32_t* sizes18) {
    if (!cfg) return FFN_E_CONFIG;
    ParamLayout lo = make_param_layout(cfg->F, cfg->ND, cfg->NC);
    for (int i = 0; i < P_COUNT; ++i) {
        if (offsets18) offsets18[i] = lo.off[i];
        if (sizes18) sizes18[i] = lo.size[i];
    }
    return lo.total;
}

int ffn_create(const ffn_config* cfg, int device, ffn_ctx** out) {
    if (!cfg || !out) return fail(nullptr, FFN_E_CONFIG, "null argument");
    *out = nullptr;
    std::string why;
    if (check_config(cfg, &why) != FFN_OK) return fail(nullptr, FFN_E_CONFIG, why);
    ffn_ctx* c = new ffn_ctx();
    c->cfg = *cfg;
    c->device = device;
    c->lo = make_param_layout(cfg->F, cfg->ND, cfg->NC);
    c->Pw = c->lo.total;
    uint64_t entries = 0;
    for (int l = 0; l < L; ++l) entries += 1ull << cfg->level_log2[l];
    c->table_floats = (size_t)entries * cfg->F;
    fill_dev_config(c);
    if (!select_kernel(c)) {
        delete c;
        return fail(nullptr, FFN_E_CONFIG, "this (F, ND, NC) combination is not compiled: supported are NC=2 with "
                                           "(F, ND) in {(2,1), (4,1), (2,2), (4,2)}");
    }
    DeviceGuard guard(device);
    cudaError_t e;
    int sms = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) {
        delete c;
        return cuda_fail(nullptr, e, "device query");
    }
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if ((int)c->smem > max_smem) {
        delete c;
        return fail(nullptr, FFN_E_CONFIG, "configuration needs more shared memory than the device offers");
    }
    if ((e = cudaFuncSetAttribute(c->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->smem)) != cudaSuccess ||
        (c->kernel_staged &&
         (e = cudaFuncSetAttribute(c->kernel_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->smem)) != cudaSuccess)) {
        delete c;
        return cuda_fail(nullptr, e, "shared-memory attribute");
    }
    c->max_grid = sms * c->ctas_per_sm;
    const size_t Pb = (size_t)c->Pw * sizeof(float);
    const size_t Tb = c->table_floats * sizeof(float);
    const size_t Gb = (size_t)cfg->G * cfg->G * cfg->G * sizeof(uint32_t);
    struct { void** p; size_t n; } allocs[] = {
        {(void**)&c->params, Pb}, {(void**)&c->adam_m, Pb}, {(void**)&c->adam_v, Pb},
        {(void**)&c->table, Tb}, {(void**)&c->occ_in, Gb}, {(void**)&c->occ_st, Gb},
        {(void**)&c->grads, Tb + Pb}, {(void**)&c->partials, (size_t)c->max_grid * c->groups * Pb},
        {(void**)&c->status, sizeof(int)}};
    for (auto& al : allocs) {
        if ((e = cudaMalloc(al.p, al.n)) != cudaSuccess) { ffn_destroy(c); return cuda_fail(nullptr, e, "device allocation"); }
        cudaMemset(*al.p, 0, al.n);
    }
    if (c->kernel_staged) {
        struct { void** p; size_t n; } st_allocs[] = {
            // fp32 rows (fp32 MLP) or the hi and lo fp16 operand tiles (tensor-core MLP): 4 B per feature
            {(void**)&c->x0_stage, (size_t)STAGE_SAMPLES * 16 * cfg->F * 4},
            {(void**)&c->tdt_stage, (size_t)STAGE_SAMPLES * sizeof(float2)},
            {(void**)&c->pn_stage, (size_t)STAGE_SAMPLES * sizeof(float4)},
            {(void**)&c->ray_stage, (size_t)(STAGE_SAMPLES / 16) * sizeof(uint4)}};
        for (auto& al : st_allocs)
            if ((e = cudaMalloc(al.p, al.n)) != cudaSuccess) { ffn_destroy(c); return cuda_fail(nullptr, e, "device allocation"); }
    }
    if (cfg->table_optimizer == 1) {
        if ((e = cudaMalloc((void**)&c->table_m, Tb)) != cudaSuccess || (e = cudaMalloc((void**)&c->table_v, Tb)) != cudaSuccess) {
            ffn_destroy(c);
            return cuda_fail(nullptr, e, "device allocation");
        }
        cudaMemset(c->table_m, 0, Tb);
        cudaMemset(c->table_v, 0, Tb);
    }
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) { ffn_destroy(c); return cuda_fail(nullptr, e, "initialisation"); }
    *out = c;
    return FFN_OK;
}

int ffn_destroy(ffn_ctx* c) {
    if (!c) return FFN_OK;
    DeviceGuard guard(c->device);
    cudaDeviceSynchronize();
    if (c->dp) {
        for (int p = 0; p < c->dp->peers.world; ++p) {
            if (!c->dp->opened[p]) continue;
            if (c->dp->peers.grads[p]) cudaIpcCloseMemHandle(c->dp->peers.grads[p]);
            if (c->dp->peers.table[p]) cudaIpcCloseMemHandle(c->dp->peers.table[p]);
            cudaIpcCloseMemHandle(c->dp->peers.flags[p]);
        }
        if (c->dp->flags) cudaFree(c->dp->flags);
        if (c->dp->done_counter) cudaFree(c->dp->done_counter);
        delete c->dp;
        c->dp = nullptr;
    }
    void* ptrs[] = {c->params, c->adam_m, c->adam_v, c->ext_table ? nullptr : c->table, c->table_m, c->table_v,
                    c->occ_in, c->occ_st, c->ext_grads ? nullptr : c->grads, c->partials, c->status, c->x0_stage,
                    c->tdt_stage, c->pn_stage, c->ray_stage};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    delete c;
    return FFN_OK;
}

int ffn_buffer(ffn_ctx* c, int id, void** dev, size_t* bytes) {
    if (!c || !dev || !bytes) return fail(c, FFN_E_CONFIG, "null argument");
    const size_t Pb = (size_t)c->Pw * sizeof(float), Tb = c->table_floats * sizeof(float);
    const size_t Gb = (size_t)c->cfg.G * c->cfg.G * c->cfg.G * sizeof(uint32_t);
    switch (id) {
        case FFN_BUF_PARAMS: *dev = c->params; *bytes = Pb; break;
        case FFN_BUF_ADAM_M: *dev = c->adam_m; *bytes = Pb; break;
        case FFN_BUF_ADAM_V: *dev = c->adam_v; *bytes = Pb; break;
        case FFN_BUF_TABLE: *dev = c->table; *bytes = Tb; break;
        case FFN_BUF_OCC_IN: *dev = c->occ_in; *bytes = Gb; break;
        case FFN_BUF_OCC_ST: *dev = c->occ_st; *bytes = Gb; break;
        case FFN_BUF_GRADS: *dev = c->grads; *bytes = Tb + Pb; break;
        case FFN_BUF_TABLE_M: *dev = c->table_m; *bytes = c->table_m ? Tb : 0; break;
        case FFN_BUF_TABLE_V: *dev = c->table_v; *bytes = c->table_v ? Tb : 0; break;
        default: return fail(c, FFN_E_NAME, "unknown buffer id");
    }
    return FFN_OK;
}

int ffn_grad_buffer(ffn_ctx* c, void** dev, size_t* n_floats) {
    if (!c || !dev || !n_floats) return fail(c, FFN_E_CONFIG, "null argument");
    *dev = c->grads;
    *n_floats = c->table_floats + (size_t)c->Pw;
    return FFN_OK;
}

static int check_io(ffn_ctx* c, const void* rays, const void* out, uint32_t n, const ffn_step_scalars* s) {
    if (!c) return FFN_E_CONFIG;
    if (!s) return fail(c, FFN_E_CONFIG, "null step scalars");
    if (s->spr != 0 && s->spr != 16 && s->spr != 32 && s->spr != 64)
        return fail(c, FFN_E_CONFIG, "samples_per_ray must be 16, 32 or 64 (power of two, <= S_MAX=64)");
    if (n == 0) return FFN_OK;
    if (!rays || !out) return fail(c, FFN_E_CONFIG, "rays and out must be device pointers");
    if (!aligned16(rays) || !aligned16(out)) return fail(c, FFN_E_CONFIG, "rays/out must be 16-byte aligned");
    if ((uint64_t)n * 64ull >= (1ull << 31)) return fail(c, FFN_E_CAPACITY, "too many rays in one call");
    return FFN_OK;
}

int ffn_forward_backward(ffn_ctx* c, const void* rays, const void* targets, void* out, uint32_t n,
                         const ffn_step_scalars* s, void* stream) {
    int rc = check_io(c, rays, out, n, s);
    if (rc != FFN_OK || n == 0) return rc;
    if (!targets || !aligned16(targets)) return fail(c, FFN_E_CONFIG, "targets must be a 16-byte aligned device pointer");
    DeviceGuard guard(c->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((s->flags & FFN_STEP_TABLE_IMMEDIATE) && c->cfg.table_optimizer != 0)
        return fail(c, FFN_E_CONFIG, "immediate table updates need the SGD table optimizer");
    if (c->kernel_staged) return forward_backward_staged(c, rays, targets, out, n, s, st);
    StepArgs a = base_args(c, rays, targets, out, n, s);
    a.do_train = 1;
    int parts = 0;
    if ((rc = launch_fused(c, a, st, &parts)) != FFN_OK) return rc;
    reduce_partials<<<(c->Pw + 255) / 256, 256, 0, st>>>(c->partials, parts, c->Pw, c->grads + c->table_floats,
                                                            c->status);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "gradient reduction launch");
}

int ffn_apply_updates(ffn_ctx* c, const ffn_step_scalars* s, void* stream) {
    if (!c || !s) return fail(c, FFN_E_CONFIG, "null argument");
    DeviceGuard guard(c->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const ffn_config& g = c->cfg;
    mlp_adam_kernel<<<(c->Pw + 255) / 256, 256, 0, st>>>(c->params, c->grads + c->table_floats, c->adam_m,
                                                         c->adam_v, c->Pw, c->lo.off[P_WC_IN], c->lo.off[P_BD_0],
                                                         c->lo.off[P_BC_0], s->lr_t, s->color_rel_lr,
                                                         g.adam_beta1, g.adam_beta2, g.adam_eps);
    ++c->launches;
    LevelCoef lc{};
    for (int l = 0; l < L; ++l) {
        lc.start[l] = g.level_offset[l] * (uint32_t)g.F;
        lc.coef[l] = g.table_optimizer == 1 ? s->table_lr_t * g.hash_lr_scale[l]
                                            : -(s->lr_f * g.hash_lr_scale[l]) * 0.5f;   // HASH_LR_RATE
    }
    lc.start[L] = (uint32_t)c->table_floats;
    const uint32_t n4 = (uint32_t)(c->table_floats / 4);
    const int blocks = grid_for(n4, 256, 16);
    if (s->flags & (FFN_STEP_TABLE_IMMEDIATE | FFN_STEP_TABLE_APPLIED)) {
        // the table was updated inside the forward/backward pass or by ffn_dp_reduce_apply
    } else if (g.table_optimizer == 1) {
        table_adam_kernel<<<blocks, 256, 0, st>>>(c->table, c->grads, c->table_m, c->table_v, n4, lc,
                                                   g.adam_beta1, g.adam_beta2, g.table_adam_eps);
        ++c->launches;
    } else {
        table_sgd_kernel<<<blocks, 256, 0, st>>>(c->table, c->grads, n4, lc);
        ++c->launches;
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "update launch");
}

int ffn_train_step(ffn_ctx* c, const void* rays, const void* targets, void* out, uint32_t n,
                   const ffn_step_scalars* s, void* stream) {
    int rc = ffn_forward_backward(c, rays, targets, out, n, s, stream);
    if (rc != FFN_OK) return rc;
    return ffn_apply_updates(c, s, stream);
}

int ffn_render(ffn_ctx* c, const void* rays, void* out, uint32_t n, const ffn_step_scalars* s, void* stream) {
    int rc = check_io(c, rays, out, n, s);
    if (rc != FFN_OK || n == 0) return rc;
    DeviceGuard guard(c->device);
    StepArgs a = base_args(c, rays, nullptr, out, n, s);
    a.do_train = 0;
    a.partials = nullptr;
    return launch_fused(c, a, static_cast<cudaStream_t>(stream), nullptr);
}

int ffn_probe(ffn_ctx* c, const void* rays, const void* targets, void* out, uint32_t n,
              const ffn_step_scalars* s, const void* bypass, float* t, float* dt, int32_t* idx,
              uint32_t* flags, float* sigma, float* rgb, float* trans, void* stream) {
    int rc = check_io(c, rays, out, n, s);
    if (rc != FFN_OK || n == 0) return rc;
    if (bypass && !aligned16(bypass)) return fail(c, FFN_E_CONFIG, "bypass must be 16-byte aligned");
    DeviceGuard guard(c->device);
    StepArgs a = base_args(c, rays, targets, out, n, s);
    a.do_train = 1;
    a.partials = nullptr;
    a.probe = 1;
    a.bypass = static_cast<const float4*>(bypass);
    a.dbg_t = t; a.dbg_dt = dt; a.dbg_idx = idx; a.dbg_flags = flags;
    a.dbg_sigma = sigma; a.dbg_rgb = rgb; a.dbg_trans = trans;
    return launch_fused(c, a, static_cast<cudaStream_t>(stream), nullptr);
}

int ffn_occ_st_bytes(ffn_ctx* c, uint8_t* bytes, int to_bytes, void* stream) {
    if (!c || !bytes) return fail(c, FFN_E_CONFIG, "null argument");
    if (!aligned16(bytes)) return fail(c, FFN_E_CONFIG, "bytes must be 16-byte aligned");
    DeviceGuard guard(c->device);
    const uint32_t n = (uint32_t)c->cfg.G * c->cfg.G * c->cfg.G;
    const int blocks = grid_for(n, 256, 8);
    occ_bytes_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(c->occ_st, bytes, n, to_bytes);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "occupancy byte conversion launch");
}

int ffn_occ_maintenance(ffn_ctx* c, uint32_t decay_q24, uint32_t seed, void* stream) {
    if (!c) return FFN_E_CONFIG;
    if (decay_q24 > (1u << 24)) return fail(c, FFN_E_CONFIG, "decay_q24 must be in [0, 2^24]");
    DeviceGuard guard(c->device);
    const uint32_t n = (uint32_t)c->cfg.G * c->cfg.G * c->cfg.G;
    const int blocks = grid_for(n, 256, 8);
    occ_decay_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(c->occ_in, c->occ_st, n, decay_q24, seed);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "decay launch");
}

int ffn_hash_encode(ffn_ctx* c, const float* pts, float* enc, int64_t n, void* stream) {
    if (!c || (n > 0 && (!pts || !enc))) return fail(c, FFN_E_CONFIG, "null argument");
    if (n <= 0) return FFN_OK;
    if (!aligned16(enc)) return fail(c, FFN_E_CONFIG, "enc must be 16-byte aligned");
    DeviceGuard guard(c->device);
    const int64_t items = (n + 15) / 16;   // blocks of 16 points x 16 levels
    const int sms = c->max_grid / c->ctas_per_sm;
    const int blocks = (int)(items < (int64_t)sms * 16 ? items : (int64_t)sms * 16);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (c->cfg.F == 2) hash_fwd_kernel<2><<<blocks, 256, 0, st>>>(c->dc, c->table, pts, n, enc);
    else hash_fwd_kernel<4><<<blocks, 256, 0, st>>>(c->dc, c->table, pts, n, enc);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "hash encode launch");
}

int ffn_hash_encode_bwd(ffn_ctx* c, const float* pts, const float* denc, int64_t n, void* stream) {
    if (!c || (n > 0 && (!pts || !denc))) return fail(c, FFN_E_CONFIG, "null argument");
    if (n <= 0) return FFN_OK;
    if (!aligned16(denc)) return fail(c, FFN_E_CONFIG, "denc must be 16-byte aligned");
    DeviceGuard guard(c->device);
    const int64_t items = (n + 15) / 16;   // blocks of 16 points x 16 levels
    const int sms = c->max_grid / c->ctas_per_sm;
    const int blocks = (int)(items < (int64_t)sms * 16 ? items : (int64_t)sms * 16);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (c->cfg.F == 2) hash_bwd_kernel<2><<<blocks, 256, 0, st>>>(c->dc, c->grads, pts, denc, n);
    else hash_bwd_kernel<4><<<blocks, 256, 0, st>>>(c->dc, c->grads, pts, denc, n);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "hash scatter launch");
}

int ffn_hash_encode_f16(ffn_ctx* c, const void* table16, const float* pts, void* enc16, int64_t n, void* stream) {
    if (!c || (n > 0 && (!table16 || !pts || !enc16))) return fail(c, FFN_E_CONFIG, "null argument");
    if (n <= 0) return FFN_OK;
    if (!aligned16(table16) || !aligned16(enc16)) return fail(c, FFN_E_CONFIG, "table16 and enc16 must be 16-byte aligned");
    DeviceGuard guard(c->device);
    const int64_t items = (n + 15) / 16;   // blocks of 16 points x 16 levels
    const int sms = c->max_grid / c->ctas_per_sm;
    const int blocks = (int)(items < (int64_t)sms * 16 ? items : (int64_t)sms * 16);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const __half* tab = static_cast<const __half*>(table16);
    __half* enc = static_cast<__half*>(enc16);
    if (c->cfg.F == 2) hash_fwd_f16_kernel<2><<<blocks, 256, 0, st>>>(c->dc, tab, pts, n, enc);
    else hash_fwd_f16_kernel<4><<<blocks, 256, 0, st>>>(c->dc, tab, pts, n, enc);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "fp16 hash encode launch");
}

int ffn_hash_encode_bwd_f16(ffn_ctx* c, void* grad16, const float* pts, const float* denc, int64_t n, void* stream) {
    if (!c || (n > 0 && (!grad16 || !pts || !denc))) return fail(c, FFN_E_CONFIG, "null argument");
    if (n <= 0) return FFN_OK;
    if (!aligned16(grad16) || !aligned16(denc)) return fail(c, FFN_E_CONFIG, "grad16 and denc must be 16-byte aligned");
    DeviceGuard guard(c->device);
    const int64_t items = (n + 15) / 16;
    const int sms = c->max_grid / c->ctas_per_sm;
    const int blocks = (int)(items < (int64_t)sms * 16 ? items : (int64_t)sms * 16);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    __half* g = static_cast<__half*>(grad16);
    if (c->cfg.F == 2) hash_bwd_f16_kernel<2><<<blocks, 256, 0, st>>>(c->dc, g, pts, denc, n);
    else hash_bwd_f16_kernel<4><<<blocks, 256, 0, st>>>(c->dc, g, pts, denc, n);
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "fp16 hash scatter launch");
}

int ffn_pack_x0(ffn_ctx* c, const void* x16, void* tiles, int64_t n, void* stream) {
    if (!c || (n > 0 && (!x16 || !tiles))) return fail(c, FFN_E_CONFIG, "null argument");
    if (n <= 0) return FFN_OK;
    if (n % 128 != 0) return fail(c, FFN_E_CONFIG, "n must be a multiple of 128 (the tile height)");
    if (!aligned16(x16) || !aligned16(tiles)) return fail(c, FFN_E_CONFIG, "x16 and tiles must be 16-byte aligned");
    DeviceGuard guard(c->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t threads = n * (L * c->cfg.F / 8);
    const int blocks = (int)((threads + 255) / 256);
    if (c->cfg.F == 2) pack_x0_kernel<2><<<blocks, 256, 0, st>>>(static_cast<const __half*>(x16), n,
                                                                 static_cast<unsigned char*>(tiles));
    else pack_x0_kernel<4><<<blocks, 256, 0, st>>>(static_cast<const __half*>(x16), n, static_cast<unsigned char*>(tiles));
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(c, e, "pack launch");
}

int ffn_mlp_bench(ffn_ctx* c, const void* tiles, int64_t n, void* stream) { return mlp_bench<false>(c, tiles, n, stream); }
int ffn_mlp_bench_f16(ffn_ctx* c, const void* tiles, int64_t n, void* stream) { return mlp_bench<true>(c, tiles, n, stream); }

uint64_t ffn_kernel_launches(const ffn_ctx* c) { return c ? c->launches : 0u; }

int ffn_batch_generate(const void* images, int img_f32, int channels, const uint8_t* weights, const float* c2w,
                       const float* K, int k_per_image, int n_img, int W, int H, uint32_t n, float uniform_frac,
                       uint32_t seed, uint32_t max_tries, void* rays, void* targets, int32_t* im, int32_t* x,
                       int32_t* y, void* stream) {
    if (n == 0) return FFN_OK;
    if (!images || !weights || !c2w || !rays || !targets) return fail(nullptr, FFN_E_CONFIG, "null argument");
    if (n_img < 1 || W < 1 || H < 1 || channels < 3) return fail(nullptr, FFN_E_CONFIG, "need >= 1 image of >= 3 channels");
    if ((im || x || y) && !(im && x && y)) return fail(nullptr, FFN_E_CONFIG, "im, x and y are given together");
    if (!aligned16(rays) || !aligned16(targets)) return fail(nullptr, FFN_E_CONFIG, "rays/targets must be 16-byte aligned");
    if (!(uniform_frac >= 0.0f && uniform_frac <= 1.0f)) return fail(nullptr, FFN_E_CONFIG, "uniform_frac must be in [0, 1]");
    ffn::BatchGen g{images, img_f32, weights, c2w, K, k_per_image, n_img, W, H, channels, n, uniform_frac, seed, max_tries};
    const int blocks = grid_for(n, 256, 8);
    ffn::batch_generate_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        g, static_cast<float4*>(rays), static_cast<float4*>(targets), im, x, y);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(nullptr, e, "batch generation launch");
}

int ffn_camera_rays(const float* c2w, const float* K, int W, int H, uint32_t first, uint32_t n, void* rays,
                    void* stream) {
    if (n == 0) return FFN_OK;
    if (!c2w || !rays) return fail(nullptr, FFN_E_CONFIG, "null argument");
    if (W < 1 || H < 1 || (uint64_t)first + n > (uint64_t)W * (uint64_t)H)
        return fail(nullptr, FFN_E_CONFIG, "pixel range outside the view");
    if (!aligned16(rays)) return fail(nullptr, FFN_E_CONFIG, "rays must be 16-byte aligned");
    ffn::ViewCam v{};
    std::memcpy(v.c2w, c2w, sizeof(v.c2w));
    if (K) std::memcpy(v.k, K, sizeof(v.k));
    v.has_k = K != nullptr;
    v.W = W;
    v.H = H;
    const int blocks = grid_for(n, 256, 8);
    ffn::camera_rays_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(v, first, n, static_cast<float4*>(rays));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(nullptr, e, "camera rays launch");
}

int ffn_batch_errors(const void* out, const void* targets, uint32_t n, float* err, double* sum_sq, void* stream) {
    if (n == 0) return FFN_OK;
    if (!out || !targets || (!err && !sum_sq)) return fail(nullptr, FFN_E_CONFIG, "null argument");
    if (!aligned16(out) || !aligned16(targets)) return fail(nullptr, FFN_E_CONFIG, "out/targets must be 16-byte aligned");
    const int blocks = grid_for(n, 256, 8);
    ffn::batch_error_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float4*>(out), static_cast<const float4*>(targets), n, err, sum_sq);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(nullptr, e, "error launch");
}

int ffn_batch_feedback(uint8_t* weights, const void* images, int img_f32, int channels, int W, int H,
                       const int32_t* im, const int32_t* x, const int32_t* y, const float* err, uint32_t n,
                       const float* median, double ema, int bg_cap, int fg_tau, void* stream) {
    if (n == 0) return FFN_OK;
    if (!weights || !images || !im || !x || !y || !err || !median) return fail(nullptr, FFN_E_CONFIG, "null argument");
    const int blocks = grid_for(n, 256, 8);
    ffn::batch_feedback_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        weights, images, img_f32, channels, W, H, im, x, y, err, n, median, ema, bg_cap, fg_tau);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(nullptr, e, "feedback launch");
}

int ffn_status(ffn_ctx* c, uint32_t* status) {
    if (!c || !status) return fail(c, FFN_E_CONFIG, "null argument");
    DeviceGuard guard(c->device);
    int h = 0;
    cudaError_t e = cudaMemcpy(&h, c->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(c, e, "status read");
    cudaMemset(c->status, 0, sizeof(int));
    *status = (uint32_t)h;
    return FFN_OK;
}

int ffn_dp_ipc_handles(ffn_ctx* c, void* out) {
    if (!c || !out) return fail(c, FFN_E_CONFIG, "null argument");
    DeviceGuard guard(c->device);
    cudaError_t e;
    if (!c->dp) {
        c->dp = new DpState();
        if ((e = cudaMalloc((void**)&c->dp->flags, 2 * ffn::DP_MAX_RANKS * sizeof(uint32_t))) != cudaSuccess ||
            (e = cudaMalloc((void**)&c->dp->done_counter, sizeof(unsigned int))) != cudaSuccess)
            return cuda_fail(c, e, "flag allocation");
        cudaMemset(c->dp->flags, 0, 2 * ffn::DP_MAX_RANKS * sizeof(uint32_t));
        cudaMemset(c->dp->done_counter, 0, sizeof(unsigned int));
        if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(c, e, "flag initialisation");
    }
    cudaIpcMemHandle_t h[3];
    std::memset(h, 0, sizeof(h));
    // buffers bound from outside (multicast-capable allocations) are not exported: the NVLS exchange
    // reaches them through their multicast address
    if ((!c->ext_grads && (e = cudaIpcGetMemHandle(&h[0], c->grads)) != cudaSuccess) ||
        (!c->ext_table && (e = cudaIpcGetMemHandle(&h[1], c->table)) != cudaSuccess) ||
        (e = cudaIpcGetMemHandle(&h[2], c->dp->flags)) != cudaSuccess)
        return cuda_fail(c, e, "IPC handle");
    std::memcpy(out, h, sizeof(h));
    return FFN_OK;
}

int ffn_dp_attach(ffn_ctx* c, int rank, int world, const void* handles) {
    if (!c || !handles) return fail(c, FFN_E_CONFIG, "null argument");
    if (!c->dp) return fail(c, FFN_E_STATE, "ffn_dp_ipc_handles must be called first");
    if (world < 1 || world > ffn::DP_MAX_RANKS || rank < 0 || rank >= world)
        return fail(c, FFN_E_CONFIG, "world must be 1..8 and 0 <= rank < world");
    if (c->dp->peers.world) return fail(c, FFN_E_STATE, "already attached");
    DeviceGuard guard(c->device);
    const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
    ffn::DpPeers& P = c->dp->peers;
    for (int p = 0; p < world; ++p) {
        if (p == rank) {
            P.grads[p] = c->grads; P.table[p] = c->table; P.flags[p] = c->dp->flags;
            continue;
        }
        void *g = nullptr, *t = nullptr, *f = nullptr;
        cudaError_t e = cudaSuccess;
        const bool flags_only = c->ext_grads || c->ext_table;   // NVLS exchange: peers' buffers via multicast
        if ((!flags_only && (e = cudaIpcOpenMemHandle(&g, h[3 * p], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) ||
            (!flags_only && (e = cudaIpcOpenMemHandle(&t, h[3 * p + 1], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) ||
            (e = cudaIpcOpenMemHandle(&f, h[3 * p + 2], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) {
            if (g) cudaIpcCloseMemHandle(g);
            if (t) cudaIpcCloseMemHandle(t);
            return cuda_fail(c, e, "opening a peer's IPC handle");
        }
        P.grads[p] = static_cast<float*>(g); P.table[p] = static_cast<float*>(t); P.flags[p] = static_cast<uint32_t*>(f);
        c->dp->opened[p] = true;
    }
    P.rank = rank;
    P.world = world;
    return FFN_OK;
}

int ffn_bind_external(ffn_ctx* c, int id, void* dev_ptr, size_t bytes) {
    if (!c || !dev_ptr) return fail(c, FFN_E_CONFIG, "null argument");
    if (id != FFN_BUF_TABLE && id != FFN_BUF_GRADS) return fail(c, FFN_E_NAME, "only the table and the gradient buffer can be bound");
    if (c->dp && c->dp->peers.world) return fail(c, FFN_E_STATE, "bind buffers before ffn_dp_attach");
    if (!aligned16(dev_ptr)) return fail(c, FFN_E_CONFIG, "buffer must be 16-byte aligned");
    const size_t need = (c->table_floats + (id == FFN_BUF_GRADS ? (size_t)c->Pw : 0)) * sizeof(float);
    if (bytes < need) return fail(c, FFN_E_CAPACITY, "buffer smaller than the context's");
    DeviceGuard guard(c->device);
    float*& slot = id == FFN_BUF_TABLE ? c->table : c->grads;
    bool& ext = id == FFN_BUF_TABLE ? c->ext_table : c->ext_grads;
    cudaError_t e;
    if ((e = cudaDeviceSynchronize()) != cudaSuccess ||
        (e = cudaMemcpy(dev_ptr, slot, need, cudaMemcpyDeviceToDevice)) != cudaSuccess)
        return cuda_fail(c, e, "copy into the bound buffer");
    if (!ext) cudaFree(slot);
    slot = static_cast<float*>(dev_ptr);
    ext = true;
    return FFN_OK;
}

int ffn_dp_attach_multicast(ffn_ctx* c, void* mc_grads, void* mc_table) {
    if (!c || !mc_grads || !mc_table) return fail(c, FFN_E_CONFIG, "null argument");
    if (!c->dp || !c->dp->peers.world) return fail(c, FFN_E_STATE, "ffn_dp_attach must be called first");
    if (!c->ext_grads || !c->ext_table) return fail(c, FFN_E_STATE, "bind the multicast-backed buffers first");
    if (!aligned16(mc_grads) || !aligned16(mc_table)) return fail(c, FFN_E_CONFIG, "multicast addresses must be 16-byte aligned");
    c->dp->mc_grads = static_cast<float*>(mc_grads);
    c->dp->mc_table = static_cast<float*>(mc_table);
    return FFN_OK;
}

int ffn_dp_reduce_apply(ffn_ctx* c, const ffn_step_scalars* s, void* stream) {
    if (!c || !s) return fail(c, FFN_E_CONFIG, "null argument");
    if (!c->dp || !c->dp->peers.world) return fail(c, FFN_E_STATE, "ffn_dp_attach must be called first");
    if (c->cfg.table_optimizer != 0) return fail(c, FFN_E_CONFIG, "the fused exchange applies the SGD table update only");
    DeviceGuard guard(c->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const ffn_config& g = c->cfg;
    LevelCoef lc{};
    for (int l = 0; l < L; ++l) {
        lc.start[l] = g.level_offset[l] * (uint32_t)g.F;
        lc.coef[l] = -(s->lr_f * g.hash_lr_scale[l]) * 0.5f;   // HASH_LR_RATE
    }
    lc.start[L] = (uint32_t)c->table_floats;
    const uint32_t table4 = (uint32_t)(c->table_floats / 4);
    const uint32_t total4 = (uint32_t)((c->table_floats + (size_t)c->Pw) / 4);
    const int sms = c->max_grid / c->ctas_per_sm;
    if (!c->dp->mc_grads && (c->ext_grads || c->ext_table))
        return fail(c, FFN_E_STATE, "externally bound buffers need ffn_dp_attach_multicast");
    const uint32_t epoch = ++c->dp->epoch;
    if (c->dp->mc_grads)
        ffn::dp_reduce_apply_nvls_kernel<<<sms * 4, 256, 0, st>>>(c->dp->peers, c->dp->mc_grads, c->dp->mc_table,
                                                                  c->table, table4, total4, lc, epoch, c->status,
                                                                  c->dp->done_counter, c->dp->wait_limit);
    else {
        // registers sized for the world: two float4 per thread and iteration up to 4 ranks, one at 8
        auto kern = c->dp->peers.world <= 2 ? ffn::dp_reduce_apply_kernel<2, 2>
                  : c->dp->peers.world <= 4 ? ffn::dp_reduce_apply_kernel<4, 2> : ffn::dp_reduce_apply_kernel<8, 1>;
        kern<<<sms * 4, 256, 0, st>>>(c->dp->peers, table4, total4, lc, epoch, c->status, c->dp->done_counter,
                                      c->dp->wait_limit);
    }
    ++c->launches;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(c, e, "exchange launch");
    // every rank has read this rank's table gradients: clear them for the next step
    if ((e = cudaMemsetAsync(c->grads, 0, c->table_floats * sizeof(float), st)) != cudaSuccess)
        return cuda_fail(c, e, "gradient clear");
    return FFN_OK;
}

int ffn_dp_set_wait_limit(ffn_ctx* c, uint32_t polls) {
    if (!c) return FFN_E_CONFIG;
    if (!c->dp) return fail(c, FFN_E_STATE, "ffn_dp_ipc_handles must be called first");
    if (polls == 0) return fail(c, FFN_E_CONFIG, "the wait limit must be at least one poll");
    c->dp->wait_limit = polls;
    return FFN_OK;
}

int ffn_adam(float* p, const float* g, float* m, float* v, int64_t n, float lr_t, float b1, float b2,
             float eps, void* stream) {
    if (n <= 0) return FFN_OK;
    if (!p || !g || !m || !v) return FFN_E_CONFIG;
    if (!aligned16(p) || !aligned16(g) || !aligned16(m) || !aligned16(v)) return FFN_E_CONFIG;
    const int64_t n4 = (n + 3) / 4;
    const int blocks = grid_for((uint64_t)n4, 256, 16);
    adam_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p, g, m, v, n, lr_t, b1, b2, eps);
    return cudaGetLastError() == cudaSuccess ? FFN_OK : FFN_E_CUDA;
}

}  // extern "C"

#include "ffn_noalloc.cu"
#include "ffn_probe.cu"
