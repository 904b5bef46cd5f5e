// ffn_noalloc.cu -- ffn_forward_backward_noalloc: the fused forward/backward step for callers that
// cannot allocate device memory.  Included into ffn_capi.cu's translation unit (it uses that
// file's config check, error and device-guard helpers and the fused kernels).
//
// Who needs it: code that runs inside another runtime's device-memory budget -- a rendering or
// simulation engine that owns every device allocation through its own pool, or a serving process
// whose memory is reserved up front -- where the library may not call cudaMalloc itself (the
// engine's accounting would not see the memory, and cudaMalloc/cudaFree can synchronise the
// device in the middle of the caller's frame).  Such callers hold the model's buffers themselves
// and pass them in; ffn_create, which allocates, is not for them.
//
// The one piece of memory the step needs beyond its inputs and outputs is the weight-gradient
// partial sums (one row of Pw floats per tile group of the fused kernel, summed in a fixed order
// by reduce_partials).  Here it lives in a file-scope __device__ array of
// FFN_NOALLOC_SCRATCH_BYTES (24 MiB) that every GPU which loads this library holds until the
// process exits.  Its first 256 bytes hold a status word for callers that pass no status output.
#include <mutex>

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)24 << 20;   // FFN_NOALLOC_SCRATCH_BYTES
constexpr size_t NOALLOC_HEADER_BYTES = 256;                 // status word, then the partials
constexpr int NOALLOC_MAX_DEVICES = 64;

// Shared by every call on a device.  In host code this name is a host-side stand-in, not a device
// address: the address kernels use comes from cudaGetSymbolAddress (noalloc_setup).
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

struct NoallocKernel {
    void (*fn)(StepArgs) = nullptr;
    int rows = 0;          // samples per tile
    int threads = 0;       // threads per block
    int groups = 1;        // tiles side by side per block (one partial row each)
    int ctas_per_sm = 1;
    size_t smem = 0;
};

struct NoallocDevice {
    bool ready = false;                 // set-up succeeded; a failed set-up is retried by the next call
    unsigned char* scratch = nullptr;   // device address of g_noalloc_scratch on this device
    int sms = 0;
    int max_smem = 0;                   // opt-in dynamic shared memory per block
};

std::mutex g_noalloc_mu;
NoallocDevice g_noalloc_dev[NOALLOC_MAX_DEVICES];

template <int F, int ND, int NC, int ROWS>
NoallocKernel noalloc_kernel_for(int mlp_precision, int Pw) {
    NoallocKernel k;
    if (mlp_precision == 1) {
        using PL = TcPlan<F, ND>;
        k.fn = fused_step_tc_kernel<F, ND>;
        k.rows = PL::ROWS;
        k.threads = PL::THREADS;
        k.groups = PL::GROUPS;
        k.smem = PL::BYTES;
        k.ctas_per_sm = PL::CTAS_PER_SM;
    } else {
        k.fn = fused_step_kernel<F, ND, NC, ROWS>;
        k.rows = ROWS;
        k.threads = ROWS;
        k.smem = (size_t)Smem<F, ND, NC, ROWS>::floats(Pw) * sizeof(float);
        k.ctas_per_sm = 1;
    }
    return k;
}

// The same (F, ND, NC) -> kernel choice as ffn_create.
bool noalloc_pick(int F, int ND, int NC, int mlp_precision, NoallocKernel* k) {
    if (NC != 2) return false;
    const int Pw = make_param_layout(F, ND, NC).total;
    if (F == 2 && ND == 1) { *k = noalloc_kernel_for<2, 1, 2, 128>(mlp_precision, Pw); return true; }
    if (F == 4 && ND == 1) { *k = noalloc_kernel_for<4, 1, 2, 128>(mlp_precision, Pw); return true; }
    if (F == 2 && ND == 2) { *k = noalloc_kernel_for<2, 2, 2, 64>(mlp_precision, Pw); return true; }
    if (F == 4 && ND == 2) { *k = noalloc_kernel_for<4, 2, 2, 64>(mlp_precision, Pw); return true; }
    return false;
}

// A failed set-up is not remembered: the device stays "not ready" and the next call tries again
// (a transient error, such as a context that was still being created, does not disable the entry
// point for the rest of the process).
int noalloc_setup_fail(char* err, size_t err_size, int code, const char* what, cudaError_t e) {
    snprintf(err, err_size, "%s%s%s", what, e != cudaSuccess ? ": " : "", e != cudaSuccess ? cudaGetErrorString(e) : "");
    return code;
}

// Once per device, with that device current: resolve the scratch array's device address and
// raise the dynamic shared-memory limit of every compiled fused kernel that fits the device.  Runs
// inside the first successful call on each device.
int noalloc_setup(int dev, NoallocDevice** out, char* err, size_t err_size) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoallocDevice& d = g_noalloc_dev[dev];
    *out = &d;
    if (d.ready) return FFN_OK;
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return noalloc_setup_fail(err, err_size, FFN_E_CUDA, "scratch symbol address", e);
    if ((reinterpret_cast<uintptr_t>(p) & 255u) != 0)
        return noalloc_setup_fail(err, err_size, FFN_E_CUDA, "scratch not 256-byte aligned", cudaSuccess);
    int sms = 0, max_smem = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return noalloc_setup_fail(err, err_size, FFN_E_CUDA, "device query", e);
    if ((e = cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
        return noalloc_setup_fail(err, err_size, FFN_E_CUDA, "device query", e);
    const int combos[4][2] = {{2, 1}, {4, 1}, {2, 2}, {4, 2}};
    for (const auto& fd : combos) {
        for (int prec = 0; prec < 2; ++prec) {
            NoallocKernel k;
            noalloc_pick(fd[0], fd[1], 2, prec, &k);
            if ((int)k.smem > max_smem) continue;   // such a kernel is refused per call (FFN_E_CONFIG)
            if ((e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)k.smem)) != cudaSuccess)
                return noalloc_setup_fail(err, err_size, FFN_E_CUDA, "shared-memory attribute", e);
        }
    }
    d.scratch = static_cast<unsigned char*>(p);
    d.sms = sms;
    d.max_smem = max_smem;
    d.ready = true;
    return FFN_OK;
}

}  // namespace

extern "C" int ffn_forward_backward_noalloc(const ffn_config* cfg, const float* params, float* table,
                                            const uint32_t* occ_in, uint32_t* occ_st, const void* rays,
                                            const void* targets, void* out, float* grads, int* status,
                                            uint32_t n, const ffn_step_scalars* s, void* stream) {
    if (!cfg || !s) return fail(nullptr, FFN_E_CONFIG, "null configuration or step scalars");
    std::string why;
    if (check_config(cfg, &why) != FFN_OK) return fail(nullptr, FFN_E_CONFIG, why);
    if (s->spr != 0 && s->spr != 16 && s->spr != 32 && s->spr != 64)
        return fail(nullptr, FFN_E_CONFIG, "samples_per_ray must be 16, 32 or 64 (power of two, <= S_MAX=64)");
    if ((s->flags & FFN_STEP_TABLE_IMMEDIATE) && cfg->table_optimizer != 0)
        return fail(nullptr, FFN_E_CONFIG, "immediate table updates need the SGD table optimizer");
    NoallocKernel k;
    if (!noalloc_pick(cfg->F, cfg->ND, cfg->NC, cfg->mlp_precision, &k))
        return fail(nullptr, FFN_E_CONFIG, "this (F, ND, NC) combination is not compiled: supported are NC=2 with "
                                           "(F, ND) in {(2,1), (4,1), (2,2), (4,2)}");
    if (n == 0) return FFN_OK;
    if (!params || !table || !occ_in || !occ_st || !rays || !targets || !out || !grads)
        return fail(nullptr, FFN_E_CONFIG, "params, table, occupancy grids, rays, targets, out and grads must be device pointers");
    if (!aligned16(rays) || !aligned16(targets) || !aligned16(out))
        return fail(nullptr, FFN_E_CONFIG, "rays/targets/out must be 16-byte aligned");
    if ((uint64_t)n * 64ull >= (1ull << 31)) return fail(nullptr, FFN_E_CAPACITY, "too many rays in one call");

    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "current device");
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(nullptr, FFN_E_CONFIG, "device index beyond 63");
    NoallocDevice* d = nullptr;
    char setup_err[160] = {0};
    const int setup_rc = noalloc_setup(dev, &d, setup_err, sizeof(setup_err));
    if (setup_rc != FFN_OK) return fail(nullptr, setup_rc, setup_err);
    if (k.smem > (size_t)d->max_smem) {
        char msg[160];
        snprintf(msg, sizeof(msg), "the fused kernel for this configuration needs %zu bytes of shared memory per block; "
                 "this device allows %d", k.smem, d->max_smem);
        return fail(nullptr, FFN_E_CONFIG, msg);
    }

    const ParamLayout lo = make_param_layout(cfg->F, cfg->ND, cfg->NC);
    const int spr = s->spr ? (int)s->spr : cfg->spr;
    const int rpt = k.rows / spr;
    const int n_tiles = (int)((n + (uint32_t)rpt - 1) / (uint32_t)rpt);
    const int max_grid = d->sms * k.ctas_per_sm;
    const int blocks = (n_tiles + k.groups - 1) / k.groups;
    const int grid = blocks < max_grid ? blocks : max_grid;
    const int parts = grid * k.groups;
    const size_t need = NOALLOC_HEADER_BYTES + (size_t)parts * lo.total * sizeof(float);
    if (need > NOALLOC_SCRATCH_BYTES) {
        char msg[200];
        snprintf(msg, sizeof(msg), "this call needs %zu bytes of weight-gradient scratch (%d partial rows x %d floats); "
                 "the static scratch holds %zu", need, parts, lo.total, NOALLOC_SCRATCH_BYTES);
        return fail(nullptr, FFN_E_CAPACITY, msg);
    }
    uint64_t entries = 0;
    for (int l = 0; l < L; ++l) entries += 1ull << cfg->level_log2[l];
    const size_t table_floats = (size_t)entries * cfg->F;

    StepArgs a{};
    DevConfig& dc = a.c;
    dc.F = cfg->F; dc.ND = cfg->ND; dc.NC = cfg->NC; dc.spr = spr; dc.G = cfg->G; dc.background = cfg->background;
    for (int l = 0; l < L; ++l) {
        dc.level_log2[l] = cfg->level_log2[l];
        dc.level_offset[l] = cfg->level_offset[l];
        dc.level_res[l] = cfg->level_res[l];
        dc.hash_lr_scale[l] = cfg->hash_lr_scale[l];
    }
    for (int i = 0; i < 3; ++i) { dc.bmin[i] = cfg->box_min[i]; dc.bmax[i] = cfg->box_max[i]; }
    dc.rho_min = cfg->rho_min; dc.rho_max = cfg->rho_max; dc.dt_min = cfg->dt_min; dc.dt_max = cfg->dt_max;
    dc.t_near = cfg->t_near; dc.t_far = cfg->t_far;
    dc.transfer = cfg->transfer_fmt ? cfg->transfer_fmt : 32;
    a.lo = lo;
    a.params = params;
    a.table = table;
    a.occ_in = occ_in;
    a.occ_st = occ_st;
    a.rays = static_cast<const float4*>(rays);
    a.targets = static_cast<const float4*>(targets);
    a.out = static_cast<float4*>(out);
    a.grad_table = grads;
    for (int l = 0; l < L; ++l) a.hash_coef[l] = 1.0f;
    if (s->flags & FFN_STEP_TABLE_IMMEDIATE) {
        a.grad_table = table;
        for (int l = 0; l < L; ++l) a.hash_coef[l] = -(s->lr_f * cfg->hash_lr_scale[l]) * 0.5f;   // HASH_LR_RATE
    }
    float* partials = reinterpret_cast<float*>(d->scratch + NOALLOC_HEADER_BYTES);
    a.partials = partials;
    a.status = status ? status : reinterpret_cast<int*>(d->scratch);
    a.n_rays = n;
    a.ray_offset = s->ray_offset;
    a.sh_mult = s->sh_mult;
    a.occ_strength = s->occ_strength;
    a.seed = s->rng_u32;
    a.do_train = 1;

    // What must start at zero: the gradient output (accumulated by atomics) and the status word.
    // Every partial row the kernel reads back is written in full by its CTA first.
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((e = cudaMemsetAsync(grads, 0, (table_floats + (size_t)lo.total) * sizeof(float), st)) != cudaSuccess)
        return cuda_fail(nullptr, e, "gradient clear");
    if ((e = cudaMemsetAsync(a.status, 0, sizeof(int), st)) != cudaSuccess) return cuda_fail(nullptr, e, "status clear");
    k.fn<<<grid, k.threads, k.smem, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(nullptr, e, "fused step launch");
    reduce_partials<<<(lo.total + 255) / 256, 256, 0, st>>>(partials, parts, lo.total, grads + table_floats, a.status);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(nullptr, e, "gradient reduction launch");
    return FFN_OK;
}
