// ffn_probe.cu -- achievable rates of random 8-byte accesses on this GPU (no reference
// counterpart).  Included into ffn_capi.cu's translation unit.
//
// The hash-grid encode and its gradient scatter are not bandwidth-bound in the streaming sense:
// every trilinear corner is an independent 8-byte load (F = 2: a float2) from a random table
// entry, and every gradient corner an independent 8-byte vector reduction (red.global.add.v2.f32).
// Each such access moves a 32-byte sector through L1/L2 (and from HBM when the table does not fit
// L2), so the copy bandwidth is not an attainable ceiling for them.  These two kernels measure the
// ceiling that is: the rate of fully random float2 loads (read-only path, like the encoders) and of
// fully random float2 reductions over a buffer of a given size, with every thread keeping eight
// independent accesses in flight.  Rates for an L2-resident buffer (the 67 MB cfg3 table) and an
// HBM-resident one (537 MB) bound the encode and scatter kernels from above; their fraction of it is
// the roofline figure the benchmark reports beside the HBM fraction.
namespace ffn {

constexpr int PROBE_ILP = 8;

__device__ __forceinline__ uint32_t probe_index(uint32_t seed, uint64_t op, uint32_t mask) {
    return hash_u32(seed ^ (uint32_t)op ^ (uint32_t)(op >> 32) * 0x9E3779B9u) & mask;
}

// sink[0] receives a thread's sum only when it equals a value no sum takes (keeps the loads live).
__global__ void __launch_bounds__(256) probe_gather_kernel(const float2* __restrict__ buf, uint32_t mask,
                                                           uint64_t n_ops, uint32_t seed, float* __restrict__ sink) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    float acc = 0.0f;
    for (uint64_t base = tid * PROBE_ILP; base < n_ops; base += stride * PROBE_ILP) {
        float2 v[PROBE_ILP];
#pragma unroll
        for (int k = 0; k < PROBE_ILP; ++k)
            v[k] = base + k < n_ops ? __ldg(buf + probe_index(seed, base + k, mask)) : make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < PROBE_ILP; ++k) acc += v[k].x + v[k].y;
    }
    if (acc == -1.2345e-38f) sink[0] = acc;
}

__global__ void __launch_bounds__(256) probe_red_kernel(float* __restrict__ buf, uint32_t mask, uint64_t n_ops,
                                                        uint32_t seed) {
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t base = tid * PROBE_ILP; base < n_ops; base += stride * PROBE_ILP) {
#pragma unroll
        for (int k = 0; k < PROBE_ILP; ++k)
            if (base + k < n_ops) red_add2(buf + 2 * (size_t)probe_index(seed, base + k, mask), 1.0e-30f, 1.0e-30f);
    }
}

}  // namespace ffn

extern "C" int ffn_probe_random_access(void* buf, size_t bytes, int mode, uint64_t n_ops, uint32_t seed,
                                       void* stream) {
    if (!buf || bytes < 8) return fail(nullptr, FFN_E_CONFIG, "need a device buffer of at least 8 bytes");
    if (mode != 0 && mode != 1) return fail(nullptr, FFN_E_CONFIG, "mode must be 0 (gather) or 1 (reduction)");
    if (!aligned16(buf)) return fail(nullptr, FFN_E_CONFIG, "buf must be 16-byte aligned");
    uint64_t entries = bytes / 8;
    if (entries > (1ull << 31)) entries = 1ull << 31;
    uint32_t mask = 1u;
    while ((uint64_t)mask * 2u <= entries) mask *= 2u;     // largest power of two <= entries
    mask -= 1u;
    if (n_ops == 0) return FFN_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int blocks = grid_for((n_ops + ffn::PROBE_ILP - 1) / ffn::PROBE_ILP, 256, 8);
    if (mode == 0)
        ffn::probe_gather_kernel<<<blocks, 256, 0, st>>>(static_cast<const float2*>(buf), mask, n_ops, seed,
                                                          static_cast<float*>(buf));
    else
        ffn::probe_red_kernel<<<blocks, 256, 0, st>>>(static_cast<float*>(buf), mask, n_ops, seed);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FFN_OK : cuda_fail(nullptr, e, "probe launch");
}
