// ffn_dp.cu -- the data-parallel exchange of the deferred step as one kernel over NVLink peer
// memory: gradient reduction across ranks fused with the table SGD step and the broadcast of the
// updated table.  Included into ffn_capi.cu's translation unit.
//
// Every rank owns a contiguous shard (in float4 units) of the gradient buffer [table | MLP].  For
// each float4 of its shard it loads the W ranks' gradients over NVLink (plain peer loads), sums
// them in rank order, and
//   * table part: applies table += coef_l * g (the reference's SGD step, ffnerf_OG.cl:2155-2168)
//     and stores the new value into every rank's table (peer stores);
//   * MLP part: stores the summed gradient into every rank's MLP gradient, for the local Adam.
// That is a reduce-scatter, the SGD update of the shard and an all-gather in one pass: each byte of
// table crosses NVLink once in each direction.  The table part of every rank's gradient buffer is
// cleared locally (ffn_dp_reduce_apply, after the kernel) once every rank has read it.
//
// Ordering between ranks uses flag words in each rank's own memory (IPC-mapped by the peers):
//   entry: block 0 of rank r stores epoch into slot r of every rank's entry flags (release, system
//          scope), then every block waits until all W entry slots of its own rank reach epoch
//          (acquire), i.e. every rank's gradients are complete;
//   exit:  the last block of rank r to finish stores epoch into slot r of every rank's exit flags,
//          then waits until all W exit slots reach epoch, so that no rank's next step reads a
//          table or writes a gradient buffer that a peer is still reading or writing.
// Every wait is bounded (wait_limit polls of about 1 us each, DP_WAIT_LIMIT_DEFAULT unless the
// caller set another with ffn_dp_set_wait_limit); a wait that runs out sets status bit 8 and the
// kernel skips its work, so no rank can hang the others.  After a timeout the ranks' epochs no
// longer agree: the exchange is not used again until the ranks re-attach.
#include <cuda_runtime.h>

namespace ffn {

constexpr int DP_MAX_RANKS = 8;
constexpr uint32_t DP_WAIT_LIMIT_DEFAULT = 1u << 24;   // polls of ~1 us each (~16 s) before giving up

struct DpPeers {
    float* grads[DP_MAX_RANKS];      // every rank's gradient buffer (this rank's included)
    float* table[DP_MAX_RANKS];      // every rank's table
    uint32_t* flags[DP_MAX_RANKS];   // every rank's flag words: [0, W) entry, [W, 2W) exit
    int rank, world;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until flags[first .. first + n) all reach epoch (wrap-safe compare).
__device__ __forceinline__ bool dp_wait(const uint32_t* flags, int first, int n, uint32_t epoch, uint32_t limit) {
    for (uint32_t it = 0; it < limit; ++it) {
        bool all = true;
        for (int k = 0; k < n; ++k) all &= (int32_t)(ld_acquire_sys(flags + first + k) - epoch) >= 0;
        if (all) return true;
        __nanosleep(1000);
    }
    return false;
}

// U float4 of the shard per thread and iteration, all of their loads (every rank's gradients and
// the local table) issued before any sum, so that U * (W + 1) loads are in flight per thread; WMAX
// bounds the ranks the registers are sized for.
template <int WMAX, int U>
__global__ void __launch_bounds__(256, 4) dp_reduce_apply_kernel(const DpPeers P, uint32_t table4, uint32_t total4,
                                                                 const LevelCoef lc, uint32_t epoch, int* status,
                                                                 unsigned int* done_counter, uint32_t wait_limit) {
    __shared__ int ok;
    const int W = P.world, r = P.rank;
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0) {
            __threadfence_system();
            for (int p = 0; p < W; ++p) st_release_sys(P.flags[p] + r, epoch);
        }
        ok = dp_wait(P.flags[r], 0, W, epoch, wait_limit) ? 1 : 0;
        if (!ok) atomicOr(status, ST_DP_TIMEOUT);
    }
    __syncthreads();
    if (ok) {
        const uint32_t per = (total4 + (uint32_t)W - 1) / (uint32_t)W;
        const uint32_t lo = (uint32_t)r * per;
        const uint32_t hi = lo + per < total4 ? lo + per : total4;
        const uint32_t S = gridDim.x * blockDim.x;
        for (uint32_t i0 = lo + blockIdx.x * blockDim.x + threadIdx.x; i0 < hi; i0 += U * S) {
            float4 g[U][WMAX], t[U];
            bool has[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t i = i0 + (uint32_t)u * S;
                has[u] = i < hi;
                t[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (!has[u]) continue;
#pragma unroll
                for (int p = 0; p < WMAX; ++p)
                    if (p < W) g[u][p] = reinterpret_cast<const float4*>(P.grads[p])[i];
                if (i < table4) t[u] = reinterpret_cast<const float4*>(P.table[r])[i];
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (!has[u]) continue;
                const uint32_t i = i0 + (uint32_t)u * S;
                float4 s = g[u][0];
#pragma unroll
                for (int p = 1; p < WMAX; ++p)
                    if (p < W) { s.x = fa(s.x, g[u][p].x); s.y = fa(s.y, g[u][p].y); s.z = fa(s.z, g[u][p].z); s.w = fa(s.w, g[u][p].w); }
                if (i < table4) {
                    const float cf = lc.coef[level_of(lc, i * 4u)];
                    float4 tv = t[u];
                    tv.x = fa(tv.x, fm(cf, s.x)); tv.y = fa(tv.y, fm(cf, s.y));
                    tv.z = fa(tv.z, fm(cf, s.z)); tv.w = fa(tv.w, fm(cf, s.w));
#pragma unroll
                    for (int p = 0; p < WMAX; ++p)
                        if (p < W) reinterpret_cast<float4*>(P.table[p])[i] = tv;
                } else {
#pragma unroll
                    for (int p = 0; p < WMAX; ++p)
                        if (p < W) reinterpret_cast<float4*>(P.grads[p])[i] = s;
                }
            }
        }
    }
    // exit: the last block of this rank publishes completion and waits for every rank's
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int prev = atomicAdd(done_counter, 1u);
        if (prev == gridDim.x - 1) {
            *done_counter = 0u;
            __threadfence_system();
            for (int p = 0; p < W; ++p) st_release_sys(P.flags[p] + W + r, epoch);
            if (!dp_wait(P.flags[r], W, W, epoch, wait_limit)) atomicOr(status, ST_DP_TIMEOUT);
        }
    }
}

// The same exchange through the NVSwitch (NVLS): the gradient buffer and the table of every rank are
// bound to one multicast object each, so multimem.ld_reduce on the multicast address returns the
// sum over all ranks (the switch adds) and multimem.st writes one value into every rank's copy.
// Each rank moves only its shard once in each direction.  Flags and waits as above.
__device__ __forceinline__ float4 mc_ld_reduce_add(const float* mc) {
    float4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(mc) : "memory");
    return v;
}
__device__ __forceinline__ void mc_st(float* mc, float4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
                 :: "l"(mc), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}

__global__ void __launch_bounds__(256) dp_reduce_apply_nvls_kernel(const DpPeers P, float* mc_grads, float* mc_table,
                                                                   const float* __restrict__ table, uint32_t table4,
                                                                   uint32_t total4, const LevelCoef lc, uint32_t epoch,
                                                                   int* status, unsigned int* done_counter,
                                                                   uint32_t wait_limit) {
    __shared__ int ok;
    const int W = P.world, r = P.rank;
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0) {
            __threadfence_system();
            for (int p = 0; p < W; ++p) st_release_sys(P.flags[p] + r, epoch);
        }
        ok = dp_wait(P.flags[r], 0, W, epoch, wait_limit) ? 1 : 0;
        if (!ok) atomicOr(status, ST_DP_TIMEOUT);
    }
    __syncthreads();
    if (ok) {
        const uint32_t per = (total4 + (uint32_t)W - 1) / (uint32_t)W;
        const uint32_t lo = (uint32_t)r * per;
        const uint32_t hi = lo + per < total4 ? lo + per : total4;
        // two float4 of the shard per thread and iteration, both reductions and table loads in flight
        const uint32_t S = gridDim.x * blockDim.x;
        for (uint32_t i0 = lo + blockIdx.x * blockDim.x + threadIdx.x; i0 < hi; i0 += 2 * S) {
            float4 s[2], t[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const uint32_t i = i0 + (uint32_t)u * S;
                s[u] = t[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i >= hi) continue;
                s[u] = mc_ld_reduce_add(mc_grads + 4 * (size_t)i);
                if (i < table4) t[u] = reinterpret_cast<const float4*>(table)[i];
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const uint32_t i = i0 + (uint32_t)u * S;
                if (i >= hi) continue;
                if (i < table4) {
                    const float cf = lc.coef[level_of(lc, i * 4u)];
                    float4 tv = t[u];
                    tv.x = fa(tv.x, fm(cf, s[u].x)); tv.y = fa(tv.y, fm(cf, s[u].y));
                    tv.z = fa(tv.z, fm(cf, s[u].z)); tv.w = fa(tv.w, fm(cf, s[u].w));
                    mc_st(mc_table + 4 * (size_t)i, tv);
                } else {
                    mc_st(mc_grads + 4 * (size_t)i, s[u]);
                }
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int prev = atomicAdd(done_counter, 1u);
        if (prev == gridDim.x - 1) {
            *done_counter = 0u;
            __threadfence_system();
            for (int p = 0; p < W; ++p) st_release_sys(P.flags[p] + W + r, epoch);
            if (!dp_wait(P.flags[r], W, W, epoch, wait_limit)) atomicOr(status, ST_DP_TIMEOUT);
        }
    }
}

}  // namespace ffn

namespace {

struct DpState {
    ffn::DpPeers peers{};
    float* mc_grads = nullptr;              // multicast addresses (NVLS exchange), or null
    float* mc_table = nullptr;
    uint32_t* flags = nullptr;              // this rank's flag words [2 * world]
    unsigned int* done_counter = nullptr;
    bool opened[ffn::DP_MAX_RANKS] = {};    // which peer mappings this rank opened (and closes)
    uint32_t epoch = 0;
    uint32_t wait_limit = ffn::DP_WAIT_LIMIT_DEFAULT;   // polls per cross-rank wait (ffn_dp_set_wait_limit)
};

}  // namespace
