// ffn_tcgen05.cuh -- the sm_100a tensor-core primitives the fused MLP uses (inline PTX).
//
// Shared-memory operand layout ("core-matrix interleaved", no swizzle): a tile of R rows x C
// columns of 16-bit values is stored as 8x8 core matrices of 128 contiguous bytes,
//     byte(r, c) = (r / 8) * SBO + (c / 8) * 128 + (r % 8) * 16 + (c % 8) * 2,  SBO = (C / 8) * 128.
// The same bytes describe the tile
//   * K-major   (rows = M or N, columns = K): LBO = 128 (next 8 columns), SBO = (C/8)*128, and
//   * MN-major  (columns = M or N, rows = K): SBO = 128 (next 8 columns), LBO = (C/8)*128,
// so one copy of an activation tile [sample][feature] feeds the forward GEMM (K = feature), the
// backward-data GEMM and the weight-gradient GEMM (K = sample) without a transposed copy.
//
// Matrix descriptor (64 bit): start address >> 4 in [0,14), LBO >> 4 in [16,30), SBO >> 4 in
// [32,46), version 1 in [46,48), layout type 0 (no swizzle) in [61,64).
// Instruction descriptor (kind::f16): D format F32 at [4,6), A/B format F16 at [7,10)/[10,13),
// A/B major (0 = K, 1 = MN) at bit 15/16, N >> 3 at [17,23), M >> 4 at [24,29).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace ffn {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Descriptor of a tile with `cols` columns, K-major (K runs along the columns).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr, int cols) {
    return make_desc(saddr, 128u, (uint32_t)(cols / 8) * 128u);
}
// Descriptor of the same tile read MN-major (M or N runs along the columns, K along the rows).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr, int cols) {
    return make_desc(saddr, (uint32_t)(cols / 8) * 128u, 128u);
}

__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// Byte offset of element (r, c) in a tile with `cols` columns.
__device__ __forceinline__ uint32_t tile_off(int r, int c, int cols) {
    return (uint32_t)((r >> 3) * (cols >> 3) * 128 + (c >> 3) * 128 + (r & 7) * 16 + (c & 7) * 2);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one instruction (issued by one thread).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        :
        : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void commit(uint64_t* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(mbar)) : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(mbar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Waits for the mbarrier phase `parity` to complete; gives up after `limit` polls and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, uint32_t limit) {
    const uint32_t a = smem_u32(mbar);
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// TMEM allocation by one full warp; the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (warp w reads lanes 32w..32w+31).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Saturating fp32 -> fp16 (keeps +-65504 instead of producing inf).
__device__ __forceinline__ __half to_half_sat(float x) {
    return __float2half_rn(fminf(fmaxf(x, -65504.0f), 65504.0f));
}

// Two fp32 values -> one packed fp16 pair (x0 in the low half), rounded to nearest even; magnitudes
// above 65504 saturate to +-65504, a NaN stays NaN.  One conversion instruction for both values.
__device__ __forceinline__ uint32_t pack_half2_sat(float x0, float x1) {
    uint32_t r;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    return r;
}
__device__ __forceinline__ float2 unpack_half2(uint32_t h) {
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Stores 8 values as one 16-byte core-matrix row chunk.
__device__ __forceinline__ void st_chunk8(unsigned char* tile, int r, int c0, int cols, const float* v) {
    uint4 h;
    h.x = pack_half2_sat(v[0], v[1]);
    h.y = pack_half2_sat(v[2], v[3]);
    h.z = pack_half2_sat(v[4], v[5]);
    h.w = pack_half2_sat(v[6], v[7]);
    *reinterpret_cast<uint4*>(tile + tile_off(r, c0, cols)) = h;
}
// Stores 8 values as a compensated pair of fp16 chunks: hi = fp16(x) into `hi_tile`, lo = fp16(x - hi)
// into `lo_tile` (same position), so that hi + lo carries about 22 significant bits.  A product
// with an operand pair is formed as hi*hi' + hi*lo' + lo*hi' (the split-fp16 scheme of Markidis et
// al., "NVIDIA Tensor Core Programmability, Performance & Precision", IPDPSW 2018, and Ootomo &
// Yokota, "Recovering single-precision accuracy from Tensor Cores while surpassing the FP32
// theoretical peak", IJHPCA 2022); the lo*lo' term is below fp32 rounding and is left out.
__device__ __forceinline__ void st_chunk8_hilo(unsigned char* hi_tile, unsigned char* lo_tile, int r, int c0, int cols,
                                               const float* v) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        h[i] = pack_half2_sat(v[2 * i], v[2 * i + 1]);
        const float2 b = unpack_half2(h[i]);
        l[i] = pack_half2_sat(v[2 * i] - b.x, v[2 * i + 1] - b.y);
    }
    const uint32_t off = tile_off(r, c0, cols);
    *reinterpret_cast<uint4*>(hi_tile + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_tile + off) = make_uint4(l[0], l[1], l[2], l[3]);
}
__device__ __forceinline__ void ld_chunk8(const unsigned char* tile, int r, int c0, int cols, float* v) {
    uint4 u = *reinterpret_cast<const uint4*>(tile + tile_off(r, c0, cols));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

}  // namespace tc
}  // namespace ffn
