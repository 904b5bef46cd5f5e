// clemu.h -- TEST INFRASTRUCTURE ONLY.
//
// A minimal OpenCL C 1.2 execution layer for the CPU, just large enough to compile the
// reference's three .cl files (after the mechanical rewrite in ref_build.py) as C++ and run them
// with real work-group semantics:
//   * every work-item is a fiber with its own stack; barrier() switches to the next fiber of
//     the work-group, so all work-items reach barrier k before any passes it;
//   * __local variables become thread_local statics, shared by the fibers of the work-group
//     that runs on this OS thread;
//   * vector types float3/float4 with the operators, swizzle (.xyz) and builtins the kernels use;
//   * atomics map to GCC __atomic builtins (work-groups may run on several OS threads).
// Math builtins map to the C library (exp -> expf, powr -> powf, native_sqrt -> sqrtf,
// rsqrt -> 1/sqrtf, length -> sqrtf(x*x+y*y+z*z)).
#pragma once
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <functional>

namespace clemu {

typedef unsigned int uint;
typedef unsigned long ulong;
typedef unsigned char uchar;
typedef _Float16 half;     // cl_khr_fp16 storage type (the fp16 transfer format)
inline half convert_half_rte(float x) { return (half)x; }   // IEEE round to nearest even
inline float convert_float(half h) { return (float)h; }

// ----------------------------------------------------------------- vector types
struct float3 { float x, y, z, w_; };
struct float4 {
    float x, y, z, w;
    float3 xyz() const { return float3{x, y, z, 0.0f}; }
};
inline float3 f3_make(float a, float b, float c) { return float3{a, b, c, 0.0f}; }
inline float3 f3_bcast(float a) { return float3{a, a, a, 0.0f}; }
inline float4 f4_bcast(float a) { return float4{a, a, a, a}; }
inline float3 operator+(float3 a, float3 b) { return f3_make(a.x + b.x, a.y + b.y, a.z + b.z); }
inline float3 operator-(float3 a, float3 b) { return f3_make(a.x - b.x, a.y - b.y, a.z - b.z); }
inline float3 operator*(float3 a, float3 b) { return f3_make(a.x * b.x, a.y * b.y, a.z * b.z); }
inline float3 operator/(float3 a, float3 b) { return f3_make(a.x / b.x, a.y / b.y, a.z / b.z); }
inline float3 operator*(float s, float3 a) { return f3_make(s * a.x, s * a.y, s * a.z); }
inline float3 operator*(float3 a, float s) { return f3_make(a.x * s, a.y * s, a.z * s); }
inline float3 operator/(float3 a, float s) { return f3_make(a.x / s, a.y / s, a.z / s); }
inline float3 operator+(float3 a, float s) { return f3_make(a.x + s, a.y + s, a.z + s); }
inline float3 operator-(float3 a, float s) { return f3_make(a.x - s, a.y - s, a.z - s); }

// ----------------------------------------------------------------- scalar builtins
inline float fmin(float a, float b) { return std::fmin(a, b); }
inline float fmax(float a, float b) { return std::fmax(a, b); }
inline float3 fmin(float3 a, float3 b) { return f3_make(std::fmin(a.x, b.x), std::fmin(a.y, b.y), std::fmin(a.z, b.z)); }
inline float3 fmax(float3 a, float3 b) { return f3_make(std::fmax(a.x, b.x), std::fmax(a.y, b.y), std::fmax(a.z, b.z)); }
inline float clamp(float x, float lo, float hi) { return std::fmin(std::fmax(x, lo), hi); }
inline int clamp(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }
inline uint clamp(uint x, uint lo, uint hi) { return x < lo ? lo : (x > hi ? hi : x); }
inline float3 clamp(float3 v, float lo, float hi) { return f3_make(clamp(v.x, lo, hi), clamp(v.y, lo, hi), clamp(v.z, lo, hi)); }
inline float mix(float a, float b, float t) { return a + (b - a) * t; }
inline float floor(float x) { return std::floor(x); }
inline float rint(float x) { return std::rint(x); }
inline float fabs(float x) { return std::fabs(x); }
inline float sqrt(float x) { return std::sqrt(x); }
inline float native_sqrt(float x) { return std::sqrt(x); }
inline float rsqrt(float x) { return 1.0f / std::sqrt(x); }
inline float exp(float x) { return std::exp(x); }
inline float log1p(float x) { return std::log1p(x); }
inline float pow(float x, float y) { return std::pow(x, y); }
inline float powr(float x, float y) { return std::pow(x, y); }
inline float fma(float a, float b, float c) { return std::fma(a, b, c); }
inline float copysign(float a, float b) { return std::copysign(a, b); }
inline float frexp(float x, int* e) { return std::frexp(x, e); }
inline float ldexp(float x, int e) { return std::ldexp(x, e); }
inline bool isfinite(float x) { return std::isfinite(x); }
inline float length(float3 v) { return std::sqrt(v.x * v.x + v.y * v.y + v.z * v.z); }
inline uint popcount(uint x) { return (uint)__builtin_popcount(x); }

inline float as_float(int i) { float f; std::memcpy(&f, &i, 4); return f; }
inline float as_float(uint i) { float f; std::memcpy(&f, &i, 4); return f; }
inline int as_int(uint u) { int i; std::memcpy(&i, &u, 4); return i; }
inline int as_int(float f) { int i; std::memcpy(&i, &f, 4); return i; }
inline uint as_uint(float f) { uint u; std::memcpy(&u, &f, 4); return u; }
inline uint as_uint(int i) { uint u; std::memcpy(&u, &i, 4); return u; }

inline int atomic_cmpxchg(volatile int* p, int cmp, int val) {
    int expected = cmp;
    __atomic_compare_exchange_n((int*)p, &expected, val, false, __ATOMIC_SEQ_CST, __ATOMIC_SEQ_CST);
    return expected;
}
inline int atomic_or(volatile int* p, int val) {
    return __atomic_fetch_or((int*)p, val, __ATOMIC_SEQ_CST);
}

// ----------------------------------------------------------------- work-group runtime
enum { CLK_LOCAL_MEM_FENCE = 1, CLK_GLOBAL_MEM_FENCE = 2 };

struct WorkGroup;
struct Fiber {
    void* sp = nullptr;
    char* stack = nullptr;
    bool done = false;
};

constexpr int kMaxLocals = 64;    // __local variables per kernel

struct WorkGroup {
    int n = 0;
    size_t group_id[2] = {0, 0}, local_size[2] = {1, 1};
    int cur = 0;
    void* sched_sp = nullptr;
    Fiber* fibers = nullptr;
    std::function<void()> body;
    void* locals[kMaxLocals] = {};  // this group's __local memory, one block per declaration
    void free_locals() {
        for (void*& p : locals) { std::free(p); p = nullptr; }
    }
};

extern thread_local WorkGroup* tls_wg;

// The __local variable `id` of the running work-group: zeroed on the group's first use, then shared
// by its work-items (ref_build.py rewrites each __local declaration into a reference to it).
template <typename T>
T& local_ref(int id) {
    void*& p = tls_wg->locals[id];
    if (!p) p = std::calloc(1, sizeof(T));
    return *reinterpret_cast<T*>(p);
}

inline size_t get_group_id(int d) { return tls_wg->group_id[d]; }
inline size_t get_local_size(int d) { return tls_wg->local_size[d]; }
inline size_t get_local_id(int d) {
    return d == 0 ? (size_t)tls_wg->cur % tls_wg->local_size[0] : (size_t)tls_wg->cur / tls_wg->local_size[0];
}
inline size_t get_global_id(int d) { return tls_wg->group_id[d] * tls_wg->local_size[d] + get_local_id(d); }
void barrier(int flags);

// Runs `body` once per work-item of a (lx * ly)-item work-group with ids (gx, gy).
void run_work_group(size_t gx, size_t gy, size_t lx, size_t ly, const std::function<void()>& body);

// Runs work-groups 0 .. n_groups-1 (lx work-items each) in lockstep: every work-item of every group
// reaches barrier k before any passes it, as on a device that holds all the groups at once.  The
// groups are spread over n_threads OS threads that meet at a thread barrier after every barrier
// interval.
void run_work_groups_lockstep(size_t n_groups, size_t lx, const std::function<void()>& body, int n_threads);

}  // namespace clemu
