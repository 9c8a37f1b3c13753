// kvb_common.cuh -- element types, 16-byte vector helpers, reductions and the
// device-side error word shared by every kernel of libkvasir_b200.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "kvasir_b200.h"  // include/ (on the compiler's include path)

namespace kvb {

// ---------------------------------------------------------------- element traits
template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
    static constexpr int kDtype = KVB_BF16;
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
    // two packed elements <-> float2
    static __device__ __forceinline__ float2 unpack(uint32_t u) {
        return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    }
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

template <>
struct Elem<__half> {
    static constexpr int kDtype = KVB_F16;
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ float2 unpack(uint32_t u) {
        __half2 h = *reinterpret_cast<__half2*>(&u);
        return __half22float2(h);
    }
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// 8 elements (16 bytes) <-> 8 floats
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
    float2 a = Elem<T>::unpack(v.x), b = Elem<T>::unpack(v.y);
    float2 c = Elem<T>::unpack(v.z), d = Elem<T>::unpack(v.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
    uint4 v;
    v.x = Elem<T>::pack(f[0], f[1]);
    v.y = Elem<T>::pack(f[2], f[3]);
    v.z = Elem<T>::pack(f[4], f[5]);
    v.w = Elem<T>::pack(f[6], f[7]);
    return v;
}

// Two floats as a packed 16-bit pair `hi` (round to nearest) plus the packed
// 16-bit remainder `lo` = round(x - hi): hi + lo carries ~16 significant bits.
template <typename T>
__device__ __forceinline__ void split_pack(float a, float b, uint32_t& hi, uint32_t& lo) {
    hi = Elem<T>::pack(a, b);
    const float2 h = Elem<T>::unpack(hi);
    lo = Elem<T>::pack(a - h.x, b - h.y);
}

// streaming 16-byte loads/stores (data touched once)
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------- device error word
// Kernels never trap: a bounded wait that gives up, or an argument that a
// kernel finds invalid at run time, ORs a code into this word and the kernel
// returns.  kvb_device_error() reads and clears it.
enum DevError : uint32_t {
    kDevErrWaitTimeout = 1u,   // an mbarrier / TMA wait exceeded its time limit
    kDevErrBadLength = 2u,     // a per-sequence length outside [0, max_len]
    kDevErrBadPosition = 4u,   // a per-sequence position outside the cache / table
    kDevErrSelfTest = 8u,      // the deliberate timeout of kvb_selftest_wait_timeout
};

// All device code of the library is one translation unit (kvb_api.cu), so the
// word is defined here with internal linkage.
static __device__ uint32_t g_dev_error = 0;

__device__ __forceinline__ void raise_dev_error(uint32_t code) { atomicOr(&g_dev_error, code); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- thread-block clusters
// Distributed shared memory: the same variable in CTA `rank` of this cluster.
template <typename T>
__device__ __forceinline__ T dsmem_ld(const T* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(remote)
                 : "r"((uint32_t)__cvta_generic_to_shared(local)), "r"(rank));
    T v;
    static_assert(sizeof(T) == 4, "32-bit values only");
    uint32_t u;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(u) : "r"(remote));
    memcpy(&v, &u, 4);
    return v;
}
// The address of `local` in CTA `rank` of this cluster, and a 32-bit load from such an address.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(remote)
                 : "r"((uint32_t)__cvta_generic_to_shared(local)), "r"(rank));
    return remote;
}
__device__ __forceinline__ uint32_t dsmem_ld_at(uint32_t addr) {
    uint32_t u;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(u) : "r"(addr));
    return u;
}
// Cluster-wide barrier with release / acquire semantics for shared memory.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Time limit of every device-side wait.  Copies finish in microseconds; the
// limit only bounds a wait that would otherwise never end.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

}  // namespace kvb
