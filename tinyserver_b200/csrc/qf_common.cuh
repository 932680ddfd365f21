// Shared device helpers of libqwen3fused: dtype traits with the rounding rule
// of each storage type, 16-byte streaming loads/stores, launch bookkeeping.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "qwen3fused.h"

namespace qf {

// ---------------------------------------------------------------------------
// Storage dtypes.  Every op of the reference computes in fp32 and stores its
// result in the tensor dtype; `rnd` is that store-and-reload, so a kernel that
// calls it at the same points as the reference rounds where the reference does.
template <typename T>
struct Dt;

template <>
struct Dt<float> {
    static constexpr int kPerVec = 4;  // elements per 16 bytes
    __device__ __forceinline__ static float to_f(float v) { return v; }
    __device__ __forceinline__ static float from_f(float v) { return v; }
};

template <>
struct Dt<__nv_bfloat16> {
    static constexpr int kPerVec = 8;
    __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <>
struct Dt<__half> {
    static constexpr int kPerVec = 8;
    __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
    __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
};

template <typename T>
__device__ __forceinline__ float rnd(float v) {
    return Dt<T>::to_f(Dt<T>::from_f(v));
}
template <>
__device__ __forceinline__ float rnd<float>(float v) {
    return v;
}

// ---------------------------------------------------------------------------
// 16-byte global memory access.  Streamed data (read once) bypasses L1 and
// asks L2 for a 256-byte prefetch; streamed outputs are marked evict-first.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint2 ld_stream8(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(p));
    return r;
}

// Read-only data shared by many CTAs (weights, tables): normal caching.
__device__ __forceinline__ uint4 ld_shared_ro16(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ void st_stream16(void* p, const uint4& v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void st16(void* p, const uint4& v) {
    *reinterpret_cast<uint4*>(p) = v;
}

// Unpack/pack 16 bytes <-> kPerVec floats.
template <typename T>
__device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < Dt<T>::kPerVec; ++i) f[i] = Dt<T>::to_f(e[i]);
}

template <typename T>
__device__ __forceinline__ uint4 pack(const float* f) {
    uint4 v;
    T* e = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int i = 0; i < Dt<T>::kPerVec; ++i) e[i] = Dt<T>::from_f(f[i]);
    return v;
}

__device__ __forceinline__ int64_t load_index(const void* p, int64_t i, int index_type) {
    return index_type == QF_I64 ? __ldg(reinterpret_cast<const long long*>(p) + i)
                                : (int64_t)__ldg(reinterpret_cast<const int*>(p) + i);
}

__device__ __forceinline__ void flag(int32_t* status, int32_t bits) {
    if (status) atomicOr(reinterpret_cast<int*>(status), bits);
}

// ---------------------------------------------------------------------------
// Host side.
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per-device SM count, cached (device attributes are constant for a process).
int sm_count();

// Record a launch failure for qf_last_cuda_error; returns QF_ERR_LAUNCH.
int launch_failed(cudaError_t e);

// Check the launch that was just issued.
inline int check_launch() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QF_OK : launch_failed(e);
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace qf
