// Shared device helpers of libqwen3fused: dtype traits with the rounding rule
// of each storage type, 16-byte streaming loads/stores, launch bookkeeping.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

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
// 16-byte global memory access.  Streamed data (read once) is read through
// the non-coherent read-only path with no cache hint: on B200 the c4 step ran
// 242.7 us with L1::no_allocate + L2::256B on these loads and 235.4 us
// without (every kernel faster; L1::evict_first measured like no_allocate).
// Streamed outputs are marked evict-first.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint2 ld_stream8(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];"
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

// ---------------------------------------------------------------------------
// Two 16-bit values in one 32-bit register (element 0 in the low half, as in
// memory).  The arithmetic is the IEEE round-to-nearest op of the storage
// type with an explicit .rn (never contracted into an FMA), and it equals
// torch's "compute in fp32, round to the dtype" for these operands:
//  * a product of two bf16 (8-bit significands) or two fp16 (11-bit) values
//    is exact in fp32, so rounding it once is what torch's mul does;
//  * a sum of two such values is exact in fp32 unless their exponents differ
//    by more than 24 - p bits; then the smaller one lies far below half an
//    ulp of the larger, so the fp32 rounding cannot move the sum across a
//    rounding midpoint of the 16-bit type and double rounding changes nothing.
template <typename T>
struct Packed;

template <>
struct Packed<__nv_bfloat16> {
    __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    // round two floats to the storage type and pack them (lo at the low half)
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        uint32_t d;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
        return d;
    }
    __device__ __forceinline__ static float lo(uint32_t v) { return __uint_as_float(v << 16); }
    __device__ __forceinline__ static float hi(uint32_t v) {
        return __uint_as_float(v & 0xffff0000u);
    }
};

template <>
struct Packed<__half> {
    __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        uint32_t d;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
        return d;
    }
    __device__ __forceinline__ static float lo(uint32_t v) {
        return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu)));
    }
    __device__ __forceinline__ static float hi(uint32_t v) {
        return __half2float(__ushort_as_half((unsigned short)(v >> 16)));
    }
};

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ void set_word(uint4& v, int i, uint32_t w) {
    if (i == 0) v.x = w;
    else if (i == 1) v.y = w;
    else if (i == 2) v.z = w;
    else v.w = w;
}

// Sum of squares of the elements of one 16-byte vector (fp32 accumulation).
template <typename T>
__device__ __forceinline__ float sum_sq16(const uint4& v) {
    float s = 0.f;
    if constexpr (sizeof(T) == 2) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float lo = Packed<T>::lo(word(v, i)), hi = Packed<T>::hi(word(v, i));
            s = fmaf(lo, lo, s);
            s = fmaf(hi, hi, s);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float f = __uint_as_float(word(v, i));
            s = fmaf(f, f, s);
        }
    }
    return s;
}

// Elementwise rnd(a + b) of two 16-byte vectors (torch's same-dtype add).
template <typename T>
__device__ __forceinline__ uint4 add16(const uint4& a, const uint4& b) {
    uint4 r;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (sizeof(T) == 2)
            set_word(r, i, Packed<T>::add(word(a, i), word(b, i)));
        else
            set_word(r, i, __float_as_uint(__fadd_rn(__uint_as_float(word(a, i)),
                                                     __uint_as_float(word(b, i)))));
    }
    return r;
}

// Qwen3RMSNorm's scaling of one 16-byte vector: rnd(w * rnd(h * inv)).
template <typename T>
__device__ __forceinline__ uint4 norm16(const uint4& h, float inv, const uint4& w) {
    uint4 r;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t hv = word(h, i);
        if constexpr (sizeof(T) == 2) {
            using P = Packed<T>;
            set_word(r, i, P::mul(P::pack(__fmul_rn(P::lo(hv), inv), __fmul_rn(P::hi(hv), inv)),
                                  word(w, i)));
        } else {
            set_word(r, i, __float_as_uint(__fmul_rn(__uint_as_float(word(w, i)),
                                                     __fmul_rn(__uint_as_float(hv), inv))));
        }
    }
    return r;
}

// Resident CTAs per SM of one kernel at one block size and dynamic shared
// memory size, cached per kernel (fixed for a process on one architecture).
template <auto Kernel>
int resident_ctas(int threads, size_t smem = 0) {
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, int> cache;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find({threads, smem});
        if (it != cache.end()) return it->second;
    }
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, Kernel, threads, smem) != cudaSuccess ||
        v < 1)
        v = 1;
    std::lock_guard<std::mutex> lock(mu);
    cache[{threads, smem}] = v;
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
// Programmatic dependent launch (sm_90+).  The hot-path kernels are launched
// with programmatic stream serialization: the next kernel in the stream may be
// launched -- its CTAs scheduled onto SMs as the previous kernel's retire --
// before the previous one has finished.  Every kernel launched that way calls
// pdl_wait() before its first access to memory that earlier work in the
// stream may still write, which blocks until the preceding grid has completed
// and its writes are visible, so the overlap is only launch latency, CTA
// rasterisation and loads of inputs known to be final, never data that is in
// flight.  pdl_trigger()
// allows the following grid to begin launching.
#ifndef QF_PDL
#define QF_PDL 1
#endif

__device__ __forceinline__ void pdl_wait() {
#if QF_PDL
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

__device__ __forceinline__ void pdl_trigger() {
#if QF_PDL
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
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

// Launch a kernel that calls pdl_wait() before touching global memory, with
// programmatic stream serialization (see pdl_wait).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, unsigned block, size_t smem,
               cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = QF_PDL;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
    return e == cudaSuccess ? QF_OK : launch_failed(e);
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace qf
