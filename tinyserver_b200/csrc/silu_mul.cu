// SiLU-and-mul: out = rnd(rnd(silu(gate)) * up).
//
// Replaces Qwen3MLP's `act_fn(gate_proj(x)) * up_proj(x)` (transformers 5.5.0
// modeling_qwen3.py:82), which the reference runs as two eager kernels (silu,
// then mul: 3 reads + 2 writes of T*I elements).  One pass here: 2 reads and
// 1 write, 16-byte vectors, streaming cache hints.
//
// torch's silu is x / (1 + exp(-x)) in fp32, rounded to the dtype.  For 16-bit
// dtypes the kernel evaluates it with the hardware exp2 unit (__expf) and the
// fast divide: their error (a few fp32 ulp) is far below the bf16/fp16
// rounding that follows, and the full-precision path would make the kernel
// ALU-bound at B200 bandwidth.  fp32 keeps expf and the IEEE divide.
#include "qf_common.cuh"

namespace qf {
namespace {

struct SiluArgs {
    const char* gate;
    int64_t gs;
    const char* up;
    int64_t us;
    char* out;
    int64_t os;
    int64_t rows, I;
};

template <typename T>
__device__ __forceinline__ float silu(float g) {
    return __fdividef(g, 1.0f + __expf(-g));
}
template <>
__device__ __forceinline__ float silu<float>(float g) {
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}

// rnd(rnd(silu(g)) * u) on one 16-byte vector; 16-bit types multiply with a
// packed .rn op (the product of two 16-bit values is exact in fp32, so one
// rounding is what torch's mul does).
template <typename T>
__device__ __forceinline__ uint4 silu_mul16(const uint4& g, const uint4& u) {
    uint4 r;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t gw = word(g, i);
        if constexpr (sizeof(T) == 2) {
            using P = Packed<T>;
            set_word(r, i, P::mul(P::pack(silu<T>(P::lo(gw)), silu<T>(P::hi(gw))), word(u, i)));
        } else {
            set_word(r, i, __float_as_uint(__fmul_rn(silu<T>(__uint_as_float(gw)),
                                                     __uint_as_float(word(u, i)))));
        }
    }
    return r;
}

// blockIdx.x enumerates (row, chunk); a chunk is blockDim.x * VPT vectors.
template <typename T, int VPT>
__global__ void __launch_bounds__(256) silu_mul_vec_kernel(const SiluArgs a, const int64_t nvec,
                                                           const int64_t chunks) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x / chunks;
    const int64_t chunk = blockIdx.x - row * chunks;
    const char* g = a.gate + row * a.gs * (int64_t)sizeof(T);
    const char* u = a.up + row * a.us * (int64_t)sizeof(T);
    char* o = a.out + row * a.os * (int64_t)sizeof(T);
    const int64_t v0 = chunk * (int64_t)blockDim.x * VPT + threadIdx.x;
    uint4 gv[VPT], uv[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int64_t v = v0 + (int64_t)j * blockDim.x;
        if (v < nvec) {
            gv[j] = ld_stream16(g + v * 16);
            uv[j] = ld_stream16(u + v * 16);
        }
    }
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int64_t v = v0 + (int64_t)j * blockDim.x;
        if (v < nvec) st_stream16(o + v * 16, silu_mul16<T>(gv[j], uv[j]));
    }
}

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_scalar_kernel(const SiluArgs a) {
    const int64_t total = a.rows * a.I;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / a.I, c = i - r * a.I;
        const float g = Dt<T>::to_f(reinterpret_cast<const T*>(a.gate)[r * a.gs + c]);
        const float u = Dt<T>::to_f(reinterpret_cast<const T*>(a.up)[r * a.us + c]);
        reinterpret_cast<T*>(a.out)[r * a.os + c] =
            Dt<T>::from_f(__fmul_rn(rnd<T>(silu<T>(g)), u));
    }
}

template <typename T>
int dispatch(const SiluArgs& a, cudaStream_t stream) {
    constexpr int EPV = Dt<T>::kPerVec;
    constexpr int VPT = 2;
    const int64_t es = sizeof(T);
    const bool vec = a.I % EPV == 0 && aligned16(a.gate) && aligned16(a.up) &&
                     aligned16(a.out) && (a.gs * es) % 16 == 0 && (a.us * es) % 16 == 0 &&
                     (a.os * es) % 16 == 0;
    if (vec) {
        const int64_t nvec = a.I / EPV;
        const int threads = (int)std::min<int64_t>(256, ceil_div(ceil_div(nvec, VPT), 32) * 32);
        const int64_t chunks = ceil_div(nvec, (int64_t)threads * VPT);
        const int64_t blocks = a.rows * chunks;
        if (blocks <= 0x7fffffffLL) {
            return launch_pdl(silu_mul_vec_kernel<T, VPT>, (unsigned)blocks, threads, 0, stream,
                              a, nvec, chunks);
        }
    }
    const int64_t blocks =
        std::min<int64_t>(ceil_div(a.rows * a.I, 256), (int64_t)sm_count() * 32);
    silu_mul_scalar_kernel<T><<<(unsigned)blocks, 256, 0, stream>>>(a);
    return check_launch();
}

}  // namespace
}  // namespace qf

extern "C" int qf_silu_and_mul(const void* gate, int64_t gate_row_stride, const void* up,
                               int64_t up_row_stride, void* out, int64_t out_row_stride,
                               int64_t num_rows, int64_t intermediate, int dtype,
                               cudaStream_t stream) {
    if (num_rows < 0 || intermediate < 0) return QF_ERR_INVALID;
    if (num_rows == 0 || intermediate == 0) return QF_OK;
    if (!gate || !up || !out) return QF_ERR_INVALID;
    qf::SiluArgs a{static_cast<const char*>(gate), gate_row_stride,
                   static_cast<const char*>(up),   up_row_stride,
                   static_cast<char*>(out),        out_row_stride,
                   num_rows,                       intermediate};
    switch (dtype) {
    case QF_F32: return qf::dispatch<float>(a, stream);
    case QF_F16: return qf::dispatch<__half>(a, stream);
    case QF_BF16: return qf::dispatch<__nv_bfloat16>(a, stream);
    default: return QF_ERR_INVALID;
    }
}
