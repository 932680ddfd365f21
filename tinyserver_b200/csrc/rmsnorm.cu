// RMSNorm and residual-add + RMSNorm over hidden-size rows.
//
// Replaces Qwen3RMSNorm.forward (transformers 5.5.0 modeling_qwen3.py:59-64)
// and the decoder layer's residual adds (modeling_qwen3.py:327, :333) that
// feed it.  The reference runs ~7 eager kernels per norm (cast, pow, mean,
// add, rsqrt, mul, cast, mul), each a full HBM pass; here one CTA reads each
// row once, keeps it in registers across the block reduction, and writes the
// new residual and the normed row once.
//
// CTAs are persistent (grid = min(rows, resident CTAs)) and keep the weight
// vector in registers for every row they process.  Rounding follows the
// reference op by op: h = rnd(res + x); y = rnd(w * rnd(h * rsqrt(var + eps))).
#include "qf_common.cuh"

// Threads per row for rows up to 4 * QF_RMS_MAX_THREADS 16-byte vectors
// (compile-time knob; rows are split into 1, 2 or 4 vectors per thread).
#ifndef QF_RMS_MAX_THREADS
#define QF_RMS_MAX_THREADS 256
#endif

namespace qf {
namespace {

struct NormArgs {
    const char* x;
    int64_t xs;  // row strides, elements
    const char* res;
    int64_t rs;
    const char* w;
    char* res_out;
    int64_t ros;
    char* out;
    int64_t os;
    int64_t rows;
    int64_t H;
    int64_t nvec;  // H / elements-per-16-bytes
    float eps;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// 1 / sqrt(mean + eps), IEEE-rounded at each step as torch's fp32 ops are.
__device__ __forceinline__ float inv_rms(float sum_sq, int64_t H, float eps) {
    const float var = __fdiv_rn(sum_sq, (float)H);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// One CTA per row at a time, persistent over rows.  Thread i holds vectors
// i, i + nthr, ... of the row (VPT of them) as raw 16-byte words; the weight
// stays in registers for every row.  The next row's loads are issued before
// the current row's block reduction, so a CTA always has a row in flight
// while it reduces, scales and stores the previous one.  16-bit types add and
// scale with packed .rn ops (see Packed): the same roundings as torch's
// separate add, cast and mul kernels.
template <typename T, int VPT, bool ADD>
__global__ void __launch_bounds__(VPT == 8 ? 512 : QF_RMS_MAX_THREADS) rmsnorm_vec_kernel(const NormArgs a) {
    __shared__ float red[2][32];
    const int tid = threadIdx.x;
    const int nthr = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
    constexpr int64_t ES = sizeof(T);
    pdl_wait();
    pdl_trigger();

    uint4 w[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int64_t v = tid + (int64_t)j * nthr;
        w[j] = v < a.nvec ? ld_shared_ro16(a.w + v * 16) : make_uint4(0, 0, 0, 0);
    }

    uint4 xr[VPT], rr[VPT];
    auto load_row = [&](int64_t row) {
        const char* xp = a.x + row * a.xs * ES;
        const char* rp = ADD ? a.res + row * a.rs * ES : nullptr;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const int64_t v = tid + (int64_t)j * nthr;
            if (v < a.nvec) {
                xr[j] = ld_stream16(xp + v * 16);
                if (ADD) rr[j] = ld_stream16(rp + v * 16);
            }
        }
    };

    int64_t row = blockIdx.x;
    if (row < a.rows) load_row(row);
    for (int parity = 0; row < a.rows; row += gridDim.x, parity ^= 1) {
        uint4 h[VPT];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const int64_t v = tid + (int64_t)j * nthr;
            h[j] = make_uint4(0, 0, 0, 0);
            if (v < a.nvec) {
                h[j] = ADD ? add16<T>(rr[j], xr[j]) : xr[j];
                ss += sum_sq16<T>(h[j]);
            }
        }
        // prefetch: this CTA's next row is in flight during the reduction
        if (row + gridDim.x < a.rows) load_row(row + gridDim.x);
        ss = warp_sum(ss);
        if (lane == 0) red[parity][warp] = ss;
        __syncthreads();
        float tot = 0.f;
        for (int i = 0; i < nwarps; ++i) tot += red[parity][i];
        const float inv = inv_rms(tot, a.H, a.eps);

        char* outr = a.out + row * a.os * ES;
        char* rout = ADD ? a.res_out + row * a.ros * ES : nullptr;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const int64_t v = tid + (int64_t)j * nthr;
            if (v < a.nvec) {
                if (ADD) st16(rout + v * 16, h[j]);
                st16(outr + v * 16, norm16<T>(h[j], inv, w[j]));
            }
        }
    }
}

// Any hidden size / alignment: one CTA per row, two passes over the row.
template <typename T, bool ADD>
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(const NormArgs a) {
    __shared__ float red[32];
    const T* x = reinterpret_cast<const T*>(a.x) + blockIdx.x * a.xs;
    const T* r = ADD ? reinterpret_cast<const T*>(a.res) + blockIdx.x * a.rs : nullptr;
    const T* w = reinterpret_cast<const T*>(a.w);
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < a.H; i += blockDim.x) {
        float h = Dt<T>::to_f(x[i]);
        if (ADD) h = rnd<T>(__fadd_rn(Dt<T>::to_f(r[i]), h));
        ss = fmaf(h, h, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    const float inv = inv_rms(tot, a.H, a.eps);
    T* out = reinterpret_cast<T*>(a.out) + blockIdx.x * a.os;
    T* rout = ADD ? reinterpret_cast<T*>(a.res_out) + blockIdx.x * a.ros : nullptr;
    for (int64_t i = threadIdx.x; i < a.H; i += blockDim.x) {
        float h = Dt<T>::to_f(x[i]);
        if (ADD) h = rnd<T>(__fadd_rn(Dt<T>::to_f(r[i]), h));
        const float y = __fmul_rn(Dt<T>::to_f(w[i]), rnd<T>(__fmul_rn(h, inv)));
        // every thread reads its own elements before writing them, so out/rout may alias x/r
        if (ADD) rout[i] = Dt<T>::from_f(h);
        out[i] = Dt<T>::from_f(y);
    }
}

template <typename T, int VPT, bool ADD>
int launch_vec(const NormArgs& a, cudaStream_t stream) {
    const int threads = (int)std::min<int64_t>(VPT == 8 ? 512 : QF_RMS_MAX_THREADS,
                                               ceil_div(ceil_div(a.nvec, VPT), 32) * 32);
    const int per_sm = resident_ctas<rmsnorm_vec_kernel<T, VPT, ADD>>(threads);
    const int64_t grid = std::min<int64_t>(a.rows, (int64_t)sm_count() * per_sm);
    return launch_pdl(rmsnorm_vec_kernel<T, VPT, ADD>, (unsigned)grid, threads, 0, stream, a);
}

template <typename T, bool ADD>
int dispatch(NormArgs& a, cudaStream_t stream) {
    constexpr int EPV = Dt<T>::kPerVec;
    const int64_t es = sizeof(T);
    bool vec = a.H % EPV == 0 && aligned16(a.x) && aligned16(a.w) && aligned16(a.out) &&
               (a.xs * es) % 16 == 0 && (a.os * es) % 16 == 0;
    if (ADD)
        vec = vec && aligned16(a.res) && aligned16(a.res_out) && (a.rs * es) % 16 == 0 &&
              (a.ros * es) % 16 == 0;
    if (vec) {
        a.nvec = a.H / EPV;
        // at most 256 threads per row where possible: more rows in flight per SM
        if (a.nvec <= QF_RMS_MAX_THREADS) return launch_vec<T, 1, ADD>(a, stream);
        if (a.nvec <= 2 * QF_RMS_MAX_THREADS) return launch_vec<T, 2, ADD>(a, stream);
        if (a.nvec <= 4 * QF_RMS_MAX_THREADS) return launch_vec<T, 4, ADD>(a, stream);
        if (a.nvec <= 4096) return launch_vec<T, 8, ADD>(a, stream);
    }
    if (a.rows > 0x7fffffffLL) return QF_ERR_UNSUPPORTED;
    rmsnorm_scalar_kernel<T, ADD><<<(unsigned)a.rows, 256, 0, stream>>>(a);
    return check_launch();
}

template <bool ADD>
int run(NormArgs& a, int dtype, cudaStream_t stream) {
    if (a.rows < 0 || a.H <= 0) return QF_ERR_INVALID;
    if (a.rows == 0) return QF_OK;
    if (!a.x || !a.w || !a.out || (ADD && (!a.res || !a.res_out))) return QF_ERR_INVALID;
    switch (dtype) {
    case QF_F32: return dispatch<float, ADD>(a, stream);
    case QF_F16: return dispatch<__half, ADD>(a, stream);
    case QF_BF16: return dispatch<__nv_bfloat16, ADD>(a, stream);
    default: return QF_ERR_INVALID;
    }
}

}  // namespace
}  // namespace qf

extern "C" int qf_rmsnorm(const void* x, int64_t x_row_stride, const void* weight, void* out,
                          int64_t out_row_stride, int64_t num_rows, int64_t hidden, float eps,
                          int dtype, cudaStream_t stream) {
    qf::NormArgs a{};
    a.x = static_cast<const char*>(x);
    a.xs = x_row_stride;
    a.w = static_cast<const char*>(weight);
    a.out = static_cast<char*>(out);
    a.os = out_row_stride;
    a.rows = num_rows;
    a.H = hidden;
    a.eps = eps;
    return qf::run<false>(a, dtype, stream);
}

extern "C" int qf_add_rmsnorm(const void* x, int64_t x_row_stride, const void* residual,
                              int64_t residual_row_stride, const void* weight,
                              void* residual_out, int64_t residual_out_row_stride, void* out,
                              int64_t out_row_stride, int64_t num_rows, int64_t hidden,
                              float eps, int dtype, cudaStream_t stream) {
    qf::NormArgs a{};
    a.x = static_cast<const char*>(x);
    a.xs = x_row_stride;
    a.res = static_cast<const char*>(residual);
    a.rs = residual_row_stride;
    a.w = static_cast<const char*>(weight);
    a.res_out = static_cast<char*>(residual_out);
    a.ros = residual_out_row_stride;
    a.out = static_cast<char*>(out);
    a.os = out_row_stride;
    a.rows = num_rows;
    a.H = hidden;
    a.eps = eps;
    return qf::run<true>(a, dtype, stream);
}
