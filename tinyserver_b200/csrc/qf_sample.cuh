// Pieces the two sampling paths share: the order key and fixed-point mass of
// a scaled logit, the counter-hash uniform, and the batch-wide path's entry
// (sampler_wide.cu), which sampler.cu's entry point calls.
//
// Both paths compute the same integers from the same s = logit / temperature:
// a mass is exp(s - max) x 2^40 rounded to a u64, so every sum of masses is
// exact and independent of the order of addition, and the two paths pick the
// same token.
#pragma once

#include "qf_common.cuh"

namespace qf {

using u64 = unsigned long long;

constexpr float kMassScale = 1099511627776.0f;  // 2^40

// s's float bits with the sign folded, so that unsigned comparison follows s.
__device__ __forceinline__ uint32_t order_key(float s) {
    const uint32_t b = __float_as_uint(s);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// The inverse of order_key.
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ u64 mass_of(float s, float m) {
    return __float2ull_rn(expf(s - m) * kMassScale);
}

// (s desc, index asc): the rank order of the reference's stable sort.
__device__ __forceinline__ bool better(float s, uint32_t i, float t, uint32_t j) {
    return s > t || (s == t && i < j);
}

// splitmix64 of (seed, step), top 53 bits as a double in [0, 1), clamped to
// the largest float32 below 1 -- uniform_from_hash, determinism.py:30-51.
__device__ __forceinline__ float uniform_from_hash(uint64_t seed, uint64_t step) {
    uint64_t x = seed * 0x9E3779B97F4A7C15ull + step;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    x ^= x >> 31;
    const double u = fmin((double)(x >> 11) * 0x1p-53, 1.0 - 0x1p-24);
    return __double2float_rn(u);
}

template <typename T>
__device__ __forceinline__ float scaled(T x, float tc) {
    const float s = __fdiv_rn(Dt<T>::to_f(x), tc);
    return s == 0.0f ? 0.0f : s;  // -0 ranks with +0, as in the sort
}

// ---------------------------------------------------------------------------
// The batch-wide path (sampler_wide.cu): every row's max, histogram,
// boundary search, candidate compaction and candidate selection run as
// grid-wide passes over all rows at once.  A row it cannot finish is listed
// for the per-row cluster kernel.
struct WideArgs {
    const void* logits;
    int64_t row_stride;  // elements
    int64_t batch, vocab;
    int dtype;
    int vec;             // 16-byte loads (aligned rows)
    const float* temperature;
    const void* top_k;
    int top_k_i64;
    const float* top_p;
    const float* uniforms;
    const int64_t* seeds;
    const int64_t* steps;
    int64_t* out;
    void* workspace;
};

// Bytes of workspace the batch-wide path needs for `batch` rows.
int64_t sample_wide_workspace_bytes(int64_t batch);

// Enqueue the batch-wide passes.  Afterwards *slow_n (device) rows, listed
// in slow_rows (device), still need the cluster kernel; both point into the
// workspace.
int sample_wide_passes(const WideArgs& a, cudaStream_t stream, const uint32_t** slow_rows,
                       const uint32_t** slow_n);

}  // namespace qf
