// Device-side arguments of the prefill varlen attention kernels, shared by the
// mma.sync path (varlen_attention.cu) and the tcgen05 path
// (varlen_attention_tc.cu).
#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

namespace qf {

struct VarlenDev {
    const char* q;
    const char* k;
    const char* v;
    char* out;
    int64_t qt, qh, kt, kh, vt, vh, ot, oh;  // token / head strides, elements
    const int32_t* cu_q;
    const int32_t* cu_k;
    int batch, Hq, Hkv;
    int causal;
    float scale;
    int32_t* status;
    int64_t total_q, total_k;  // rows of q and of k / v
    int32_t* work_counter;     // tcgen05 path: persistent CTAs claim items here
};

// The tcgen05 kernel (head_dim 128, 16-bit types).  bf16: 1 for bfloat16, 0
// for float16.  Returns a QF_* code.
int launch_varlen_tc(const VarlenDev& a, int bf16, int max_q, cudaStream_t stream);

}  // namespace qf
