// Library-wide entry points of libqwen3fused: status word, errors, version.
#include <stdio.h>
#include <string.h>

#include "qf_common.cuh"

namespace qf {

namespace {
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];  // 0 = not queried yet (benign race: same value)
thread_local char g_last_error[256];
}  // namespace

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < kMaxDevices && g_sm_count[dev] > 0) return g_sm_count[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        n = 148;
    if (dev < kMaxDevices) g_sm_count[dev] = n;
    return n;
}

int launch_failed(cudaError_t e) {
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e),
             cudaGetErrorString(e));
    return QF_ERR_LAUNCH;
}

}  // namespace qf

extern "C" int qf_read_status(int32_t* status_dev, int32_t* flags_out, int clear,
                              cudaStream_t stream) {
    if (!status_dev || !flags_out) return QF_ERR_INVALID;
    int32_t host = 0;
    cudaError_t e = cudaMemcpyAsync(&host, status_dev, sizeof(int32_t), cudaMemcpyDeviceToHost,
                                    stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(status_dev, 0, sizeof(int32_t), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return qf::launch_failed(e);
    *flags_out = host;
    return host ? QF_ERR_DEVICE : QF_OK;
}

extern "C" const char* qf_last_cuda_error(void) { return qf::g_last_error; }

extern "C" size_t qf_qk_norm_rope_args_size(void) { return sizeof(qf_qk_norm_rope_args); }

extern "C" size_t qf_paged_attention_args_size(void) { return sizeof(qf_paged_attention_args); }

extern "C" size_t qf_varlen_attention_args_size(void) { return sizeof(qf_varlen_attention_args); }

extern "C" size_t qf_sample_args_size(void) { return sizeof(qf_sample_args); }

extern "C" const char* qf_version(void) { return "qwen3fused 0.1.0 sm_100a"; }
