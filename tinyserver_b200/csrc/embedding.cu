// Embedding gather: out[t, :] = table[ids[t], :].
//
// Replaces nn.Embedding.forward as Qwen3Model calls it (transformers 5.5.0
// modeling_qwen3.py:392).  A bit-exact row copy in 16-byte chunks; an id
// outside [0, vocab) writes a zero row and sets QF_FLAG_BAD_TOKEN instead of
// reading outside the table.
#include "qf_common.cuh"

namespace qf {
namespace {

struct EmbArgs {
    const void* ids;
    int index_type;
    const char* table;
    int64_t V, trs;  // vocab, table row stride (elements)
    char* out;
    int64_t ors;
    int64_t T, H, es;
    int32_t* status;
};

template <int VPT>
__global__ void __launch_bounds__(256) embedding_vec_kernel(const EmbArgs a, const int64_t nvec,
                                                            const int64_t chunks) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x / chunks;
    const int64_t chunk = blockIdx.x - row * chunks;
    const int64_t id = load_index(a.ids, row, a.index_type);
    const bool ok = id >= 0 && id < a.V;
    if (!ok && chunk == 0 && threadIdx.x == 0) flag(a.status, QF_FLAG_BAD_TOKEN);
    const char* src = a.table + (ok ? id : 0) * a.trs * a.es;
    char* dst = a.out + row * a.ors * a.es;
    const int64_t v0 = chunk * (int64_t)blockDim.x * VPT + threadIdx.x;
    uint4 r[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int64_t v = v0 + (int64_t)j * blockDim.x;
        r[j] = make_uint4(0, 0, 0, 0);
        if (ok && v < nvec) r[j] = ld_stream16(src + v * 16);
    }
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int64_t v = v0 + (int64_t)j * blockDim.x;
        if (v < nvec) st_stream16(dst + v * 16, r[j]);
    }
}

__global__ void __launch_bounds__(256) embedding_scalar_kernel(const EmbArgs a) {
    const int64_t total = a.T * a.H;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / a.H, c = i - t * a.H;
        const int64_t id = load_index(a.ids, t, a.index_type);
        const bool ok = id >= 0 && id < a.V;
        if (!ok && c == 0) flag(a.status, QF_FLAG_BAD_TOKEN);
        char* dst = a.out + (t * a.ors + c) * a.es;
        const char* src = a.table + ((ok ? id : 0) * a.trs + c) * a.es;
        for (int64_t b = 0; b < a.es; ++b) dst[b] = ok ? src[b] : 0;
    }
}

}  // namespace
}  // namespace qf

extern "C" int qf_embedding(const void* ids, int index_type, const void* table, int64_t vocab,
                            int64_t table_row_stride, void* out, int64_t out_row_stride,
                            int64_t num_tokens, int64_t hidden, int64_t elem_size,
                            int32_t* status, cudaStream_t stream) {
    if (num_tokens < 0 || hidden < 0 || vocab < 0 || elem_size <= 0) return QF_ERR_INVALID;
    if (index_type != QF_I32 && index_type != QF_I64) return QF_ERR_INVALID;
    if (num_tokens == 0 || hidden == 0) return QF_OK;
    if (!ids || !table || !out) return QF_ERR_INVALID;
    qf::EmbArgs a{ids, index_type, static_cast<const char*>(table), vocab, table_row_stride,
                  static_cast<char*>(out), out_row_stride, num_tokens, hidden, elem_size, status};
    const int64_t row_bytes = hidden * elem_size;
    const bool vec = row_bytes % 16 == 0 && qf::aligned16(table) && qf::aligned16(out) &&
                     (table_row_stride * elem_size) % 16 == 0 &&
                     (out_row_stride * elem_size) % 16 == 0;
    if (vec) {
        constexpr int VPT = 2;
        const int64_t nvec = row_bytes / 16;
        const int threads =
            (int)std::min<int64_t>(256, qf::ceil_div(qf::ceil_div(nvec, VPT), 32) * 32);
        const int64_t chunks = qf::ceil_div(nvec, (int64_t)threads * VPT);
        const int64_t blocks = num_tokens * chunks;
        if (blocks <= 0x7fffffffLL) {
            return qf::launch_pdl(qf::embedding_vec_kernel<VPT>, (unsigned)blocks, threads, 0,
                                  stream, a, nvec, chunks);
        }
    }
    const int64_t blocks =
        std::min<int64_t>(qf::ceil_div(num_tokens * hidden, 256), (int64_t)qf::sm_count() * 32);
    qf::embedding_scalar_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a);
    return qf::check_launch();
}
