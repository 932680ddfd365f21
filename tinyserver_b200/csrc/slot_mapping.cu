// Per-token block/slot mapping of the paged KV cache, built on the device.
//
// The reference builds it on the host: a Python loop over every token of a
// prefill batch, per layer (server/model/patches/qwen3.py:296-310), and in
// decode one `.item()` sync + one H2D block table + one store launch per
// sequence per layer (qwen3.py:335-357).  Here one launch per forward turns
// (cu_seqlens, positions, padded block tables) into the (block, slot) arrays
// every layer's fused store then reads:
//   block_mapping[t] = block_tables[s, positions[t] / B],  slot_mapping[t] = positions[t] % B
// which is the address rule of kv_cache.py:49-58 (per sequence) and of the
// reference tests' mapping recipe (tests/model/test_kv_cache_kernels.py:16-37).
#include "qf_common.cuh"

namespace qf {
namespace {

__global__ void __launch_bounds__(256) build_slot_mapping_kernel(
    const int32_t* __restrict__ cu, int64_t S, const int64_t* __restrict__ pos, int64_t T,
    const int32_t* __restrict__ bt, int64_t bt_stride, int64_t max_blocks, int64_t B,
    int64_t* __restrict__ bm, int64_t* __restrict__ sm, int32_t* status) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T;
         t += (int64_t)gridDim.x * blockDim.x) {
        // sequence s with cu[s] <= t < cu[s + 1] (binary search; cu is sorted)
        int64_t lo = 0, hi = S;
        while (hi - lo > 1) {
            const int64_t mid = (lo + hi) >> 1;
            if ((int64_t)__ldg(cu + mid) <= t) lo = mid;
            else hi = mid;
        }
        const int64_t p = __ldg(pos + t);
        const bool in_seq = (int64_t)__ldg(cu + lo) <= t && t < (int64_t)__ldg(cu + S);
        const int64_t logical = p >= 0 ? p / B : -1;
        if (!in_seq || p < 0 || logical >= max_blocks) {
            flag(status, QF_FLAG_BAD_TABLE);
            bm[t] = -1;
            sm[t] = 0;
            continue;
        }
        bm[t] = (int64_t)__ldg(bt + lo * bt_stride + logical);
        sm[t] = p - logical * B;
    }
}

}  // namespace
}  // namespace qf

extern "C" int qf_build_slot_mapping(const int32_t* cu_seqlens, int64_t num_seqs,
                                     const int64_t* positions, int64_t num_tokens,
                                     const int32_t* block_tables,
                                     int64_t block_tables_row_stride, int64_t max_blocks,
                                     int64_t block_size, int64_t* block_mapping,
                                     int64_t* slot_mapping, int32_t* status,
                                     cudaStream_t stream) {
    if (num_seqs < 0 || num_tokens < 0 || max_blocks < 0 || block_size <= 0)
        return QF_ERR_INVALID;
    if (num_tokens == 0) return QF_OK;
    if (num_seqs == 0 || !cu_seqlens || !positions || !block_mapping || !slot_mapping ||
        (max_blocks > 0 && !block_tables))
        return QF_ERR_INVALID;
    const int64_t blocks =
        std::min<int64_t>(qf::ceil_div(num_tokens, 256), (int64_t)qf::sm_count() * 8);
    qf::build_slot_mapping_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
        cu_seqlens, num_seqs, positions, num_tokens, block_tables, block_tables_row_stride,
        max_blocks, block_size, block_mapping, slot_mapping, status);
    return qf::check_launch();
}
