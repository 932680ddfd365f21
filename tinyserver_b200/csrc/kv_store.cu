// Paged KV-cache store: scatter of K/V head rows into (N, Hkv, B, D) pages.
//
// Replaces the reference's two Triton store kernels
// (server/model/kernels/kv_cache.py:6-70 per sequence, :122-191 batched).
// The store is a pure copy, so the kernels move whole 16-byte chunks of each
// head row (a 128-dim bf16 row is 16 chunks) and never convert values:
// placement and contents are bit-exact by construction.
// Addresses are int64 throughout (a long-context cache holds ~60 G elements).
// A block/slot outside the cache is skipped and reported in *status.
#include "qf_common.cuh"

namespace qf {
namespace {

enum { kBatched = 0, kSeq = 1 };

struct KvArgs {
    const char* k_src;
    const char* v_src;
    int64_t ks[3], vs[3];  // source strides (head, token, dim), elements
    char* k_cache;
    char* v_cache;
    int64_t kc[4], vc[4];  // cache strides (block, head, slot, dim), elements
    const void* block_mapping;
    const void* slot_mapping;
    int index_type;
    int64_t start;
    const void* table;
    int64_t table_len;
    int64_t T, Hkv, D, N, B, es;
    int32_t* status;
};

// Physical (block, slot) of token t, or false if it falls outside the cache.
template <int MODE>
__device__ __forceinline__ bool resolve(const KvArgs& a, int64_t t, int64_t& blk, int64_t& slot,
                                        bool report) {
    if (MODE == kBatched) {
        blk = load_index(a.block_mapping, t, a.index_type);
        slot = load_index(a.slot_mapping, t, a.index_type);
    } else {
        const int64_t pos = a.start + t;
        const int64_t logical = pos / a.B;
        slot = pos - logical * a.B;
        if (logical >= a.table_len) {
            if (report) flag(a.status, QF_FLAG_BAD_TABLE);
            return false;
        }
        blk = load_index(a.table, logical, a.index_type);
    }
    bool ok = true;
    if (blk < 0 || blk >= a.N) {
        if (report) flag(a.status, QF_FLAG_BAD_BLOCK);
        ok = false;
    }
    if (slot < 0 || slot >= a.B) {
        if (report) flag(a.status, QF_FLAG_BAD_SLOT);
        ok = false;
    }
    return ok;
}

// One thread per 16-byte chunk of a (token, head) row; K and V together.
// IT is the index type of the flattened loop (32-bit when it fits).
template <int MODE, typename IT>
__global__ void __launch_bounds__(256) kv_store_vec_kernel(const KvArgs a, const int64_t cpr) {
    const IT per_token = (IT)(a.Hkv * cpr);
    const IT total = (IT)a.T * per_token;
    const IT step = (IT)gridDim.x * blockDim.x;
    for (IT i = (IT)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        const IT t = i / per_token;
        const IT r = i - t * per_token;
        const IT h = r / (IT)cpr;
        const IT c = r - h * (IT)cpr;
        int64_t blk, slot;
        if (!resolve<MODE>(a, (int64_t)t, blk, slot, r == 0)) continue;
        const int64_t hh = (int64_t)h, tt = (int64_t)t, cb = (int64_t)c * 16;
        const uint4 kv = ld_stream16(a.k_src + (hh * a.ks[0] + tt * a.ks[1]) * a.es + cb);
        const uint4 vv = ld_stream16(a.v_src + (hh * a.vs[0] + tt * a.vs[1]) * a.es + cb);
        st16(a.k_cache + (blk * a.kc[0] + hh * a.kc[1] + slot * a.kc[2]) * a.es + cb, kv);
        st16(a.v_cache + (blk * a.vc[0] + hh * a.vc[1] + slot * a.vc[2]) * a.es + cb, vv);
    }
}

// Per-head tiles for rows of CPR 16-byte chunks (D * es = 16 * CPR bytes):
// block (x, h) takes head h of 256 / CPR consecutive tokens, thread (r, c)
// chunk c of token r's row.  Its K and V loads are issued together with the
// token's index loads, then the two stores: little state per thread, so many
// blocks per SM keep loads in flight.  Plain read-only loads: on B200 they
// measured faster here than streaming loads with a 256-byte L2 prefetch.
template <int MODE, int CPR>
__global__ void __launch_bounds__(256) kv_store_head_kernel(const KvArgs a) {
    constexpr int TT = 256 / CPR;  // tokens per block
    const int c = threadIdx.x % CPR, r = threadIdx.x / CPR;
    const int64_t t = (int64_t)blockIdx.x * TT + r;
    const int64_t h = blockIdx.y;
    if (t >= a.T) return;
    const int64_t cb = (int64_t)c * 16;
    const uint4 kv =
        __ldg(reinterpret_cast<const uint4*>(a.k_src + (h * a.ks[0] + t * a.ks[1]) * a.es + cb));
    const uint4 vv =
        __ldg(reinterpret_cast<const uint4*>(a.v_src + (h * a.vs[0] + t * a.vs[1]) * a.es + cb));
    int64_t blk, slot;
    if (!resolve<MODE>(a, t, blk, slot, c == 0 && h == 0)) return;
    st16(a.k_cache + (blk * a.kc[0] + h * a.kc[1] + slot * a.kc[2]) * a.es + cb, kv);
    st16(a.v_cache + (blk * a.vc[0] + h * a.vc[1] + slot * a.vc[2]) * a.es + cb, vv);
}

template <typename W>
__device__ __forceinline__ void copy_el(char* dst, const char* src) {
    *reinterpret_cast<W*>(dst) = *reinterpret_cast<const W*>(src);
}

__device__ __forceinline__ void copy_es(char* dst, const char* src, int64_t es) {
    switch (es) {
    case 1: copy_el<uint8_t>(dst, src); break;
    case 2: copy_el<uint16_t>(dst, src); break;
    case 4: copy_el<uint32_t>(dst, src); break;
    default: copy_el<uint64_t>(dst, src); break;
    }
}

// Any strides, any element size: one thread per element.
template <int MODE>
__global__ void __launch_bounds__(256) kv_store_scalar_kernel(const KvArgs a) {
    const int64_t per_token = a.Hkv * a.D;
    const int64_t total = a.T * per_token;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        const int64_t t = i / per_token;
        const int64_t r = i - t * per_token;
        const int64_t h = r / a.D;
        const int64_t d = r - h * a.D;
        int64_t blk, slot;
        if (!resolve<MODE>(a, t, blk, slot, r == 0)) continue;
        copy_es(a.k_cache + (blk * a.kc[0] + h * a.kc[1] + slot * a.kc[2] + d * a.kc[3]) * a.es,
                a.k_src + (h * a.ks[0] + t * a.ks[1] + d * a.ks[2]) * a.es, a.es);
        copy_es(a.v_cache + (blk * a.vc[0] + h * a.vc[1] + slot * a.vc[2] + d * a.vc[3]) * a.es,
                a.v_src + (h * a.vs[0] + t * a.vs[1] + d * a.vs[2]) * a.es, a.es);
    }
}

bool vectorizable(const KvArgs& a) {
    if ((a.D * a.es) % 16) return false;
    if (a.ks[2] != 1 || a.vs[2] != 1 || a.kc[3] != 1 || a.vc[3] != 1) return false;
    if (!aligned16(a.k_src) || !aligned16(a.v_src) || !aligned16(a.k_cache) ||
        !aligned16(a.v_cache))
        return false;
    const int64_t s[] = {a.ks[0], a.ks[1], a.vs[0], a.vs[1], a.kc[0], a.kc[1], a.kc[2],
                         a.vc[0], a.vc[1], a.vc[2]};
    for (int64_t v : s)
        if ((v * a.es) % 16) return false;
    return true;
}

template <int MODE>
int launch(const KvArgs& a, cudaStream_t stream) {
    const int threads = 256;
    const int64_t max_blocks = (int64_t)sm_count() * 32;
    if (vectorizable(a)) {
        const int64_t cpr = a.D * a.es / 16;
        if ((cpr == 8 || cpr == 16 || cpr == 32) && a.Hkv <= 65535) {
            const dim3 grid((unsigned)ceil_div(a.T, 256 / cpr), (unsigned)a.Hkv);
            if (cpr == 8) kv_store_head_kernel<MODE, 8><<<grid, threads, 0, stream>>>(a);
            else if (cpr == 16) kv_store_head_kernel<MODE, 16><<<grid, threads, 0, stream>>>(a);
            else kv_store_head_kernel<MODE, 32><<<grid, threads, 0, stream>>>(a);
            return check_launch();
        }
        const int64_t total = a.T * a.Hkv * cpr;
        const int64_t blocks = std::min<int64_t>(ceil_div(total, threads), max_blocks);
        if (total < (int64_t(1) << 31))
            kv_store_vec_kernel<MODE, uint32_t><<<(unsigned)blocks, threads, 0, stream>>>(a, cpr);
        else
            kv_store_vec_kernel<MODE, uint64_t><<<(unsigned)blocks, threads, 0, stream>>>(a, cpr);
    } else {
        const int64_t total = a.T * a.Hkv * a.D;
        const int64_t blocks = std::min<int64_t>(ceil_div(total, threads), max_blocks);
        kv_store_scalar_kernel<MODE><<<(unsigned)blocks, threads, 0, stream>>>(a);
    }
    return check_launch();
}

int fill_common(KvArgs& a, const void* k_src, const int64_t* ks, const void* v_src,
                const int64_t* vs, void* k_cache, const int64_t* kc, void* v_cache,
                const int64_t* vc, int64_t T, int64_t Hkv, int64_t D, int64_t N, int64_t B,
                int64_t es, int32_t* status) {
    if (T < 0 || Hkv < 0 || D < 0 || N < 0 || B <= 0) return QF_ERR_INVALID;
    if (es != 1 && es != 2 && es != 4 && es != 8) return QF_ERR_INVALID;
    if (!ks || !vs || !kc || !vc) return QF_ERR_INVALID;
    if (T > 0 && Hkv > 0 && D > 0 && (!k_src || !v_src || !k_cache || !v_cache))
        return QF_ERR_INVALID;
    a.k_src = static_cast<const char*>(k_src);
    a.v_src = static_cast<const char*>(v_src);
    a.k_cache = static_cast<char*>(k_cache);
    a.v_cache = static_cast<char*>(v_cache);
    for (int i = 0; i < 3; ++i) {
        a.ks[i] = ks[i];
        a.vs[i] = vs[i];
    }
    for (int i = 0; i < 4; ++i) {
        a.kc[i] = kc[i];
        a.vc[i] = vc[i];
    }
    a.T = T;
    a.Hkv = Hkv;
    a.D = D;
    a.N = N;
    a.B = B;
    a.es = es;
    a.status = status;
    return QF_OK;
}

}  // namespace
}  // namespace qf

extern "C" int qf_kv_store_batched(const void* k_src, const int64_t k_src_strides[3],
                                   const void* v_src, const int64_t v_src_strides[3],
                                   void* k_cache, const int64_t k_cache_strides[4],
                                   void* v_cache, const int64_t v_cache_strides[4],
                                   const void* block_mapping, const void* slot_mapping,
                                   int index_type, int64_t num_tokens, int64_t num_kv_heads,
                                   int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                   int64_t elem_size, int32_t* status, cudaStream_t stream) {
    qf::KvArgs a{};
    int rc = qf::fill_common(a, k_src, k_src_strides, v_src, v_src_strides, k_cache,
                             k_cache_strides, v_cache, v_cache_strides, num_tokens, num_kv_heads,
                             head_dim, num_blocks, block_size, elem_size, status);
    if (rc) return rc;
    if (index_type != QF_I32 && index_type != QF_I64) return QF_ERR_INVALID;
    if (num_tokens == 0 || num_kv_heads == 0 || head_dim == 0) return QF_OK;
    if (!block_mapping || !slot_mapping) return QF_ERR_INVALID;
    a.block_mapping = block_mapping;
    a.slot_mapping = slot_mapping;
    a.index_type = index_type;
    return qf::launch<qf::kBatched>(a, stream);
}

extern "C" int qf_kv_store_seq(int64_t start_position, const void* block_table,
                               int64_t table_len, int index_type, const void* k_src,
                               const int64_t k_src_strides[3], const void* v_src,
                               const int64_t v_src_strides[3], void* k_cache,
                               const int64_t k_cache_strides[4], void* v_cache,
                               const int64_t v_cache_strides[4], int64_t num_tokens,
                               int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
                               int64_t block_size, int64_t elem_size, int32_t* status,
                               cudaStream_t stream) {
    qf::KvArgs a{};
    int rc = qf::fill_common(a, k_src, k_src_strides, v_src, v_src_strides, k_cache,
                             k_cache_strides, v_cache, v_cache_strides, num_tokens, num_kv_heads,
                             head_dim, num_blocks, block_size, elem_size, status);
    if (rc) return rc;
    if (index_type != QF_I32 && index_type != QF_I64) return QF_ERR_INVALID;
    if (start_position < 0 || table_len < 0) return QF_ERR_INVALID;
    if (num_tokens == 0 || num_kv_heads == 0 || head_dim == 0) return QF_OK;
    if (!block_table && table_len > 0) return QF_ERR_INVALID;
    a.start = start_position;
    a.table = block_table;
    a.table_len = table_len;
    a.index_type = index_type;
    return qf::launch<qf::kSeq>(a, stream);
}
