/*
 * qwen3fused.h -- C ABI of libqwen3fused.so, the B200 (sm_100a) kernels of the
 * Qwen3 decoder layer's memory-bound op path in tinyserver's server/model.
 *
 * Conventions (every entry point):
 *  - Pointers are device pointers unless stated otherwise; the caller owns all
 *    memory.  No entry point allocates or frees.
 *  - Sizes and strides are int64 and strides count ELEMENTS, not bytes.
 *  - Work is enqueued on `stream` (the caller's current stream) and is not
 *    waited for.  Entry points are stateless and reentrant.
 *  - Return value: QF_OK, or a QF_ERR_* code for a rejected argument
 *    (checked on the host before any launch) or a launch failure.
 *  - Index errors found on the device (a token id outside the vocabulary, a
 *    block or slot outside the cache) never fault: the kernel skips that
 *    write and ORs a QF_FLAG_* bit into *status (when status is not NULL).
 *    qf_read_status() fetches and clears the word.
 *
 * Element dtype tags: QF_F32, QF_F16, QF_BF16.  Index dtype tags: QF_I32,
 * QF_I64 (the reference passes int64 mappings from the model and int32 ones
 * in its tests; both are accepted).
 */
#ifndef QWEN3FUSED_H
#define QWEN3FUSED_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { QF_F32 = 0, QF_F16 = 1, QF_BF16 = 2 };
enum { QF_I32 = 0, QF_I64 = 1 };

enum {
    QF_OK = 0,
    QF_ERR_INVALID = 1,     /* null pointer, negative size, unknown tag */
    QF_ERR_UNSUPPORTED = 2, /* a shape this library has no kernel for */
    QF_ERR_LAUNCH = 3,      /* the CUDA launch failed (see qf_last_cuda_error) */
    QF_ERR_DEVICE = 4,      /* qf_read_status found a flagged index error */
    QF_ERR_SCRATCH = 5      /* the call needs more scratch than the fixed array of
                               qf_paged_attention_decode_noalloc holds */
};

enum {
    QF_FLAG_BAD_BLOCK = 1, /* block index < 0 or >= num_blocks */
    QF_FLAG_BAD_SLOT = 2,  /* slot index < 0 or >= block_size */
    QF_FLAG_BAD_TOKEN = 4, /* token id < 0 or >= vocab */
    QF_FLAG_BAD_TABLE = 8, /* logical block beyond the block table's length */
    QF_FLAG_TIMEOUT = 16   /* a kernel gave up waiting on its own tensor-core work */
};

/* ---------------------------------------------------------------------- */
/* Paged KV-cache store, batched form.
 * Replaces store_kv_cache_batched (server/model/kernels/kv_cache.py:194-251;
 * Triton kernel kv_cache.py:122-191):
 *   k_cache[block_mapping[t], h, slot_mapping[t], :] = k_src[h, t, :]  (and V)
 * k_src/v_src: (num_kv_heads, num_tokens, head_dim) with strides *_src_strides.
 * k_cache/v_cache: (num_blocks, num_kv_heads, block_size, head_dim) with
 * strides *_cache_strides (per-layer views of the 6-D pool are fine).
 * elem_size: bytes per element (the store is a copy; any 1/2/4/8-byte dtype). */
int qf_kv_store_batched(const void* k_src, const int64_t k_src_strides[3],
                        const void* v_src, const int64_t v_src_strides[3],
                        void* k_cache, const int64_t k_cache_strides[4],
                        void* v_cache, const int64_t v_cache_strides[4],
                        const void* block_mapping, const void* slot_mapping, int index_type,
                        int64_t num_tokens, int64_t num_kv_heads, int64_t head_dim,
                        int64_t num_blocks, int64_t block_size, int64_t elem_size,
                        int32_t* status, cudaStream_t stream);

/* Paged KV-cache store, one sequence.
 * Replaces store_kv_cache (kv_cache.py:73-119; Triton kernel kv_cache.py:6-70):
 *   pos = start_position + i; blk = block_table[pos / block_size];
 *   k_cache[blk, h, pos % block_size, :] = k_src[h, i, :]  (and V)
 * block_table: (table_len,) int32 or int64 (index_type). */
int qf_kv_store_seq(int64_t start_position, const void* block_table, int64_t table_len,
                    int index_type,
                    const void* k_src, const int64_t k_src_strides[3],
                    const void* v_src, const int64_t v_src_strides[3],
                    void* k_cache, const int64_t k_cache_strides[4],
                    void* v_cache, const int64_t v_cache_strides[4],
                    int64_t num_tokens, int64_t num_kv_heads, int64_t head_dim,
                    int64_t num_blocks, int64_t block_size, int64_t elem_size,
                    int32_t* status, cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* RMSNorm over rows of `hidden` elements.
 * Replaces Qwen3RMSNorm.forward (transformers 5.5.0
 * models/qwen3/modeling_qwen3.py:59-64) with its rounding points:
 *   out = rnd(w * rnd(x * rsqrt(mean(x^2) + eps)))   (fp32 math, rnd = to dtype)
 * x, weight and out share `dtype`; rows have their own strides; out may alias x. */
int qf_rmsnorm(const void* x, int64_t x_row_stride, const void* weight,
               void* out, int64_t out_row_stride, int64_t num_rows, int64_t hidden,
               float eps, int dtype, cudaStream_t stream);

/* Residual add + RMSNorm in one pass.
 * Replaces the decoder layer's `residual + hidden_states` (modeling_qwen3.py:327
 * and :333) followed by the next Qwen3RMSNorm (modeling_qwen3.py:331 / :316):
 *   h = rnd(residual + x);  residual_out = h;  out = RMSNorm(h)
 * residual_out may alias residual (in-place update of the residual stream). */
int qf_add_rmsnorm(const void* x, int64_t x_row_stride,
                   const void* residual, int64_t residual_row_stride,
                   const void* weight,
                   void* residual_out, int64_t residual_out_row_stride,
                   void* out, int64_t out_row_stride,
                   int64_t num_rows, int64_t hidden, float eps, int dtype,
                   cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* RoPE tables.  Replaces Qwen3RotaryEmbedding.forward (modeling_qwen3.py:137-148),
 * default rope type:
 *   f = inv_freq[i mod head_dim/2] * float(positions[t]);
 *   cos[t, i] = rnd(cos(f) * scaling);  sin[t, i] = rnd(sin(f) * scaling)
 * positions: (num_tokens,) int32/int64; inv_freq: device, head_dim/2 floats
 * (computed by the caller exactly as compute_default_rope_parameters does);
 * cos/sin: (num_tokens, head_dim) contiguous. */
int qf_rope_cos_sin(const void* positions, int index_type, const float* inv_freq,
                    int64_t num_tokens, int64_t head_dim, float scaling, int dtype,
                    void* cos, void* sin, cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Fused q_norm/k_norm + RoPE + paged KV store (one pass over q, k, v).
 * Replaces, in server/model/patches/qwen3.py's attention forward, the chain
 * q_norm/k_norm (qwen3.py:268-271 -> modeling_qwen3.py:248-249),
 * apply_rotary_pos_emb (qwen3.py:287 -> modeling_qwen3.py:159-181) and
 * store_kv_cache_batched of the rotated K and of V (qwen3.py:311-318).
 * Each optional part switches off with a NULL pointer:
 *   q_weight/k_weight NULL -> no norm (plain apply_rotary_pos_emb);
 *   cos NULL -> cos/sin computed in-kernel from positions + inv_freq, rounded
 *               to dtype exactly as the table would be;
 *   k_out NULL -> rotated K only goes to the cache;
 *   k_cache NULL -> no store (v, caches and mappings unused).
 * Layouts: q (T, Hq, D), k/v (T, Hkv, D), q_out (T, Hq, D), k_out (T, Hkv, D),
 * each given by a token stride and a head stride (head_dim contiguous);
 * cos/sin (T, D) rows with cos_sin_token_stride; caches (N, Hkv, B, D).
 * head_dim must be 64, 128 or 256. */
typedef struct {
    const void* q; int64_t q_stride_token, q_stride_head;
    const void* k; int64_t k_stride_token, k_stride_head;
    const void* v; int64_t v_stride_token, v_stride_head;
    const void* q_weight;
    const void* k_weight;
    float eps;
    const void* cos; const void* sin; int64_t cos_sin_token_stride;
    const void* positions; int positions_type; const float* inv_freq;
    void* q_out; int64_t q_out_stride_token, q_out_stride_head;
    void* k_out; int64_t k_out_stride_token, k_out_stride_head;
    void* k_cache; void* v_cache; int64_t cache_strides[4];
    int64_t num_blocks, block_size;
    const void* block_mapping; const void* slot_mapping; int index_type;
    int64_t num_tokens, num_q_heads, num_kv_heads, head_dim;
    int dtype;
    int32_t* status;
} qf_qk_norm_rope_args;

int qf_qk_norm_rope_store(const qf_qk_norm_rope_args* args, cudaStream_t stream);

/* sizeof(qf_qk_norm_rope_args) as compiled into the library, so a binding
 * (ctypes, cgo, ...) can check its mirror of the struct. */
size_t qf_qk_norm_rope_args_size(void);

/* ---------------------------------------------------------------------- */
/* SiLU-and-mul.  Replaces Qwen3MLP's `act_fn(gate_proj(x)) * up_proj(x)`
 * (modeling_qwen3.py:82, act_fn = silu):
 *   out = rnd(rnd(g / (1 + exp(-g))) * u)
 * gate/up/out rows have their own strides, so a merged [T, 2I] gate|up
 * projection (up = gate + I) and separate tensors both work. */
int qf_silu_and_mul(const void* gate, int64_t gate_row_stride,
                    const void* up, int64_t up_row_stride,
                    void* out, int64_t out_row_stride,
                    int64_t num_rows, int64_t intermediate, int dtype,
                    cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Embedding gather.  Replaces nn.Embedding.forward as Qwen3Model calls it
 * (embed_tokens(input_ids), modeling_qwen3.py:392):
 *   out[t, :] = table[ids[t], :]   (bit-exact copy; elem_size bytes/element)
 * An id outside [0, vocab) writes a zero row and sets QF_FLAG_BAD_TOKEN. */
int qf_embedding(const void* ids, int index_type, const void* table, int64_t vocab,
                 int64_t table_row_stride, void* out, int64_t out_row_stride,
                 int64_t num_tokens, int64_t hidden, int64_t elem_size,
                 int32_t* status, cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Per-token block/slot mapping built on the device.
 * Replaces the reference's per-token Python loop in the prefill branch
 * (qwen3.py:296-310) and the per-sequence start-position lookup of the decode
 * branch (qwen3.py:335-357):
 *   token t belongs to sequence s with cu_seqlens[s] <= t < cu_seqlens[s+1];
 *   pos = positions[t]; block_mapping[t] = block_tables[s, pos / block_size];
 *   slot_mapping[t] = pos % block_size
 * cu_seqlens: (num_seqs + 1,) int32; positions: (num_tokens,) int64;
 * block_tables: (num_seqs, max_blocks) int32 with row stride
 * block_tables_row_stride; outputs: (num_tokens,) int64.
 * A logical block >= max_blocks, or a negative position, sets
 * QF_FLAG_BAD_TABLE and writes block -1 (which every store then skips). */
int qf_build_slot_mapping(const int32_t* cu_seqlens, int64_t num_seqs,
                          const int64_t* positions, int64_t num_tokens,
                          const int32_t* block_tables, int64_t block_tables_row_stride,
                          int64_t max_blocks, int64_t block_size,
                          int64_t* block_mapping, int64_t* slot_mapping,
                          int32_t* status, cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Decode paged attention: one query token per sequence against its cached
 * tokens.  Replaces paged_attention_forward (server/model/kernels/
 * paged_attention.py:124-192; Triton kernel :8-121):
 *   out[s, h, :] = softmax(q[s, h] . K_s^T * scale) @ V_s      (fp32 math)
 * where token j < seq_lens[s] of sequence s sits at
 * cache[block_tables[s, j / block_size], h / (Hq / Hkv), j % block_size, :].
 * q, out: (num_seqs, Hq, head_dim) with sequence/head strides, head_dim
 * contiguous; caches (N, Hkv, B, D) with strides (head_dim contiguous, rows
 * 16-byte aligned); block_tables: int32 rows; seq_lens: int32.
 * head_dim 64/128/256; Hq / Hkv in {1, 2, 4, 8}.
 * workspace: fp32 scratch that lets one sequence be split over several CTAs;
 * pass at least qf_paged_attention_workspace_bytes(...) bytes for the
 * longest sequence the block tables allow (max_blocks_per_seq * block_size),
 * or NULL to run one CTA per (sequence, kv head).  A block index outside the
 * cache is skipped and sets QF_FLAG_BAD_BLOCK; a seq_lens[s] longer than
 * max_blocks_per_seq * block_size is cut to that length and sets
 * QF_FLAG_BAD_TABLE.  max_blocks_per_seq * block_size must stay below 2^31
 * (QF_ERR_UNSUPPORTED otherwise). */
typedef struct {
    const void* q; int64_t q_stride_seq, q_stride_head;
    const void* k_cache; const void* v_cache; int64_t cache_strides[4];
    int64_t num_blocks, block_size;
    const int32_t* block_tables; int64_t block_tables_row_stride, max_blocks_per_seq;
    const int32_t* seq_lens;
    int64_t num_seqs, num_q_heads, num_kv_heads, head_dim;
    float scale;
    void* out; int64_t out_stride_seq, out_stride_head;
    void* workspace; int64_t workspace_bytes;
    int dtype;
    int32_t* status;
} qf_paged_attention_args;

int qf_paged_attention_decode(const qf_paged_attention_args* args, cudaStream_t stream);

/* Workspace bytes qf_paged_attention_decode needs to split sequences of up to
 * max_seq_len tokens (0: nothing to split). */
size_t qf_paged_attention_workspace_bytes(int64_t num_seqs, int64_t num_q_heads,
                                          int64_t head_dim, int64_t max_seq_len);

/* sizeof(qf_paged_attention_args) as compiled into the library. */
size_t qf_paged_attention_args_size(void);

/* The same decode attention for callers that cannot allocate device memory.
 * No counterpart in the reference.  Some callers must not call cudaMalloc: a
 * host framework that hands this library only raw pointers and owns every
 * allocation, a runtime that reserves all device memory at start, or a
 * latency-bound loop that cannot take the device synchronisation an
 * allocation implies.  This entry point allocates nothing: the split-K
 * partials live in a fixed device array of qf_paged_attention_noalloc_capacity()
 * bytes (128 MiB) inside the library, which every GPU that loads the library
 * holds until the process exits.  args->workspace and workspace_bytes are
 * ignored; q, caches, tables and out are still the caller's.
 *  - A call whose partials would exceed the array (see
 *    qf_paged_attention_workspace_bytes) returns QF_ERR_SCRATCH before any
 *    device work.
 *  - The first call on each device looks up the array's device address with
 *    cudaGetSymbolAddress (with that device current); make that first call
 *    before any stream capture.
 *  - All calls on a device share the array and it keeps the last call's
 *    contents (nothing in it needs to start at zero); calls that overlap on
 *    the GPU, e.g. on two streams, race on it. */
int qf_paged_attention_decode_noalloc(const qf_paged_attention_args* args, cudaStream_t stream);

/* Bytes of the fixed array qf_paged_attention_decode_noalloc uses. */
size_t qf_paged_attention_noalloc_capacity(void);

/* ---------------------------------------------------------------------- */
/* Prefill attention over variable-length packed sequences.  Replaces
 * flash_attn_varlen_func (server/model/kernels/varlen_attention.py:145-218;
 * Triton kernel :8-142): sequence b owns query rows [cu_seqlens_q[b],
 * cu_seqlens_q[b+1]) and key/value rows [cu_seqlens_k[b], cu_seqlens_k[b+1]);
 *   out[t, h] = softmax(q[t, h] . K_b^T * scale, causal: key j <= query i
 *               within the sequence) @ V_b,   kv head h / (Hq / Hkv)
 * fp32 math; for 16-bit types the probabilities are rounded to the value
 * dtype before the product with V, as the reference does.  q, out: (Tq, Hq,
 * D); k, v: (Tk, Hkv, D); token and head strides, head_dim contiguous, rows
 * 16-byte aligned; cu_seqlens int32 (batch + 1); head_dim 64 or 128. */
typedef struct {
    const void* q; int64_t q_stride_token, q_stride_head;
    const void* k; int64_t k_stride_token, k_stride_head;
    const void* v; int64_t v_stride_token, v_stride_head;
    void* out; int64_t out_stride_token, out_stride_head;
    const int32_t* cu_seqlens_q; const int32_t* cu_seqlens_k;
    int64_t batch, max_seqlen_q, num_q_heads, num_kv_heads, head_dim;
    int causal;
    float scale;
    int dtype;
    int32_t* status;  /* optional: QF_FLAG_TIMEOUT */
    int64_t total_q, total_k;  /* rows of q and of k/v (the tensor-core path's
                                  bulk copies stay inside them); 0 = unknown */
    int32_t* work_counter;     /* optional, 2 words of device memory, zero
                                  before their first use: the tensor-core path
                                  then runs one CTA per SM, claiming work from
                                  it, and leaves it at zero again when the call
                                  completes.  Calls that may overlap on the GPU
                                  (other streams) need counters of their own.
                                  NULL: one CTA per 256-query tile pair. */
} qf_varlen_attention_args;

int qf_varlen_attention(const qf_varlen_attention_args* args, cudaStream_t stream);

/* sizeof(qf_varlen_attention_args) as compiled into the library. */
size_t qf_varlen_attention_args_size(void);

/* ---------------------------------------------------------------------- */
/* Batched token sampling.  Replaces sample_tokens
 * (server/model/sampling.py:118-194): per row b of logits (batch, vocab),
 *   s = float(logits[b]) / max(temperature[b], 1e-5)
 *   order: s descending, ties by ascending index (a stable sort)
 *   top-k: keep the first k ranks (top_k <= 0 or >= vocab keeps all)
 *   softmax over the kept ranks; top-p: drop every rank whose probability
 *   mass before it exceeds top_p (rank 0 always stays)
 *   out[b] = the first rank whose cumulative mass reaches
 *            uniforms[b] * (kept mass), as a token id;
 *   temperature <= 0: out[b] = argmax (lowest index among equal maxima).
 * No sort: a radix select over the order-preserving bits of s, with the
 * probability masses held as exact fixed-point integers.
 * The uniforms come either from `uniforms` (float32) or, when that is NULL,
 * from the counter hash of (seeds[b], steps[b]) that
 * uniforms_from_seeds (server/model/determinism.py:30-73) computes on the
 * host.  temperature, top_p: float32; top_k: int32 or int64 (top_k_type);
 * seeds, steps: int64 (bits read as unsigned); out: int64.  logits rows are
 * contiguous, `logits_row_stride` elements apart. */
typedef struct {
    const void* logits; int64_t logits_row_stride;
    int64_t batch, vocab;
    int dtype;
    const float* temperature;
    const void* top_k; int top_k_type;
    const float* top_p;
    const float* uniforms;
    const int64_t* seeds; const int64_t* steps;
    int64_t* out;
    /* Scratch for the batch-wide path, at least qf_sample_workspace_bytes(batch)
     * bytes, 256-byte aligned; its contents need no initialisation.  Calls
     * that may overlap on the GPU need workspaces of their own.  NULL: every
     * row runs on the per-row cluster kernel. */
    void* workspace; int64_t workspace_bytes;
    /* QF_SAMPLE_PATH_AUTO: the batch-wide path when a workspace is given and
     * the batch is large enough; QF_SAMPLE_PATH_CLUSTER: the per-row cluster
     * kernel; QF_SAMPLE_PATH_WIDE: the batch-wide path (needs the workspace,
     * at most 65535 rows).  Every path returns the same tokens. */
    int path;
} qf_sample_args;

enum { QF_SAMPLE_PATH_AUTO = 0, QF_SAMPLE_PATH_CLUSTER = 1, QF_SAMPLE_PATH_WIDE = 2 };

int qf_sample_tokens(const qf_sample_args* args, cudaStream_t stream);

/* Bytes of workspace the batch-wide sampling path needs for `batch` rows
 * (~66 KB a row, whatever the vocabulary).  No counterpart in the reference,
 * whose sort allocates its own temporaries. */
int64_t qf_sample_workspace_bytes(int64_t batch);

/* sizeof(qf_sample_args) as compiled into the library. */
size_t qf_sample_args_size(void);

/* out[i] = uniform_from_hash(seeds[i], steps[i])
 * (server/model/determinism.py:30-51): splitmix64 of (seed, step), top 53
 * bits scaled by 2^-53, clamped to 1 - 2^-24, rounded to float32. */
int qf_uniforms_from_seeds(const int64_t* seeds, const int64_t* steps, int64_t n, float* out,
                           cudaStream_t stream);

/* ---------------------------------------------------------------------- */
/* Status word: copy *status_dev to *flags_out (host) after the work queued
 * on `stream` so far, then zero it when `clear` is set.  Synchronises
 * `stream`.  Returns QF_ERR_DEVICE when any flag was set. */
int qf_read_status(int32_t* status_dev, int32_t* flags_out, int clear, cudaStream_t stream);

/* Text of the last CUDA error seen by any entry point of this library in the
 * calling thread ("" when none). */
const char* qf_last_cuda_error(void);

/* Library version string, e.g. "qwen3fused 0.1.0 sm_100a". */
const char* qf_version(void);

#ifdef __cplusplus
}
#endif

#endif /* QWEN3FUSED_H */
