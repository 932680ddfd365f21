/*
 * qwen3_oracle.c -- CPU restatement of the Qwen3 decoder layer's memory-bound
 * op path, as the reference (nosyndicate/tinyserver, server/model) runs it.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  The
 * product path (tinyserver_b200) never links, imports or calls it, and has no
 * CPU fallback.
 *
 * Parity pin: every function here is checked against golden vectors produced
 * by the reference's own code (transformers 5.5.0 Qwen3 modules, which hold
 * the arithmetic the reference calls, and the reference's Triton KV-store
 * kernels run under TRITON_INTERPRET=1) -- see tests/golden/make_golden.py and
 * tests/test_oracle_golden.py.
 *
 * Where the reference is PyTorch eager code, each torch op rounds its result
 * to the tensor dtype.  The oracle reproduces those rounding points one by one
 * (compute in fp32, round to the storage dtype after every op), because that
 * is what makes a bf16 result "the reference's result".
 *
 * Third-party source of the arithmetic: transformers 5.5.0,
 * transformers/models/qwen3/modeling_qwen3.py (cited below as "HF:<line>").
 * Reference files are cited by their path inside the tinyserver project.
 *
 * Storage dtypes: 0 = float32, 1 = float16, 2 = bfloat16 (same tags as
 * include/qwen3fused.h).  Strides are in elements.  Return 0 on success,
 * nonzero on a bad argument or an out-of-range index.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };

static int esize(int dtype) {
    switch (dtype) {
    case OR_F32: return 4;
    case OR_F16: return 2;
    case OR_BF16: return 2;
    default: return 0;
    }
}

/* float32 -> bfloat16, round to nearest even (torch's c10::BFloat16 rule). */
static inline uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bf16_bits_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float load_el(const void* base, int64_t i, int dtype) {
    switch (dtype) {
    case OR_F32: return ((const float*)base)[i];
    case OR_F16: return (float)((const _Float16*)base)[i];
    default: return bf16_bits_to_f32(((const uint16_t*)base)[i]);
    }
}

static inline void store_el(void* base, int64_t i, float v, int dtype) {
    switch (dtype) {
    case OR_F32: ((float*)base)[i] = v; break;
    case OR_F16: ((_Float16*)base)[i] = (_Float16)v; break;
    default: ((uint16_t*)base)[i] = f32_to_bf16_bits(v); break;
    }
}

/* The value a torch op leaves behind when its fp32 result is stored in dtype. */
static inline float rnd(float v, int dtype) {
    switch (dtype) {
    case OR_F32: return v;
    case OR_F16: return (float)(_Float16)v;
    default: return bf16_bits_to_f32(f32_to_bf16_bits(v));
    }
}

static inline int64_t load_index(const void* p, int64_t i, int index_is_64) {
    return index_is_64 ? ((const int64_t*)p)[i] : (int64_t)((const int32_t*)p)[i];
}

/* ------------------------------------------------------------------------ */
/* Embedding gather: nn.Embedding forward, called as embed_tokens(input_ids)
 * at HF:392 (module built at HF:363).  out[t, :] = table[ids[t], :], a pure
 * copy; an id outside [0, V) is an error (torch raises IndexError). */
int oracle_embedding(const int64_t* ids, int64_t T, const void* table, int64_t V,
                     int64_t H, int64_t table_row_stride, int dtype, void* out,
                     int64_t out_row_stride) {
    int es = esize(dtype);
    if (!es || T < 0 || H < 0) return 1;
    for (int64_t t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= V) return 2;
    for (int64_t t = 0; t < T; ++t)
        memcpy((char*)out + t * out_row_stride * es,
               (const char*)table + ids[t] * table_row_stride * es, (size_t)(H * es));
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Qwen3RMSNorm.forward (HF:59-64) on one row, with the optional residual add
 * of the decoder layer (HF:327 / HF:333: `hidden_states = residual +
 * hidden_states`, a dtype-rounded add) in front of it:
 *   h   = rnd(res + x)                       (only when res != NULL)
 *   var = mean(float(h)^2)                   (fp32; HF:61-62)
 *   n   = rnd(float(h) * rsqrt(var + eps))   (HF:63, then .to(input_dtype) HF:64)
 *   y   = rnd(w * n)                         (HF:64, weight in the same dtype)
 * torch's CPU rsqrt on float is 1/sqrt, which is what is used here. */
static void rmsnorm_row(const void* x, const void* res, const void* w, int64_t H,
                        float eps, int dtype, void* h_out, void* y_out) {
    double acc = 0.0;
    for (int64_t i = 0; i < H; ++i) {
        float h = load_el(x, i, dtype);
        if (res) h = rnd(load_el(res, i, dtype) + h, dtype);
        acc += (double)h * (double)h;
    }
    float var = (float)(acc / (double)H);
    float inv = 1.0f / sqrtf(var + eps);
    for (int64_t i = 0; i < H; ++i) {
        float h = load_el(x, i, dtype);
        if (res) h = rnd(load_el(res, i, dtype) + h, dtype);
        float n = rnd(h * inv, dtype);
        float y = rnd(load_el(w, i, dtype) * n, dtype);
        if (h_out) store_el(h_out, i, h, dtype);
        store_el(y_out, i, y, dtype);
    }
}

int oracle_rmsnorm(const void* x, int64_t x_row_stride, const void* w, int64_t T, int64_t H,
                   float eps, int dtype, void* out, int64_t out_row_stride) {
    int es = esize(dtype);
    if (!es || T < 0 || H <= 0) return 1;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        rmsnorm_row((const char*)x + t * x_row_stride * es, NULL, w, H, eps, dtype, NULL,
                    (char*)out + t * out_row_stride * es);
    return 0;
}

/* Residual add + RMSNorm; rows are contiguous with row stride H.
 * h_out receives the new residual stream (residual + x), y_out the normed row. */
int oracle_add_rmsnorm(const void* x, const void* res, const void* w, int64_t T, int64_t H,
                       float eps, int dtype, void* h_out, void* y_out) {
    int es = esize(dtype);
    if (!es || T < 0 || H <= 0) return 1;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        rmsnorm_row((const char*)x + t * H * es, (const char*)res + t * H * es, w, H, eps, dtype,
                    (char*)h_out + t * H * es, (char*)y_out + t * H * es);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Qwen3RotaryEmbedding.forward (HF:137-148), default rope type:
 *   freqs[t, i] = inv_freq[i] * float(pos[t])          (fp32, HF:143; a K=1 matmul)
 *   emb = cat(freqs, freqs)                             (HF:144)
 *   cos = rnd(cos(emb) * scaling), sin likewise         (HF:145-148)
 * inv_freq (D/2 floats) is passed in: the caller computes it exactly as
 * compute_default_rope_parameters does (HF:125-132) with torch. */
int oracle_rope_cos_sin(const int64_t* pos, int64_t T, const float* inv_freq, int64_t D,
                        float scaling, int dtype, void* cos_out, void* sin_out) {
    int es = esize(dtype);
    if (!es || T < 0 || D <= 0 || (D & 1)) return 1;
    int64_t half = D / 2;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        float p = (float)pos[t];
        for (int64_t i = 0; i < D; ++i) {
            float f = inv_freq[i % half] * p;
            store_el(cos_out, t * D + i, cosf(f) * scaling, dtype);
            store_el(sin_out, t * D + i, sinf(f) * scaling, dtype);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* apply_rotary_pos_emb + rotate_half (HF:151-155, HF:159-181) on one head row
 * of length D (neox layout: element i pairs with i + D/2):
 *   out[i]       = rnd(rnd(x[i] * cos[i])           + rnd(-x[i+D/2] * sin[i]))
 *   out[i+D/2]   = rnd(rnd(x[i+D/2] * cos[i+D/2])   + rnd( x[i]     * sin[i+D/2]))
 * x is the dtype-rounded input (q_norm/k_norm output in the reference). */
static void rope_row(const float* x, const void* cos_row, const void* sin_row, int64_t D,
                     int dtype, float* out) {
    int64_t half = D / 2;
    for (int64_t i = 0; i < D; ++i) {
        float rot = (i < half) ? -x[i + half] : x[i - half];
        float a = rnd(x[i] * load_el(cos_row, i, dtype), dtype);
        float b = rnd(rot * load_el(sin_row, i, dtype), dtype);
        out[i] = rnd(a + b, dtype);
    }
}

/* ------------------------------------------------------------------------ */
/* The reference's attention pre-processing for one batch (server/model/
 * patches/qwen3.py:264-318): views of the q/k/v projections, q_norm/k_norm
 * (qwen3.py:268-271 -> HF:248-249, a Qwen3RMSNorm over head_dim), RoPE
 * (qwen3.py:287 -> HF:159-181), then the paged KV store of the rotated K and
 * the untouched V (qwen3.py:311-318 -> kv_cache.py:122-191).
 *
 * Layouts (strides in elements, last dim contiguous):
 *   q: (T, Hq, D) with strides (q_st, q_sh); k, v: (T, Hkv, D) likewise
 *   cos/sin: (T, D) rows with stride cs_st
 *   q_out: (T, Hq, D) contiguous; k_out (may be NULL): (T, Hkv, D) contiguous
 *   caches: (N, Hkv, B, D) with strides c[0..3] (may be NULL: no store)
 *   block_mapping/slot_mapping: (T,) int32 or int64
 * q_w/k_w may be NULL: no norm (plain RoPE, the apply_rotary_pos_emb drop-in).
 */
int oracle_qk_norm_rope_store(const void* q, int64_t q_st, int64_t q_sh, const void* k,
                              int64_t k_st, int64_t k_sh, const void* v, int64_t v_st,
                              int64_t v_sh, const void* q_w, const void* k_w, float eps,
                              const void* cos, const void* sin, int64_t cs_st, int64_t T,
                              int64_t Hq, int64_t Hkv, int64_t D, int dtype, void* q_out,
                              void* k_out, void* k_cache, void* v_cache, const int64_t* c,
                              int64_t N, int64_t B, const void* block_mapping,
                              const void* slot_mapping, int index_is_64) {
    int es = esize(dtype);
    if (!es || T < 0 || D <= 0 || (D & 1) || D > 1024) return 1;
    if (k_cache && (!block_mapping || !slot_mapping || !v)) return 1;
    if (k_cache) {
        for (int64_t t = 0; t < T; ++t) {
            int64_t bi = load_index(block_mapping, t, index_is_64);
            int64_t si = load_index(slot_mapping, t, index_is_64);
            if (bi < 0 || bi >= N || si < 0 || si >= B) return 2;
        }
    }
    int64_t H = Hq + Hkv;
    /* Serial order over tokens keeps the store deterministic (the last token
     * mapped to a slot wins) even for colliding mappings. */
    for (int64_t t = 0; t < T; ++t) {
        for (int64_t hh = 0; hh < H; ++hh) {
            int is_q = hh < Hq;
            int64_t h = is_q ? hh : hh - Hq;
            const char* src = is_q ? (const char*)q + (t * q_st + h * q_sh) * es
                                   : (const char*)k + (t * k_st + h * k_sh) * es;
            const void* w = is_q ? q_w : k_w;
            float xin[1024], xn[1024], xo[1024];
            for (int64_t i = 0; i < D; ++i) xin[i] = load_el(src, i, dtype);
            if (w) {
                double acc = 0.0;
                for (int64_t i = 0; i < D; ++i) acc += (double)xin[i] * (double)xin[i];
                float inv = 1.0f / sqrtf((float)(acc / (double)D) + eps);
                for (int64_t i = 0; i < D; ++i)
                    xn[i] = rnd(load_el(w, i, dtype) * rnd(xin[i] * inv, dtype), dtype);
            } else {
                for (int64_t i = 0; i < D; ++i) xn[i] = xin[i];
            }
            rope_row(xn, (const char*)cos + t * cs_st * es, (const char*)sin + t * cs_st * es, D,
                     dtype, xo);
            if (is_q) {
                for (int64_t i = 0; i < D; ++i) store_el(q_out, (t * Hq + h) * D + i, xo[i], dtype);
            } else {
                if (k_out)
                    for (int64_t i = 0; i < D; ++i)
                        store_el(k_out, (t * Hkv + h) * D + i, xo[i], dtype);
                if (k_cache) {
                    int64_t bi = load_index(block_mapping, t, index_is_64);
                    int64_t si = load_index(slot_mapping, t, index_is_64);
                    int64_t off = bi * c[0] + h * c[1] + si * c[2];
                    for (int64_t i = 0; i < D; ++i) store_el(k_cache, off + i * c[3], xo[i], dtype);
                    const char* vs = (const char*)v + (t * v_st + h * v_sh) * es;
                    for (int64_t i = 0; i < D; ++i)
                        store_el(v_cache, off + i * c[3], load_el(vs, i, dtype), dtype);
                }
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Paged KV-cache stores (server/model/kernels/kv_cache.py).  Both are byte
 * copies of whole head rows; all strides are honoured (kv_cache.py:117-118,
 * 248-250).  src: (Hkv, T, D) with strides s[0..2]; caches: (N, Hkv, B, D)
 * with strides c[0..3].  Out-of-range block/slot indices are an error (the
 * reference does not check them; its Triton kernels would write out of
 * bounds). */
static void copy_row(const void* src, const int64_t* s, int64_t h, int64_t t, void* dst,
                     int64_t dst_off, const int64_t* c, int64_t D, int es) {
    for (int64_t d = 0; d < D; ++d)
        memcpy((char*)dst + (dst_off + d * c[3]) * es,
               (const char*)src + (h * s[0] + t * s[1] + d * s[2]) * es, (size_t)es);
}

/* store_kv_cache_batched (kv_cache.py:194-251, kernel 122-191):
 *   cache[bm[t], h, sm[t], :] = src[h, t, :] for every t < T, h < Hkv. */
int oracle_kv_store_batched(const void* k_src, const int64_t* ks, const void* v_src,
                            const int64_t* vs, void* k_cache, void* v_cache, const int64_t* c,
                            const void* block_mapping, const void* slot_mapping,
                            int index_is_64, int64_t T, int64_t Hkv, int64_t D, int64_t N,
                            int64_t B, int dtype_size) {
    if (dtype_size <= 0 || T < 0) return 1;
    for (int64_t t = 0; t < T; ++t) {
        int64_t bi = load_index(block_mapping, t, index_is_64);
        int64_t si = load_index(slot_mapping, t, index_is_64);
        if (bi < 0 || bi >= N || si < 0 || si >= B) return 2;
    }
    for (int64_t t = 0; t < T; ++t) {
        int64_t bi = load_index(block_mapping, t, index_is_64);
        int64_t si = load_index(slot_mapping, t, index_is_64);
        for (int64_t h = 0; h < Hkv; ++h) {
            int64_t off = bi * c[0] + h * c[1] + si * c[2];
            copy_row(k_src, ks, h, t, k_cache, off, c, D, dtype_size);
            copy_row(v_src, vs, h, t, v_cache, off, c, D, dtype_size);
        }
    }
    return 0;
}

/* store_kv_cache (kv_cache.py:73-119, kernel 6-70), one sequence:
 *   pos = start + i; blk = block_table[pos // B]; slot = pos % B
 *   cache[blk, h, slot, :] = src[h, i, :] */
int oracle_kv_store_seq(int64_t start_position, const void* block_table, int64_t table_len,
                        int index_is_64, const void* k_src, const int64_t* ks,
                        const void* v_src, const int64_t* vs, void* k_cache, void* v_cache,
                        const int64_t* c, int64_t T, int64_t Hkv, int64_t D, int64_t N,
                        int64_t B, int dtype_size) {
    if (dtype_size <= 0 || T < 0 || B <= 0 || start_position < 0) return 1;
    for (int64_t i = 0; i < T; ++i) {
        int64_t pos = start_position + i;
        if (pos / B >= table_len) return 2;
        int64_t bi = load_index(block_table, pos / B, index_is_64);
        if (bi < 0 || bi >= N) return 2;
    }
    for (int64_t i = 0; i < T; ++i) {
        int64_t pos = start_position + i;
        int64_t bi = load_index(block_table, pos / B, index_is_64);
        int64_t si = pos % B;
        for (int64_t h = 0; h < Hkv; ++h) {
            int64_t off = bi * c[0] + h * c[1] + si * c[2];
            copy_row(k_src, ks, h, i, k_cache, off, c, D, dtype_size);
            copy_row(v_src, vs, h, i, v_cache, off, c, D, dtype_size);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Qwen3MLP's activation product (HF:81-83, `act_fn(gate_proj(x)) * up_proj(x)`
 * with act_fn = ACT2FN["silu"]): torch's silu is x / (1 + exp(-x)) in fp32,
 * rounded to the dtype; the product is rounded again:
 *   out = rnd(rnd(g / (1 + exp(-g))) * u)
 * gate/up rows have their own strides so a merged [T, 2I] (gate first) and
 * two separate [T, I] tensors are both covered. */
int oracle_silu_and_mul(const void* gate, int64_t gate_row_stride, const void* up,
                        int64_t up_row_stride, int64_t T, int64_t I, int dtype, void* out,
                        int64_t out_row_stride) {
    int es = esize(dtype);
    if (!es || T < 0 || I < 0) return 1;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const char* g = (const char*)gate + t * gate_row_stride * es;
        const char* u = (const char*)up + t * up_row_stride * es;
        char* o = (char*)out + t * out_row_stride * es;
        for (int64_t i = 0; i < I; ++i) {
            float gv = load_el(g, i, dtype);
            float s = rnd(gv / (1.0f + expf(-gv)), dtype);
            store_el(o, i, s * load_el(u, i, dtype), dtype);
        }
    }
    return 0;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
