// q_norm / k_norm + neox RoPE + paged KV store, fused; and the RoPE tables.
//
// Replaces, in the reference's attention forward (server/model/patches/
// qwen3.py:264-318), the chain
//   q_norm, k_norm          (qwen3.py:268-271 -> Qwen3RMSNorm over head_dim,
//                            transformers 5.5.0 modeling_qwen3.py:59-64, :248-249)
//   apply_rotary_pos_emb    (qwen3.py:287 -> modeling_qwen3.py:151-181)
//   .contiguous() copies + store_kv_cache_batched of K and V (qwen3.py:311-318,
//                            server/model/kernels/kv_cache.py:122-251)
// with one pass over q, k and v: each head row is read once into registers,
// normalised, rotated and written once (q_out, optionally k_out) and K/V rows
// go straight into their cache pages.
//
// Work split: a head row of D elements is handled by G = D/8 lanes; lane l
// holds elements [4l, 4l+4) of the first half and the same four of the second
// half, so the neox pairs (i, i + D/2) of the rotation sit in one register
// file and need no shuffle.  The RMS reduction is a G-lane butterfly.  A warp
// handles 32/G head rows per step and two steps per iteration (more loads in
// flight); every lane of a warp runs the same iterations, so the shuffles are
// always convergent.
//
// Rounding follows the reference op by op (all math fp32, rnd = to dtype):
//   n   = rnd(w * rnd(x * rsqrt(mean(x^2) + eps)))                   (norm)
//   out = rnd(rnd(n * cos) + rnd(rotate_half(n) * sin))               (RoPE)
// and cos/sin are the dtype-rounded table values (modeling_qwen3.py:148).
#include "qf_common.cuh"

namespace qf {
namespace {

// Four consecutive elements as one load: 8 bytes for 16-bit types, 16 for fp32.
template <typename T>
struct Quad {
    using Raw = uint2;
    __device__ __forceinline__ static Raw ld_stream(const char* p) { return ld_stream8(p); }
    __device__ __forceinline__ static Raw ld_cached(const char* p) {
        return __ldg(reinterpret_cast<const uint2*>(p));
    }
};
template <>
struct Quad<float> {
    using Raw = uint4;
    __device__ __forceinline__ static Raw ld_stream(const char* p) { return ld_stream16(p); }
    __device__ __forceinline__ static Raw ld_cached(const char* p) {
        return __ldg(reinterpret_cast<const uint4*>(p));
    }
};

template <typename T>
__device__ __forceinline__ void unpack4(const typename Quad<T>::Raw& r, float* f) {
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = Dt<T>::to_f(e[i]);
}

template <typename T>
__device__ __forceinline__ typename Quad<T>::Raw pack4(const float* f) {
    typename Quad<T>::Raw r;
    T* e = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = Dt<T>::from_f(f[i]);
    return r;
}

template <typename T>
__device__ __forceinline__ void st4(char* p, const typename Quad<T>::Raw& r) {
    *reinterpret_cast<typename Quad<T>::Raw*>(p) = r;
}

struct QkDev {
    const char* q;
    int64_t q_st, q_sh;
    const char* k;
    int64_t k_st, k_sh;
    const char* v;
    int64_t v_st, v_sh;
    const char* qw;
    const char* kw;
    float eps;
    const char* cos;
    const char* sin;
    int64_t cs_st;
    const void* pos;
    int pos_type;
    const float* inv_freq;
    char* q_out;
    int64_t qo_st, qo_sh;
    char* k_out;
    int64_t ko_st, ko_sh;
    char* k_cache;
    char* v_cache;
    int64_t c0, c1, c2;
    int64_t N, B;
    const void* bm;
    const void* sm;
    int idx_type;
    int64_t T, Hq, Hkv;
    int64_t tasks_per_token;  // Hq + Hkv, plus Hkv V rows when storing
    int store;
    int32_t* status;
};

__device__ __forceinline__ float inv_rms(float sum_sq, int n, float eps) {
    const float var = __fdiv_rn(sum_sq, (float)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

__device__ __forceinline__ bool cache_slot(const QkDev& a, int64_t t, int64_t& blk,
                                           int64_t& slot, bool report) {
    blk = load_index(a.bm, t, a.idx_type);
    slot = load_index(a.sm, t, a.idx_type);
    const bool bad_b = blk < 0 || blk >= a.N;
    const bool bad_s = slot < 0 || slot >= a.B;
    if (report && (bad_b || bad_s))
        flag(a.status, (bad_b ? QF_FLAG_BAD_BLOCK : 0) | (bad_s ? QF_FLAG_BAD_SLOT : 0));
    return !bad_b && !bad_s;
}

template <typename T, int D, typename IT>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const QkDev a) {
    constexpr int G = D / 8;      // lanes per head row
    constexpr int HPW = 32 / G;   // head rows per warp per step
    constexpr int HALF = D / 2;
    constexpr int U = 2;          // steps per iteration
    constexpr int64_t ES = sizeof(T);
    using Q = Quad<T>;
    using Raw = typename Q::Raw;

    const int lane = threadIdx.x & 31;
    const int sub = lane / G;
    const int gl = lane - sub * G;
    const int e0 = gl * 4;
    const int64_t off1 = e0 * ES, off2 = (HALF + e0) * ES;

    float qw1[4], qw2[4], kw1[4], kw2[4];
    if (a.qw) {
        unpack4<T>(Q::ld_cached(a.qw + off1), qw1);
        unpack4<T>(Q::ld_cached(a.qw + off2), qw2);
    }
    if (a.kw) {
        unpack4<T>(Q::ld_cached(a.kw + off1), kw1);
        unpack4<T>(Q::ld_cached(a.kw + off2), kw2);
    }

    const IT tpt = (IT)a.tasks_per_token;
    const IT total = (IT)a.T * tpt;
    const IT warp = ((IT)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const IT nwarp = ((IT)gridDim.x * blockDim.x) >> 5;
    const IT Hq = (IT)a.Hq, Hkv = (IT)a.Hkv;

    for (IT base = warp * (HPW * U); base < total; base += nwarp * (HPW * U)) {
        Raw r1[U], r2[U];
        int64_t tt[U], hh[U];
        int kind[U];
        bool act[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const IT task = base + (IT)(u * HPW + sub);
            act[u] = task < total;
            const IT t = act[u] ? task / tpt : 0;
            const IT hx = act[u] ? task - t * tpt : 0;
            tt[u] = (int64_t)t;
            const char* src;
            if (hx < Hq) {
                kind[u] = 0;
                hh[u] = (int64_t)hx;
                src = a.q + (tt[u] * a.q_st + hh[u] * a.q_sh) * ES;
            } else if (hx < Hq + Hkv) {
                kind[u] = 1;
                hh[u] = (int64_t)(hx - Hq);
                src = a.k + (tt[u] * a.k_st + hh[u] * a.k_sh) * ES;
            } else {
                kind[u] = 2;
                hh[u] = (int64_t)(hx - Hq - Hkv);
                src = a.v + (tt[u] * a.v_st + hh[u] * a.v_sh) * ES;
            }
            if (act[u]) {
                r1[u] = Q::ld_stream(src + off1);
                r2[u] = Q::ld_stream(src + off2);
            }
        }

        float x1[U][4], x2[U][4], ss[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            ss[u] = 0.f;
            if (act[u] && kind[u] < 2) {
                unpack4<T>(r1[u], x1[u]);
                unpack4<T>(r2[u], x2[u]);
                if (kind[u] == 0 ? a.qw != nullptr : a.kw != nullptr) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        ss[u] = fmaf(x1[u][j], x1[u][j], ss[u]);
                        ss[u] = fmaf(x2[u][j], x2[u][j], ss[u]);
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
        }

#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (!act[u]) continue;
            const int64_t t = tt[u], h = hh[u];
            if (kind[u] == 2) {  // V row: bit-exact copy into its page
                int64_t blk, slot;
                if (cache_slot(a, t, blk, slot, gl == 0 && h == 0)) {
                    char* dst = a.v_cache + (blk * a.c0 + h * a.c1 + slot * a.c2) * ES;
                    st4<T>(dst + off1, r1[u]);
                    st4<T>(dst + off2, r2[u]);
                }
                continue;
            }
            const bool is_q = kind[u] == 0;
            float n1[4], n2[4];
            const bool has_w = is_q ? a.qw != nullptr : a.kw != nullptr;
            if (has_w) {
                const float inv = inv_rms(ss[u], D, a.eps);
                const float* w1 = is_q ? qw1 : kw1;
                const float* w2 = is_q ? qw2 : kw2;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    n1[j] = rnd<T>(__fmul_rn(w1[j], rnd<T>(__fmul_rn(x1[u][j], inv))));
                    n2[j] = rnd<T>(__fmul_rn(w2[j], rnd<T>(__fmul_rn(x2[u][j], inv))));
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    n1[j] = x1[u][j];
                    n2[j] = x2[u][j];
                }
            }
            float c1[4], c2[4], s1[4], s2[4];
            if (a.cos) {
                const char* cr = a.cos + t * a.cs_st * ES;
                const char* sr = a.sin + t * a.cs_st * ES;
                unpack4<T>(Q::ld_cached(cr + off1), c1);
                unpack4<T>(Q::ld_cached(cr + off2), c2);
                unpack4<T>(Q::ld_cached(sr + off1), s1);
                unpack4<T>(Q::ld_cached(sr + off2), s2);
            } else {
                const float p = (float)load_index(a.pos, t, a.pos_type);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float sv, cv;
                    sincosf(__fmul_rn(__ldg(a.inv_freq + e0 + j), p), &sv, &cv);
                    c1[j] = c2[j] = rnd<T>(cv);
                    s1[j] = s2[j] = rnd<T>(sv);
                }
            }
            float o1[4], o2[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                o1[j] = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(n1[j], c1[j])),
                                         rnd<T>(__fmul_rn(-n2[j], s1[j]))));
                o2[j] = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(n2[j], c2[j])),
                                         rnd<T>(__fmul_rn(n1[j], s2[j]))));
            }
            const Raw p1 = pack4<T>(o1), p2 = pack4<T>(o2);
            if (is_q) {
                char* dst = a.q_out + (t * a.qo_st + h * a.qo_sh) * ES;
                st4<T>(dst + off1, p1);
                st4<T>(dst + off2, p2);
            } else {
                if (a.k_out) {
                    char* dst = a.k_out + (t * a.ko_st + h * a.ko_sh) * ES;
                    st4<T>(dst + off1, p1);
                    st4<T>(dst + off2, p2);
                }
                int64_t blk, slot;
                if (a.store && cache_slot(a, t, blk, slot, gl == 0 && h == 0)) {
                    char* dst = a.k_cache + (blk * a.c0 + h * a.c1 + slot * a.c2) * ES;
                    st4<T>(dst + off1, p1);
                    st4<T>(dst + off2, p2);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// 16-byte path (the serving layout: every row start and stride 16-byte
// aligned).  Work unit = (token, step): HPW consecutive head rows of one
// token from its row list [q heads | k heads | v heads when storing].  A head
// row is split over G lanes (2 for 16-bit D <= 256); lane g of a row holds the
// 16-byte chunks g, g + G, g + 2G, ... of the first half and the same chunks
// of the second half, so
//  * the neox pairs (i, i + D/2) of the rotation are in one lane,
//  * the G lanes of a row touch G adjacent chunks per instruction (whole
//    32-byte sectors for G = 2),
//  * the RMS reduction is log2(G) shuffles, and
//  * everything that depends only on the token (row bases, the cos/sin row,
//    the cache slot) is set up once per unit and shared by HPW rows.
// For 16-bit types the norm's weight multiply and all of RoPE run as packed
// .rn ops (see Packed), which round exactly where torch's separate kernels do.
// Lanes per head row, CTAs per SM the register budget is sized for, and warp
// steps per work unit (compile-time knobs; the defaults are the best of
// sweeps on B200 at Qwen3-8B shapes: 2/4/8 lanes per row, 1/2/3/6 steps per
// unit, with and without prefetching the next unit).
#ifndef QF_QK_LANES
#define QF_QK_LANES 4
#endif
#ifndef QF_QK_MIN_CTAS
#define QF_QK_MIN_CTAS 3
#endif
#ifndef QF_QK_STEPS
#define QF_QK_STEPS 2  // warp steps (HPW head rows each) per work unit
#endif
#ifndef QF_QK_CONTIG
#define QF_QK_CONTIG 1  // each warp takes a contiguous range of units (a token's in a row)
#endif

template <typename T, int D>
struct Wide {
    static constexpr int EPV = 16 / (int)sizeof(T);  // elements per 16-byte chunk
    static constexpr int NCH = D / 2 / EPV;          // chunks per half row
    static constexpr int G0 = QF_QK_LANES < NCH ? QF_QK_LANES : NCH;
    static constexpr int G = NCH / 8 > G0 ? NCH / 8 : G0;  // lanes per row
    static constexpr int C = NCH / G;                // chunk pairs per lane
    static constexpr int HPW = 32 / G;               // head rows per warp step
    static_assert(NCH % G == 0 && C >= 1 && C <= 8, "unsupported head_dim");
};

// norm + RoPE of one head row held as two 16-byte vectors (x1: first half, x2:
// second half); w1/w2 the weight vectors, c1/c2/s1/s2 the cos/sin vectors.
template <typename T>
__device__ __forceinline__ void norm_rope_vec(uint4& x1, uint4& x2, bool has_w, float inv,
                                              const uint4& w1, const uint4& w2, const uint4& c1,
                                              const uint4& c2, const uint4& s1,
                                              const uint4& s2) {
    if constexpr (sizeof(T) == 2) {
        using P = Packed<T>;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t a = word(x1, i), b = word(x2, i);
            if (has_w) {
                a = P::mul(P::pack(__fmul_rn(P::lo(a), inv), __fmul_rn(P::hi(a), inv)),
                           word(w1, i));
                b = P::mul(P::pack(__fmul_rn(P::lo(b), inv), __fmul_rn(P::hi(b), inv)),
                           word(w2, i));
            }
            // out1 = x1*cos1 - x2*sin1 ; out2 = x2*cos2 + x1*sin2   (rotate_half)
            set_word(x1, i, P::sub(P::mul(a, word(c1, i)), P::mul(b, word(s1, i))));
            set_word(x2, i, P::add(P::mul(b, word(c2, i)), P::mul(a, word(s2, i))));
        }
    } else {
        const float* fx1 = reinterpret_cast<const float*>(&x1);
        const float* fx2 = reinterpret_cast<const float*>(&x2);
        const float* fw1 = reinterpret_cast<const float*>(&w1);
        const float* fw2 = reinterpret_cast<const float*>(&w2);
        const float* fc1 = reinterpret_cast<const float*>(&c1);
        const float* fc2 = reinterpret_cast<const float*>(&c2);
        const float* fs1 = reinterpret_cast<const float*>(&s1);
        const float* fs2 = reinterpret_cast<const float*>(&s2);
        float o1[4], o2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float a = fx1[i], b = fx2[i];
            if (has_w) {
                a = __fmul_rn(fw1[i], __fmul_rn(a, inv));
                b = __fmul_rn(fw2[i], __fmul_rn(b, inv));
            }
            o1[i] = __fadd_rn(__fmul_rn(a, fc1[i]), __fmul_rn(-b, fs1[i]));
            o2[i] = __fadd_rn(__fmul_rn(b, fc2[i]), __fmul_rn(a, fs2[i]));
        }
        x1 = make_uint4(__float_as_uint(o1[0]), __float_as_uint(o1[1]), __float_as_uint(o1[2]),
                        __float_as_uint(o1[3]));
        x2 = make_uint4(__float_as_uint(o2[0]), __float_as_uint(o2[1]), __float_as_uint(o2[2]),
                        __float_as_uint(o2[3]));
    }
}

// 1 / sqrt(mean(x^2) + eps) with the same IEEE roundings as inv_rms, cheaper:
// for a power-of-two D the division by D is an exact multiply, and a
// correctly rounded reciprocal equals the correctly rounded 1/x division.
template <int D>
__device__ __forceinline__ float inv_rms_pow2(float sum_sq, float eps) {
    static_assert((D & (D - 1)) == 0, "D must be a power of two");
    return __frcp_rn(__fsqrt_rn(__fadd_rn(sum_sq * (1.0f / D), eps)));
}

// Per-warp staging of one token's cos and sin rows in shared memory (layout
// cos[0:D] | sin[0:D]): copied from the table, or computed in the kernel with
// each frequency evaluated once (cos[i] = cos[i + D/2], as the table built by
// cat(freqs, freqs) holds it).
template <typename T, int D>
__device__ __forceinline__ void stage_cos_sin(uint4* cs, const char* cos_row,
                                              const char* sin_row, const float* inv_freq,
                                              float p, int lane) {
    constexpr int NCHR = D * (int)sizeof(T) / 16;  // chunks per full row
    if (cos_row) {
        for (int i = lane; i < 2 * NCHR; i += 32)
            cs[i] = ld_shared_ro16(i < NCHR ? cos_row + i * 16 : sin_row + (i - NCHR) * 16);
    } else {
        constexpr int HALF = D / 2;
        T* e = reinterpret_cast<T*>(cs);
        for (int j = lane; j < HALF; j += 32) {
            float sv, cv;
            sincosf(__fmul_rn(__ldg(inv_freq + j), p), &sv, &cv);
            e[j] = e[HALF + j] = Dt<T>::from_f(cv);
            e[D + j] = e[D + HALF + j] = Dt<T>::from_f(sv);
        }
    }
}

// One warp step's rows in registers (HPW head rows of one token), and what
// they are.
template <typename T, int D>
struct StepRows {
    uint4 x1[Wide<T, D>::C], x2[Wide<T, D>::C];
    int kind;  // 0 q, 1 k, 2 v, 3 past the last row
    int h;     // head index within its kind
};

template <typename T, int D>
__device__ __forceinline__ void load_step(const QkDev& a, int64_t t, int step, int sub, int gl,
                                          StepRows<T, D>& r) {
    using W = Wide<T, D>;
    constexpr int64_t ES = sizeof(T);
    const int row = step * W::HPW + sub;
    const int Hq = (int)a.Hq, Hkv = (int)a.Hkv;
    r.kind = row < Hq ? 0 : row < Hq + Hkv ? 1 : row < (int)a.tasks_per_token ? 2 : 3;
    r.h = r.kind == 0 ? row : r.kind == 1 ? row - Hq : row - Hq - Hkv;
    const char* src = r.kind == 0   ? a.q + (t * a.q_st + (int64_t)r.h * a.q_sh) * ES
                      : r.kind == 1 ? a.k + (t * a.k_st + (int64_t)r.h * a.k_sh) * ES
                                    : a.v + (t * a.v_st + (int64_t)r.h * a.v_sh) * ES;
    if (r.kind < 3) {
#pragma unroll
        for (int m = 0; m < W::C; ++m) {
            r.x1[m] = ld_stream16(src + (gl + W::G * m) * 16);
            r.x2[m] = ld_stream16(src + (D / 2) * ES + (gl + W::G * m) * 16);
        }
    }
}

// Norm, RoPE and the stores of one warp step; csm holds the token's cos/sin
// rows and cache_off the byte offset of its (block, head 0, slot) page row.
template <typename T, int D>
__device__ __forceinline__ void process_step(const QkDev& a, int64_t t, StepRows<T, D>& r,
                                             int gl, const uint4 (*wsm)[D * sizeof(T) / 16],
                                             const uint4* csm, bool slot_ok,
                                             int64_t cache_off) {
    using W = Wide<T, D>;
    constexpr int G = W::G, C = W::C, NCH = W::NCH;
    constexpr int64_t ES = sizeof(T);
    constexpr int HALF = D / 2;
    const int kind = r.kind, h = r.h;

    const bool has_w = kind == 0 ? a.qw != nullptr : a.kw != nullptr;
    float ss = 0.f;
    if (kind < 2 && has_w) {
#pragma unroll
        for (int m = 0; m < C; ++m) ss += sum_sq16<T>(r.x1[m]) + sum_sq16<T>(r.x2[m]);
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);

    char* dst = nullptr;
    char* dst2 = nullptr;
    if (kind == 2) {  // V row: bit-exact copy into its page
        if (slot_ok) dst = a.v_cache + cache_off + (int64_t)h * a.c1 * ES;
    } else if (kind < 2) {
        const float inv = has_w ? inv_rms_pow2<D>(ss, a.eps) : 1.f;
        const uint4* w = wsm[kind];
#pragma unroll
        for (int m = 0; m < C; ++m) {
            const int c = gl + G * m;
            norm_rope_vec<T>(r.x1[m], r.x2[m], has_w, inv, w[c], w[NCH + c], csm[c],
                             csm[NCH + c], csm[2 * NCH + c], csm[3 * NCH + c]);
        }
        if (kind == 0) {
            dst = a.q_out + (t * a.qo_st + (int64_t)h * a.qo_sh) * ES;
        } else {
            if (a.k_out) dst2 = a.k_out + (t * a.ko_st + (int64_t)h * a.ko_sh) * ES;
            if (slot_ok) dst = a.k_cache + cache_off + (int64_t)h * a.c1 * ES;
        }
    }
    if (dst) {
#pragma unroll
        for (int m = 0; m < C; ++m) {
            st16(dst + (gl + G * m) * 16, r.x1[m]);
            st16(dst + HALF * ES + (gl + G * m) * 16, r.x2[m]);
        }
    }
    if (dst2) {
#pragma unroll
        for (int m = 0; m < C; ++m) {
            st16(dst2 + (gl + G * m) * 16, r.x1[m]);
            st16(dst2 + HALF * ES + (gl + G * m) * 16, r.x2[m]);
        }
    }
}

// Grid-stride over units of U warp steps of one token.  A unit issues the
// loads of all its steps first, then does the per-token work once (the
// position and cache-slot lookups, the cos/sin staging), then runs the steps'
// independent arithmetic back to back, which gives the scheduler U chains to
// interleave.
template <typename T, int D, typename IT>
__global__ void __launch_bounds__(256, Wide<T, D>::C > 4 ? 2 : QF_QK_MIN_CTAS)
    qk_norm_rope_wide_kernel(const QkDev a, const IT steps, const IT upt, const IT units) {
    using W = Wide<T, D>;
    constexpr int G = W::G, NCH = W::NCH, HPW = W::HPW;
    constexpr int U = QF_QK_STEPS;
    constexpr int NV = 2 * NCH;  // 16-byte chunks per weight vector
    constexpr int64_t ES = sizeof(T);

    __shared__ uint4 wsm[2][NV];        // q_norm and k_norm weights
    __shared__ uint4 csm[8][4 * NCH];   // per warp: the current token's cos | sin rows
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < 2 * NV; i += blockDim.x) {
        const char* w = i < NV ? a.qw : a.kw;
        const int j = i < NV ? i : i - NV;
        wsm[i < NV ? 0 : 1][j] = w ? ld_shared_ro16(w + j * 16) : make_uint4(0, 0, 0, 0);
    }
    __syncthreads();

    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int sub = lane / G;
    const int gl = lane - sub * G;
    const int Hq = (int)a.Hq;
    const IT warp = ((IT)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const IT nwarp = ((IT)gridDim.x * blockDim.x) >> 5;
    int64_t staged = -1;  // token whose cos/sin rows csm[wib] holds
#if QF_QK_CONTIG
    // consecutive units belong to one token, so the cos/sin staging and the
    // position load happen once per token and warp
    const IT u_begin = (IT)((uint64_t)units * warp / nwarp);
    const IT u_end = (IT)((uint64_t)units * (warp + 1) / nwarp);
    for (IT unit = u_begin; unit < u_end; ++unit) {
#else
    for (IT unit = warp; unit < units; unit += nwarp) {
#endif
        const IT tu = unit / upt;
        const int64_t t = (int64_t)tu;
        const int s0 = (int)(unit - tu * upt) * U;
        const int row0 = s0 * HPW, row_end = (s0 + U) * HPW;  // this unit's row range

        // per-token index loads first: they complete under the row loads
        const bool rope = row0 < Hq + (int)a.Hkv;
        const float pos = rope && !a.cos && t != staged ? (float)load_index(a.pos, t, a.pos_type)
                                                        : 0.f;
        int64_t blk = 0, slot = 0;
        const bool slot_ok = a.store && row_end > Hq &&
                             cache_slot(a, t, blk, slot, lane == 0 && row0 <= Hq);
        const int64_t cache_off = (blk * a.c0 + slot * a.c2) * ES;

        StepRows<T, D> r[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (s0 + u < (int)steps) load_step<T, D>(a, t, s0 + u, sub, gl, r[u]);
            else r[u].kind = 3;
        }
        if (rope && t != staged) {
            __syncwarp();  // the previous unit's reads of csm are done
            stage_cos_sin<T, D>(csm[wib], a.cos ? a.cos + t * a.cs_st * ES : nullptr,
                                a.cos ? a.sin + t * a.cs_st * ES : nullptr, a.inv_freq, pos,
                                lane);
            __syncwarp();
            staged = t;
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            process_step<T, D>(a, t, r[u], gl, wsm, csm[wib], slot_ok, cache_off);
    }
}

template <typename T, int D, typename IT>
int launch_qk_wide_it(const QkDev& a, int64_t steps, int64_t upt, int64_t units,
                      cudaStream_t stream) {
    constexpr auto kernel = qk_norm_rope_wide_kernel<T, D, IT>;
    const int threads = 256;
    const int64_t need = ceil_div(units, threads / 32);
    const int64_t fill = (int64_t)sm_count() * resident_ctas<kernel>(threads);
    return launch_pdl(kernel, (unsigned)std::min<int64_t>(need, fill), threads, 0, stream, a,
                      (IT)steps, (IT)upt, (IT)units);
}

template <typename T, int D>
int launch_qk_wide(const QkDev& a, cudaStream_t stream) {
    const int64_t steps = ceil_div(a.tasks_per_token, (int64_t)Wide<T, D>::HPW);
    const int64_t upt = ceil_div(steps, (int64_t)QF_QK_STEPS);  // units per token
    const int64_t units = a.T * upt;
    if (units < (int64_t(1) << 31))
        return launch_qk_wide_it<T, D, uint32_t>(a, steps, upt, units, stream);
    return launch_qk_wide_it<T, D, uint64_t>(a, steps, upt, units, stream);
}

template <typename T, int D>
int launch_qk(const QkDev& a, cudaStream_t stream) {
    constexpr int G = D / 8, HPW = 32 / G, U = 2;
    const int threads = 256;
    const int64_t total = a.T * a.tasks_per_token;
    const int64_t warps = ceil_div(total, (int64_t)HPW * U);
    const int64_t blocks = std::min<int64_t>(ceil_div(warps, threads / 32), (int64_t)sm_count() * 8);
    if (total < (int64_t(1) << 31))
        qk_norm_rope_kernel<T, D, uint32_t><<<(unsigned)blocks, threads, 0, stream>>>(a);
    else
        qk_norm_rope_kernel<T, D, uint64_t><<<(unsigned)blocks, threads, 0, stream>>>(a);
    return check_launch();
}

template <typename T, int D>
int launch_qk_best(const QkDev& a, bool vec, cudaStream_t stream) {
    return vec ? launch_qk_wide<T, D>(a, stream) : launch_qk<T, D>(a, stream);
}

template <typename T>
int dispatch_qk(const QkDev& a, int64_t D, bool vec, cudaStream_t stream) {
    switch (D) {
    case 64: return launch_qk_best<T, 64>(a, vec, stream);
    case 128: return launch_qk_best<T, 128>(a, vec, stream);
    case 256: return launch_qk_best<T, 256>(a, vec, stream);
    default: return QF_ERR_UNSUPPORTED;
    }
}

// ---------------------------------------------------------------------------
// RoPE tables (Qwen3RotaryEmbedding.forward, modeling_qwen3.py:137-148): one
// thread per (token, frequency) computes sincos once and writes both halves.
template <typename T>
__global__ void __launch_bounds__(256) rope_cos_sin_kernel(const void* pos, int pos_type,
                                                           const float* inv_freq, int64_t T_,
                                                           int64_t half, float scaling, T* cos,
                                                           T* sin) {
    const int64_t total = T_ * half;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / half, j = i - t * half;
        const float p = (float)load_index(pos, t, pos_type);
        float sv, cv;
        sincosf(__fmul_rn(__ldg(inv_freq + j), p), &sv, &cv);
        const T c = Dt<T>::from_f(__fmul_rn(cv, scaling));
        const T s = Dt<T>::from_f(__fmul_rn(sv, scaling));
        const int64_t r = t * 2 * half;
        cos[r + j] = c;
        cos[r + j + half] = c;
        sin[r + j] = s;
        sin[r + j + half] = s;
    }
}

inline bool al(const void* p, int64_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)bytes) == 0;
}

}  // namespace
}  // namespace qf

extern "C" int qf_qk_norm_rope_store(const qf_qk_norm_rope_args* p, cudaStream_t stream) {
    if (!p) return QF_ERR_INVALID;
    const qf_qk_norm_rope_args& g = *p;
    if (g.num_tokens < 0 || g.num_q_heads < 0 || g.num_kv_heads < 0) return QF_ERR_INVALID;
    if (g.dtype != QF_F32 && g.dtype != QF_F16 && g.dtype != QF_BF16) return QF_ERR_INVALID;
    const int64_t D = g.head_dim;
    if (D != 64 && D != 128 && D != 256) return QF_ERR_UNSUPPORTED;
    const bool store = g.k_cache != nullptr;
    if (g.num_tokens == 0 || (g.num_q_heads == 0 && g.num_kv_heads == 0)) return QF_OK;
    if (!g.q_out && g.num_q_heads > 0) return QF_ERR_INVALID;
    if ((g.num_q_heads > 0 && !g.q) || (g.num_kv_heads > 0 && !g.k)) return QF_ERR_INVALID;
    if (!g.cos && (!g.positions || !g.inv_freq)) return QF_ERR_INVALID;
    if (g.cos && !g.sin) return QF_ERR_INVALID;
    if (g.positions && g.positions_type != QF_I32 && g.positions_type != QF_I64)
        return QF_ERR_INVALID;
    if (store) {
        if (!g.v_cache || !g.v || !g.block_mapping || !g.slot_mapping) return QF_ERR_INVALID;
        if (g.index_type != QF_I32 && g.index_type != QF_I64) return QF_ERR_INVALID;
        if (g.num_blocks < 0 || g.block_size <= 0) return QF_ERR_INVALID;
        if (g.cache_strides[3] != 1) return QF_ERR_UNSUPPORTED;
    }
    // every 4-element quad a lane touches must be one aligned load/store
    const int64_t es = g.dtype == QF_F32 ? 4 : 2;
    const int64_t qa = 4 * es;
    const int64_t strides[] = {g.q_stride_token,     g.q_stride_head,     g.k_stride_token,
                               g.k_stride_head,      g.q_out_stride_token, g.q_out_stride_head,
                               g.cos ? g.cos_sin_token_stride : 0,
                               g.k_out ? g.k_out_stride_token : 0,
                               g.k_out ? g.k_out_stride_head : 0,
                               store ? g.v_stride_token : 0, store ? g.v_stride_head : 0,
                               store ? g.cache_strides[0] : 0, store ? g.cache_strides[1] : 0,
                               store ? g.cache_strides[2] : 0};
    for (int64_t s : strides)
        if (s % 4) return QF_ERR_UNSUPPORTED;
    const void* ptrs[] = {g.q, g.k, g.q_out, g.q_weight, g.k_weight, g.cos, g.sin, g.k_out,
                          store ? g.v : nullptr, g.k_cache, g.v_cache};
    for (const void* ptr : ptrs)
        if (ptr && !qf::al(ptr, qa)) return QF_ERR_UNSUPPORTED;
    // the 16-byte path when every row start is 16-byte aligned (the serving
    // layout); otherwise the 4-element path above
    bool vec = true;
    for (int64_t s : strides)
        if ((s * es) % 16) vec = false;
    for (const void* ptr : ptrs)
        if (ptr && !qf::al(ptr, 16)) vec = false;

    qf::QkDev a{};
    a.q = static_cast<const char*>(g.q);
    a.q_st = g.q_stride_token;
    a.q_sh = g.q_stride_head;
    a.k = static_cast<const char*>(g.k);
    a.k_st = g.k_stride_token;
    a.k_sh = g.k_stride_head;
    a.v = static_cast<const char*>(g.v);
    a.v_st = g.v_stride_token;
    a.v_sh = g.v_stride_head;
    a.qw = static_cast<const char*>(g.q_weight);
    a.kw = static_cast<const char*>(g.k_weight);
    a.eps = g.eps;
    a.cos = static_cast<const char*>(g.cos);
    a.sin = static_cast<const char*>(g.sin);
    a.cs_st = g.cos_sin_token_stride;
    a.pos = g.positions;
    a.pos_type = g.positions_type;
    a.inv_freq = g.inv_freq;
    a.q_out = static_cast<char*>(g.q_out);
    a.qo_st = g.q_out_stride_token;
    a.qo_sh = g.q_out_stride_head;
    a.k_out = static_cast<char*>(g.k_out);
    a.ko_st = g.k_out_stride_token;
    a.ko_sh = g.k_out_stride_head;
    a.k_cache = static_cast<char*>(g.k_cache);
    a.v_cache = static_cast<char*>(g.v_cache);
    a.c0 = g.cache_strides[0];
    a.c1 = g.cache_strides[1];
    a.c2 = g.cache_strides[2];
    a.N = g.num_blocks;
    a.B = g.block_size;
    a.bm = g.block_mapping;
    a.sm = g.slot_mapping;
    a.idx_type = g.index_type;
    a.T = g.num_tokens;
    a.Hq = g.num_q_heads;
    a.Hkv = g.num_kv_heads;
    a.store = store ? 1 : 0;
    a.tasks_per_token = g.num_q_heads + g.num_kv_heads + (store ? g.num_kv_heads : 0);
    a.status = g.status;
    switch (g.dtype) {
    case QF_F32: return qf::dispatch_qk<float>(a, D, vec, stream);
    case QF_F16: return qf::dispatch_qk<__half>(a, D, vec, stream);
    default: return qf::dispatch_qk<__nv_bfloat16>(a, D, vec, stream);
    }
}

extern "C" int qf_rope_cos_sin(const void* positions, int index_type, const float* inv_freq,
                               int64_t num_tokens, int64_t head_dim, float scaling, int dtype,
                               void* cos, void* sin, cudaStream_t stream) {
    if (num_tokens < 0 || head_dim <= 0 || (head_dim & 1)) return QF_ERR_INVALID;
    if (index_type != QF_I32 && index_type != QF_I64) return QF_ERR_INVALID;
    if (num_tokens == 0) return QF_OK;
    if (!positions || !inv_freq || !cos || !sin) return QF_ERR_INVALID;
    const int64_t half = head_dim / 2;
    const int64_t blocks =
        std::min<int64_t>(qf::ceil_div(num_tokens * half, 256), (int64_t)qf::sm_count() * 16);
    switch (dtype) {
    case QF_F32:
        qf::rope_cos_sin_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(
            positions, index_type, inv_freq, num_tokens, half, scaling,
            static_cast<float*>(cos), static_cast<float*>(sin));
        break;
    case QF_F16:
        qf::rope_cos_sin_kernel<__half><<<(unsigned)blocks, 256, 0, stream>>>(
            positions, index_type, inv_freq, num_tokens, half, scaling,
            static_cast<__half*>(cos), static_cast<__half*>(sin));
        break;
    case QF_BF16:
        qf::rope_cos_sin_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
            positions, index_type, inv_freq, num_tokens, half, scaling,
            static_cast<__nv_bfloat16*>(cos), static_cast<__nv_bfloat16*>(sin));
        break;
    default: return QF_ERR_INVALID;
    }
    return qf::check_launch();
}
