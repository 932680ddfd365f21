// Batched token sampling as grid-wide passes over every row at once.
//
// Same contract and the same integers as the per-row cluster kernel in
// sampler.cu (sample_tokens, server/model/sampling.py:118-194): s = logit /
// max(temperature, 1e-5), ranks by (s desc, index asc), top-k by count, top-p
// and the inverse-CDF pick by exact fixed-point mass (exp(s - max) x 2^40).
// The cluster kernel keeps one row's slice in each CTA's shared memory and
// walks the row through ~10 cluster-wide steps, so only ~37 rows are in flight
// at a time; here each step is one launch over all rows:
//
//   P1 max        every (row, chunk) CTA: the row's maximum and its lowest
//                 index (one 64-bit atomicMax per CTA); zeroes its share of
//                 the row's histograms
//   P2 histogram  every (row, chunk) CTA: a shared-memory histogram of its
//                 elements, added into the row's global one -- counts for
//                 top-k rows, masses and the total mass for the others
//   P3 bounds     one CTA per row: which bins the row's decisions can land
//                 in.  A top-k row takes its whole head down to the top-k
//                 cut.  A row without top-k takes the bin of its top-p cut
//                 (or of its pick) and, with top-p, the bins the pick can
//                 land in: the kept mass lies inside the cut bin's bounds,
//                 so u times it does too.  Greedy rows take the argmax here.
//   P4 compact    every (row, chunk) CTA: the elements of those bins, as
//                 (order desc, index asc) keys, into the row's candidates
//   P5 select     one CTA per row: candidates grouped by bin (a counting
//                 sort); the cumulative mass before each bin comes from the
//                 head itself (top-k rows) or from the histogram; each
//                 decision (the top-k mass, the top-p cut, the pick) finds
//                 its bin from the bin totals and sorts only that bin
//
// A row whose candidates overflow the buffer, or whose logits make ties the
// passes cannot see (below), is listed for the cluster kernel, which the
// entry point launches last.
//
// Bins.  Depth bins: d = max - s, bins of 1/64 for d < 16, of 1/8 for
// 16 <= d < 144, the rest in the last bin.  The bin is non-decreasing in d,
// so the elements at or above a bin are a head of the rank order, and equal s
// share a bin.  For 16-bit logits the max, the top-k counts and the
// compaction work on the logits themselves, two per 32-bit word (packed
// bf16x2 / f16x2 maxima and compares, 16-bit order keys), without the
// division: for distinct 16-bit values x < x', x / t and x' / t differ by at
// least 2^-11 relative, far above float32 rounding, so the order of s is the
// order of x wherever s is a finite normal number.  P3 checks that at the
// maximum and at every key threshold it sets (the values on either side must
// give different s) and sends the row to the cluster kernel otherwise.  Top-k
// rows of 16-bit logits count by the top 13 bits of the 16-bit key, in the 24
// such bins below the maximum's.  fp32 logits divide in every pass.
#include <cfloat>

#include "qf_sample.cuh"

namespace qf {
namespace {

#ifndef QF_WIDE_CTAS_PER_SM
#define QF_WIDE_CTAS_PER_SM 7  // row-pass CTAs per SM over the batch
#endif
#ifndef QF_WIDE_LOADS
#define QF_WIDE_LOADS 4  // 8-element groups in flight per thread
#endif
#ifndef QF_WIDE_CAND
#define QF_WIDE_CAND 2048  // candidates a row may have on this path
#endif
#ifndef QF_WIDE_SEL_THREADS
#define QF_WIDE_SEL_THREADS 256  // threads of a P5 CTA (one row)
#endif

constexpr int kWThreads = 512;
constexpr int kWWarps = kWThreads / 32;
constexpr int kDepthBins = 2048;
constexpr int kRawBins = 8192;  // 16-bit keys >> 3
constexpr uint32_t kRawWindow = 24;  // raw bins a top-k row counts below its maximum's
constexpr int kCandCap = QF_WIDE_CAND;
constexpr int kLoads = QF_WIDE_LOADS;
constexpr uint32_t kNone = 0xffffffffu;
static_assert((kCandCap & (kCandCap - 1)) == 0, "the candidate sort pads to a power of two");
static_assert(kLoads >= 1 && kLoads <= 8, "a compaction step marks its elements in 64 bits");

enum : uint32_t { kFast = 1, kDone = 2, kSlow = 3 };
enum : uint32_t { kUseK = 1, kUseP = 2 };

struct RowHdr {         // 128 bytes per row, zeroed before P1
    u64 maxkey;         // P1: (key << 32) | ~index of the best element (key of x
                        // for 16-bit logits, of s for fp32)
    u64 z_all;          // P2: total mass (rows without top-k)
    u64 k_eff;          // P3
    u64 base_mas;       // P3: mass ranked above bin d_lo (rows without top-k)
    float u, top_p, m;  // P3 (m: the row's maximum s)
    uint32_t ncand;     // P4: candidates found (more than kCandCap: the row is slow)
    uint32_t state;     // P3
    uint32_t flags;     // P3
    uint32_t d_lo, d_hi;                  // P3: the span of the candidates' depth bins
    uint32_t r1_lo, r1_hi, r2_lo, r2_hi;  // P3: the two depth-bin ranges taken
    uint32_t k1_lo, k1_hi, k2_lo, k2_hi;  // P3, 16-bit logits: the same as key ranges
    uint32_t pad[8];
};
static_assert(sizeof(RowHdr) == 128, "row header layout");

struct WideDev {
    const char* logits;
    int64_t row_stride;
    int64_t vocab;
    int chunk;  // elements per (row, chunk) CTA, a multiple of 8
    int vec;
    const float* temperature;
    const void* top_k;
    int top_k_i64;
    const float* top_p;
    const float* uniforms;
    const int64_t* seeds;
    const int64_t* steps;
    int64_t* out;
    uint32_t* slow_n;
    RowHdr* hdr;
    uint32_t* slow_rows;
    uint32_t* cnt;  // [batch][kRawBins] (fp32 logits: the first kDepthBins)
    u64* mas;       // [batch][kDepthBins]
    u64* cand;      // [batch][kCandCap]
};

// Workspace layout: slow count | row headers | slow list | counts | masses |
// candidates, each region 256-byte aligned.
struct Layout {
    int64_t hdr, rows, cnt, mas, cand, total;
};
inline int64_t up256(int64_t x) { return (x + 255) & ~int64_t(255); }
inline Layout layout(int64_t B) {
    Layout l;
    l.hdr = 256;
    l.rows = l.hdr + up256(B * (int64_t)sizeof(RowHdr));
    l.cnt = l.rows + up256(B * 4);
    l.mas = l.cnt + up256(B * kRawBins * 4);
    l.cand = l.mas + up256(B * kDepthBins * 8);
    l.total = l.cand + up256(B * (int64_t)kCandCap * 8);
    return l;
}

__device__ __forceinline__ int depth_bin(float s, float m) {
    const float d = __fsub_rn(m, s);
    const bool near = d < 16.0f;  // false for NaN: the last bin
    // d <= 0 -> 0; d >= 144, inf and NaN -> 1024 + 1023 (fminf drops the NaN)
    const float y = near ? fmaxf(d * 64.0f, 0.0f) : fminf(__fsub_rn(d, 16.0f) * 8.0f, 1023.0f);
    return (int)y + (near ? 0 : 1024);
}

__device__ __forceinline__ int64_t row_top_k(const WideDev& a, int64_t row) {
    return a.top_k_i64 ? reinterpret_cast<const int64_t*>(a.top_k)[row]
                       : (int64_t)reinterpret_cast<const int32_t*>(a.top_k)[row];
}

__device__ __forceinline__ bool row_use_k(const WideDev& a, int64_t row) {
    const int64_t k = row_top_k(a, row);
    return k > 0 && k < a.vocab;
}

// ---- 16-bit values and their 16-bit order keys ------------------------------
template <typename T>
__device__ __forceinline__ float f_of_bits16(uint32_t b) {
    if constexpr (std::is_same<T, __half>::value)
        return __half2float(__ushort_as_half((unsigned short)b));
    else
        return __bfloat162float(__ushort_as_bfloat16((unsigned short)b));
}
__device__ __forceinline__ uint32_t key16_of_bits(uint32_t b) {
    return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}
__device__ __forceinline__ uint32_t bits_of_key16(uint32_t k) {
    return (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu);
}
// both halves of a word of two 16-bit values to their keys
__device__ __forceinline__ uint32_t keys2(uint32_t w) {
    const uint32_t neg = ((w >> 15) & 0x00010001u) * 0xffffu;  // 0xffff per negative half
    return w ^ (neg | 0x80008000u);
}
template <typename T>
__device__ __forceinline__ float x_of_key16(uint32_t k) {
    return f_of_bits16<T>(bits_of_key16(k));
}
template <typename T>
__device__ __forceinline__ uint32_t key16_of_float(float v) {  // v representable in T
    const T t = Dt<T>::from_f(v);
    return key16_of_bits(*reinterpret_cast<const unsigned short*>(&t));
}

// ---- loads: a thread's 8-element groups, all issued before any is used -----
template <typename T>
struct Raw8 {
    uint4 v[sizeof(T) == 4 ? 2 : 1];
    int cnt;
};

template <typename T>
__device__ __forceinline__ void fetch8(const T* p, int n, int g, bool vec, Raw8<T>& r) {
    const int e0 = 8 * g;
    r.cnt = max(0, min(8, n - e0));
    if (r.cnt == 8 && vec) {
        r.v[0] = ld_stream16(p + e0);
        if constexpr (sizeof(T) == 4) r.v[1] = ld_stream16(p + e0 + 4);
    } else {
        if constexpr (sizeof(T) == 4) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) w[j] = j < r.cnt ? __float_as_uint(p[e0 + j]) : 0u;
            r.v[0] = make_uint4(w[0], w[1], w[2], w[3]);
            r.v[1] = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
            const unsigned short* q = reinterpret_cast<const unsigned short*>(p + e0);
            uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < r.cnt) w[j >> 1] |= (uint32_t)q[j] << (16 * (j & 1));
            r.v[0] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// Whether all of a thread's kLoads groups starting at g0 are whole and can be
// read with vector loads; then fetch them with no per-element checks.
__device__ __forceinline__ bool groups_full(bool vec, int n, int g0) {
    return vec && 8 * (g0 + (kLoads - 1) * kWThreads + (int)threadIdx.x + 1) <= n;
}
template <typename T>
__device__ __forceinline__ void fetch_full(const T* p, int g0, Raw8<T> (&r)[kLoads]) {
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
        const int e0 = 8 * (g0 + u * kWThreads + (int)threadIdx.x);
        r[u].v[0] = ld_stream16(p + e0);
        if constexpr (sizeof(T) == 4) r[u].v[1] = ld_stream16(p + e0 + 4);
        r[u].cnt = 8;
    }
}
template <typename T>
__device__ __forceinline__ void fetch_any(const T* p, int n, int g0, bool vec,
                                          Raw8<T> (&r)[kLoads]) {
#pragma unroll
    for (int u = 0; u < kLoads; ++u) fetch8<T>(p, n, g0 + u * kWThreads + threadIdx.x, vec, r[u]);
}

// Element j of a group: for 16-bit types its bits; as a float (exact).
template <typename T>
__device__ __forceinline__ uint32_t bits16(const Raw8<T>& r, int j) {
    return (word(r.v[0], j >> 1) >> (16 * (j & 1))) & 0xffffu;
}
template <typename T>
__device__ __forceinline__ float x_at(const Raw8<T>& r, int j) {
    if constexpr (sizeof(T) == 4) return __uint_as_float(word(r.v[j >> 2], j & 3));
    else return f_of_bits16<T>(bits16<T>(r, j));
}
// Packed max of two words of two 16-bit values each (a NaN half yields the
// other operand's half), and a type's -inf in both halves.
template <typename T>
__device__ __forceinline__ uint32_t hmax2u(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (std::is_same<T, __half>::value)
        asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    else
        asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// Packed a >= b and a <= b of two 16-bit values: 0xffff per true half
// (false for NaN).
template <typename T>
__device__ __forceinline__ uint32_t ge2(uint32_t a, uint32_t b) {
    if constexpr (std::is_same<T, __half>::value)
        return __hge2_mask(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    else
        return __hge2_mask(*reinterpret_cast<const __nv_bfloat162*>(&a),
                           *reinterpret_cast<const __nv_bfloat162*>(&b));
}
template <typename T>
__device__ __forceinline__ uint32_t le2(uint32_t a, uint32_t b) {
    if constexpr (std::is_same<T, __half>::value)
        return __hle2_mask(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    else
        return __hle2_mask(*reinterpret_cast<const __nv_bfloat162*>(&a),
                           *reinterpret_cast<const __nv_bfloat162*>(&b));
}
template <typename T>
__device__ __forceinline__ uint32_t ninf2() {
    return std::is_same<T, __half>::value ? 0xfc00fc00u : 0xff80ff80u;
}
// The largest value of a thread's groups (invalid elements read as -inf).
template <typename T, int L>
__device__ __forceinline__ float groups_max(const Raw8<T> (&r)[L]);

// The valid halves of word q (elements 2q, 2q+1) of a group: 0xffff each.
__device__ __forceinline__ uint32_t valid2(int cnt, int q) {
    return (2 * q < cnt ? 0x0000ffffu : 0u) | (2 * q + 1 < cnt ? 0xffff0000u : 0u);
}

// One group's elements maximised pairwise: both halves of the result hold
// candidates for the group's largest x (missing elements read as -inf).
template <typename T>
__device__ __forceinline__ uint32_t group_max2(const Raw8<T>& g) {
    uint32_t m = hmax2u<T>(hmax2u<T>(g.v[0].x, g.v[0].y), hmax2u<T>(g.v[0].z, g.v[0].w));
    if (g.cnt < 8) {  // the tail: only the elements that exist
        m = ninf2<T>();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t ok = valid2(g.cnt, q);
            m = hmax2u<T>(m, (word(g.v[0], q) & ok) | (ninf2<T>() & ~ok));
        }
    }
    return m;
}

template <typename T>
__device__ __forceinline__ float max_of2(uint32_t m) {
    return fmaxf(f_of_bits16<T>(m & 0xffffu), f_of_bits16<T>(m >> 16));
}

template <typename T, int L>
__device__ __forceinline__ float groups_max(const Raw8<T> (&r)[L]) {
    uint32_t v = ninf2<T>();
#pragma unroll
    for (int u = 0; u < L; ++u) v = hmax2u<T>(v, group_max2<T>(r[u]));
    return max_of2<T>(v);
}

// The (row, chunk) of this CTA in the row passes: its first element and count.
__device__ __forceinline__ int chunk_elems(const WideDev& a, int64_t& lo) {
    lo = (int64_t)blockIdx.x * a.chunk;
    const int64_t left = a.vocab - lo;
    return left <= 0 ? 0 : (left < a.chunk ? (int)left : a.chunk);
}

// The row's maximum s from P1's key.
template <typename T>
__device__ __forceinline__ float row_max_s(u64 maxkey, float tc) {
    const float v = key_value((uint32_t)(maxkey >> 32));
    if constexpr (sizeof(T) == 2) return scaled<float>(v, tc);  // v is the 16-bit x, exactly
    else return v;
}

// ---- P1 --------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kWThreads) wide_max_kernel(const WideDev a) {
    pdl_wait();  // the previous pass's writes are visible from here
    pdl_trigger();
    const int64_t row = blockIdx.y;
    int64_t lo;
    const int n = chunk_elems(a, lo);
    {  // this CTA's share of the row's histograms, zeroed for P2
        const int cs = (kRawBins + gridDim.x - 1) / gridDim.x;
        const int c1 = min(kRawBins, (int)(blockIdx.x + 1) * cs);
        for (int b = blockIdx.x * cs + threadIdx.x; b < c1; b += kWThreads)
            a.cnt[row * kRawBins + b] = 0;
        const int ms = (kDepthBins + gridDim.x - 1) / gridDim.x;
        const int m1 = min(kDepthBins, (int)(blockIdx.x + 1) * ms);
        for (int b = blockIdx.x * ms + threadIdx.x; b < m1; b += kWThreads)
            a.mas[row * kDepthBins + b] = 0;
    }
    const float tc = fmaxf(a.temperature[row], 1e-5f);
    const T* p = reinterpret_cast<const T*>(a.logits) + row * a.row_stride + lo;
    const int ng = (n + 7) / 8;
    // 16-bit: the largest x and its first index; fp32: the best s as the
    // cluster kernel keeps it (a thread's first element, then strictly
    // larger ones)
    float best = -INFINITY;
    uint32_t best_i = kNone;
    // one pass over a thread's groups (inlined twice: whole groups, where
    // every element check folds away, and the rest)
    auto body = [&](const Raw8<T> (&r)[kLoads], int g0) {
        if constexpr (sizeof(T) == 2) {
            // the groups' largest x by packed maxima; only when it beats the
            // running best, the first element holding it (equal x, +0 and
            // -0 included, give equal s)
            float gmu[kLoads];
            float gm = -INFINITY;
#pragma unroll
            for (int u = 0; u < kLoads; ++u) {
                gmu[u] = max_of2<T>(group_max2<T>(r[u]));
                gm = fmaxf(gm, gmu[u]);
            }
            const bool any = r[0].cnt > 0;  // group 0 holds this thread's first elements
            if (any && (best_i == kNone || gm > best)) {
                // the first group holding gm, then its first element holding it
                // (descending loops: the last match written is the first one)
                int uu = 0;
                uint4 v = r[0].v[0];
#pragma unroll
                for (int u = kLoads - 1; u >= 0; --u)
                    if (gmu[u] == gm) {
                        uu = u;
                        v = r[u].v[0];
                    }
                int jj = -1;  // stays -1 only when no element compares equal (NaN)
#pragma unroll
                for (int j = 7; j >= 0; --j)
                    if (f_of_bits16<T>((word(v, j >> 1) >> (16 * (j & 1))) & 0xffffu) == gm) jj = j;
                if (jj >= 0) {
                    best = gm;
                    best_i = 8u * (uint32_t)(g0 + uu * kWThreads + threadIdx.x) + jj;
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < kLoads; ++u) {
                const uint32_t e0 = 8u * (uint32_t)(g0 + u * kWThreads + threadIdx.x);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float v = scaled<float>(x_at<T>(r[u], j), tc);
                    if (j < r[u].cnt && (v > best || best_i == kNone)) {
                        best = v;
                        best_i = e0 + j;
                    }
                }
            }
        }
    };
    for (int g0 = 0; g0 < ng; g0 += kLoads * kWThreads) {
        Raw8<T> r[kLoads];
        if (groups_full(a.vec, n, g0)) {
            fetch_full<T>(p, g0, r);
            body(r, g0);
        } else {
            fetch_any<T>(p, n, g0, a.vec, r);
            body(r, g0);
        }
    }
    if (best_i != kNone) best_i += (uint32_t)lo;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float s2 = __shfl_down_sync(0xffffffffu, best, o);
        const uint32_t i2 = __shfl_down_sync(0xffffffffu, best_i, o);
        if (i2 != kNone && (best_i == kNone || better(s2, i2, best, best_i))) {
            best = s2;
            best_i = i2;
        }
    }
    __shared__ float ws[kWWarps];
    __shared__ uint32_t wi[kWWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        ws[warp] = best;
        wi[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = -INFINITY;
        uint32_t bi = kNone;
        for (int w = 0; w < kWWarps; ++w)
            if (wi[w] != kNone && (bi == kNone || better(ws[w], wi[w], b, bi))) {
                b = ws[w];
                bi = wi[w];
            }
        if (bi != kNone) atomicMax(&a.hdr[row].maxkey, ((u64)order_key(b) << 32) | (u64)(~bi));
    }
}

// ---- P2 --------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kWThreads) wide_hist_kernel(const WideDev a) {
    pdl_wait();  // the previous pass's writes are visible from here
    pdl_trigger();
    constexpr bool kRaw = sizeof(T) == 2;
    constexpr int kCntBins = kRaw ? kRawBins : kDepthBins;
    const int64_t row = blockIdx.y;
    const float temp = a.temperature[row];
    if (temp <= 0.0f) return;  // greedy: the argmax is all it needs
    const bool use_k = row_use_k(a, row);
    __shared__ uint32_t h[kRawBins];  // counts, or the masses' low | high words
    __shared__ u64 wz[kWWarps];
    uint32_t* h_lo = h;
    uint32_t* h_hi = h + kDepthBins;
    for (int b = threadIdx.x; b < kRawBins; b += kWThreads) h[b] = 0;
    __syncthreads();
    int64_t lo;
    const int n = chunk_elems(a, lo);
    const float tc = fmaxf(temp, 1e-5f);
    const float m = row_max_s<T>(a.hdr[row].maxkey, tc);
    const T* p = reinterpret_cast<const T*>(a.logits) + row * a.row_stride + lo;
    const int ng = (n + 7) / 8;
    u64 z = 0;
    // 16-bit top-k rows count only the kRawWindow raw bins from the maximum's
    // down (a top-k cut below them sends the row to the cluster kernel)
    uint32_t bmin = 0;
    float xmin = -INFINITY;
    if constexpr (kRaw) {
        const uint32_t kmax = key16_of_float<T>(key_value((uint32_t)(a.hdr[row].maxkey >> 32)));
        bmin = (kmax >> 3) > (uint32_t)kRawWindow ? (kmax >> 3) - kRawWindow : 0u;
        xmin = x_of_key16<T>(bmin << 3);
    }
    auto body = [&](const Raw8<T> (&r)[kLoads]) {
        // 16-bit top-k rows: nothing to count when the groups' largest x is
        // below the window
        if constexpr (kRaw)
            if (use_k && groups_max<T, kLoads>(r) < xmin) return;
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            if (use_k) {
                if constexpr (kRaw) {
                    {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint32_t k2 = keys2(word(r[u].v[0], q));
                            const uint32_t b0 = (k2 & 0xffffu) >> 3, b1 = k2 >> 19;
                            if (2 * q < r[u].cnt && b0 >= bmin) atomicAdd(&h[b0], 1u);
                            if (2 * q + 1 < r[u].cnt && b1 >= bmin) atomicAdd(&h[b1], 1u);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < r[u].cnt)
                            atomicAdd(&h[depth_bin(scaled<float>(x_at<T>(r[u], j), tc), m)], 1u);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (j < r[u].cnt) {
                        const float s = scaled<float>(x_at<T>(r[u], j), tc);
                        const int d = depth_bin(s, m);
                        const u64 w = mass_of(s, m);  // < 2^41
                        z += w;
                        const uint32_t wl = (uint32_t)w, wh = (uint32_t)(w >> 32);
                        const uint32_t old = atomicAdd(&h_lo[d], wl);
                        if (old + wl < old || wh) atomicAdd(&h_hi[d], wh + (old + wl < old));
                    }
                }
            }
        }
    };
    for (int g0 = 0; g0 < ng; g0 += kLoads * kWThreads) {
        Raw8<T> r[kLoads];
        if (groups_full(a.vec, n, g0)) {
            fetch_full<T>(p, g0, r);
            body(r);
        } else {
            fetch_any<T>(p, n, g0, a.vec, r);
            body(r);
        }
    }
    __syncthreads();
    if (use_k) {
        for (int b = threadIdx.x; b < kCntBins; b += kWThreads)
            if (h[b]) atomicAdd(&a.cnt[row * kRawBins + b], h[b]);
    } else {
        for (int b = threadIdx.x; b < kDepthBins; b += kWThreads) {
            const u64 w = ((u64)h_hi[b] << 32) | h_lo[b];
            if (w) atomicAdd(&a.mas[row * kDepthBins + b], w);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        if ((threadIdx.x & 31) == 0) wz[threadIdx.x >> 5] = z;
        __syncthreads();
        if (threadIdx.x == 0) {
            u64 t = 0;
            for (int w = 0; w < kWWarps; ++w) t += wz[w];
            atomicAdd(&a.hdr[row].z_all, t);
        }
    }
}

// ---- P3 --------------------------------------------------------------------
constexpr int kSThreads = 256;
constexpr int kSWarps = kSThreads / 32;
constexpr int kDepthPer = kDepthBins / kSThreads;  // depth bins per thread
constexpr int kRawPer = kRawBins / kSThreads;      // raw bins per thread
// The row's histogram is staged in shared memory with one pad word after
// every 32 raw bins (one pad u64 after every 16 depth bins), so that the
// threads' reads of their runs of consecutive bins fall into distinct banks.
__device__ __forceinline__ int raw_slot(int b) { return b + (b >> 5); }
__device__ __forceinline__ int depth_slot(int b) { return b + (b >> 4); }
constexpr int kStageWords = kRawBins + kRawBins / 32;
static_assert(2 * (kDepthBins + kDepthBins / 16) <= kStageWords, "depth staging fits");
constexpr int kCrossSlots = 3;  // crossings one P3 CTA takes

struct Cross {
    uint32_t pos;  // kNone: not reached
    u64 before;    // cumulative weight before it
    u64 through;   // and through it
};

struct CrossShared {
    u64 wsum[kSWarps];
    uint32_t first[kCrossSlots];
    u64 before[kCrossSlots], through[kCrossSlots];
};

// Thread t holds positions [PER t, PER t + PER) in w: the total weight of
// every position before its first.  Whole CTA, once per CTA.
template <int PER>
__device__ u64 block_before(const u64 (&w)[PER], CrossShared& sh) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    u64 sum = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) sum += w[i];
    u64 incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const u64 x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
    }
    if (lane == 31) sh.wsum[warp] = incl;
    __syncthreads();
    u64 before = incl - sum;
#pragma unroll
    for (int q = 0; q < kSWarps; ++q) before += q < warp ? sh.wsum[q] : 0;
    return before;
}

// NC crossings at once, into shared slots [slot, slot + NC) that no earlier
// call used (their `first` set to kNone before the CTA's first barrier): for
// each tau, the first position whose weight is > 0 and whose inclusive
// cumulative weight reaches tau.  `before` from block_before.  Whole CTA.
template <int PER, int NC>
__device__ void block_cross(const u64 (&w)[PER], u64 before, const u64 (&tau)[NC], int slot,
                            CrossShared& sh, Cross (&c)[NC]) {
    uint32_t mine[NC];
    u64 mb[NC], mt[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        mine[k] = kNone;
        mb[k] = mt[k] = 0;
    }
    u64 cum = before;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const u64 prev = cum;
        cum += w[i];
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            if (mine[k] == kNone && w[i] > 0 && cum >= tau[k]) {
                mine[k] = (uint32_t)(PER * threadIdx.x + i);
                mb[k] = prev;
                mt[k] = cum;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const uint32_t wmin = __reduce_min_sync(0xffffffffu, mine[k]);
        if ((threadIdx.x & 31) == 0 && wmin != kNone) atomicMin(&sh.first[slot + k], wmin);
    }
    __syncthreads();
    uint32_t first[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        first[k] = sh.first[slot + k];
        if (mine[k] != kNone && mine[k] == first[k]) {
            sh.before[slot + k] = mb[k];
            sh.through[slot + k] = mt[k];
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        c[k].pos = first[k];
        c[k].before = first[k] == kNone ? 0 : sh.before[slot + k];
        c[k].through = first[k] == kNone ? 0 : sh.through[slot + k];
    }
}

// For each of NS depth bins D: the smallest 16-bit key in [kninf, kpinf]
// whose s lands in a bin <= D (kpinf + 1 when D < 0).  s(+inf) is in bin 0
// and the bin does not increase with the key, so each search is for the
// first true value of a monotone predicate that holds at kpinf.  `clean` is
// cleared when a found key's s equals the s of the key below it.  Whole CTA;
// D uniform; `ks` zeroed (nfalse, bad) before the CTA's first barrier.
//
// A window of kKeyWin keys around the key where s = m - (the lower edge of
// bin D + 1) is tested with one key per thread, and two more threads test
// the key below the window (must be false) and the one above it (must be
// true).  When both hold, the count of false tests is the answer's offset,
// and the s values the threads found answer the `clean` check.  A search
// whose window misses (not met with finite rows) takes the whole key range
// in rounds: each splits the keys below the upper end into kSThreads runs,
// one thread tests the last key of each, and the count of false tests gives
// the run holding the first true key (65,536 keys: two rounds).
constexpr int kKeyWin = kSThreads - 2;
constexpr int kKeySearches = 4;

struct KeyShared {
    float s[kKeySearches][kSThreads];
    uint32_t nfalse[kKeySearches];
    uint32_t bad;
};

template <typename T, int NS>
__device__ void block_key_thresholds(const int (&D)[NS], float tc, float m, uint32_t kninf,
                                     uint32_t kpinf, uint32_t (&t)[NS], bool& clean,
                                     KeyShared& ks) {
    static_assert(NS <= kKeySearches, "key-search slots");
    auto s_of = [&](uint32_t q) { return scaled<float>(x_of_key16<T>(q), tc); };
    const int tid = (int)threadIdx.x, lane = tid & 31;
    uint32_t wlo[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        t[s] = kpinf + 1;
        wlo[s] = kninf;
        if (D[s] < 0) continue;
        const int e = D[s] + 1;
        const float edge = e <= 1024 ? (float)e * (1.0f / 64.0f) : 16.0f + (float)(e - 1024) * 0.125f;
        const uint32_t kc = key16_of_float<T>((m - edge) * tc);
        uint32_t w0 = kc > kninf + kKeyWin / 2 ? kc - kKeyWin / 2 : kninf;
        if (w0 > kpinf - kKeyWin) w0 = kpinf - kKeyWin;
        wlo[s] = w0;
        // thread i < kKeyWin tests w0 + i, thread kKeyWin the key below the
        // window, thread kKeyWin + 1 the window's top w0 + kKeyWin
        const bool none = tid == kKeyWin && w0 == kninf;  // no key below
        const uint32_t q = tid < kKeyWin ? w0 + tid : (tid == kKeyWin ? w0 - 1 : w0 + kKeyWin);
        float sv = 0.0f;
        bool p = false;
        if (!none) {
            sv = s_of(q);
            p = depth_bin(sv, m) <= D[s];
        }
        ks.s[s][tid] = sv;
        const bool f = tid < kKeyWin && !p;
        const bool bad = (tid == kKeyWin && p) || (tid == kKeyWin + 1 && !p);
        const uint32_t nf = (uint32_t)__popc(__ballot_sync(0xffffffffu, f));
        const bool anybad = __any_sync(0xffffffffu, bad);
        if (lane == 0) {
            if (nf) atomicAdd(&ks.nfalse[s], nf);
            if (anybad) atomicOr(&ks.bad, 1u << s);
        }
    }
    __syncthreads();
    const uint32_t bad = ks.bad;
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        if (D[s] < 0 || ((bad >> s) & 1u)) continue;
        const uint32_t nf = ks.nfalse[s];
        t[s] = wlo[s] + nf;
        if (t[s] > kninf) {  // s at the found key and at the key below it
            const float s_at = ks.s[s][nf < (uint32_t)kKeyWin ? (int)nf : kKeyWin + 1];
            const float s_below = ks.s[s][nf > 0 ? (int)nf - 1 : kKeyWin];
            clean = clean && s_below != s_at;
        }
    }
    if (bad == 0) return;
    uint32_t lo[NS], hi[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        lo[s] = kninf;
        hi[s] = D[s] >= 0 && ((bad >> s) & 1u) ? kpinf : kninf;
    }
    for (int round = 0; round < 4; ++round) {  // two rounds for 16-bit keys, a third finds nothing left
        uint32_t step[NS];
        bool f[NS];
        bool any = false;
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            const uint32_t n = hi[s] - lo[s];
            step[s] = (n + kSThreads - 1) / kSThreads;
            const uint32_t q = lo[s] + (threadIdx.x + 1) * step[s] - 1;
            f[s] = n > 0 && q < hi[s] && depth_bin(s_of(q), m) > D[s];
            any = any || n > 0;
        }
        if (!any) break;
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            const uint32_t nf = (uint32_t)__syncthreads_count(f[s]);
            if (hi[s] > lo[s]) {
                lo[s] += nf * step[s];
                hi[s] = min(hi[s], lo[s] + step[s] - 1);
            }
        }
    }
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        if (D[s] < 0 || !((bad >> s) & 1u)) continue;
        t[s] = lo[s];
        clean = clean && (lo[s] <= kninf || s_of(lo[s] - 1) != s_of(lo[s]));
    }
}

// Top-k rows of 16-bit logits: over the row's top PER x kSThreads raw bins
// (position q is bin kRawBins - 1 - q), the first position whose cumulative
// count reaches k_eff.  Whole CTA.
template <int PER>
__device__ Cross raw_crossing(const uint32_t* cnt_row, u64 k_eff, uint32_t* stage, CrossShared& xs) {
    constexpr int kPos = PER * kSThreads;
    constexpr int kVec = kPos / 4 / kSThreads;
    static_assert(kPos % (4 * kSThreads) == 0 && kPos <= kRawBins, "whole 16-byte loads");
    const uint4* src = reinterpret_cast<const uint4*>(cnt_row + (kRawBins - kPos));
    uint4 v[kVec];
#pragma unroll
    for (int i = 0; i < kVec; ++i) v[i] = src[threadIdx.x + i * kSThreads];
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
        const int b = 4 * ((int)threadIdx.x + i * kSThreads);  // from bin kRawBins - kPos
        stage[raw_slot(b)] = v[i].x;
        stage[raw_slot(b + 1)] = v[i].y;
        stage[raw_slot(b + 2)] = v[i].z;
        stage[raw_slot(b + 3)] = v[i].w;
    }
    __syncthreads();
    u64 w[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) w[i] = stage[raw_slot(kPos - 1 - (PER * (int)threadIdx.x + i))];
    const u64 before = block_before<PER>(w, xs);
    const u64 tau[1] = {k_eff};
    Cross c[1];
    block_cross<PER, 1>(w, before, tau, 0, xs, c);
    return c[0];
}
constexpr int kRawTop = 2048;  // the short scan's bins

template <typename T>
__global__ void __launch_bounds__(kSThreads) wide_bounds_kernel(const WideDev a) {
    constexpr bool kRaw = sizeof(T) == 2;
    const int64_t row = blockIdx.x;
    // The row's settings are inputs that no pass writes, and all the work
    // queued before P1 has completed by the time this grid launches (P1 is
    // launched without overlap, and P2's CTAs release this grid only after
    // their own wait on P1), so they load while the wait below runs.
    const float temp = a.temperature[row];
    const int64_t k = row_top_k(a, row);
    const float top_p = a.top_p[row];
    const float u = a.uniforms ? a.uniforms[row]
                               : uniform_from_hash((uint64_t)a.seeds[row], (uint64_t)a.steps[row]);
    pdl_wait();  // the previous pass's writes are visible from here
    pdl_trigger();
    RowHdr& h = a.hdr[row];
    const u64 maxkey = h.maxkey;
    const u64 z_all = h.z_all;
    const uint32_t argmax = ~(uint32_t)maxkey;
    const float tc = fmaxf(temp, 1e-5f);
    const float m = row_max_s<T>(maxkey, tc);
    // 16-bit logits: the order of s must be the order of x at the maximum --
    // a finite normal s, and the next lower 16-bit value giving a lower s
    bool plain = true;
    uint32_t kninf = 0, kpinf = 0, k16 = 0;  // k16: the maximum's 16-bit key
    if constexpr (kRaw) {
        kninf = key16_of_float<T>(-INFINITY);
        kpinf = key16_of_float<T>(INFINITY);
        k16 = key16_of_float<T>(key_value((uint32_t)(maxkey >> 32)));
        plain = isfinite(m) && fabsf(m) >= FLT_MIN && k16 > kninf && k16 <= kpinf &&
                scaled<float>(x_of_key16<T>(k16 - 1), tc) != m;
    }
    if (temp <= 0.0f || !plain) {
        if (threadIdx.x == 0) {
            if (plain) {  // greedy: rank 0 of the stable order
                a.out[row] = argmax;
                h.state = kDone;
            } else {
                h.state = kSlow;
                a.slow_rows[atomicAdd(a.slow_n, 1u)] = (uint32_t)row;
            }
        }
        return;
    }
    const int64_t V = a.vocab;
    const u64 k_eff = (k > 0 && k < V) ? (u64)k : (u64)V;
    const bool use_k = k_eff < (u64)V, use_p = top_p < 1.0f;
    __shared__ __align__(16) uint32_t stage[kStageWords];  // the row's histogram, padded
    __shared__ CrossShared xs;
    __shared__ KeyShared ks;
    if (threadIdx.x < kCrossSlots) xs.first[threadIdx.x] = kNone;
    if (threadIdx.x < kKeySearches) ks.nfalse[threadIdx.x] = 0;
    if (threadIdx.x == 0) ks.bad = 0;
    // depth-bin ranges [r1_lo, r1_hi] and [r2_lo, r2_hi] (empty: lo > hi)
    uint32_t r1_lo = 0, r1_hi = 0, r2_lo = 1, r2_hi = 0;
    u64 base_mas = 0;
    bool ok = true;
    uint32_t k1_lo = 1, k1_hi = 0, k2_lo = 1, k2_hi = 0;  // 16-bit key ranges (inclusive)
    if (use_k) {
        if constexpr (kRaw) {
            // P2 counted only the bins from kRawWindow below the maximum's up;
            // when those are all among the top kRawTop, only those are read
            const uint32_t bmin = (k16 >> 3) > kRawWindow ? (k16 >> 3) - kRawWindow : 0u;
            const uint32_t* cnt_row = a.cnt + row * kRawBins;
            Cross c[1];
            if (bmin >= (uint32_t)(kRawBins - kRawTop))
                c[0] = raw_crossing<kRawTop / kSThreads>(cnt_row, k_eff, stage, xs);
            else
                c[0] = raw_crossing<kRawPer>(cnt_row, k_eff, stage, xs);
            const uint32_t t16 = c[0].pos == kNone ? 0 : (uint32_t)(kRawBins - 1 - c[0].pos) << 3;
            ok = c[0].pos != kNone && c[0].through <= (u64)kCandCap && t16 > kninf && t16 <= kpinf &&
                 scaled<float>(x_of_key16<T>(t16 - 1), tc) != scaled<float>(x_of_key16<T>(t16), tc);
            if (ok) {
                k1_lo = t16;
                k1_hi = 0xffffu;
                r1_hi = (uint32_t)depth_bin(scaled<float>(x_of_key16<T>(t16), tc), m);
            }
        } else {
            u64 w[kDepthPer];
#pragma unroll
            for (int i = 0; i < kDepthPer; ++i)
                w[i] = a.cnt[row * kRawBins + kDepthPer * threadIdx.x + i];
            const u64 before = block_before<kDepthPer>(w, xs);
            const u64 tau[1] = {k_eff};
            Cross c[1];
            block_cross<kDepthPer, 1>(w, before, tau, 0, xs, c);
            ok = c[0].pos != kNone && c[0].through <= (u64)kCandCap;
            r1_hi = c[0].pos;
        }
    } else {
        u64* stage64 = reinterpret_cast<u64*>(stage);
        const uint4* src = reinterpret_cast<const uint4*>(a.mas + row * kDepthBins);
        constexpr int kVec = kDepthBins / 2 / kSThreads;
        uint4 v[kVec];
#pragma unroll
        for (int i = 0; i < kVec; ++i) v[i] = src[threadIdx.x + i * kSThreads];
#pragma unroll
        for (int i = 0; i < kVec; ++i) {
            const int b = 2 * ((int)threadIdx.x + i * kSThreads);
            stage64[depth_slot(b)] = ((u64)v[i].y << 32) | v[i].x;
            stage64[depth_slot(b + 1)] = ((u64)v[i].w << 32) | v[i].z;
        }
        __syncthreads();
        u64 w[kDepthPer];
#pragma unroll
        for (int i = 0; i < kDepthPer; ++i) w[i] = stage64[depth_slot(kDepthPer * (int)threadIdx.x + i)];
        const u64 before = block_before<kDepthPer>(w, xs);
        u64 tau[1];
        if (use_p) {
            const double theta = (double)top_p * (double)z_all;
            tau[0] = theta < 0.0 ? 0 : (u64)floor(theta) + 1;
        } else {
            tau[0] = (u64)ceil((double)u * (double)z_all);
            if (tau[0] > z_all) tau[0] = z_all;
        }
        Cross c[1];
        block_cross<kDepthPer, 1>(w, before, tau, 0, xs, c);
        ok = c[0].pos != kNone;
        r1_lo = r1_hi = c[0].pos;
        base_mas = c[0].before;
        if (ok && use_p) {
            // the kept mass lies within the cut bin's cumulative bounds, so
            // the pick's threshold u * (kept mass) lies within u times them
            u64 t2[2];
            t2[0] = (u64)ceil((double)u * (double)c[0].before);
            if (t2[0] > c[0].before) t2[0] = c[0].before;
            t2[1] = (u64)ceil((double)u * (double)c[0].through);
            if (t2[1] > c[0].through) t2[1] = c[0].through;
            Cross cl[2];
            block_cross<kDepthPer, 2>(w, before, t2, 1, xs, cl);
            ok = cl[0].pos != kNone && cl[1].pos != kNone && cl[0].pos <= cl[1].pos &&
                 cl[1].pos <= c[0].pos;
            if (ok) {
                if (cl[1].pos + 1 >= c[0].pos) {
                    r1_lo = cl[0].pos;
                } else {
                    r2_lo = r2_hi = c[0].pos;
                    r1_lo = cl[0].pos;
                    r1_hi = cl[1].pos;
                }
                base_mas = cl[0].before;
            }
        }
        if constexpr (kRaw) {
            if (ok) {
                // the smallest key whose bin is <= each range's ends
                const bool two = r2_lo <= r2_hi;
                const int D[4] = {(int)r1_hi, (int)r1_lo - 1, two ? (int)r2_hi : -1,
                                  two ? (int)r2_lo - 1 : -1};
                uint32_t t[4];
                block_key_thresholds<T, 4>(D, tc, m, kninf, kpinf, t, ok, ks);
                k1_lo = t[0];
                k1_hi = t[1] - 1;
                if (two) {
                    k2_lo = t[2];
                    k2_hi = t[3] - 1;
                }
            }
        }
    }
    if (threadIdx.x == 0) {
        h.k_eff = k_eff;
        h.base_mas = base_mas;
        h.u = u;
        h.top_p = top_p;
        h.m = m;
        h.flags = (use_k ? kUseK : 0u) | (use_p ? kUseP : 0u);
        h.r1_lo = r1_lo;
        h.r1_hi = r1_hi;
        h.r2_lo = r2_lo;
        h.r2_hi = r2_hi;
        h.d_lo = r1_lo;
        h.d_hi = r2_lo <= r2_hi ? r2_hi : r1_hi;
        h.k1_lo = k1_lo;
        h.k1_hi = k1_hi;
        h.k2_lo = k2_lo;
        h.k2_hi = k2_hi;
        h.state = ok ? kFast : kSlow;
        if (!ok) a.slow_rows[atomicAdd(a.slow_n, 1u)] = (uint32_t)row;
    }
}

// ---- P4 --------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kWThreads) wide_compact_kernel(const WideDev a) {
    pdl_wait();  // the previous pass's writes are visible from here
    pdl_trigger();
    constexpr bool kRaw = sizeof(T) == 2;
    const int64_t row = blockIdx.y;
    RowHdr& h = a.hdr[row];
    if (h.state != kFast) return;
    int64_t lo;
    const int n = chunk_elems(a, lo);
    const float tc = fmaxf(a.temperature[row], 1e-5f);
    const float m = h.m;
    const int r1_lo = (int)h.r1_lo, r1_hi = (int)h.r1_hi, r2_lo = (int)h.r2_lo,
              r2_hi = (int)h.r2_hi;
    const uint32_t k1lo = h.k1_lo, k1hi = h.k1_hi, k2lo = h.k2_lo, k2hi = h.k2_hi;
    // the key ranges as value bounds, both halves (an empty range's bounds are
    // NaN, which no value compares to); every candidate's x is at least that
    // of the lowest taken key
    float xlow = 0.0f;
    uint32_t lo1 = 0, hi1 = 0, lo2 = 0, hi2 = 0;
    if constexpr (kRaw) {
        const uint32_t kp = key16_of_float<T>(INFINITY);
        lo1 = bits_of_key16(k1lo) * 0x00010001u;
        hi1 = bits_of_key16(min(k1hi, kp)) * 0x00010001u;
        lo2 = k2lo <= k2hi ? bits_of_key16(k2lo) * 0x00010001u : ninf2<T>() | 0x00400040u;
        hi2 = k2lo <= k2hi ? bits_of_key16(min(k2hi, kp)) * 0x00010001u : lo2;
        xlow = x_of_key16<T>(k2lo <= k2hi ? min(k1lo, k2lo) : k1lo);
    }
    const T* p = reinterpret_cast<const T*>(a.logits) + row * a.row_stride + lo;
    u64* cand = a.cand + row * kCandCap;
    const int ng = (n + 7) / 8;
    const int lane = threadIdx.x & 31;
    // the loop bound is the same for every thread, so the warp-wide
    // reservations below always run with the whole warp
    // bit 8u + j of the result: element j of group u is a candidate
    auto body = [&](const Raw8<T> (&r)[kLoads]) -> u64 {
        u64 take = 0;
        bool look = true;
        if constexpr (kRaw) look = groups_max<T, kLoads>(r) >= xlow;
#pragma unroll
        for (int u = 0; u < kLoads; ++u) {
            if constexpr (kRaw) {
                if (look) {  // packed value compares against the ranges' bounds
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t w = word(r[u].v[0], q);
                        const uint32_t t = ((ge2<T>(w, lo1) & le2<T>(w, hi1)) |
                                            (ge2<T>(w, lo2) & le2<T>(w, hi2))) &
                                           valid2(r[u].cnt, q);
                        take |= (u64)((t & 1u) | ((t >> 15) & 2u)) << (8 * u + 2 * q);
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int d = depth_bin(scaled<float>(x_at<T>(r[u], j), tc), m);
                    if (j < r[u].cnt && ((d >= r1_lo && d <= r1_hi) || (d >= r2_lo && d <= r2_hi)))
                        take |= 1ull << (8 * u + j);
                }
            }
        }
        return take;
    };
    for (int g0 = 0; g0 < ng; g0 += kLoads * kWThreads) {
        Raw8<T> r[kLoads];
        u64 take;
        if (groups_full(a.vec, n, g0)) {
            fetch_full<T>(p, g0, r);
            take = body(r);
        } else {
            fetch_any<T>(p, n, g0, a.vec, r);
            take = body(r);
        }
        if (!__any_sync(0xffffffffu, take != 0)) continue;  // the usual case: nothing here
        const uint32_t mine = __popcll(take);
        uint32_t incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += x;
        }
        const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
        if (total == 0) continue;
        uint32_t base = 0;
        if (lane == 0) {
            base = atomicAdd(&h.ncand, total);
            if (base <= (uint32_t)kCandCap && base + total > (uint32_t)kCandCap)
                a.slow_rows[atomicAdd(a.slow_n, 1u)] = (uint32_t)row;  // the one overflow
        }
        base = __shfl_sync(0xffffffffu, base, 0);
        uint32_t slot = base + incl - mine;
        if (take) {
#pragma unroll
            for (int u = 0; u < kLoads; ++u)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if ((take >> (8 * u + j)) & 1ull) {
                        if (slot < (uint32_t)kCandCap) {
                            const float s = scaled<float>(x_at<T>(r[u], j), tc);
                            const uint32_t idx =
                                (uint32_t)(lo + 8 * (g0 + u * kWThreads + threadIdx.x) + j);
                            cand[slot] = ((u64)(~order_key(s)) << 32) | idx;
                        }
                        ++slot;
                    }
        }
    }
}

// ---- P5 --------------------------------------------------------------------
constexpr int kPThreads = QF_WIDE_SEL_THREADS;
constexpr int kPWarps = kPThreads / 32;
static_assert(kPWarps <= 32 && kCandCap % kPThreads == 0 && kDepthBins % kPThreads == 0,
              "select: one scan warp, whole per-thread shares");

struct SelShared {
    uint32_t cnt[kDepthBins + 1];  // candidates per bin (relative to d_lo)
    uint32_t off[kDepthBins + 1];  // their first position in the grouped order
    u64 red[kPWarps];
    uint32_t first;
};

// Inclusive prefix sums of v[0, n) in place, plus `base`.  Whole CTA.
__device__ void block_scan_u64(u64* v, int n, u64 base, SelShared& sh) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (n + kPThreads - 1) / kPThreads;
    const int i0 = min(n, (int)threadIdx.x * per), i1 = min(n, i0 + per);
    u64 run = 0;
    for (int i = i0; i < i1; ++i) {
        run += v[i];
        v[i] = run;
    }
    u64 x = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const u64 y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    __syncthreads();  // earlier readers of sh.red are done
    if (lane == 31) sh.red[warp] = x;
    __syncthreads();
    if (warp == 0) {
        u64 y = lane < kPWarps ? sh.red[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const u64 z = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += z;
        }
        if (lane < kPWarps) sh.red[lane] = y;
    }
    __syncthreads();
    const u64 off = base + (warp ? sh.red[warp - 1] : 0) + (x - run);
    for (int i = i0; i < i1; ++i) v[i] += off;
    __syncthreads();
}

__device__ __forceinline__ float s_of_cand(u64 key) { return key_value(~(uint32_t)(key >> 32)); }

// grouped keys | inclusive masses | a bin being sorted | the bins' bases
constexpr size_t kSelSmem = 3 * (size_t)kCandCap * sizeof(u64) + kDepthBins * sizeof(u64);

__global__ void __launch_bounds__(kPThreads) wide_select_kernel(const WideDev a) {
    pdl_wait();  // the previous pass's writes are visible from here
    pdl_trigger();
    extern __shared__ __align__(16) u64 wsm[];
    u64* grouped = wsm;                 // candidate keys grouped by bin
    u64* w = wsm + kCandCap;            // inclusive masses in the grouped order
    u64* scratch = wsm + 2 * kCandCap;  // a bin being sorted
    u64* bbase = wsm + 3 * kCandCap;    // the mass ranked above each bin
    __shared__ SelShared sh;
    const int64_t row = blockIdx.x;
    const RowHdr& h = a.hdr[row];
    if (h.state != kFast || h.ncand > (uint32_t)kCandCap) return;
    const int n = (int)h.ncand;
    const float m = h.m;
    const int d_lo = (int)h.d_lo;
    const int nb = max(1, min(kDepthBins, (int)h.d_hi - d_lo + 1));
    const bool use_k = h.flags & kUseK, use_p = h.flags & kUseP;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const u64* cand = a.cand + row * kCandCap;
    if (n == 0) {  // not reached: every decision's bin holds an element
        if (threadIdx.x == 0) a.slow_rows[atomicAdd(a.slow_n, 1u)] = (uint32_t)row;
        return;
    }
    auto bin_of = [&](u64 key) {
        return min(nb - 1, max(0, depth_bin(s_of_cand(key), m) - d_lo));
    };
    // a row without top-k: its histogram's masses of bins d_lo on, loaded now
    // and used once the candidates are grouped
    constexpr int kBinPer = kDepthBins / kPThreads;
    u64 hm[kBinPer];
#pragma unroll
    for (int q = 0; q < kBinPer; ++q) {
        const int b = (int)threadIdx.x + q * kPThreads;
        hm[q] = !use_k && b < nb ? a.mas[row * kDepthBins + d_lo + b] : 0;
    }
    // ---- counting sort by bin ----------------------------------------------
    // a thread's candidates, all loaded at once and kept for the scatter
    constexpr int kPer = kCandCap / kPThreads;
    u64 ck[kPer];
    int cb[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        const int i = (int)threadIdx.x + q * kPThreads;
        ck[q] = i < n ? cand[i] : 0;
    }
    for (int b = threadIdx.x; b <= nb; b += kPThreads) sh.cnt[b] = 0;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
        cb[q] = bin_of(ck[q]);
        if ((int)threadIdx.x + q * kPThreads < n) atomicAdd(&sh.cnt[cb[q]], 1u);
    }
    __syncthreads();
    for (int b = threadIdx.x; b < nb; b += kPThreads) bbase[b] = sh.cnt[b];
    __syncthreads();
    block_scan_u64(bbase, nb, 0, sh);  // bbase as scratch for the offsets
    for (int b = threadIdx.x; b < nb; b += kPThreads) {
        sh.off[b] = (uint32_t)(bbase[b] - sh.cnt[b]);
        sh.cnt[b] = 0;  // from here: the fill count
    }
    if (threadIdx.x == 0) sh.off[nb] = (uint32_t)n;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q)
        if ((int)threadIdx.x + q * kPThreads < n)
            grouped[sh.off[cb[q]] + atomicAdd(&sh.cnt[cb[q]], 1u)] = ck[q];
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kPThreads) w[i] = mass_of(s_of_cand(grouped[i]), m);
    __syncthreads();
    block_scan_u64(w, n, 0, sh);
    // the mass ranked above each bin: a top-k row holds its whole head, so
    // the sums before the bin; otherwise the row's histogram
    if (use_k) {
        for (int b = threadIdx.x; b < nb; b += kPThreads)
            bbase[b] = sh.off[b] ? w[sh.off[b] - 1] : 0;
        __syncthreads();
    } else {
        // the histogram's bin masses from d_lo on, summed onto the mass
        // ranked above d_lo: scratch[b] is the mass through bin b
#pragma unroll
        for (int q = 0; q < kBinPer; ++q) {
            const int b = (int)threadIdx.x + q * kPThreads;
            if (b < nb) scratch[b] = hm[q];
        }
        __syncthreads();
        block_scan_u64(scratch, nb, h.base_mas, sh);
#pragma unroll
        for (int q = 0; q < kBinPer; ++q) {
            const int b = (int)threadIdx.x + q * kPThreads;
            if (b < nb) bbase[b] = scratch[b] - hm[q];
        }
        __syncthreads();
        // rebase w: the grouped prefix at each bin's start, replaced by bbase
        for (int b = threadIdx.x; b < nb; b += kPThreads)
            scratch[b] = sh.off[b] ? w[sh.off[b] - 1] : 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += kPThreads) {
            const int b = bin_of(grouped[i]);
            w[i] = w[i] - scratch[b] + bbase[b];
        }
        __syncthreads();
    }
    // ---- decisions: each sorts the one bin it lands in ---------------------
    int sorted[3] = {-1, -1, -1};
    int nsorted = 0;
    auto sort_bin = [&](int b) {
        for (int q = 0; q < nsorted; ++q)
            if (sorted[q] == b) return;
        if (nsorted < 3) sorted[nsorted++] = b;
        const int o = (int)sh.off[b], c = (int)sh.off[b + 1] - o;
        if (c <= 1) return;
        const u64 before = bbase[b];
        if (c <= 32) {  // one warp: rank by counting, then a warp scan of the masses
            if (warp == 0) {
                const u64 key = lane < c ? grouped[o + lane] : ~0ull;
                int rank = 0;
                for (int j = 0; j < c; ++j) rank += __shfl_sync(0xffffffffu, key, j) < key;
                if (lane < c) scratch[rank] = key;
                __syncwarp();
                u64 x = 0;
                if (lane < c) {
                    grouped[o + lane] = scratch[lane];
                    x = mass_of(s_of_cand(scratch[lane]), m);
                }
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const u64 y = __shfl_up_sync(0xffffffffu, x, d);
                    if (lane >= d) x += y;
                }
                if (lane < c) w[o + lane] = before + x;
            }
            __syncthreads();
            return;
        }
        int P = 1;
        while (P < c) P <<= 1;
        for (int i = threadIdx.x; i < P; i += kPThreads) scratch[i] = i < c ? grouped[o + i] : ~0ull;
        __syncthreads();
        for (int kk = 2; kk <= P; kk <<= 1) {  // bitonic, ascending key = rank order
            for (int j = kk >> 1; j > 0; j >>= 1) {
                for (int i = threadIdx.x; i < P; i += kPThreads) {
                    const int l = i ^ j;
                    if (l > i) {
                        const u64 x = scratch[i], y = scratch[l];
                        if ((x > y) == ((i & kk) == 0)) {
                            scratch[i] = y;
                            scratch[l] = x;
                        }
                    }
                }
                __syncthreads();
            }
        }
        for (int i = threadIdx.x; i < c; i += kPThreads) {
            grouped[o + i] = scratch[i];
            scratch[i] = mass_of(s_of_cand(scratch[i]), m);
        }
        __syncthreads();
        block_scan_u64(scratch, c, before, sh);
        for (int i = threadIdx.x; i < c; i += kPThreads) w[o + i] = scratch[i];
        __syncthreads();
    };
    // the first position, in rank order, whose inclusive mass reaches tau
    auto first_reaching = [&](u64 tau) -> int {
        if (threadIdx.x == 0) sh.first = kNone;
        __syncthreads();
        for (int b = threadIdx.x; b < nb; b += kPThreads)
            if (sh.off[b + 1] > sh.off[b] && w[sh.off[b + 1] - 1] >= tau)
                atomicMin(&sh.first, (uint32_t)b);
        __syncthreads();
        const uint32_t b = sh.first;
        __syncthreads();
        if (b == kNone) return -1;
        sort_bin((int)b);
        const int o = (int)sh.off[b], c = (int)sh.off[b + 1] - o;
        if (threadIdx.x == 0) sh.first = kNone;
        __syncthreads();
        for (int i = threadIdx.x; i < c; i += kPThreads)
            if (w[o + i] >= tau) atomicMin(&sh.first, (uint32_t)(o + i));
        __syncthreads();
        const uint32_t r = sh.first;
        __syncthreads();
        return r == kNone ? -1 : (int)r;
    };
    const u64 k_eff = h.k_eff;
    bool ok = true;
    u64 z_k = h.z_all;
    if (use_k) {  // the whole head is here, so a position is a rank
        if (k_eff > (u64)n) {
            ok = false;
        } else {
            const int pos = (int)k_eff - 1;
            int lo_b = 0, hi_b = nb - 1;  // the last bin whose offset is <= pos
            while (lo_b < hi_b) {
                const int mid = (lo_b + hi_b + 1) >> 1;
                if ((int)sh.off[mid] <= pos) lo_b = mid;
                else hi_b = mid - 1;
            }
            sort_bin(lo_b);
            z_k = w[pos];
        }
    }
    u64 z_r = z_k;
    if (ok && use_p) {
        const double theta = (double)h.top_p * (double)z_k;
        const u64 tau = theta < 0.0 ? 0 : (u64)floor(theta) + 1;
        const int r = first_reaching(tau);
        ok = r >= 0;
        // with top-k, positions are ranks; without it the cut never reaches k
        if (ok && (!use_k || (u64)r + 1 < k_eff)) z_r = w[r];
    }
    int r = -1;
    if (ok) {
        u64 tau = (u64)ceil((double)h.u * (double)z_r);
        if (tau > z_r) tau = z_r;
        r = first_reaching(tau);
        ok = r >= 0;
    }
    if (threadIdx.x == 0) {
        if (ok) a.out[row] = (int64_t)(uint32_t)grouped[r];
        else a.slow_rows[atomicAdd(a.slow_n, 1u)] = (uint32_t)row;  // not reached
    }
}

template <typename T>
int launch_wide(const WideDev& d, int64_t B, int nchunk, cudaStream_t stream) {
    static std::atomic<uint64_t> sized{0};  // devices whose attribute is set
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = dev < 64 ? 1ull << dev : 0;
    if (!(sized.load(std::memory_order_relaxed) & bit)) {
        const cudaError_t e = cudaFuncSetAttribute(
            wide_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSelSmem);
        if (e != cudaSuccess) return launch_failed(e);
        sized.fetch_or(bit, std::memory_order_relaxed);
    }
    // the passes after the first start with programmatic dependent launch:
    // each one's launch and prologue overlap the previous pass's tail, and it
    // waits for that pass (pdl_wait) before its first global access
    const dim3 rows_grid((unsigned)nchunk, (unsigned)B);
    wide_max_kernel<T><<<rows_grid, kWThreads, 0, stream>>>(d);
    int rc = check_launch();
    if (rc == QF_OK) rc = launch_pdl(wide_hist_kernel<T>, rows_grid, kWThreads, 0, stream, d);
    if (rc == QF_OK) rc = launch_pdl(wide_bounds_kernel<T>, dim3((unsigned)B), kSThreads, 0, stream, d);
    if (rc == QF_OK) rc = launch_pdl(wide_compact_kernel<T>, rows_grid, kWThreads, 0, stream, d);
    if (rc == QF_OK)
        rc = launch_pdl(wide_select_kernel, dim3((unsigned)B), kPThreads, kSelSmem, stream, d);
    return rc;
}

}  // namespace

int64_t sample_wide_workspace_bytes(int64_t batch) { return layout(batch).total; }

int sample_wide_passes(const WideArgs& a, cudaStream_t stream, const uint32_t** slow_rows,
                       const uint32_t** slow_n) {
    const int64_t B = a.batch;
    const Layout l = layout(B);
    char* ws = static_cast<char*>(a.workspace);
    WideDev d{};
    d.logits = static_cast<const char*>(a.logits);
    d.row_stride = a.row_stride;
    d.vocab = a.vocab;
    // CTAs per row in the row passes: about QF_WIDE_CTAS_PER_SM per SM over
    // the batch (each thread keeps only a few loads in flight, so the passes
    // need many CTAs to cover the memory latency)
    const int64_t want = std::max<int64_t>(
        1, std::min<int64_t>(16, (QF_WIDE_CTAS_PER_SM * sm_count() + B / 2) / B));
    d.chunk = (int)std::max<int64_t>(8, ceil_div(ceil_div(a.vocab, want), 8) * 8);
    d.vec = a.vec;
    d.temperature = a.temperature;
    d.top_k = a.top_k;
    d.top_k_i64 = a.top_k_i64;
    d.top_p = a.top_p;
    d.uniforms = a.uniforms;
    d.seeds = a.seeds;
    d.steps = a.steps;
    d.out = a.out;
    d.slow_n = reinterpret_cast<uint32_t*>(ws);
    d.hdr = reinterpret_cast<RowHdr*>(ws + l.hdr);
    d.slow_rows = reinterpret_cast<uint32_t*>(ws + l.rows);
    d.cnt = reinterpret_cast<uint32_t*>(ws + l.cnt);
    d.mas = reinterpret_cast<u64*>(ws + l.mas);
    d.cand = reinterpret_cast<u64*>(ws + l.cand);
    *slow_rows = d.slow_rows;
    *slow_n = d.slow_n;
    const int nchunk = (int)ceil_div(a.vocab, (int64_t)d.chunk);
    // the slow count and every row header start at zero
    const cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)l.rows, stream);
    if (e != cudaSuccess) return launch_failed(e);
    switch (a.dtype) {
    case QF_F32: return launch_wide<float>(d, B, nchunk, stream);
    case QF_F16: return launch_wide<__half>(d, B, nchunk, stream);
    default: return launch_wide<__nv_bfloat16>(d, B, nchunk, stream);
    }
}

}  // namespace qf
