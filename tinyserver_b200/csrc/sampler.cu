// Batched token sampling without a sort.
//
// Replaces sample_tokens (server/model/sampling.py:118-194).  For row b:
//   s_i = float(logits[b, i]) / max(temperature[b], 1e-5)          (:166-168)
//   ranks: s descending, equal s by ascending index (stable sort, :172-174)
//   top-k keeps ranks < k (k <= 0 or >= V keeps all, :178-180)
//   p = softmax over the kept ranks (:182)
//   top-p keeps rank r when the mass of ranks < r is <= top_p (:186-189)
//   token = the first rank whose cumulative mass is >= u * (kept mass)
//           (inverse-CDF pick, :193-198); temperature <= 0: the argmax (:203-205).
//
// Every step above is "the first rank, in (s desc, index asc) order, whose
// cumulative weight reaches a threshold": top-k by count, top-p and the pick
// by mass.  This kernel finds each such rank with a radix select instead of a
// sort.  The order key of s is its float bits with the sign folded so that
// unsigned comparison follows s; its top 11, middle 11 and low 10 bits are
// three digit levels.  Per level, every CTA histograms its elements (count
// and mass) by digit, the cluster adds the histograms over distributed shared
// memory, and a descending scan finds the digit where the cumulative weight
// crosses the threshold; the next level only counts elements under that
// prefix.  After three levels the key is exact; elements with equal keys have
// equal s, equal mass and consecutive ranks in index order, so the rank inside
// that group is arithmetic, and for the pick one CTA walks its slice in index
// order to name the token.
//
// Masses are exp(s - max) as fixed-point integers (x 2^40, u64): integer sums
// do not depend on the order of addition, so the per-CTA histograms, their
// cluster sum and every deeper level agree exactly, and the result does not
// depend on how the vocabulary is split.  Thresholds: top-p keeps ranks up to
// and including the first whose inclusive mass exceeds top_p * (kept mass);
// the pick is the first rank whose inclusive mass is >= ceil(u * kept mass).
//
// One cluster of kClusterCtas CTAs per row; each CTA keeps its slice of the
// row in shared memory as fp32 s, so the row is read from HBM once.
#include <cooperative_groups.h>

#include "qf_sample.cuh"

namespace cg = cooperative_groups;

namespace qf {
namespace {

#ifndef QF_SAMPLE_CLUSTER
#define QF_SAMPLE_CLUSTER 8
#endif
#ifndef QF_SAMPLE_LOADS
#define QF_SAMPLE_LOADS 5  // 16-byte loads in flight per thread: a whole slice in one batch
#endif
#ifndef QF_SAMPLE_WIDE_MIN_ROWS
#define QF_SAMPLE_WIDE_MIN_ROWS 128  // auto: the batch-wide path from this many rows on
#endif
#ifndef QF_SAMPLE_PREFETCH
#define QF_SAMPLE_PREFETCH 1  // prefetch into L2 the slice the next wave of clusters reads
#endif

constexpr int kClusterCtas = QF_SAMPLE_CLUSTER;
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 2048;                     // digits per level (level 3 uses 1024)
constexpr int kOwn = kBins / kClusterCtas;      // combined bins each CTA holds
constexpr int kGroup = 32;                      // bins per group (one warp's scan)
constexpr int kGroups = kBins / kGroup;         // 64: two per lane of the scanning warp
constexpr int kOwnGroups = kOwn / kGroup;
static_assert(kOwn <= kThreads && kOwn % kGroup == 0 && kGroups == 64, "cluster size 4..64");

struct SampleDev {
    const char* logits;
    int64_t row_stride;  // elements
    int64_t vocab;
    int slice;           // elements per CTA, a multiple of 8
    int vec;             // 16-byte loads (aligned rows)
    int ahead;           // rows between a cluster and the one a wave later (0: no prefetch)
    const float* temperature;
    const void* top_k;
    int top_k_i64;
    const float* top_p;
    const float* uniforms;
    const int64_t* seeds;
    const int64_t* steps;
    int64_t* out;
    // optional: the rows to sample, rows[0 .. *nrows) (device), one cluster
    // each; clusters past *nrows exit at once.  NULL: cluster c samples row c.
    const uint32_t* rows;
    const uint32_t* nrows;
};

// The crossing found by a descending scan: its digit, the cumulative weight
// of everything ranked above it, and its own weight.
struct Crossing {
    int found;
    int digit;
    u64 above_cnt, above_mas, cnt, mas;
};

// Candidates of one select: the elements under a digit prefix, at most
// kCand of them across the cluster.
constexpr int kCand = 512;
// Candidates of the one-pass path: every element whose level-1 digit is at or
// above the boundary digit, at most kUni of them across the cluster.  Rank 0
// sorts them as (u64 key, u64 mass) pairs in its own slice's shared memory,
// which the launcher sizes to at least kUni * 16 bytes.  The path is taken up
// to kUniTake candidates: a larger sort by one CTA costs more than the
// cluster-wide selects (on Qwen3's vocabulary, 2048 candidates took ~8%
// longer per row than top-k and a pick by selects).
constexpr int kUni = 2048;
#ifndef QF_SAMPLE_UNI_TAKE
#define QF_SAMPLE_UNI_TAKE 512
#endif
constexpr int kUniTake = QF_SAMPLE_UNI_TAKE;
static_assert(kUniTake <= kUni, "one-pass candidates fit the buffers");

struct SampleShared {
    union {
        struct {  // this CTA's histogram at the current level; the mass is a
                  // u64 kept as two u32 words (shared-memory u32 atomics are
                  // native, u64 ones are not), the carry added explicitly
            uint32_t cnt[kBins];
            uint32_t mas_lo[kBins];
            uint32_t mas_hi[kBins];
        } h;
        struct {  // candidate selects, two buffers used in turn
            float s[2][kCand];      // this CTA's matching elements
            uint32_t idx[2][kCand]; // and their vocabulary indices
            u64 key[kCand];         // all of the cluster's: (order desc, index asc) as a u64
            u64 w[kCand];           // and masses
        } c;
        struct {  // the one-pass path: this CTA's elements at or above the boundary digit
            float s[kUni];
            uint32_t idx[kUni];
        } x;
    } u;
    // A level's histogram summed over the cluster: this CTA's range of bins,
    // and every 32-bin group's totals (pushed here by the group's owner).
    // lv[0]: level 1 (kept for every select of the row); lv[1]: levels 2, 3.
    struct Level {
        u64 own_mas[kOwn];
        uint32_t own_cnt[kOwn];
        u64 grp_mas[kGroups];
        uint32_t grp_cnt[kGroups];
    } lv[2];
    float max_s;  // this CTA's maximum and its lowest global index
    uint32_t max_idx;
    u64 red_mas[kWarps];
    uint32_t red_cnt[kWarps];
    Crossing res;
    float row_max;
    uint32_t row_argmax;
    u64 z_all;
    int owner;
    uint32_t owner_j;
    uint32_t cand_n[2];                     // this CTA's candidates, per buffer
    uint32_t cand_pre[kClusterCtas + 1];    // the cluster's, prefix by rank
    struct {
        int found;
        uint32_t idx;
        u64 incl_cnt, incl_mas;
    } cres;
};

template <typename F>
__device__ __forceinline__ void for_each_s(const float* sv, int n, F&& f) {
    const int n4 = n >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(sv);
    for (int q = threadIdx.x; q < n4; q += kThreads) {
        const float4 v = s4[q];
        f(v.x);
        f(v.y);
        f(v.z);
        f(v.w);
    }
    for (int i = (n4 << 2) + (int)threadIdx.x; i < n; i += kThreads) f(sv[i]);
}

// Load this CTA's slice, write s to shared memory, return the thread's best
// (s, local index).
template <typename T>
__device__ __forceinline__ void load_slice(const SampleDev& a, const T* row, int n, float tc,
                                           float* sv, float& best, uint32_t& best_i) {
    if (a.vec) {
        constexpr int PV = Dt<T>::kPerVec;
        constexpr int U = QF_SAMPLE_LOADS;
        const int nv = n / PV;
        for (int c0 = threadIdx.x; c0 < nv; c0 += U * kThreads) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + u * kThreads;
                if (c < nv) raw[u] = ld_stream16(row + (int64_t)c * PV);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + u * kThreads;
                if (c >= nv) break;
                const T* x = reinterpret_cast<const T*>(&raw[u]);
                float v[PV];
#pragma unroll
                for (int j = 0; j < PV; ++j) {
                    v[j] = scaled<T>(x[j], tc);
                    if (v[j] > best || best_i == 0xffffffffu) {
                        best = v[j];
                        best_i = (uint32_t)(c * PV + j);
                    }
                }
#pragma unroll
                for (int j = 0; j < PV; j += 4)
                    *reinterpret_cast<float4*>(sv + c * PV + j) =
                        make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            }
        }
        for (int i = nv * PV + (int)threadIdx.x; i < n; i += kThreads) {
            const float v = scaled<T>(row[i], tc);
            sv[i] = v;
            if (v > best || best_i == 0xffffffffu) {
                best = v;
                best_i = (uint32_t)i;
            }
        }
    } else {
        for (int i = threadIdx.x; i < n; i += kThreads) {
            const float v = scaled<T>(row[i], tc);
            sv[i] = v;
            if (v > best || best_i == 0xffffffffu) {
                best = v;
                best_i = (uint32_t)i;
            }
        }
    }
}

__device__ __forceinline__ void zero_hist(SampleShared& sm) {
    for (int i = threadIdx.x; i < kBins; i += kThreads) {
        sm.u.h.cnt[i] = 0;
        sm.u.h.mas_lo[i] = 0;
        sm.u.h.mas_hi[i] = 0;
    }
}

// Histogram of this CTA's elements whose key has `prefix` above bit `hi`,
// by the digit (key >> shift) & mask.  hi == 32: no prefix.
__device__ __forceinline__ void build_hist(SampleShared& sm, const float* sv, int n, float m,
                                           int hi, uint32_t prefix, int shift, uint32_t mask) {
    for_each_s(sv, n, [&](float s) {
        const uint32_t k = order_key(s);
        if (hi == 32 || (k >> hi) == prefix) {
            const uint32_t d = (k >> shift) & mask;
            atomicAdd(&sm.u.h.cnt[d], 1u);
            const u64 w = mass_of(s, m);  // < 2^41
            const uint32_t wl = (uint32_t)w, wh = (uint32_t)(w >> 32);
            if (wl) {
                const uint32_t old = atomicAdd(&sm.u.h.mas_lo[d], wl);
                if (old + wl < old) atomicAdd(&sm.u.h.mas_hi[d], 1u);  // carry
            }
            if (wh) atomicAdd(&sm.u.h.mas_hi[d], wh);
        }
    });
}

// Sum the cluster's histograms over this CTA's bin range into lv[level], and
// push each 32-bin group's totals into every CTA's lv[level].  Call between
// two cluster barriers.
__device__ void combine(const cg::cluster_group& cl, SampleShared& sm, int level) {
    const int rank = (int)cl.block_rank();
    if (threadIdx.x < kOwn) {
        const int b = rank * kOwn + threadIdx.x;
        u64 m = 0;
        uint32_t c = 0;
#pragma unroll
        for (int q = 0; q < kClusterCtas; ++q) {
            const SampleShared* r = cl.map_shared_rank(&sm, q);
            m += ((u64)r->u.h.mas_hi[b] << 32) | r->u.h.mas_lo[b];
            c += r->u.h.cnt[b];
        }
        sm.lv[level].own_mas[threadIdx.x] = m;
        sm.lv[level].own_cnt[threadIdx.x] = c;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            m += __shfl_xor_sync(0xffffffffu, m, o);
            c += __shfl_xor_sync(0xffffffffu, c, o);
        }
        const int lane = threadIdx.x & 31;
        const int g = rank * kOwnGroups + (threadIdx.x >> 5);
        if (lane < kClusterCtas) {
            SampleShared* r = cl.map_shared_rank(&sm, lane);
            r->lv[level].grp_mas[g] = m;
            r->lv[level].grp_cnt[g] = c;
        }
    }
}

__device__ __forceinline__ void scan_up(uint32_t& c, u64& m, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t xc = __shfl_up_sync(0xffffffffu, c, o);
        const u64 xm = __shfl_up_sync(0xffffffffu, m, o);
        if (lane >= o) {
            c += xc;
            m += xm;
        }
    }
}

// Warp 0: the first combined bin, in descending digit order, that is not empty
// and whose inclusive cumulative weight (count or mass, starting from
// above_*) reaches tau.  The group totals are local; the 32 bins of the
// chosen group are read from the CTA that owns them.  Every lane returns the
// same result.
__device__ Crossing search(const cg::cluster_group& cl, SampleShared& sm, int level,
                           bool by_mass, u64 tau, u64 above_cnt, u64 above_mas) {
    const int lane = threadIdx.x & 31;
    const SampleShared::Level& L = sm.lv[level];
    Crossing f{};
    // groups, highest digits first: lane l takes groups 63 - 2l and 62 - 2l
    const int ga = kGroups - 1 - 2 * lane, gb = ga - 1;
    const uint32_t ca = L.grp_cnt[ga], cb = L.grp_cnt[gb];
    const u64 ma = L.grp_mas[ga], mb = L.grp_mas[gb];
    uint32_t ic = ca + cb;
    u64 im = ma + mb;
    scan_up(ic, im, lane);
    const uint32_t lc = ca + cb;
    bool cond = lc > 0 && (by_mass ? above_mas + im : above_cnt + ic) >= tau;
    unsigned bal = __ballot_sync(0xffffffffu, cond);
    if (!bal) return f;
    int W = __ffs(bal) - 1;
    u64 ec = above_cnt + ic - lc, em = above_mas + im - (ma + mb);
    int g = ga;
    if (!(ca > 0 && (by_mass ? em + ma : ec + ca) >= tau)) {
        g = gb;
        ec += ca;
        em += ma;
    }
    g = __shfl_sync(0xffffffffu, g, W);
    above_cnt = __shfl_sync(0xffffffffu, ec, W);
    above_mas = __shfl_sync(0xffffffffu, em, W);
    // that group's bins, highest first: lane l takes bin 31 - l
    const int rho = g / kOwnGroups;
    const int b = (g % kOwnGroups) * kGroup + kGroup - 1 - lane;
    const SampleShared::Level& R = cl.map_shared_rank(&sm, rho)->lv[level];
    const uint32_t bc = R.own_cnt[b];
    const u64 bm = R.own_mas[b];
    ic = bc;
    im = bm;
    scan_up(ic, im, lane);
    cond = bc > 0 && (by_mass ? above_mas + im : above_cnt + ic) >= tau;
    bal = __ballot_sync(0xffffffffu, cond);
    if (!bal) return f;  // unreachable: the group total crossed
    W = __ffs(bal) - 1;
    f.found = 1;
    f.digit = rho * kOwn + __shfl_sync(0xffffffffu, b, W);
    f.above_cnt = above_cnt + __shfl_sync(0xffffffffu, ic - bc, W);
    f.above_mas = above_mas + __shfl_sync(0xffffffffu, im - bm, W);
    f.cnt = __shfl_sync(0xffffffffu, bc, W);
    f.mas = __shfl_sync(0xffffffffu, bm, W);
    return f;
}

// Run `search` on warp 0 and hand the result to the whole CTA.
__device__ __forceinline__ Crossing search_all(const cg::cluster_group& cl, SampleShared& sm,
                                               int level, bool by_mass, u64 tau, u64 above_cnt,
                                               u64 above_mas) {
    __syncthreads();  // everyone has read the previous result
    if (threadIdx.x < 32) {
        const Crossing f = search(cl, sm, level, by_mass, tau, above_cnt, above_mas);
        if (threadIdx.x == 0) sm.res = f;
    }
    __syncthreads();
    return sm.res;
}

// One deeper level: histogram under `prefix`, cluster sum, scan.
__device__ __forceinline__ Crossing deeper(const cg::cluster_group& cl, SampleShared& sm,
                                           const float* sv, int n, float m, int hi,
                                           uint32_t prefix, int shift, uint32_t mask, bool by_mass,
                                           u64 tau, const Crossing& parent) {
    cl.sync();  // no CTA still reads another's candidate buffers (they share the histogram)
    zero_hist(sm);
    __syncthreads();
    build_hist(sm, sv, n, m, hi, prefix, shift, mask);
    cl.sync();  // every CTA's histogram is complete
    combine(cl, sm, 1);
    cl.sync();  // every CTA's combined range and group totals are complete
    return search_all(cl, sm, 1, by_mass, tau, parent.above_cnt, parent.above_mas);
}

// The rank where the cumulative weight first reaches tau.
struct Selected {
    int found;
    int has_idx;        // idx is the rank's vocabulary index
    uint32_t idx;
    uint32_t key;       // otherwise: the order key of the rank's s,
    uint32_t low_digit; // its level-3 digit (this CTA's cnt[] holds its local count)
    u64 j;              // and its position inside the group of equal keys (index order)
    u64 incl_cnt;       // ranks up to and including it
    u64 incl_mas;       // their mass
};

// Select among the elements whose key has `prefix` above bit `hi` -- at most
// kCand of them in the cluster -- the first (key desc, index asc) whose
// cumulative weight, starting from above_*, reaches tau.  Every CTA gathers
// all candidates over distributed shared memory and ranks each against the
// others.  One cluster barrier; the candidate buffers alternate between
// selects, so a CTA may fill the next buffer while others still read this one
// (the buffer after that is only refilled once every CTA passed the next
// select's barrier, i.e. finished reading).
__device__ Selected select_candidates(const cg::cluster_group& cl, SampleShared& sm,
                                      const float* sv, int n, int64_t base, float m, int hi,
                                      uint32_t prefix, bool by_mass, u64 tau, u64 above_cnt,
                                      u64 above_mas, int buf) {
    if (threadIdx.x == 0) {
        sm.cand_n[buf] = 0;
        sm.cres.found = 0;
    }
    __syncthreads();
    auto take = [&](float s, int i) {
        if ((order_key(s) >> hi) == prefix) {
            const uint32_t slot = atomicAdd(&sm.cand_n[buf], 1u);
            if (slot < kCand) {
                sm.u.c.s[buf][slot] = s;
                sm.u.c.idx[buf][slot] = (uint32_t)(base + i);
            }
        }
    };
    const int n4 = n >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(sv);
    for (int q = threadIdx.x; q < n4; q += kThreads) {
        const float4 v = s4[q];
        take(v.x, 4 * q);
        take(v.y, 4 * q + 1);
        take(v.z, 4 * q + 2);
        take(v.w, 4 * q + 3);
    }
    for (int i = (n4 << 2) + (int)threadIdx.x; i < n; i += kThreads) take(sv[i], i);
    cl.sync();  // every CTA's candidates are in place
    const int lane = threadIdx.x & 31;
    if (threadIdx.x < 32) {
        uint32_t c = 0;
        if (lane < kClusterCtas)
            c = min(cl.map_shared_rank(&sm, lane)->cand_n[buf], (uint32_t)kCand);
        uint32_t incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += x;
        }
        if (lane < kClusterCtas) sm.cand_pre[lane + 1] = incl;
        if (lane == 0) sm.cand_pre[0] = 0;
    }
    __syncthreads();
    const int total = (int)min(sm.cand_pre[kClusterCtas], (uint32_t)kCand);
    const int t = threadIdx.x;
    u64 key = 0, w = 0;
    uint32_t idx = 0;
    if (t < total) {
        int q = 0;
        while (q + 1 < kClusterCtas && (int)sm.cand_pre[q + 1] <= t) ++q;
        const SampleShared* r = cl.map_shared_rank(&sm, q);
        const float s = r->u.c.s[buf][t - sm.cand_pre[q]];
        idx = r->u.c.idx[buf][t - sm.cand_pre[q]];
        key = ((u64)(~order_key(s)) << 32) | idx;
        w = mass_of(s, m);
        sm.u.c.key[t] = key;
        sm.u.c.w[t] = w;
    }
    __syncthreads();
    if (t < total) {
        uint32_t bc = 0;
        u64 bm = 0;
        int v = 0;
        for (; v + 4 <= total; v += 4) {
            u64 kv[4], wv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                kv[j] = sm.u.c.key[v + j];
                wv[j] = sm.u.c.w[v + j];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (kv[j] < key) {
                    ++bc;
                    bm += wv[j];
                }
        }
        for (; v < total; ++v) {
            if (sm.u.c.key[v] < key) {
                ++bc;
                bm += sm.u.c.w[v];
            }
        }
        const u64 ec = above_cnt + bc, em = above_mas + bm;
        const bool hit = by_mass ? (em + w >= tau && (em < tau || (tau == 0 && bc == 0)))
                                 : ec + 1 == tau;
        if (hit) {
            sm.cres.found = 1;
            sm.cres.idx = idx;
            sm.cres.incl_cnt = ec + 1;
            sm.cres.incl_mas = em + w;
        }
    }
    __syncthreads();
    Selected out{};
    out.found = sm.cres.found;
    out.has_idx = 1;
    out.idx = sm.cres.idx;
    out.incl_cnt = sm.cres.incl_cnt;
    out.incl_mas = sm.cres.incl_mas;
    return out;
}

// `known`: the level-1 crossing of this same threshold, when the caller has it.
__device__ Selected select_rank(const cg::cluster_group& cl, SampleShared& sm, const float* sv,
                                int n, int64_t base, float m, bool by_mass, u64 tau, int& nsel,
                                const Crossing* known = nullptr) {
    Selected out{};
    const Crossing f1 = known ? *known : search_all(cl, sm, 0, by_mass, tau, 0, 0);
    if (!f1.found) return out;
    const uint32_t p1 = (uint32_t)f1.digit;
    if (f1.cnt <= (u64)kCand)
        return select_candidates(cl, sm, sv, n, base, m, 21, p1, by_mass, tau, f1.above_cnt,
                                 f1.above_mas, nsel++ & 1);
    const Crossing f2 = deeper(cl, sm, sv, n, m, 21, p1, 10, 2047u, by_mass, tau, f1);
    if (!f2.found) return out;
    const uint32_t p2 = (p1 << 11) | (uint32_t)f2.digit;
    if (f2.cnt <= (u64)kCand)
        return select_candidates(cl, sm, sv, n, base, m, 10, p2, by_mass, tau, f2.above_cnt,
                                 f2.above_mas, nsel++ & 1);
    const Crossing f3 = deeper(cl, sm, sv, n, m, 10, p2, 0, 1023u, by_mass, tau, f2);
    if (!f3.found) return out;
    out.found = 1;
    out.key = (p2 << 10) | (uint32_t)f3.digit;
    out.low_digit = (uint32_t)f3.digit;
    const u64 w = f3.mas / f3.cnt;  // equal keys, equal masses
    if (by_mass)
        out.j = (w == 0 || tau <= f3.above_mas) ? 0 : (tau - f3.above_mas + w - 1) / w - 1;
    else
        out.j = tau - f3.above_cnt - 1;
    out.incl_cnt = f3.above_cnt + out.j + 1;
    out.incl_mas = f3.above_mas + (out.j + 1) * w;
    return out;
}

// The j-th element (in index order) of this CTA's slice whose key is `key`;
// the caller knows it exists.  Returns the local index (all threads).
__device__ int nth_with_key(SampleShared& sm, const float* sv, int n, uint32_t key, uint32_t j) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int span = ((n + kWarps - 1) / kWarps + 31) & ~31;
    const int lo = warp * span, hi = min(n, lo + span);
    uint32_t c = 0;
    for (int b = lo; b < hi; b += 32) {
        const int i = b + lane;
        c += __popc(__ballot_sync(0xffffffffu, i < hi && order_key(sv[i]) == key));
    }
    if (lane == 0) sm.red_cnt[warp] = c;
    sm.owner = -1;
    __syncthreads();
    uint32_t before = 0;
    for (int w = 0; w < warp; ++w) before += sm.red_cnt[w];
    if (j >= before && j < before + c) {
        uint32_t jj = j - before;
        for (int b = lo; b < hi; b += 32) {
            const int i = b + lane;
            const unsigned bal = __ballot_sync(0xffffffffu, i < hi && order_key(sv[i]) == key);
            const uint32_t pc = __popc(bal);
            if (jj < pc) {
                if (((bal >> lane) & 1u) && __popc(bal & ((1u << lane) - 1u)) == (int)jj)
                    sm.owner = i;
                break;
            }
            jj -= pc;
        }
    }
    __syncthreads();
    return sm.owner;
}

// First position r of the nondecreasing incl[0, n) with incl[r] >= tau, or -1.
// Whole CTA.
__device__ int first_reaching(SampleShared& sm, const u64* incl, int n, u64 tau) {
    if (threadIdx.x == 0) sm.owner = -1;
    __syncthreads();
    for (int r = threadIdx.x; r < n; r += kThreads)
        if (incl[r] >= tau && (r == 0 || incl[r - 1] < tau)) sm.owner = r;  // one such r
    __syncthreads();
    const int r = sm.owner;
    __syncthreads();
    return r;
}

// The one-pass path.  Every rank that top-k, top-p and the pick can land on
// has its level-1 digit >= dstar, and ncand <= kUni elements of the row do
// (the caller checked).  Every CTA compacts its own; rank 0 gathers them,
// sorts them by (s desc, index asc) -- the rank order -- sums their masses in
// that order and reads the three thresholds off the sums.  These are the same
// integers the select path computes (the top-k cut's inclusive mass, the first
// rank whose inclusive mass reaches tau), so the token is the same.  Called by
// every CTA of the cluster; returns with all of them past the final barrier.
__device__ void sample_unified(const cg::cluster_group& cl, SampleShared& sm, float* sv, int n,
                               int64_t base, float m, uint32_t dstar, bool use_k, u64 k_eff,
                               bool use_p, float top_p, u64 z_all, float u, int64_t* out) {
    const int rank = (int)cl.block_rank();
    if (threadIdx.x == 0) sm.cand_n[0] = 0;
    __syncthreads();
    auto take = [&](float s, int i) {
        if ((order_key(s) >> 21) >= dstar) {
            const uint32_t slot = atomicAdd(&sm.cand_n[0], 1u);
            if (slot < kUni) {  // always: this CTA's share of at most kUni
                sm.u.x.s[slot] = s;
                sm.u.x.idx[slot] = (uint32_t)(base + i);
            }
        }
    };
    const int n4 = n >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(sv);
    for (int q = threadIdx.x; q < n4; q += kThreads) {
        const float4 v = s4[q];
        take(v.x, 4 * q);
        take(v.y, 4 * q + 1);
        take(v.z, 4 * q + 2);
        take(v.w, 4 * q + 3);
    }
    for (int i = (n4 << 2) + (int)threadIdx.x; i < n; i += kThreads) take(sv[i], i);
    cl.sync();  // every CTA's candidates are in place
    if (rank == 0) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        if (threadIdx.x < 32) {
            uint32_t c = 0;
            if (lane < kClusterCtas)
                c = min(cl.map_shared_rank(&sm, lane)->cand_n[0], (uint32_t)kUni);
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += x;
            }
            if (lane < kClusterCtas) sm.cand_pre[lane + 1] = incl;
            if (lane == 0) sm.cand_pre[0] = 0;
        }
        __syncthreads();
        const int total = (int)min(sm.cand_pre[kClusterCtas], (uint32_t)kUni);
        int P = 1;
        while (P < total) P <<= 1;
        // (key, mass) pairs over this CTA's slice, which it no longer needs
        u64* yk = reinterpret_cast<u64*>(sv);
        u64* yw = yk + kUni;
        for (int t = threadIdx.x; t < P; t += kThreads) {
            u64 key = ~0ull, w = 0;  // padding sorts last
            if (t < total) {
                int q = 0;
                while (q + 1 < kClusterCtas && (int)sm.cand_pre[q + 1] <= t) ++q;
                const SampleShared* r = cl.map_shared_rank(&sm, q);
                const float s = r->u.x.s[t - sm.cand_pre[q]];
                key = ((u64)(~order_key(s)) << 32) | r->u.x.idx[t - sm.cand_pre[q]];
                w = mass_of(s, m);
            }
            yk[t] = key;
            yw[t] = w;
        }
        __syncthreads();
        // bitonic sort, ascending key = rank order
        for (int k = 2; k <= P; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int i = threadIdx.x; i < P; i += kThreads) {
                    const int l = i ^ j;
                    if (l > i) {
                        const u64 x = yk[i], y = yk[l];
                        if ((x > y) == ((i & k) == 0)) {
                            yk[i] = y;
                            yk[l] = x;
                            const u64 t = yw[i];
                            yw[i] = yw[l];
                            yw[l] = t;
                        }
                    }
                }
                __syncthreads();
            }
        }
        // inclusive sums of the masses in rank order: a run of `per` per thread
        const int per = (P + kThreads - 1) / kThreads;
        const int i0 = min(P, (int)threadIdx.x * per), i1 = min(P, i0 + per);
        u64 run = 0;
        for (int i = i0; i < i1; ++i) {
            run += yw[i];
            yw[i] = run;
        }
        u64 x = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const u64 y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) sm.red_mas[warp] = x;
        __syncthreads();
        if (warp == 0) {
            u64 y = lane < kWarps ? sm.red_mas[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const u64 z = __shfl_up_sync(0xffffffffu, y, o);
                if (lane >= o) y += z;
            }
            if (lane < kWarps) sm.red_mas[lane] = y;
        }
        __syncthreads();
        const u64 off = (warp ? sm.red_mas[warp - 1] : 0) + (x - run);
        for (int i = i0; i < i1; ++i) yw[i] += off;
        __syncthreads();
        // top-k: the mass of ranks < k; top-p: up to the first rank whose
        // inclusive mass exceeds top_p * that; the pick: the first rank whose
        // inclusive mass is >= ceil(u * the kept mass)
        const u64 z_k = use_k ? yw[k_eff - 1] : z_all;
        u64 z_r = z_k;
        if (use_p) {
            const double theta = (double)top_p * (double)z_k;
            const u64 tau = theta < 0.0 ? 0 : (u64)floor(theta) + 1;
            const int r = first_reaching(sm, yw, total, tau);
            if (r >= 0 && (u64)r + 1 < k_eff) z_r = yw[r];
        }
        u64 tau = (u64)ceil((double)u * (double)z_r);
        if (tau > z_r) tau = z_r;
        const int r = first_reaching(sm, yw, total, tau);
        if (threadIdx.x == 0) *out = r >= 0 ? (int64_t)(uint32_t)yk[r] : (int64_t)sm.row_argmax;
    }
    cl.sync();  // no CTA leaves while rank 0 may read its shared memory
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2) sample_kernel(const SampleDev a) {
    extern __shared__ __align__(16) float sv[];
    __shared__ SampleShared sm;
    const cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank();
    int64_t row = blockIdx.x / kClusterCtas;
    if (a.rows) {  // every CTA of a cluster reads the same count and entry
        if ((uint32_t)row >= *a.nrows) return;
        row = a.rows[row];
        if (row >= (int64_t)(gridDim.x / kClusterCtas)) return;  // not a row of the batch
    }
    const int64_t base = (int64_t)rank * a.slice;
    const int64_t left = a.vocab - base;
    const int n = left <= 0 ? 0 : (left < a.slice ? (int)left : a.slice);
    const T* lrow = reinterpret_cast<const T*>(a.logits) + row * a.row_stride + base;
    // Rows run one cluster each, about `ahead` clusters at a time, in row
    // order: the cluster that takes row + ahead starts when one of this wave
    // ends, so its slice is fetched into L2 now, one bulk prefetch per CTA.
    if (QF_SAMPLE_PREFETCH && threadIdx.x == 0 && a.vec && a.ahead > 0 && n > 0 &&
        row + a.ahead < (int64_t)(gridDim.x / kClusterCtas)) {
        const uint32_t bytes = (uint32_t)(((int64_t)n * (int64_t)sizeof(T)) & ~(int64_t)15);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                         reinterpret_cast<uint64_t>(lrow + a.ahead * a.row_stride)),
                     "r"(bytes)
                     : "memory");
    }

    const float temp = a.temperature[row];
    const float tc = fmaxf(temp, 1e-5f);

    // ---- load the slice, row maximum --------------------------------------
    float best = -INFINITY;
    uint32_t best_i = 0xffffffffu;
    load_slice<T>(a, lrow, n, tc, sv, best, best_i);
    if (best_i != 0xffffffffu) best_i += (uint32_t)base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float s2 = __shfl_down_sync(0xffffffffu, best, o);
        const uint32_t i2 = __shfl_down_sync(0xffffffffu, best_i, o);
        if (i2 != 0xffffffffu && (best_i == 0xffffffffu || better(s2, i2, best, best_i))) {
            best = s2;
            best_i = i2;
        }
    }
    if (lane == 0) {
        sm.red_mas[warp] = __float_as_uint(best);
        sm.red_cnt[warp] = best_i;
    }
    zero_hist(sm);
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = -INFINITY;
        uint32_t bi = 0xffffffffu;
        for (int w = 0; w < kWarps; ++w) {
            const float s2 = __uint_as_float((uint32_t)sm.red_mas[w]);
            const uint32_t i2 = sm.red_cnt[w];
            if (i2 != 0xffffffffu && (bi == 0xffffffffu || better(s2, i2, b, bi))) {
                b = s2;
                bi = i2;
            }
        }
        sm.max_s = b;
        sm.max_idx = bi;
    }
    cl.sync();
    if (threadIdx.x < 32) {  // lane q reads CTA q's maximum
        float b = -INFINITY;
        uint32_t bi = 0xffffffffu;
        if (lane < kClusterCtas) {
            const SampleShared* r = cl.map_shared_rank(&sm, lane);
            b = r->max_s;
            bi = r->max_idx;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float s2 = __shfl_xor_sync(0xffffffffu, b, o);
            const uint32_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (i2 != 0xffffffffu && (bi == 0xffffffffu || better(s2, i2, b, bi))) {
                b = s2;
                bi = i2;
            }
        }
        if (lane == 0) {
            sm.row_max = b;
            sm.row_argmax = bi;
        }
    }
    __syncthreads();
    const float m = sm.row_max;

    if (temp <= 0.0f) {  // greedy: rank 0 of the stable order
        if (rank == 0 && threadIdx.x == 0) a.out[row] = sm.row_argmax;
        cl.sync();  // no CTA leaves while others may read its shared memory
        return;
    }

    // ---- level 1 over the whole row: counts and masses ---------------------
    build_hist(sm, sv, n, m, 32, 0, 21, 2047u);
    cl.sync();
    combine(cl, sm, 0);
    cl.sync();
    if (threadIdx.x < 32) {
        u64 z = sm.lv[0].grp_mas[lane] + sm.lv[0].grp_mas[lane + 32];
#pragma unroll
        for (int o = 16; o; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        if (lane == 0) sm.z_all = z;
    }
    __syncthreads();
    const u64 z_all = sm.z_all;
    int nsel = 0;  // candidate selects so far (picks their buffer)

    // ---- settings ----------------------------------------------------------
    const int64_t V = a.vocab;
    const int64_t k = a.top_k_i64 ? reinterpret_cast<const int64_t*>(a.top_k)[row]
                                  : (int64_t)reinterpret_cast<const int32_t*>(a.top_k)[row];
    const u64 k_eff = (k > 0 && k < V) ? (u64)k : (u64)V;
    const float top_p = a.top_p[row];
    const float u = a.uniforms ? a.uniforms[row]
                               : uniform_from_hash((uint64_t)a.seeds[row], (uint64_t)a.steps[row]);
    const bool use_k = k_eff < (u64)V, use_p = top_p < 1.0f;

    // ---- one pass when the filtered head of the order is small --------------
    // Every answer ranks at or above the top-k cut, or without top-k at or
    // above the top-p cut (its threshold taken on the whole mass), so the
    // level-1 digit of that cut bounds all three.
    Crossing f0{};  // that cut's level-1 crossing, reused by its select below
    if (use_k || use_p) {
        u64 tau_b = k_eff;
        if (!use_k) {
            const double theta = (double)top_p * (double)z_all;
            tau_b = theta < 0.0 ? 0 : (u64)floor(theta) + 1;
        }
        f0 = search_all(cl, sm, 0, !use_k, tau_b, 0, 0);
        if (f0.found && f0.above_cnt + f0.cnt <= (u64)kUniTake) {
            sample_unified(cl, sm, sv, n, base, m, (uint32_t)f0.digit, use_k, k_eff, use_p, top_p,
                           z_all, u, a.out + row);
            return;
        }
    }

    // ---- top-k -------------------------------------------------------------
    u64 z_k = z_all;
    if (use_k) {
        const Selected c = select_rank(cl, sm, sv, n, base, m, false, k_eff, nsel, &f0);
        if (c.found) z_k = c.incl_mas;
    }

    // ---- top-p -------------------------------------------------------------
    u64 z_r = z_k;
    if (use_p) {
        const double theta = (double)top_p * (double)z_k;
        const u64 tau = theta < 0.0 ? 0 : (u64)floor(theta) + 1;
        // without top-k, z_k is z_all and tau the threshold f0 was found for
        const Selected c =
            select_rank(cl, sm, sv, n, base, m, true, tau, nsel, use_k ? nullptr : &f0);
        if (c.found && c.incl_cnt < k_eff) z_r = c.incl_mas;
    }

    // ---- the pick ----------------------------------------------------------
    u64 tau = (u64)ceil((double)u * (double)z_r);
    if (tau > z_r) tau = z_r;
    const Selected pick = select_rank(cl, sm, sv, n, base, m, true, tau, nsel);
    if (pick.found && pick.has_idx) {
        if (rank == 0 && threadIdx.x == 0) a.out[row] = pick.idx;
    } else if (pick.found) {
        // which CTA holds the pick: prefix over the CTAs' counts of the key
        if (threadIdx.x < 32) {
            uint32_t c = 0;
            if (lane < kClusterCtas) c = cl.map_shared_rank(&sm, lane)->u.h.cnt[pick.low_digit];
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += x;
            }
            const bool own = lane < kClusterCtas && pick.j >= incl - c && pick.j < incl;
            const unsigned bal = __ballot_sync(0xffffffffu, own);
            if (lane == 0) {
                sm.owner = bal ? __ffs(bal) - 1 : -1;
                sm.owner_j = 0;
            }
            __syncwarp();
            if (own) sm.owner_j = (uint32_t)(pick.j - (incl - c));
        }
        __syncthreads();
        const int owner = sm.owner;
        const uint32_t jj = sm.owner_j;
        __syncthreads();
        if (owner == rank) {
            const int li = nth_with_key(sm, sv, n, pick.key, jj);
            if (threadIdx.x == 0) a.out[row] = li >= 0 ? base + li : (int64_t)sm.row_argmax;
        } else if (owner < 0 && rank == 0 && threadIdx.x == 0) {
            a.out[row] = sm.row_argmax;  // unreachable: some CTA holds the pick
        }
    } else if (rank == 0 && threadIdx.x == 0) {
        a.out[row] = sm.row_argmax;  // unreachable: tau <= kept mass
    }
    cl.sync();  // no CTA leaves while others may read its shared memory
}

__global__ void uniforms_kernel(const int64_t* seeds, const int64_t* steps, int64_t n,
                                float* out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = uniform_from_hash((uint64_t)seeds[i], (uint64_t)steps[i]);
}

template <typename T>
int launch_sample(const SampleDev& a, int64_t batch, cudaStream_t stream) {
    constexpr auto kernel = sample_kernel<T>;
    static std::atomic<int> max_dyn{-1};
    if (max_dyn.load(std::memory_order_relaxed) < 0) {
        int dev = 0, optin = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        const int dyn = optin - (int)sizeof(SampleShared) - 1024;
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
        if (e != cudaSuccess) return launch_failed(e);
        max_dyn.store(dyn, std::memory_order_relaxed);
    }
    // the slice as fp32, and room for the one-pass path's sorted pairs
    const size_t smem = std::max((size_t)a.slice * sizeof(float), (size_t)kUni * 2 * sizeof(u64));
    if ((int64_t)smem > max_dyn.load(std::memory_order_relaxed)) return QF_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(batch * kClusterCtas));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kClusterCtas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // clusters resident at once for this slice size (queried once per size)
    static std::atomic<int64_t> wave_key{-1};
    static std::atomic<int> wave{0};
    const int64_t key = (int64_t)smem;
    if (wave_key.load(std::memory_order_relaxed) != key) {
        int nc = 0;
        if (cudaOccupancyMaxActiveClusters(&nc, kernel, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            nc = 0;
        }
        wave.store(nc, std::memory_order_relaxed);
        wave_key.store(key, std::memory_order_relaxed);
    }
    SampleDev b = a;
    b.ahead = a.rows ? 0 : wave.load(std::memory_order_relaxed);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, b);
    return e == cudaSuccess ? QF_OK : launch_failed(e);
}

}  // namespace
}  // namespace qf

extern "C" int qf_sample_tokens(const qf_sample_args* p, cudaStream_t stream) {
    if (!p) return QF_ERR_INVALID;
    const qf_sample_args& g = *p;
    if (g.batch < 0 || g.vocab <= 0) return QF_ERR_INVALID;
    if (g.batch == 0) return QF_OK;
    if (!g.logits || !g.temperature || !g.top_k || !g.top_p || !g.out) return QF_ERR_INVALID;
    if (!g.uniforms && (!g.seeds || !g.steps)) return QF_ERR_INVALID;
    if (g.dtype != QF_F32 && g.dtype != QF_F16 && g.dtype != QF_BF16) return QF_ERR_INVALID;
    if (g.top_k_type != QF_I32 && g.top_k_type != QF_I64) return QF_ERR_INVALID;
    if (g.logits_row_stride < g.vocab && g.batch > 1) return QF_ERR_INVALID;
    if (g.vocab >= (int64_t)1 << 31 || g.batch > (int64_t)1 << 24) return QF_ERR_UNSUPPORTED;
    const int64_t es = g.dtype == QF_F32 ? 4 : 2;
    qf::SampleDev a{};
    a.logits = static_cast<const char*>(g.logits);
    a.row_stride = g.logits_row_stride;
    a.vocab = g.vocab;
    a.slice = (int)(qf::ceil_div(qf::ceil_div(g.vocab, qf::kClusterCtas), 8) * 8);
    a.vec = qf::aligned16(g.logits) && (g.logits_row_stride * es) % 16 == 0;
    a.temperature = g.temperature;
    a.top_k = g.top_k;
    a.top_k_i64 = g.top_k_type == QF_I64;
    a.top_p = g.top_p;
    a.uniforms = g.uniforms;
    a.seeds = g.seeds;
    a.steps = g.steps;
    a.out = g.out;
    // the batch-wide passes, when asked for or when the batch is large enough
    // to keep the GPU busy with them; rows they leave go to the cluster kernel
    const bool ws_ok = g.workspace &&
                       g.workspace_bytes >= qf::sample_wide_workspace_bytes(g.batch) &&
                       (reinterpret_cast<uintptr_t>(g.workspace) & 255u) == 0;
    bool wide = false;
    switch (g.path) {
    case QF_SAMPLE_PATH_AUTO:
        wide = ws_ok && g.batch >= QF_SAMPLE_WIDE_MIN_ROWS && g.batch <= 65535;
        break;
    case QF_SAMPLE_PATH_CLUSTER: break;
    case QF_SAMPLE_PATH_WIDE:
        if (!ws_ok) return QF_ERR_INVALID;
        if (g.batch > 65535) return QF_ERR_UNSUPPORTED;
        wide = true;
        break;
    default: return QF_ERR_INVALID;
    }
    if (wide) {
        qf::WideArgs w{};
        w.logits = g.logits;
        w.row_stride = g.logits_row_stride;
        w.batch = g.batch;
        w.vocab = g.vocab;
        w.dtype = g.dtype;
        w.vec = a.vec;
        w.temperature = g.temperature;
        w.top_k = g.top_k;
        w.top_k_i64 = a.top_k_i64;
        w.top_p = g.top_p;
        w.uniforms = g.uniforms;
        w.seeds = g.seeds;
        w.steps = g.steps;
        w.out = g.out;
        w.workspace = g.workspace;
        const int rc = qf::sample_wide_passes(w, stream, &a.rows, &a.nrows);
        if (rc != QF_OK) return rc;
    }
    switch (g.dtype) {
    case QF_F32: return qf::launch_sample<float>(a, g.batch, stream);
    case QF_F16: return qf::launch_sample<__half>(a, g.batch, stream);
    default: return qf::launch_sample<__nv_bfloat16>(a, g.batch, stream);
    }
}

extern "C" int64_t qf_sample_workspace_bytes(int64_t batch) {
    return batch <= 0 ? 0 : qf::sample_wide_workspace_bytes(batch);
}

extern "C" int qf_uniforms_from_seeds(const int64_t* seeds, const int64_t* steps, int64_t n,
                                      float* out, cudaStream_t stream) {
    if (n < 0) return QF_ERR_INVALID;
    if (n == 0) return QF_OK;
    if (!seeds || !steps || !out) return QF_ERR_INVALID;
    const int threads = 256;
    qf::uniforms_kernel<<<(unsigned)qf::ceil_div(n, threads), threads, 0, stream>>>(seeds, steps,
                                                                                    n, out);
    return qf::check_launch();
}
