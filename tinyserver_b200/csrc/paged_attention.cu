// Decode-phase paged attention over the (N, Hkv, B, D) KV pages.
//
// Replaces paged_attention_forward (server/model/kernels/paged_attention.py:
// 124-192; Triton kernel :8-121): for every sequence s and query head h, one
// query token against the sequence's first seq_lens[s] cached tokens,
//   out[s, h, :] = softmax(q[s, h] . K_s^T * scale) @ V_s       (fp32 math)
// with K_s/V_s gathered through block_tables[s] (token j at block
// block_tables[s, j / B], slot j % B) and kv head h / (Hq / Hkv) (GQA).
//
// B200 shape of the computation (flash-decoding):
//  * one CTA per (sequence, kv head, partition of kPart keys); the CTA serves
//    all G = Hq/Hkv query heads of its kv head, so every K and V row crosses
//    HBM once per layer, not once per query head (the reference's grid is
//    (sequence, query head));
//  * 4 warps take 32-key tiles in turn; in QK a lane owns one key and walks
//    its row with 16-byte loads against q in shared memory (broadcast reads);
//    online softmax per warp and head in fp32; in PV a lane owns D/32
//    elements of the output and reads each V row coalesced;
//  * the warps merge through shared memory; a sequence longer than one
//    partition leaves per-partition (max, sum, acc) in a caller-provided fp32
//    workspace and a second kernel merges them.
// Keys past seq_len are never read; a block index outside the cache is
// skipped and flagged (QF_FLAG_BAD_BLOCK); a seq_len longer than its
// block-table row is cut to the row and flagged (QF_FLAG_BAD_TABLE).
#include <math.h>

#include "qf_common.cuh"
#include "qf_mma.cuh"

// Keys per CTA when a workspace allows splitting a sequence: the longest
// partition (fewest partials, best on B200 at the c3 decode shape) unless the
// batch has too few sequences to fill the GPU that way; then it halves, down
// to the shortest, until there are at least kAttnTargetParts
// (sequence, partition) pairs.  Compile-time knobs.
#ifndef QF_ATTN_PARTITION
#define QF_ATTN_PARTITION 2048
#endif
#ifndef QF_ATTN_MIN_PARTITION
#define QF_ATTN_MIN_PARTITION 256
#endif
constexpr int64_t kAttnTargetParts = 512;

namespace qf {
namespace {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = 32 * kAttnWarps;
#ifndef QF_ATTN_PV_BATCH
#define QF_ATTN_PV_BATCH 8
#endif
constexpr int kPvBatch = QF_ATTN_PV_BATCH;  // V rows in flight per lane in PV

struct AttnDev {
    const char* q;
    int64_t qs, qh;  // query strides (sequence, head), elements
    const char* kc;
    const char* vc;
    int64_t c0, c1, c2;  // cache strides (block, head, slot), elements
    int64_t N, B;
    const int32_t* bt;
    int64_t bts, max_blocks;
    const int32_t* lens;
    int S, Hq, Hkv;
    float scale;
    char* out;
    int64_t os, oh;
    float* ws;  // [S][Hq][P][D + 2]: acc[0:D], max, sum
    int P;      // partitions per sequence in the workspace layout
    int part;   // keys per partition
    int32_t* status;
};

// Keys of sequence s that the kernels may read: seq_lens[s], clamped to what
// its block-table row can describe (max_blocks * B).  A longer length would
// index past the row and need more partitions than the workspace holds, so it
// is cut to the row and flagged QF_FLAG_BAD_TABLE (by one thread of each CTA).
__device__ __forceinline__ int seq_keys(const AttnDev& a, int s) {
    int L = __ldg(a.lens + s);
    const int64_t cap = a.max_blocks * a.B;
    if ((int64_t)L > cap) {
        if (threadIdx.x == 0) flag(a.status, QF_FLAG_BAD_TABLE);
        L = (int)cap;
    }
    return L;
}

// Load PER elements of one row (PER * sizeof(T) bytes: 4, 8 or a multiple of
// 16) as floats.
template <typename T, int PER>
__device__ __forceinline__ void load_row_slice(const char* p, float* f) {
    constexpr int BYTES = PER * (int)sizeof(T);
    if constexpr (BYTES % 16 == 0) {
#pragma unroll
        for (int c = 0; c < BYTES / 16; ++c) unpack<T>(ld_shared_ro16(p + c * 16), f + c * Dt<T>::kPerVec);
    } else {
        static_assert(BYTES == 4 || BYTES == 8, "slice size");
        uint2 r;
        if constexpr (BYTES == 8) r = __ldg(reinterpret_cast<const uint2*>(p));
        else r = make_uint2(__ldg(reinterpret_cast<const unsigned*>(p)), 0);
        const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
        for (int i = 0; i < PER; ++i) f[i] = Dt<T>::to_f(e[i]);
    }
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kAttnThreads) paged_decode_kernel(const AttnDev a) {
    constexpr int ES = sizeof(T);
    constexpr int EPV = 16 / ES;       // elements per 16-byte chunk
    constexpr int NCH = D / EPV;       // 16-byte chunks per row
    constexpr int PER = D / 32;        // output elements per lane in PV
    const int p = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
    const int L = seq_keys(a, s);
    const int k_begin = p * a.part;
    if (p > 0 && k_begin >= L) return;  // partition past the sequence (p = 0 always runs)
    const int k_end = min(L, k_begin + a.part);
    const int nparts = L > a.part ? (L + a.part - 1) / a.part : 1;

    __shared__ __align__(16) float qs[G][D];
    __shared__ float ps[kAttnWarps][G][32];
    __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
    __shared__ __align__(16) float wacc[kAttnWarps][G][D];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < G * D; i += kAttnThreads) {
        const int h = i / D, d = i - h * D;
        const T* qp = reinterpret_cast<const T*>(a.q) + (int64_t)s * a.qs +
                      (int64_t)(g * G + h) * a.qh + d;
        qs[h][d] = Dt<T>::to_f(*qp);
    }
    __syncthreads();

    float m[G], l[G], acc[G][PER];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[h][e] = 0.f;
    }

    const int ntiles = (k_end - k_begin + 31) / 32;
    const int32_t* bt = a.bt + (int64_t)s * a.bts;
    for (int tile = warp; tile < ntiles; tile += kAttnWarps) {
        const int j0 = k_begin + tile * 32;
        const int j = j0 + lane;
        bool valid = j < k_end;
        int64_t row_off = 0;  // (block, head g, slot) element offset of key j
        if (valid) {
            const int64_t lb = j / a.B;
            const int64_t blk = __ldg(bt + lb);
            if (blk < 0 || blk >= a.N) {
                flag(a.status, QF_FLAG_BAD_BLOCK);
                valid = false;
            } else {
                row_off = blk * a.c0 + (int64_t)g * a.c1 + (j - lb * a.B) * a.c2;
            }
        }

        // QK: lane = key, the row in 16-byte chunks, 8 in flight
        float sc[G];
#pragma unroll
        for (int h = 0; h < G; ++h) sc[h] = 0.f;
        if (valid) {
            const char* kr = a.kc + row_off * ES;
#pragma unroll
            for (int c0 = 0; c0 < NCH; c0 += 8) {
                uint4 kv[8];
#pragma unroll
                for (int c = 0; c < 8; ++c)  // L1-cached: a lane's 16-byte loads share sectors
                    if (c0 + c < NCH) kv[c] = ld_shared_ro16(kr + (c0 + c) * 16);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    if (c0 + c >= NCH) break;
                    float x[EPV];
                    unpack<T>(kv[c], x);
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const float* qv = &qs[h][(c0 + c) * EPV];
#pragma unroll
                        for (int e = 0; e < EPV; ++e) sc[h] = fmaf(qv[e], x[e], sc[h]);
                    }
                }
            }
        }

        // online softmax, per head
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float v = valid ? sc[h] * a.scale : -INFINITY;
            const float mnew = fmaxf(m[h], warp_max(v));
            const float pj = valid ? exp_rel(v, mnew) : 0.f;
            const float corr = exp_rel(m[h], mnew);
            l[h] = l[h] * corr + warp_sum(pj);
#pragma unroll
            for (int e = 0; e < PER; ++e) acc[h][e] *= corr;
            m[h] = mnew;
            ps[warp][h][lane] = pj;
        }
        __syncwarp();

        // PV: lane = D/32 output elements; V rows coalesced, kPvBatch keys' loads
        // in flight at a time.  A key that is not valid has p = 0 and reads a
        // safe row (offset 0 of the cache), so the loop has no branch.
        const int nk = min(32, k_end - j0);
        for (int jb = 0; jb < nk; jb += kPvBatch) {
            float v[kPvBatch][PER];
#pragma unroll
            for (int u = 0; u < kPvBatch; ++u) {
                const int jj = jb + u < nk ? jb + u : nk - 1;
                const int64_t off = __shfl_sync(0xffffffffu, row_off, jj);
                load_row_slice<T, PER>(a.vc + (off + lane * PER) * ES, v[u]);
            }
#pragma unroll
            for (int u = 0; u < kPvBatch; ++u) {
                if (jb + u >= nk) break;
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float pj = ps[warp][h][jb + u];
#pragma unroll
                    for (int e = 0; e < PER; ++e) acc[h][e] = fmaf(pj, v[u][e], acc[h][e]);
                }
            }
        }
        __syncwarp();
    }

    // merge the warps
#pragma unroll
    for (int h = 0; h < G; ++h) {
        if (lane == 0) {
            wm[warp][h] = m[h];
            wl[warp][h] = l[h];
        }
#pragma unroll
        for (int e = 0; e < PER; ++e) wacc[warp][h][lane * PER + e] = acc[h][e];
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kAttnThreads) {
        const int h = i / D, d = i - h * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][h]);
        float Ls = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = exp_rel(wm[w][h], M);
            Ls += wl[w][h] * f;
            A += wacc[w][h][d] * f;
        }
        const int hq = g * G + h;
        if (nparts == 1) {
            T* o = reinterpret_cast<T*>(a.out) + (int64_t)s * a.os + (int64_t)hq * a.oh;
            o[d] = Dt<T>::from_f(A / Ls);
        } else {
            float* w = a.ws + (((int64_t)s * a.Hq + hq) * a.P + p) * (D + 2);
            w[d] = A;
            if (d == 0) {
                w[D] = M;
                w[D + 1] = Ls;
            }
        }
    }
}

// Merge the partitions of sequences longer than one partition.
template <typename T, int D>
__global__ void __launch_bounds__(128) paged_decode_merge_kernel(const AttnDev a) {
    const int hq = blockIdx.x, s = blockIdx.y;
    const int L = seq_keys(a, s);
    const int nparts = L > a.part ? (L + a.part - 1) / a.part : 1;
    if (nparts == 1) return;
    const float* w = a.ws + ((int64_t)s * a.Hq + hq) * a.P * (D + 2);
    float M = -INFINITY;
    for (int p = 0; p < nparts; ++p) M = fmaxf(M, w[p * (D + 2) + D]);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float Ls = 0.f, A = 0.f;
        for (int p = 0; p < nparts; ++p) {
            const float* wp = w + p * (D + 2);
            const float f = exp_rel(wp[D], M);
            Ls += wp[D + 1] * f;
            A += wp[d] * f;
        }
        T* o = reinterpret_cast<T*>(a.out) + (int64_t)s * a.os + (int64_t)hq * a.oh;
        o[d] = Dt<T>::from_f(A / Ls);
    }
}

// ---------------------------------------------------------------------------
// 16-bit path on the tensor cores.  Same work split (CTA = sequence, kv head,
// partition; warps take tiles in turn) with a 16-key tile per warp step:
//  * the tile's K and V rows are copied into the warp's own shared-memory
//    double buffer with cp.async (16 bytes per lane, the next tile in flight
//    while the current one is computed), chunk index XOR-swizzled by row so
//    ldmatrix reads are free of bank conflicts;
//  * S = Q K^T on mma.sync m16n8k16 (bf16/f16 in, fp32 accumulate): the G
//    query heads are the M rows (padded to 16), keys the N columns;
//  * online softmax in fp32 on the accumulator fragments (each row's values
//    live in one quad of lanes);
//  * O += P V on mma.sync, with P split into a 16-bit high part and the
//    16-bit rounding of its remainder (P = hi + lo to ~16 significant bits,
//    so the product keeps fp32-class accuracy), V fragments by ldmatrix.trans.
template <int D>
struct MmaTile {
    static constexpr int TK = 16;            // keys per warp step
    static constexpr int NCH = D * 2 / 16;   // 16-byte chunks per row
    static constexpr int ROW = D * 2;        // bytes per row
    static constexpr int MAT = TK * ROW;     // bytes of one K or V tile
    static constexpr int STAGE = 2 * MAT;    // K and V
    static constexpr int WARP = 2 * STAGE;   // double buffer
    static constexpr int QS = 16 * ROW;      // Q (16 rows, rows >= G zero)
    static constexpr int SMEM = QS + kAttnWarps * WARP;
    // byte offset of logical 16-byte chunk c of row r in a swizzled tile
    __device__ __forceinline__ static int off(int r, int c) { return r * ROW + ((c ^ (r & 7)) << 4); }
};

template <typename T, int D, int G>
__global__ void __launch_bounds__(kAttnThreads) paged_decode_mma_kernel(const AttnDev a) {
    using MT = MmaTile<D>;
    using P = Packed<T>;
    constexpr int TK = MT::TK, NCH = MT::NCH, NT = D / 8, KS = D / 16;
    const int p = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
    const int L = seq_keys(a, s);
    const int k_begin = p * a.part;
    if (p > 0 && k_begin >= L) return;
    const int k_end = min(L, k_begin + a.part);
    const int nparts = L > a.part ? (L + a.part - 1) / a.part : 1;

    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* qsm = smem;  // [16][D] T, unswizzled
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned char* wbuf = smem + MT::QS + warp * MT::WARP;

    for (int i = tid; i < 16 * D; i += kAttnThreads) {
        const int r = i / D, d = i - r * D;
        T v = Dt<T>::from_f(0.f);
        if (r < G)
            v = reinterpret_cast<const T*>(a.q)[(int64_t)s * a.qs + (int64_t)(g * G + r) * a.qh + d];
        reinterpret_cast<T*>(qsm)[i] = v;
    }
    __syncthreads();

    const int gid = lane >> 2, tig = lane & 3;
    uint32_t qa[KS][4];  // Q A-fragments, one per 16-dim k-step
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        const int r = ((lane >> 3) & 1) * 8 + (lane & 7), c = 2 * ks + (lane >> 4);
        ldsm_x4(qa[ks], qsm + r * MT::ROW + c * 16);
    }

    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows gid, gid + 8
    const int32_t* bt = a.bt + (int64_t)s * a.bts;

    // issue the cp.async copies of the tile starting at key j0 into buffer b;
    // returns the tile's valid-key mask (bit k: key j0 + k is read)
    auto issue = [&](int j0, int b) -> unsigned {
        int64_t row_off = 0;
        bool valid = false;
        if (lane < TK && j0 + lane < k_end) {
            const int j = j0 + lane;
            const int64_t lb = j / a.B;
            const int64_t blk = __ldg(bt + lb);
            if (blk < 0 || blk >= a.N) {
                flag(a.status, QF_FLAG_BAD_BLOCK);
            } else {
                valid = true;
                row_off = blk * a.c0 + (int64_t)g * a.c1 + (j - lb * a.B) * a.c2;
            }
        }
        const unsigned mask = __ballot_sync(0xffffffffu, valid);
        unsigned char* kt = wbuf + b * MT::STAGE;
        unsigned char* vt = kt + MT::MAT;
#pragma unroll
        for (int i = lane; i < TK * NCH; i += 32) {
            const int k = i / NCH, c = i - k * NCH;
            const int64_t off = __shfl_sync(0xffffffffu, row_off, k);
            const int bytes = (mask >> k) & 1 ? 16 : 0;
            cp_async16(kt + MT::off(k, c), a.kc + off * 2 + c * 16, bytes);
            cp_async16(vt + MT::off(k, c), a.vc + off * 2 + c * 16, bytes);
        }
        return mask;
    };

    int j0 = k_begin + warp * TK;
    unsigned mask_cur = j0 < k_end ? issue(j0, 0) : 0u;
    cp_async_commit();
    for (int it = 0; j0 < k_end; ++it, j0 += kAttnWarps * TK) {
        const int jn = j0 + kAttnWarps * TK;
        const unsigned mask_next = jn < k_end ? issue(jn, (it + 1) & 1) : 0u;
        cp_async_commit();
        cp_async_wait<1>();  // this tile has landed (the next may still be in flight)
        __syncwarp();
        const unsigned char* kt = wbuf + (it & 1) * MT::STAGE;
        const unsigned char* vt = kt + MT::MAT;

        // S = Q K^T for the 16 keys (two n-tiles of 8)
        float sc[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < KS / 2; ++kk) {
                uint32_t b[4];
                ldsm_x4(b, kt + MT::off(n * 8 + (lane & 7), kk * 4 + (lane >> 3)));
                Mma<T>::run(sc[n], qa[2 * kk], b[0], b[1]);
                Mma<T>::run(sc[n], qa[2 * kk + 1], b[2], b[3]);
            }
        }
        // online softmax: row gid holds sc[n][0..1], row gid + 8 holds sc[n][2..3]
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const bool ok = (mask_cur >> (n * 8 + 2 * tig + e)) & 1;
                sc[n][e] = ok ? sc[n][e] * a.scale : -INFINITY;
                sc[n][2 + e] = ok ? sc[n][2 + e] * a.scale : -INFINITY;
                mx0 = fmaxf(mx0, sc[n][e]);
                mx1 = fmaxf(mx1, sc[n][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float cr0 = exp_rel(m0, mn0), cr1 = exp_rel(m1, mn1);
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                sc[n][e] = exp_rel(sc[n][e], mn0);
                sc[n][2 + e] = exp_rel(sc[n][2 + e], mn1);
                sum0 += sc[n][e];
                sum1 += sc[n][2 + e];
            }
        }
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
        l0 = l0 * cr0 + sum0;
        l1 = l1 * cr1 + sum1;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            o[n][0] *= cr0;
            o[n][1] *= cr0;
            o[n][2] *= cr1;
            o[n][3] *= cr1;
        }
        // P as A-fragments (C layout of the two n-tiles = A layout of k16), hi + lo
        uint32_t ph[4], pl[4];
        {
            const float* f[4] = {&sc[0][0], &sc[0][2], &sc[1][0], &sc[1][2]};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                ph[r] = P::pack(f[r][0], f[r][1]);
                pl[r] = P::pack(f[r][0] - P::lo(ph[r]), f[r][1] - P::hi(ph[r]));
            }
        }
        // O += P V, two output n-tiles per ldmatrix.x4.trans
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b[4];
            ldsm_x4_t(b, vt + MT::off(((lane >> 3) & 1) * 8 + (lane & 7), 2 * np + (lane >> 4)));
            Mma<T>::run(o[2 * np], ph, b[0], b[1]);
            Mma<T>::run(o[2 * np], pl, b[0], b[1]);
            Mma<T>::run(o[2 * np + 1], ph, b[2], b[3]);
            Mma<T>::run(o[2 * np + 1], pl, b[2], b[3]);
        }
        __syncwarp();  // every lane is done with this buffer before it is refilled
        mask_cur = mask_next;
    }
    cp_async_wait<0>();
    __syncthreads();  // all warps done: the tile buffers become the merge area

    // merge the warps (rows r < G only; row gid's values: o[n][0..1], m0, l0)
    float* wm_ = reinterpret_cast<float*>(smem + MT::QS);   // [warps][G]
    float* wl_ = wm_ + kAttnWarps * G;                        // [warps][G]
    float* wacc_ = wl_ + kAttnWarps * G;                      // [warps][G][D]
    if (gid < G) {
        if (tig == 0) {
            wm_[warp * G + gid] = m0;
            wl_[warp * G + gid] = l0;
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            float* dst = wacc_ + (warp * G + gid) * D + n * 8 + 2 * tig;
            dst[0] = o[n][0];
            dst[1] = o[n][1];
        }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kAttnThreads) {
        const int h = i / D, d = i - h * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm_[w * G + h]);
        float Ls = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = exp_rel(wm_[w * G + h], M);
            Ls += wl_[w * G + h] * f;
            A += wacc_[(w * G + h) * D + d] * f;
        }
        const int hq = g * G + h;
        if (nparts == 1) {
            T* out = reinterpret_cast<T*>(a.out) + (int64_t)s * a.os + (int64_t)hq * a.oh;
            out[d] = Dt<T>::from_f(A / Ls);
        } else {
            float* w = a.ws + (((int64_t)s * a.Hq + hq) * a.P + p) * (D + 2);
            w[d] = A;
            if (d == 0) {
                w[D] = M;
                w[D + 1] = Ls;
            }
        }
    }
}

template <typename T, int D, int G>
int launch_attn_mma(const AttnDev& a, cudaStream_t stream) {
    constexpr auto kernel = paged_decode_mma_kernel<T, D, G>;
    constexpr int smem = MmaTile<D>::SMEM;
    static_assert(MmaTile<D>::QS + 2 * kAttnWarps * G * 4 + kAttnWarps * G * D * 4 <= smem,
                  "merge area must fit in the tile buffers");
    static std::atomic<bool> configured{false};
    if (!configured.load(std::memory_order_relaxed)) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return launch_failed(e);
        configured.store(true, std::memory_order_relaxed);
    }
    const dim3 grid((unsigned)a.P, (unsigned)a.Hkv, (unsigned)a.S);
    kernel<<<grid, kAttnThreads, smem, stream>>>(a);
    int rc = check_launch();
    if (rc || a.P == 1) return rc;
    paged_decode_merge_kernel<T, D><<<dim3((unsigned)a.Hq, (unsigned)a.S), 128, 0, stream>>>(a);
    return check_launch();
}

template <typename T, int D, int G>
int launch_attn(const AttnDev& a, cudaStream_t stream) {
    const dim3 grid((unsigned)a.P, (unsigned)a.Hkv, (unsigned)a.S);
    paged_decode_kernel<T, D, G><<<grid, kAttnThreads, 0, stream>>>(a);
    int rc = check_launch();
    if (rc || a.P == 1) return rc;
    paged_decode_merge_kernel<T, D><<<dim3((unsigned)a.Hq, (unsigned)a.S), 128, 0, stream>>>(a);
    return check_launch();
}

template <typename T, int D, int G>
int launch_best(const AttnDev& a, cudaStream_t stream) {
#ifndef QF_ATTN_NO_MMA
    if constexpr (sizeof(T) == 2) return launch_attn_mma<T, D, G>(a, stream);
#endif
    return launch_attn<T, D, G>(a, stream);
}

template <typename T, int D>
int dispatch_g(const AttnDev& a, int G, cudaStream_t stream) {
    switch (G) {
    case 1: return launch_best<T, D, 1>(a, stream);
    case 2: return launch_best<T, D, 2>(a, stream);
    case 4: return launch_best<T, D, 4>(a, stream);
    case 8: return launch_best<T, D, 8>(a, stream);
    default: return QF_ERR_UNSUPPORTED;
    }
}

template <typename T>
int dispatch_d(const AttnDev& a, int64_t D, int G, cudaStream_t stream) {
    switch (D) {
    case 64: return dispatch_g<T, 64>(a, G, stream);
    case 128: return dispatch_g<T, 128>(a, G, stream);
    case 256: return dispatch_g<T, 256>(a, G, stream);
    default: return QF_ERR_UNSUPPORTED;
    }
}

int partitions(int64_t max_seq_len, int64_t part) {
    return (int)std::max<int64_t>(1, ceil_div(max_seq_len, part));
}

int64_t partition_keys(int64_t num_seqs, int64_t max_seq_len) {
    int64_t part = QF_ATTN_PARTITION;
    while (part > QF_ATTN_MIN_PARTITION && num_seqs * partitions(max_seq_len, part) < kAttnTargetParts)
        part /= 2;
    return part;
}

}  // namespace
}  // namespace qf

extern "C" size_t qf_paged_attention_workspace_bytes(int64_t num_seqs, int64_t num_q_heads,
                                                     int64_t head_dim, int64_t max_seq_len) {
    if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_seq_len <= 0) return 0;
    const int64_t P = qf::partitions(max_seq_len, qf::partition_keys(num_seqs, max_seq_len));
    if (P == 1) return 0;
    int64_t n = 0;  // num_seqs * num_q_heads * P * (head_dim + 2) floats; SIZE_MAX on overflow
    if (__builtin_mul_overflow(num_seqs, num_q_heads, &n) || __builtin_mul_overflow(n, P, &n) ||
        __builtin_mul_overflow(n, head_dim + 2, &n) ||
        __builtin_mul_overflow(n, (int64_t)sizeof(float), &n))
        return SIZE_MAX;
    return (size_t)n;
}

namespace {
// Argument checks shared by both decode entry points, before any device work.
int check_decode_args(const qf_paged_attention_args& g) {
    if (g.num_seqs < 0 || g.num_q_heads <= 0 || g.num_kv_heads <= 0 || g.block_size <= 0 ||
        g.num_blocks < 0 || g.max_blocks_per_seq < 0)
        return QF_ERR_INVALID;
    if (g.num_seqs == 0) return QF_OK;
    if (!g.q || !g.k_cache || !g.v_cache || !g.block_tables || !g.seq_lens || !g.out)
        return QF_ERR_INVALID;
    if (g.num_q_heads % g.num_kv_heads) return QF_ERR_INVALID;
    if (g.num_seqs > 65535 || g.num_kv_heads > 65535) return QF_ERR_UNSUPPORTED;
    // key indices are int on the device: a block-table row describes < 2^31 keys
    if (g.max_blocks_per_seq > INT32_MAX / g.block_size) return QF_ERR_UNSUPPORTED;
    if (g.dtype != QF_F32 && g.dtype != QF_F16 && g.dtype != QF_BF16) return QF_ERR_INVALID;
    const int64_t D = g.head_dim;
    const int64_t es = g.dtype == QF_F32 ? 4 : 2;
    // K rows are read in 16-byte chunks, V row slices in D/32-element pieces
    if ((D * es) % 16 || (g.cache_strides[0] * es) % 16 || (g.cache_strides[1] * es) % 16 ||
        (g.cache_strides[2] * es) % 16 || g.cache_strides[3] != 1 || !qf::aligned16(g.k_cache) ||
        !qf::aligned16(g.v_cache))
        return QF_ERR_UNSUPPORTED;
    return QF_OK;
}
}  // namespace

extern "C" int qf_paged_attention_decode(const qf_paged_attention_args* p, cudaStream_t stream) {
    if (!p) return QF_ERR_INVALID;
    const qf_paged_attention_args& g = *p;
    const int rc = check_decode_args(g);
    if (rc || g.num_seqs == 0) return rc;
    const int64_t D = g.head_dim;
    qf::AttnDev a{};
    a.q = static_cast<const char*>(g.q);
    a.qs = g.q_stride_seq;
    a.qh = g.q_stride_head;
    a.kc = static_cast<const char*>(g.k_cache);
    a.vc = static_cast<const char*>(g.v_cache);
    a.c0 = g.cache_strides[0];
    a.c1 = g.cache_strides[1];
    a.c2 = g.cache_strides[2];
    a.N = g.num_blocks;
    a.B = g.block_size;
    a.bt = g.block_tables;
    a.bts = g.block_tables_row_stride;
    a.max_blocks = g.max_blocks_per_seq;
    a.lens = g.seq_lens;
    a.S = (int)g.num_seqs;
    a.Hq = (int)g.num_q_heads;
    a.Hkv = (int)g.num_kv_heads;
    a.scale = g.scale;
    a.out = static_cast<char*>(g.out);
    a.os = g.out_stride_seq;
    a.oh = g.out_stride_head;
    a.status = g.status;
    // the longest sequence the block tables can describe bounds the partitions
    const int64_t max_len = std::max<int64_t>(1, g.max_blocks_per_seq * g.block_size);
    const int64_t need = (int64_t)qf_paged_attention_workspace_bytes(g.num_seqs, g.num_q_heads,
                                                                     D, max_len);
    if (need > 0 && g.workspace && g.workspace_bytes >= need) {
        a.part = (int)qf::partition_keys(g.num_seqs, max_len);
        a.P = qf::partitions(max_len, a.part);
        a.ws = static_cast<float*>(g.workspace);
    } else if (need > 0 && g.workspace) {
        return QF_ERR_INVALID;  // a workspace was given but is too small
    } else {
        a.part = (int)std::min<int64_t>(max_len, 1 << 30);  // one partition per sequence
        a.P = 1;
        a.ws = nullptr;
    }
    const int G = (int)(g.num_q_heads / g.num_kv_heads);
    switch (g.dtype) {
    case QF_F32: return qf::dispatch_d<float>(a, D, G, stream);
    case QF_F16: return qf::dispatch_d<__half>(a, D, G, stream);
    default: return qf::dispatch_d<__nv_bfloat16>(a, D, G, stream);
    }
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory: a
// host framework that hands this library only raw pointers and owns every
// allocation itself, a runtime that reserves all device memory once at start
// and forbids cudaMalloc afterwards, or a latency-bound loop where the device
// synchronisation that cudaMalloc/cudaFree imply is not acceptable.  They
// call qf_paged_attention_decode_noalloc, whose split-K partials live in the
// fixed array below instead of a caller workspace.
//
// The array is a file-scope device global: every GPU that loads this library
// holds its kNoAllocScratchBytes until the process exits.  All calls on a
// device share it and it keeps the last call's contents; nothing in it has to
// start at zero (each call writes every partial it later reads), but calls
// that overlap on the GPU (two streams, two threads) race on it.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(128) << 20;  // 128 MiB
__device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices];  // device address of g_attn_scratch, per device

// The array's device address on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress, once per device, with that device current.
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qf::launch_failed(e);
    if (dev < 0 || dev >= kMaxDevices) return QF_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess) return qf::launch_failed(e);
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return QF_OK;
}
}  // namespace

extern "C" size_t qf_paged_attention_noalloc_capacity(void) { return kNoAllocScratchBytes; }

extern "C" int qf_paged_attention_decode_noalloc(const qf_paged_attention_args* p,
                                                 cudaStream_t stream) {
    if (!p) return QF_ERR_INVALID;
    const int rc0 = check_decode_args(*p);  // an invalid call is refused as such, not as too big
    if (rc0 || p->num_seqs == 0) return rc0;
    // check_decode_args bounds max_blocks_per_seq * block_size below 2^31
    const int64_t max_len = std::max<int64_t>(1, p->max_blocks_per_seq * p->block_size);
    if (qf_paged_attention_workspace_bytes(p->num_seqs, p->num_q_heads, p->head_dim, max_len) >
        kNoAllocScratchBytes)
        return QF_ERR_SCRATCH;  // checked before any device work
    qf_paged_attention_args a = *p;
    void* ptr = nullptr;
    const int rc = scratch_address(&ptr);
    if (rc) return rc;
    a.workspace = ptr;
    a.workspace_bytes = (int64_t)kNoAllocScratchBytes;
    return qf_paged_attention_decode(&a, stream);
}
