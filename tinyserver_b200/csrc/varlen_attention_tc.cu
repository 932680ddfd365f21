// Prefill varlen attention on the 5th-generation tensor cores (tcgen05, TMEM,
// TMA), warp-specialised.
//
// Same contract as the mma.sync kernel in varlen_attention.cu -- the
// reference's flash_attn_varlen_func (server/model/kernels/
// varlen_attention.py:145-218): packed sequences, causal masking with query i
// keeping key j when i >= j (indices within the sequence, :111-114), GQA by
// h / (Hq / Hkv), fp32 softmax, probabilities rounded to the value dtype
// before they meet V (:121) -- for head_dim 128 in bf16 / fp16.
//
// A work item is two 128-row query tiles of one sequence that read the same
// K and V: the same rows of two query heads of one GQA group when the group
// size is even, else 256 consecutive rows of one head.  Persistent CTAs (one
// per SM) take items in turn; each has ten warps:
//   warps 0-3   softmax of tile 0 (thread t owns query row t: tensor-memory
//               lane t), warps 4-7 the same for tile 1;
//   warp 8      issues the MMAs (one thread);
//   warp 9      issues the TMA copies (one thread).
// Per 128-key block j and tile t:
//   S_t = Q_t K_j^T   tcgen05.mma, Q and K from shared memory, S in TMEM
//   softmax           the tile's warps read S_t (tcgen05.ld), mask, update the
//                     running max m and sum l, rescale their rows of O_t when
//                     m grows, and write P_t (rounded to the value dtype) over
//                     the first 64 columns of S_t (tcgen05.st)
//   O_t += P_t V_j    tcgen05.mma with A = P_t from TMEM, B = V_j from smem
// The MMA thread orders the tensor core's work as S_0,0 S_1,0 | PV_0,0 S_0,1
// PV_1,0 S_1,1 | ... so the tensor core runs one tile's P V and next S while
// the other tile's warps are in their softmax.  tcgen05 operations of one
// thread execute in issue order, which is what lets S_t,j+1 reuse the columns
// P_t,j was read from.  K and V tiles arrive by TMA (3-D tensor maps over
// head_dim x heads x tokens, 128-byte swizzle) into a two-stage ring guarded
// by full / empty mbarriers.  Every wait is bounded: one that runs out sets
// QF_FLAG_TIMEOUT and the kernel finishes without its result.
//
// Operand layout in shared memory: a 128-row tile of 128 16-bit elements is
// two 16 KB slabs of 64 elements (128 bytes) per row in the canonical
// 128-byte swizzle (row r at r * 128, 16-byte chunk c at (c ^ r % 8) * 16),
// which is what a TMA box of 64 x 1 x 128 with SWIZZLE_128B writes.  Q and K
// are read K-major, V MN-major (rows = keys, the reduction dimension).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "qf_common.cuh"
#include "qf_varlen.cuh"

namespace qf {
namespace {

constexpr int kRows = 128;                // rows per tile, keys per block
constexpr int kSlab = kRows * 128;        // 16 KB
constexpr int kTile = 2 * kSlab;          // 32 KB: one 128 x 128 tile
constexpr int kStage = 4096;              // a softmax warp's epilogue staging: 32 rows x 128 B
constexpr int kSmem = 6 * kTile + 8 * kStage + 1024;  // Q[2], K[2], V[2], staging, alignment
constexpr int kThreads = 320;
constexpr int kMmaWarp = 8, kTmaWarp = 9;
constexpr uint32_t kTmemCols = 512;       // S_0 | S_1 | O_0 | O_1
constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at the boost clock
constexpr float kRedoLog2 = 32.f;  // one-pass softmax: p up to 2^32 kept, beyond redone

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulator, A and B both bf16 (or
// both fp16), A K-major, B K-major or MN-major, M = N = 128.
__device__ __forceinline__ uint32_t idesc(uint32_t ab_bf16, uint32_t b_mn_major) {
    return (1u << 4) | (ab_bf16 << 7) | (ab_bf16 << 10) | (b_mn_major << 16) |
           ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t id,
                                       uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id,
                                       uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(id), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Bounded wait for the completion of phase `parity`.  False when it ran out
// (the first wait to run out raises *abort) or, for a wait that watches
// `abort`, as soon as another wait has raised it: every role then leaves its
// loop without waiting out each remaining phase.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        if (abort && *abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            if (abort) *abort = 1;
            return false;
        }
    }
}

// TMA: box {64 elements, 1 head, 128 tokens} at (x, head, token) into `dst`.
__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, int x, int head,
                                         int token, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(head), "r"(token), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_tile(char* tile, const CUtensorMap* map, int head, int token,
                                         uint64_t* bar) {
    tma_load(tile, map, 0, head, token, bar);
    tma_load(tile + kSlab, map, 64, head, token, bar);
}

// TMA store of a {64 elements, 1 head, 32 tokens} box from `src` (128-byte
// swizzled, as the map says) at (x, head, token); one bulk group per call.
__device__ __forceinline__ void tma_store(const CUtensorMap* map, int x, int head, int token,
                                          const void* src) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];\n\t"
        "cp.async.bulk.commit_group;" ::"l"(reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(head), "r"(token), "r"(smem_u32(src))
        : "memory");
}
// This thread's bulk stores have read their shared memory / are complete.
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void tma_store_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

#define QF_TMEM_REGS32(r)                                                                       \
    "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),         \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),           \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),           \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define QF_TMEM_IN32(r)                                                                          \
    "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),      \
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),        \
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),      \
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),      \
        "r"(r[29]), "r"(r[30]), "r"(r[31])

// 32 consecutive columns of this thread's lane (warp w reads lanes 32 (w % 4)..).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : QF_TMEM_REGS32(r)
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "
        "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, "
        "%27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        QF_TMEM_IN32(r)
        : "memory");
}

// 16 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "
        "%10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

// 2^x with one MUFU instruction (subnormal results flush to 0).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// (d0, d1) = (a0 * b + c, a1 * b + c) as one packed fp32x2 FMA.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\tmov.b64 rc, {%5, %5};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b), "f"(c));
}

// (s0, s1) += (a0, a1) as one packed fp32x2 add.
__device__ __forceinline__ void add2(float& s0, float& s1, float a0, float a1) {
    asm("{\n\t.reg .b64 rs, ra;\n\t"
        "mov.b64 rs, {%0, %1};\n\tmov.b64 ra, {%2, %3};\n\t"
        "add.f32x2 rs, rs, ra;\n\tmov.b64 {%0, %1}, rs;\n\t}"
        : "+f"(s0), "+f"(s1)
        : "f"(a0), "f"(a1));
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// This warp's rows of O_t times f (each thread its own row; 1 keeps it).
__device__ __forceinline__ void scale_o(uint32_t sO, float f) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(sO + 32 * c, o);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
        tmem_st32(sO + 32 * c, o);
    }
}

// Columns [lim, 128) of a 32-column quarter starting at column c0 set to -inf.
__device__ __forceinline__ void mask_quarter(uint32_t* sr, int c0, int lim) {
#pragma unroll
    for (int e = 0; e < 32; ++e)
        if (c0 + e >= lim) sr[e] = __float_as_uint(-INFINITY);
}

// p = 2^(s * sl2 - mref) for the 128 columns of S, rounded to T and packed in
// pairs, quarter by quarter; each quarter's P goes over S columns
// [16q, 16q + 16), read already and below the quarter in flight.  Returns
// the row sum of p (two packed accumulator pairs), and in *mx the row max of
// the raw scores (four three-input max chains).  A row with no reference max
// yet (mref = -inf: its first block) takes the max of the block's first
// quarter, which the max chains hold once that quarter is in; the reference
// used comes back in *mused.
template <typename T>
__device__ __forceinline__ float p_pass(uint32_t sS, float sl2, float mref, bool edge, int lim,
                                        uint32_t* sr, float* mx, float* mused) {
    using P = Packed<T>;
    float ps0 = 0.f, ps1 = 0.f, ps2 = 0.f, ps3 = 0.f;
    float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
    uint32_t pk[16];
    tmem_ld32(sS, sr);
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t nx[32];
        if (q < 3) tmem_ld32(sS + 32 * (q + 1), nx);
        if (edge) mask_quarter(sr, 32 * q, lim);  // -inf * sl2 - mref = -inf: p = 0
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
            mx0 = max3(mx0, __uint_as_float(sr[e]), __uint_as_float(sr[e + 1]));
            mx1 = max3(mx1, __uint_as_float(sr[e + 2]), __uint_as_float(sr[e + 3]));
            mx2 = max3(mx2, __uint_as_float(sr[e + 4]), __uint_as_float(sr[e + 5]));
            mx3 = max3(mx3, __uint_as_float(sr[e + 6]), __uint_as_float(sr[e + 7]));
        }
        if (q == 0 && mref == -INFINITY) {  // (no valid key in the quarter: 0, every p 0)
            const float q0 = max3(mx0, mx1, fmaxf(mx2, mx3));
            mref = q0 == -INFINITY ? 0.f : q0 * sl2;
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            float x0, x1;
            fma2(x0, x1, __uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1]), sl2, -mref);
            const float p0 = ex2(x0), p1 = ex2(x1);
            if (e & 1)
                add2(ps2, ps3, p0, p1);
            else
                add2(ps0, ps1, p0, p1);
            pk[e] = P::pack(p0, p1);
        }
        tmem_st16(sS + 16 * q, pk);
        if (q < 3) {
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) sr[e] = nx[e];
        }
    }
    *mx = max3(mx0, mx1, fmaxf(mx2, mx3));
    *mused = mref;
    return (ps0 + ps1) + (ps2 + ps3);
}

// q_r . k_c in fp32 on the CUDA cores (head_dim 128).
template <typename T>
__device__ __forceinline__ float dot128(const T* q, const T* k) {
    float acc = 0.f;
#pragma unroll 4
    for (int d = 0; d < 128; d += 8) {
        const uint4 qa = *reinterpret_cast<const uint4*>(q + d);
        const uint4 ka = *reinterpret_cast<const uint4*>(k + d);
        const T* qe = reinterpret_cast<const T*>(&qa);
        const T* ke = reinterpret_cast<const T*>(&ka);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(Dt<T>::to_f(qe[i]), Dt<T>::to_f(ke[i]), acc);
    }
    return acc;
}

// The rare path of the one-pass softmax: a row whose block max exceeds its
// reference max by more than 2^kRedoLog2 had its p computed against a max far
// too low (large or infinite values), so the block's P is computed again for
// that row against the block's own max -- its scores recomputed on the CUDA
// cores from q and k in global memory, the tensor-core S being overwritten by
// P already -- and its O is rescaled before this block's P V.  Rows with
// `redo` false keep their P (read and written back: the tensor-memory copies
// are warp-wide).  Called by whole warps.
struct RowState {
    float m, l;
};

template <typename T>
__device__ __noinline__ RowState redo_rows(const T* qp, const char* kp0, int64_t k_bytes, int lim,
                                           bool redo, uint32_t sS, uint32_t sO, float sl2,
                                           RowState st) {
    using P = Packed<T>;
    // qp: this row's query; kp0: the block's first key row, k_bytes apart
    auto kp = [&](int c) { return reinterpret_cast<const T*>(kp0 + (int64_t)c * k_bytes); };
    const int n = min(lim, kRows);
    float mnew = -INFINITY;
    if (redo)
        for (int c = 0; c < n; ++c) mnew = fmaxf(mnew, dot128(qp, kp(c)));
    mnew *= sl2;
    const float corr = redo ? ex2(st.m - mnew) : 1.f;
    float ps = 0.f;
    for (int q = 0; q < 4; ++q) {
        uint32_t pk[16];
        tmem_ld16(sS + 16 * q, pk);
        tmem_wait_ld();
        if (redo) {
            for (int e = 0; e < 16; ++e) {
                const int c0 = 32 * q + 2 * e;
                const float p0 = c0 < n ? ex2(fmaf(dot128(qp, kp(c0)), sl2, -mnew)) : 0.f;
                const float p1 = c0 + 1 < n ? ex2(fmaf(dot128(qp, kp(c0 + 1)), sl2, -mnew)) : 0.f;
                ps += p0 + p1;
                pk[e] = P::pack(p0, p1);
            }
        }
        tmem_st16(sS + 16 * q, pk);
    }
    tmem_wait_st();
    scale_o(sO, corr);
    if (redo) st = RowState{mnew, st.l * corr + ps};
    return st;
}

// S_t = Q_t K_s^T (head_dim in steps of 16), then commit to `bar`.
__device__ __forceinline__ void issue_s(uint32_t tmem, uint32_t ubase, int t, int s, uint32_t id,
                                        uint64_t* bar) {
    const uint32_t q = ubase + (uint32_t)(t * kTile), k = ubase + (uint32_t)((2 + s) * kTile);
    const uint32_t d = tmem + (uint32_t)(t * kRows);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (uint32_t)((kk >> 2) * kSlab + (kk & 3) * 32);
        mma_ss(d, sdesc(q + off, 16, 1024), sdesc(k + off, 16, 1024), id, kk > 0 ? 1u : 0u);
    }
    mma_commit(bar);
}

struct TcBars {
    uint64_t q_full, q_empty;
    uint64_t k_full[2], v_full[2], k_empty[2], v_empty[2];
    uint64_t s_full[2], p_full[2], o_final[2];
    uint64_t item_full[2], item_empty[2];
    uint64_t drain;
};

// Readers of each published work item: the V producer, the MMA thread and the
// eight softmax warps (one arrival per warp).
constexpr int kItemReaders = 10;

// Two query tiles share each work item's K and V blocks.  When query heads
// come in pairs per KV head (an even group size Hq / Hkv), a tile pair is the
// same 128 query rows of two heads of one group: both tiles see the same keys,
// so they have the same number of key blocks and the same causal diagonal and
// alternate evenly to the end.  Otherwise a tile pair is 256 consecutive query
// rows of one head.
__device__ __forceinline__ bool head_pairs(const VarlenDev& a) {
    return ((a.Hq / a.Hkv) & 1) == 0;
}

// One work item: two 128-row query tiles of one sequence, tile t at query row
// r_t of head h_t.  nblk < 0: the item holds no query row.
struct Item {
    int h0, h1, r0, r1;  // tiles' query heads and first rows within the sequence
    int hk, q0, q_len, k0, k_len, nb0, nb1, nblk;
};

// Items are numbered heaviest first for causal attention: every (sequence,
// head or head pair) of the last tile row, then the row before it, ...
__device__ __forceinline__ Item decode_item(const VarlenDev& a, int it, int ny) {
    const bool pair = head_pairs(a);
    const int hx = pair ? a.Hq / 2 : a.Hq;  // head units per sequence
    const int nbh = a.batch * hx;
    const int y = it / nbh, x = it - y * nbh;
    const int b = x / hx, u = x - b * hx;
    const int m0 = (ny - 1 - y) * (pair ? kRows : 2 * kRows);
    Item w;
    w.h0 = pair ? 2 * u : u;
    w.h1 = pair ? 2 * u + 1 : u;
    w.r0 = m0;
    w.r1 = pair ? m0 : m0 + kRows;
    w.hk = w.h0 / (a.Hq / a.Hkv);
    w.q0 = __ldg(a.cu_q + b);
    w.q_len = __ldg(a.cu_q + b + 1) - w.q0;
    w.k0 = __ldg(a.cu_k + b);
    w.k_len = __ldg(a.cu_k + b + 1) - w.k0;
    w.nb0 = w.nb1 = 0;
    w.nblk = -1;
    if (w.r0 >= w.q_len) return w;
    int nbx[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {  // key blocks per tile (tile 1 may hold no rows)
        const int r0 = t ? w.r1 : w.r0;
        const int kend = r0 >= w.q_len ? 0 : a.causal ? min(w.k_len, r0 + kRows) : w.k_len;
        nbx[t] = (kend + kRows - 1) / kRows;
    }
    w.nb0 = nbx[0];
    w.nb1 = nbx[1];
    w.nblk = max(nbx[0], nbx[1]);
    return w;
}

// Persistent when `work` is given: gridDim.x CTAs (one per SM) claim items
// from the counter work[0] (heaviest first, so the last items to finish are
// short ones), and the last CTA to finish, counted in work[1], sets both
// words back to zero for the next call.  Without `work`, CTA i does item i.
//
// The TMA warp's lane 0 claims items and publishes each in a two-slot ring
// (item_slot / item_full / item_empty) for the other roles, then loads its Q
// tiles and K blocks; barrier phases run on across items (counters of items,
// key blocks and tile blocks, kept alike by every role).  While one item's
// last blocks and its epilogue run, the next item's Q, K and V are loaded and
// its first S is computed.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    varlen_attn_tc_kernel(const VarlenDev a, const __grid_constant__ CUtensorMap tq,
                          const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv,
                          const __grid_constant__ CUtensorMap to, int ny, int total,
                          int* work) {
    using P = Packed<T>;
    extern __shared__ __align__(1024) char dsm[];
    __shared__ TcBars bars;
    __shared__ uint32_t tmem_slot;
    __shared__ int item_slot[2];
    __shared__ int abort_flag;
    volatile int* abort = &abort_flag;
    volatile int* slots = item_slot;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // operand tiles at 1024-byte aligned offsets: Q_t at t, K_s at 2 + s, V_s at 4 + s
    const uint32_t raw = smem_u32(dsm);
    char* base = dsm + (((raw + 1023u) & ~1023u) - raw);
    const uint32_t ubase = smem_u32(base);

    if (tid == 0) {
        mbar_init(&bars.q_full, 1);
        mbar_init(&bars.q_empty, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bars.k_full[s], 1);
            mbar_init(&bars.v_full[s], 1);
            mbar_init(&bars.k_empty[s], 1);
            mbar_init(&bars.v_empty[s], 1);
            mbar_init(&bars.s_full[s], 1);
            mbar_init(&bars.p_full[s], kRows);
            mbar_init(&bars.o_final[s], 1);
            mbar_init(&bars.item_full[s], 1);
            mbar_init(&bars.item_empty[s], kItemReaders);
        }
        mbar_init(&bars.drain, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    // Launched with programmatic dependent launch: the set-up above (shared
    // memory, tensor memory, parameters only) overlaps the previous kernel's
    // tail; every global memory access -- the inputs, cu_seqlens, the work
    // counter -- comes after the previous grid has completed.
    pdl_wait();
    pdl_trigger();

    if (warp == kTmaWarp) {
        if (lane == 0) {
            // ---- scheduler + Q / K producer.  A K stage is refilled once the
            // S MMAs that read it are done, Q once the item's last S MMAs are.
            uint32_t n = 0, nq = 0, g = 0;  // items published, items loaded, K blocks
            int next = work ? atomicAdd(work, 1) : (int)blockIdx.x;
            while (true) {
                const int slot = (int)(n & 1);
                if (n >= 2 && !mbar_wait(&bars.item_empty[slot], ((n - 2) >> 1) & 1, abort)) break;
                int it = next;
                Item w;
                w.nblk = -1;
                while (it < total) {  // skip tile pairs past their sequence's end
                    w = decode_item(a, it, ny);
                    if (w.nblk >= 0) break;
                    it = work ? atomicAdd(work, 1) : total;
                }
                const bool done = it >= total;
                // claim the following item now: its index is back by the time
                // this one's blocks are queued
                if (!done) next = work ? atomicAdd(work, 1) : total;
                slots[slot] = done ? -1 : it;
                mbar_arrive(&bars.item_full[slot]);
                ++n;
                if (done) break;
                if (w.nblk == 0) continue;  // no keys: nothing to load
                // after a wait that gave up, no further copy is issued: the
                // stage may still be read by the tensor core
                if (nq > 0 && !mbar_wait(&bars.q_empty, (nq - 1) & 1, abort)) break;
                const int ntile = w.nb1 > 0 ? 2 : 1;
                mbar_expect_tx(&bars.q_full, (uint32_t)(ntile * kTile));
                for (int t = 0; t < ntile; ++t)
                    tma_tile(base + t * kTile, &tq, t ? w.h1 : w.h0, w.q0 + (t ? w.r1 : w.r0),
                             &bars.q_full);
                ++nq;
                bool ok = true;
                for (int j = 0; j < w.nblk; ++j, ++g) {
                    const int s = (int)(g & 1);
                    if (g >= 2 && !mbar_wait(&bars.k_empty[s], ((g - 2) >> 1) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&bars.k_full[s], (uint32_t)kTile);
                    tma_tile(base + (2 + s) * kTile, &tk, w.hk, w.k0 + j * kRows, &bars.k_full[s]);
                }
                if (!ok) break;
            }
            // every copy issued has landed before the CTA can leave
            if (nq > 0) mbar_wait(&bars.q_full, (nq - 1) & 1, nullptr);
            for (uint32_t d = g > 2 ? g - 2 : 0; d < g; ++d)
                mbar_wait(&bars.k_full[d & 1], (d >> 1) & 1, nullptr);
        } else if (lane == 1) {
            // ---- V producer: a V stage is refilled once its P V MMAs are done
            uint32_t n = 0, g = 0;
            while (true) {
                const int slot = (int)(n & 1);
                if (!mbar_wait(&bars.item_full[slot], (n >> 1) & 1, abort)) break;
                const int it = slots[slot];
                mbar_arrive(&bars.item_empty[slot]);
                ++n;
                if (it < 0) break;
                const Item w = decode_item(a, it, ny);
                bool ok = true;
                for (int j = 0; j < w.nblk; ++j, ++g) {
                    const int s = (int)(g & 1);
                    if (g >= 2 && !mbar_wait(&bars.v_empty[s], ((g - 2) >> 1) & 1, abort)) {
                        ok = false;  // gave up: issue no further copy
                        break;
                    }
                    mbar_expect_tx(&bars.v_full[s], (uint32_t)kTile);
                    tma_tile(base + (4 + s) * kTile, &tv, w.hk, w.k0 + j * kRows, &bars.v_full[s]);
                }
                if (!ok) break;
            }
            for (uint32_t d = g > 2 ? g - 2 : 0; d < g; ++d)
                mbar_wait(&bars.v_full[d & 1], (d >> 1) & 1, nullptr);
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issue, per item: S_0,0 S_1,0 | PV_0,j S_0,j+1 PV_1,j S_1,j+1 | ...
        if (lane == 0) {
            const uint32_t bf = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
            const uint32_t id_qk = idesc(bf, 0u), id_pv = idesc(bf, 1u);
            uint32_t n = 0, nq = 0, g = 0, tb0 = 0, tb1 = 0;
            while (true) {
                const int slot = (int)(n & 1);
                if (!mbar_wait(&bars.item_full[slot], (n >> 1) & 1, abort)) break;
                const int it = slots[slot];
                mbar_arrive(&bars.item_empty[slot]);
                ++n;
                if (it < 0) break;
                const Item w = decode_item(a, it, ny);
                const int nb0 = w.nb0, nb1 = w.nb1, nblk = w.nblk;
                if (nblk == 0) continue;
                mbar_wait(&bars.q_full, nq & 1, abort);
                mbar_wait(&bars.k_full[g & 1], (g >> 1) & 1, abort);
                tc_fence_after();
                issue_s(tmem, ubase, 0, (int)(g & 1), id_qk, &bars.s_full[0]);
                if (nb1 > 0) issue_s(tmem, ubase, 1, (int)(g & 1), id_qk, &bars.s_full[1]);
                mma_commit(&bars.k_empty[g & 1]);  // K of block 0 is free once these are done
                if (nblk == 1) mma_commit(&bars.q_empty);
                for (int j = 0; j < nblk; ++j) {
                    const uint32_t gj = g + (uint32_t)j;
                    const int s = (int)(gj & 1);
                    mbar_wait(&bars.v_full[s], (gj >> 1) & 1, abort);
                    if (j + 1 < nblk) mbar_wait(&bars.k_full[s ^ 1], ((gj + 1) >> 1) & 1, abort);
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const int nbt = t ? nb1 : nb0;
                        if (j >= nbt) continue;
                        mbar_wait(&bars.p_full[t], ((t ? tb1 : tb0) + (uint32_t)j) & 1, abort);
                        tc_fence_after();
                        const uint32_t o = tmem + 256u + (uint32_t)(t * kRows);
                        const uint32_t p = tmem + (uint32_t)(t * kRows);
                        const uint32_t v = ubase + (uint32_t)((4 + s) * kTile);
#pragma unroll
                        for (int k = 0; k < 8; ++k)  // keys in steps of 16
                            mma_ts(o, p + 8u * k, sdesc(v + k * 2048, kSlab, 1024), id_pv,
                                   (j > 0 || k > 0) ? 1u : 0u);
                        if (j + 1 < nbt)
                            issue_s(tmem, ubase, t, s ^ 1, id_qk, &bars.s_full[t]);
                        else  // O_t is final once this tile's MMAs so far are done
                            mma_commit(&bars.o_final[t]);
                    }
                    mma_commit(&bars.v_empty[s]);                        // V_j read
                    if (j + 1 < nblk) mma_commit(&bars.k_empty[s ^ 1]);  // K_j+1 read
                    if (j + 2 == nblk) mma_commit(&bars.q_empty);        // the last S issued
                }
                g += (uint32_t)nblk;
                tb0 += (uint32_t)nb0;
                tb1 += (uint32_t)nb1;
                ++nq;
            }
            // every MMA issued has completed before the CTA can leave
            mma_commit(&bars.drain);
            mbar_wait(&bars.drain, 0u, nullptr);
        }
    } else {
        // ---- softmax of tile t, one query row per thread
        const int t = warp >> 2;
        const int r = tid & (kRows - 1);
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t sS = tmem + lane_base + (uint32_t)(t * kRows);
        const uint32_t sO = tmem + lane_base + 256u + (uint32_t)(t * kRows);
        const float sl2 = a.scale * 1.4426950408889634f;  // scores in log2 units
        constexpr int64_t ES = sizeof(T);
        // items read, blocks of tile 0 and of tile 1 so far, items with keys
        uint32_t n = 0, tb0 = 0, tb1 = 0, nit = 0;
        uint32_t sr[64];  // 32 used in the loop, 64 in the epilogue
        while (true) {
            const int slot = (int)(n & 1);
            const bool got = mbar_wait(&bars.item_full[slot], (n >> 1) & 1, abort);
            if (!__all_sync(0xffffffffu, got)) break;
            const int it = slots[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.item_empty[slot]);
            ++n;
            if (it < 0) break;
            const Item w = decode_item(a, it, ny);
            const int nbt = t ? w.nb1 : w.nb0;
            const int trow = t ? w.r1 : w.r0;  // this tile's first query row and head
            const int thead = t ? w.h1 : w.h0;
            const int qi = trow + r;  // query row within the sequence
            const uint32_t base0 = tb0, base1 = tb1;  // blocks of each tile before this item
            tb0 += (uint32_t)w.nb0;
            tb1 += (uint32_t)w.nb1;
            if (nbt == 0) {
                if (qi < w.q_len) {  // no keys: 0 / 0, as the reference's acc / l
                    T* out = reinterpret_cast<T*>(
                        a.out + ((int64_t)(w.q0 + qi) * a.ot + (int64_t)thead * a.oh) * ES);
                    for (int d = 0; d < 128; ++d) out[d] = Dt<T>::from_f(__int_as_float(0x7fc00000));
                }
                continue;
            }
            const int klim = a.causal ? min(w.k_len, qi + 1) : w.k_len;  // keys [0, klim) count
            // running reference max m (log2 units), sum l, and a rescale of O
            // that the block before left for this one
            float m = -INFINITY, l = 0.f, pend = 1.f;
            const uint32_t tbs = t ? base1 : base0;
            for (int j = 0; j < nbt; ++j) {
                mbar_wait(&bars.s_full[t], (tbs + (uint32_t)j) & 1, abort);
                tc_fence_after();
                const int kb = j * kRows;
                // masking only on the blocks that reach past the sequence or the diagonal
                const bool edge =
                    kb + kRows > w.k_len || (a.causal && kb + kRows - 1 > trow);
                const int lim = klim - kb;  // columns [lim, 128) are masked
                // the block before's P V is done (S_j was issued after it)
                if (__any_sync(0xffffffffu, pend != 1.f)) scale_o(sO, pend);
                pend = 1.f;
                // One pass per block (sl2 > 0: the launcher sends other scales to
                // the mma.sync kernel): P against the row's reference max m, the
                // block max on the side; a row's first block takes the max of its
                // first quarter as m.  m moves when the row max has grown by more
                // than 2^8 (O / l is the same either way): l at once, O at the next
                // block's start (or in 1 / l after the last), when this block's
                // P V is done.  Growth beyond 2^kRedoLog2 (p possibly infinite)
                // redoes the row.
                float mx, mu;
                const float ps = p_pass<T>(sS, sl2, m, edge, lim, sr, &mx, &mu);
                mx *= sl2;
                if (m == -INFINITY && mx > -INFINITY) m = mu;  // the first reference
                // (rows past the sequence, whose O is never stored, are left as they are)
                const bool redo = m > -INFINITY && qi < w.q_len && mx > m + kRedoLog2;
                if (__any_sync(0xffffffffu, redo)) {
                    const RowState st = redo_rows<T>(
                        reinterpret_cast<const T*>(
                            a.q + ((int64_t)(w.q0 + qi) * a.qt + (int64_t)thead * a.qh) * ES),
                        a.k + ((int64_t)(w.k0 + kb) * a.kt + (int64_t)w.hk * a.kh) * ES,
                        a.kt * ES, lim, redo, sS, sO, sl2, RowState{m, l});
                    m = st.m;
                    l = st.l;
                }
                if (!redo) {
                    if (mx > m + 8.f) {
                        const float corr = ex2(m - mx);
                        l = (l + ps) * corr;
                        pend = corr;
                        m = mx;
                    } else {
                        l += ps;
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bars.p_full[t]);
            }
            mbar_wait(&bars.o_final[t], nit & 1, abort);
            ++nit;
            tc_fence_after();
            // O / l, 64 columns at a time: each thread packs its row into the
            // warp's staging buffer (16-byte chunk c of row r at chunk c ^ r % 8:
            // no bank conflicts, and the 128-byte swizzle a TMA box reads).  A
            // warp whose 32 rows all lie in the sequence hands the box to a TMA
            // store (lane 0) and goes on; at the sequence's end the warp writes
            // its rows itself, 4 whole 128-byte row segments per instruction.
            const float inv = pend / l;  // a rescale the last block left
            char* stage = base + 6 * kTile + warp * kStage;
            const int row0 = trow + (warp & 3) * 32;  // the warp's first row
            const bool write = !*abort;
            const bool whole = write && row0 + 32 <= w.q_len;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                tmem_ld32(sO + 64 * h, sr);
                tmem_ld32(sO + 64 * h + 32, sr + 32);
                if (lane == 0) tma_store_wait_read();  // the buffer's last store has read it
                __syncwarp();
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint4 v;
                    v.x = P::pack(__uint_as_float(sr[8 * c]) * inv, __uint_as_float(sr[8 * c + 1]) * inv);
                    v.y = P::pack(__uint_as_float(sr[8 * c + 2]) * inv, __uint_as_float(sr[8 * c + 3]) * inv);
                    v.z = P::pack(__uint_as_float(sr[8 * c + 4]) * inv, __uint_as_float(sr[8 * c + 5]) * inv);
                    v.w = P::pack(__uint_as_float(sr[8 * c + 6]) * inv, __uint_as_float(sr[8 * c + 7]) * inv);
                    *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) * 16)) = v;
                }
                if (whole) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) tma_store(&to, 64 * h, thead, w.q0 + row0, stage);
                } else {
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rr = 4 * i + (lane >> 3), c = lane & 7;
                        const uint4 v =
                            *reinterpret_cast<const uint4*>(stage + rr * 128 + ((c ^ (rr & 7)) * 16));
                        if (write && row0 + rr < w.q_len) {
                            T* dst = reinterpret_cast<T*>(
                                a.out + ((int64_t)(w.q0 + row0 + rr) * a.ot + (int64_t)thead * a.oh) * ES);
                            *reinterpret_cast<uint4*>(dst + 64 * h + 8 * c) = v;
                        }
                    }
                }
                __syncwarp();
            }
            // the next item's first P V overwrites O: these loads are ordered
            // before it by the fence ahead of that item's first p_full arrival
        }
    }

    if (warp < 8 && lane == 0) tma_store_wait_all();  // output stores complete
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        if (abort_flag) flag(a.status, QF_FLAG_TIMEOUT);
        if (work) {
            __threadfence();
            if (atomicAdd(work + 1, 1) == (int)gridDim.x - 1) {  // the last CTA out
                atomicExch(work, 0);
                atomicExch(work + 1, 0);
            }
        }
    }
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// cuTensorMapEncodeTiled, looked up once through the runtime.
PFN_cuTensorMapEncodeTiled encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
    });
    return fn;
}

// A 3-D map over (head_dim = 128, heads, tokens) with 64 x 1 x 128 boxes.
bool make_map(CUtensorMap* map, const char* ptr, int bf16, int64_t heads, int64_t tokens,
              int64_t head_stride, int64_t token_stride, int rows = kRows) {
    PFN_cuTensorMapEncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)tokens};
    const cuuint64_t strides[2] = {(cuuint64_t)head_stride * 2, (cuuint64_t)token_stride * 2};
    const cuuint32_t box[3] = {64, 1, (cuuint32_t)rows};
    const cuuint32_t estride[3] = {1, 1, 1};
    return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
              const_cast<char*>(ptr), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
int launch_tc(const VarlenDev& a, int max_q, cudaStream_t stream) {
    constexpr auto kernel = varlen_attn_tc_kernel<T>;
    static std::atomic<bool> configured{false};
    if (!configured.load(std::memory_order_relaxed)) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        if (e != cudaSuccess) return launch_failed(e);
        configured.store(true, std::memory_order_relaxed);
    }
    const int bf = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
    CUtensorMap tq, tk, tv, to;
    if (!make_map(&tq, a.q, bf, a.Hq, a.total_q, a.qh, a.qt) ||
        !make_map(&tk, a.k, bf, a.Hkv, a.total_k, a.kh, a.kt) ||
        !make_map(&tv, a.v, bf, a.Hkv, a.total_k, a.vh, a.vt) ||
        !make_map(&to, a.out, bf, a.Hq, a.total_q, a.oh, a.ot, 32))
        return QF_ERR_UNSUPPORTED;
    // items: (batch x query heads, or head pairs) x tile rows (128 queries for
    // head pairs, else 256); every CTA claims one past the last, so the
    // counter reaches total + grid
    const bool pair = a.Hkv > 0 && ((a.Hq / a.Hkv) & 1) == 0;  // as head_pairs()
    const int64_t ny = ceil_div(max_q, pair ? kRows : 2 * kRows);
    const int64_t total = (int64_t)a.batch * (pair ? a.Hq / 2 : a.Hq) * ny;
    const int64_t sms = sm_count();
    if (total + sms >= ((int64_t)1 << 31)) return QF_ERR_UNSUPPORTED;
    if (total == 0) return QF_OK;
    const int64_t grid = a.work_counter ? std::min<int64_t>(total, sms) : total;
    return launch_pdl(kernel, (unsigned)grid, (unsigned)kThreads, (size_t)kSmem, stream, a, tq, tk,
                      tv, to, (int)ny, (int)total, a.work_counter);
}

}  // namespace

int launch_varlen_tc(const VarlenDev& a, int bf16, int max_q, cudaStream_t stream) {
    if (a.total_q <= 0 || a.total_k <= 0 || a.total_q >= (1ll << 31) || a.total_k >= (1ll << 31))
        return QF_ERR_UNSUPPORTED;
    if (!(a.scale > 0.f) || isinf(a.scale)) return QF_ERR_UNSUPPORTED;  // max(s) * scale is the max
    if (reinterpret_cast<uintptr_t>(a.work_counter) % alignof(int32_t)) return QF_ERR_INVALID;
    return bf16 ? launch_tc<__nv_bfloat16>(a, max_q, stream) : launch_tc<__half>(a, max_q, stream);
}

}  // namespace qf
