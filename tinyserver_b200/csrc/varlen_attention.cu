// Prefill attention over variable-length packed sequences.
//
// Replaces flash_attn_varlen_func (server/model/kernels/varlen_attention.py:
// 145-218; Triton kernel :8-142): tokens of all sequences packed along the
// first axis, sequence b owning query rows [cu_q[b], cu_q[b+1]) and key rows
// [cu_k[b], cu_k[b+1]); query head h reads kv head h / (Hq / Hkv);
//   out[t, h] = softmax(q[t, h] . K_b^T * scale (+ causal mask)) @ V_b
// with the causal mask keeping key j for query i when i >= j (indices within
// the sequence, varlen_attention.py:111-114), fp32 math, and -- as the
// reference does (p_ij.to(v.dtype), :121) -- the probabilities rounded to the
// value dtype before they meet V.
//
// 16-bit path (tensor cores): one CTA per (64-query block, sequence, query
// head), 4 warps of 16 query rows.  The CTA streams 64-key K/V tiles through a
// shared-memory double buffer filled by cp.async (XOR-swizzled rows,
// conflict-free ldmatrix); S = Q K^T and O += P V run on mma.sync m16n8k16
// with fp32 accumulate, the online softmax on the accumulator fragments; the
// key loop stops at the causal limit of the query block.
// fp32 path (the reference's "ieee" dot products): CUDA cores, one warp per
// query row.
#include "qf_common.cuh"
#include "qf_mma.cuh"
#include "qf_varlen.cuh"

namespace qf {
namespace {

template <int D>
struct VarTile {
    static constexpr int BM = 64, BN = 64;
    static constexpr int ROW = D * 2;          // bytes per row (16-bit)
    static constexpr int NCH = ROW / 16;       // 16-byte chunks per row
    static constexpr int QS = BM * ROW;        // Q tile
    static constexpr int MAT = BN * ROW;       // one K or V tile
    static constexpr int STAGE = 2 * MAT;
    // the Q tile lives in stage 1 until its fragments are in registers (stage
    // 1 is first refilled after that)
    static constexpr int SMEM = 2 * STAGE;
    static_assert(QS <= STAGE, "Q tile must fit in one stage");
    __device__ __forceinline__ static int off(int r, int c) {
        return r * ROW + ((c ^ (r & 7)) << 4);
    }
};

template <typename T, int D>
__global__ void __launch_bounds__(128, 3) varlen_attn_mma_kernel(const VarlenDev a) {
    using VT = VarTile<D>;
    using P = Packed<T>;
    constexpr int BM = VT::BM, BN = VT::BN, NCH = VT::NCH, KS = D / 16, NT = D / 8;
    const int qb = blockIdx.x, b = blockIdx.y, hq = blockIdx.z;
    const int hk = hq / (a.Hq / a.Hkv);
    const int q0 = __ldg(a.cu_q + b), q_len = __ldg(a.cu_q + b + 1) - q0;
    const int k0 = __ldg(a.cu_k + b), k_len = __ldg(a.cu_k + b + 1) - k0;
    if (qb * BM >= q_len) return;

    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* stages = smem;
    unsigned char* qs = smem + VT::STAGE;  // stage 1
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gid = lane >> 2, tig = lane & 3;

    // Q tile (rows past the sequence read as zeros)
    for (int i = tid; i < BM * NCH; i += 128) {
        const int r = i / NCH, c = i - r * NCH;
        const int qi = qb * BM + r;
        const bool ok = qi < q_len;
        const char* src = a.q + ((int64_t)(q0 + (ok ? qi : 0)) * a.qt + (int64_t)hq * a.qh) * 2;
        cp_async16(qs + VT::off(r, c), src + c * 16, ok ? 16 : 0);
    }
    cp_async_commit();

    const int kv_end = a.causal ? min(k_len, qb * BM + BM) : k_len;
    const int nkb = (kv_end + BN - 1) / BN;
    auto issue = [&](int kb, int st) {
        unsigned char* kt = stages + st * VT::STAGE;
        unsigned char* vt = kt + VT::MAT;
        for (int i = tid; i < BN * NCH; i += 128) {
            const int r = i / NCH, c = i - r * NCH;
            const int kj = kb * BN + r;
            const bool ok = kj < k_len;
            const int64_t tok = k0 + (ok ? kj : 0);
            cp_async16(kt + VT::off(r, c), a.k + (tok * a.kt + (int64_t)hk * a.kh) * 2 + c * 16,
                       ok ? 16 : 0);
            cp_async16(vt + VT::off(r, c), a.v + (tok * a.vt + (int64_t)hk * a.vh) * 2 + c * 16,
                       ok ? 16 : 0);
        }
    };
    if (nkb > 0) issue(0, 0);
    cp_async_commit();

    cp_async_wait<1>();  // the Q tile has landed
    __syncthreads();
    uint32_t qa[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        const int r = warp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        ldsm_x4(qa[ks], qs + VT::off(r, 2 * ks + (lane >> 4)));
    }
    __syncthreads();  // every warp holds its Q fragments: stage 1 may be refilled

    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int qi0 = qb * BM + warp * 16 + gid, qi1 = qi0 + 8;  // this thread's two query rows

    for (int kb = 0; kb < nkb; ++kb) {
        if (kb + 1 < nkb) issue(kb + 1, (kb + 1) & 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const unsigned char* kt = stages + (kb & 1) * VT::STAGE;
        const unsigned char* vt = kt + VT::MAT;

        // S = Q K^T: k-steps outer, the 8 key n-tiles inner, so consecutive
        // mma.sync instructions write different accumulators
        float sc[BN / 8][4];
#pragma unroll
        for (int n = 0; n < BN / 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS / 2; ++kk) {
            uint32_t bf[BN / 8][4];
#pragma unroll
            for (int n = 0; n < BN / 8; ++n)
                ldsm_x4(bf[n], kt + VT::off(n * 8 + (lane & 7), kk * 4 + (lane >> 3)));
#pragma unroll
            for (int n = 0; n < BN / 8; ++n) Mma<T>::run(sc[n], qa[2 * kk], bf[n][0], bf[n][1]);
#pragma unroll
            for (int n = 0; n < BN / 8; ++n)
                Mma<T>::run(sc[n], qa[2 * kk + 1], bf[n][2], bf[n][3]);
        }
        // Online softmax and P V in 32-key halves: the reference updates its
        // running max every BLOCK_N = 32 keys (varlen_attention.py:190) and
        // rounds P against it, so the rounding points line up.
        // Scores are kept in log2 units (scale * log2(e) folded into one
        // multiply) so that exp2 gives the exponentials.  Every row has a
        // valid key in the first 32 keys (key 0), so the running max is finite
        // from the first half on and the exponentials need no -inf guard.
        // Masks only where this warp's rows can see a masked key: the block's
        // tail past the sequence, or keys beyond the warp's first row (causal).
        const float sl2 = a.scale * 1.4426950408889634f;
        const bool full = (kb + 1) * BN <= k_len &&
                          (!a.causal || (kb + 1) * BN <= qb * BM + warp * 16 + 1);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int n = 4 * hf; n < 4 * hf + 4; ++n) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float s0 = sc[n][e] * sl2, s1 = sc[n][2 + e] * sl2;
                    if (!full) {
                        const int kj = kb * BN + n * 8 + 2 * tig + e;
                        s0 = kj < k_len && (!a.causal || qi0 >= kj) ? s0 : -INFINITY;
                        s1 = kj < k_len && (!a.causal || qi1 >= kj) ? s1 : -INFINITY;
                    }
                    sc[n][e] = s0;
                    sc[n][2 + e] = s1;
                    mx0 = fmaxf(mx0, s0);
                    mx1 = fmaxf(mx1, s1);
                }
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            const float cr0 = exp2f(m0 - mn0), cr1 = exp2f(m1 - mn1);  // 0 on the first half
            float sum0 = 0.f, sum1 = 0.f;
            uint32_t pa[2][4];  // P rounded to T: A-fragments of this half's two k-steps
#pragma unroll
            for (int n = 4 * hf; n < 4 * hf + 4; ++n) {
                const float p0 = exp2f(sc[n][0] - mn0), p1 = exp2f(sc[n][1] - mn0);
                const float p2 = exp2f(sc[n][2] - mn1), p3 = exp2f(sc[n][3] - mn1);
                sum0 += p0 + p1;
                sum1 += p2 + p3;
                pa[(n / 2) & 1][(n & 1) * 2 + 0] = P::pack(p0, p1);
                pa[(n / 2) & 1][(n & 1) * 2 + 1] = P::pack(p2, p3);
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
#pragma unroll
            for (int kh = 0; kh < 2; ++kh) {
                const int ks2 = 2 * hf + kh;  // 16-key k-step within the tile
#pragma unroll
                for (int np = 0; np < NT / 2; ++np) {
                    uint32_t bf[4];
                    ldsm_x4_t(bf, vt + VT::off(ks2 * 16 + ((lane >> 3) & 1) * 8 + (lane & 7),
                                               2 * np + (lane >> 4)));
                    Mma<T>::run(o[2 * np], pa[kh], bf[0], bf[1]);
                    Mma<T>::run(o[2 * np + 1], pa[kh], bf[2], bf[3]);
                }
            }
        }
        __syncthreads();  // every warp is done with this stage before it is refilled
    }
    cp_async_wait<0>();

    const float inv0 = 1.f / l0, inv1 = 1.f / l1;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const int d = n * 8 + 2 * tig;
        if (qi0 < q_len) {
            T* dst = reinterpret_cast<T*>(a.out) + (int64_t)(q0 + qi0) * a.ot + (int64_t)hq * a.oh + d;
            *reinterpret_cast<uint32_t*>(dst) = P::pack(o[n][0] * inv0, o[n][1] * inv0);
        }
        if (qi1 < q_len) {
            T* dst = reinterpret_cast<T*>(a.out) + (int64_t)(q0 + qi1) * a.ot + (int64_t)hq * a.oh + d;
            *reinterpret_cast<uint32_t*>(dst) = P::pack(o[n][2] * inv1, o[n][3] * inv1);
        }
    }
}

// fp32: one warp per query row, lanes over keys for QK and over head_dim for PV.
template <int D>
__global__ void __launch_bounds__(128) varlen_attn_f32_kernel(const VarlenDev a, int max_q) {
    constexpr int PER = D / 32;
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), b = blockIdx.y, hq = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hk = hq / (a.Hq / a.Hkv);
    const int q0 = __ldg(a.cu_q + b), q_len = __ldg(a.cu_q + b + 1) - q0;
    const int k0 = __ldg(a.cu_k + b), k_len = __ldg(a.cu_k + b + 1) - k0;
    __shared__ float qsh[4][D];
    __shared__ float psh[4][32];
    if (row >= q_len) return;  // whole warps leave; no block-wide barrier follows
    const float* qr = reinterpret_cast<const float*>(a.q) + (int64_t)(q0 + row) * a.qt + (int64_t)hq * a.qh;
    for (int d = lane; d < D; d += 32) qsh[warp][d] = qr[d];
    __syncwarp();
    const int kv_end = a.causal ? min(k_len, row + 1) : k_len;
    float m = -INFINITY, l = 0.f, acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.f;
    for (int j0 = 0; j0 < kv_end; j0 += 32) {
        const int j = j0 + lane;
        float s = -INFINITY;
        if (j < kv_end) {
            const float* kr = reinterpret_cast<const float*>(a.k) + (int64_t)(k0 + j) * a.kt + (int64_t)hk * a.kh;
            float dot = 0.f;
            for (int d = 0; d < D; d += 4) {
                const float4 kv = __ldg(reinterpret_cast<const float4*>(kr + d));
                dot = fmaf(qsh[warp][d], kv.x, dot);
                dot = fmaf(qsh[warp][d + 1], kv.y, dot);
                dot = fmaf(qsh[warp][d + 2], kv.z, dot);
                dot = fmaf(qsh[warp][d + 3], kv.w, dot);
            }
            s = dot * a.scale;
        }
        const float mn = fmaxf(m, warp_max(s));
        const float p = j < kv_end ? exp_rel(s, mn) : 0.f;
        const float cr = exp_rel(m, mn);
        l = l * cr + warp_sum(p);
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] *= cr;
        m = mn;
        psh[warp][lane] = p;
        __syncwarp();
        const int nk = min(32, kv_end - j0);
        for (int jj = 0; jj < nk; ++jj) {
            const float* vr = reinterpret_cast<const float*>(a.v) + (int64_t)(k0 + j0 + jj) * a.vt + (int64_t)hk * a.vh;
            const float pj = psh[warp][jj];
#pragma unroll
            for (int e = 0; e < PER; ++e) acc[e] = fmaf(pj, vr[lane * PER + e], acc[e]);
        }
        __syncwarp();
    }
    float* o = reinterpret_cast<float*>(a.out) + (int64_t)(q0 + row) * a.ot + (int64_t)hq * a.oh;
#pragma unroll
    for (int e = 0; e < PER; ++e) o[lane * PER + e] = acc[e] / l;
}

template <typename T, int D>
int launch_varlen(const VarlenDev& a, int max_q, cudaStream_t stream) {
    if constexpr (sizeof(T) == 4) {
        const dim3 grid((unsigned)ceil_div(max_q, 4), (unsigned)a.batch, (unsigned)a.Hq);
        varlen_attn_f32_kernel<D><<<grid, 128, 0, stream>>>(a, max_q);
        return check_launch();
    } else {
        using VT = VarTile<D>;
        constexpr auto kernel = varlen_attn_mma_kernel<T, D>;
        static std::atomic<bool> configured{false};
        if (!configured.load(std::memory_order_relaxed)) {
            const cudaError_t e = cudaFuncSetAttribute(
                kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, VT::SMEM);
            if (e != cudaSuccess) return launch_failed(e);
            configured.store(true, std::memory_order_relaxed);
        }
        const dim3 grid((unsigned)ceil_div(max_q, VT::BM), (unsigned)a.batch, (unsigned)a.Hq);
        kernel<<<grid, 128, VT::SMEM, stream>>>(a);
        return check_launch();
    }
}

#ifndef QF_VARLEN_TC
#define QF_VARLEN_TC 1  // head_dim 128, 16-bit: the tcgen05 kernel
#endif

template <typename T>
int dispatch_varlen(const VarlenDev& a, int64_t D, int max_q, cudaStream_t stream) {
    if constexpr (sizeof(T) == 2) {
        if (QF_VARLEN_TC && D == 128) {
            const int rc = launch_varlen_tc(a, std::is_same<T, __nv_bfloat16>::value ? 1 : 0,
                                            max_q, stream);
            if (rc != QF_ERR_UNSUPPORTED) return rc;  // else: the mma.sync kernel below
        }
    }
    switch (D) {
    case 64: return launch_varlen<T, 64>(a, max_q, stream);
    case 128: return launch_varlen<T, 128>(a, max_q, stream);
    default: return QF_ERR_UNSUPPORTED;
    }
}

}  // namespace
}  // namespace qf

extern "C" int qf_varlen_attention(const qf_varlen_attention_args* p, cudaStream_t stream) {
    if (!p) return QF_ERR_INVALID;
    const qf_varlen_attention_args& g = *p;
    if (g.batch < 0 || g.num_q_heads <= 0 || g.num_kv_heads <= 0 || g.max_seqlen_q < 0)
        return QF_ERR_INVALID;
    if (g.batch == 0 || g.max_seqlen_q == 0) return QF_OK;
    if (!g.q || !g.k || !g.v || !g.out || !g.cu_seqlens_q || !g.cu_seqlens_k)
        return QF_ERR_INVALID;
    if (g.num_q_heads % g.num_kv_heads) return QF_ERR_INVALID;
    if (g.batch > 65535 || g.num_q_heads > 65535) return QF_ERR_UNSUPPORTED;
    if (g.dtype != QF_F32 && g.dtype != QF_F16 && g.dtype != QF_BF16) return QF_ERR_INVALID;
    const int64_t es = g.dtype == QF_F32 ? 4 : 2;
    const int64_t strides[] = {g.q_stride_token, g.q_stride_head, g.k_stride_token,
                               g.k_stride_head,  g.v_stride_token, g.v_stride_head,
                               g.out_stride_token, g.out_stride_head};
    for (int64_t s : strides)
        if ((s * es) % 16) return QF_ERR_UNSUPPORTED;
    const void* ptrs[] = {g.q, g.k, g.v, g.out};
    for (const void* ptr : ptrs)
        if (!qf::aligned16(ptr)) return QF_ERR_UNSUPPORTED;
    qf::VarlenDev a{};
    a.q = static_cast<const char*>(g.q);
    a.k = static_cast<const char*>(g.k);
    a.v = static_cast<const char*>(g.v);
    a.out = static_cast<char*>(g.out);
    a.qt = g.q_stride_token;
    a.qh = g.q_stride_head;
    a.kt = g.k_stride_token;
    a.kh = g.k_stride_head;
    a.vt = g.v_stride_token;
    a.vh = g.v_stride_head;
    a.ot = g.out_stride_token;
    a.oh = g.out_stride_head;
    a.cu_q = g.cu_seqlens_q;
    a.cu_k = g.cu_seqlens_k;
    a.batch = (int)g.batch;
    a.Hq = (int)g.num_q_heads;
    a.Hkv = (int)g.num_kv_heads;
    a.causal = g.causal ? 1 : 0;
    a.scale = g.scale;
    a.status = g.status;
    a.total_q = g.total_q;
    a.total_k = g.total_k;
    a.work_counter = g.work_counter;
    const int max_q = (int)std::min<int64_t>(g.max_seqlen_q, 1 << 30);
    switch (g.dtype) {
    case QF_F32: return qf::dispatch_varlen<float>(a, g.head_dim, max_q, stream);
    case QF_F16: return qf::dispatch_varlen<__half>(a, g.head_dim, max_q, stream);
    default: return qf::dispatch_varlen<__nv_bfloat16>(a, g.head_dim, max_q, stream);
    }
}
