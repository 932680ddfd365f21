"""ctypes front end of the C oracle (``qwen3_oracle.c``).

TEST INFRASTRUCTURE ONLY: the parity checker for tinyserver_b200's CUDA path.
Only ``tests/``, ``__graft_entry__.smoke()``, ``bench.py``'s CPU-baseline leg
and ``bench.py``'s validation of sampled outputs (the checker's role, outside
every timed region) may import this module.  The product never does.

Every function takes and returns CPU torch tensors and mirrors one op of the
reference path (citations are in the C source):

* :func:`embedding`       -- ``nn.Embedding`` gather (HF:363, HF:392)
* :func:`rmsnorm`         -- ``Qwen3RMSNorm.forward`` (HF:59-64)
* :func:`add_rmsnorm`     -- residual add (HF:327/333) + ``Qwen3RMSNorm``
* :func:`rope_cos_sin`    -- ``Qwen3RotaryEmbedding.forward`` (HF:137-148)
* :func:`qk_norm_rope_store` -- q_norm/k_norm + ``apply_rotary_pos_emb`` + paged
  store, as ``server/model/patches/qwen3.py:264-318`` runs them
* :func:`kv_store_batched` / :func:`kv_store_seq` -- ``server/model/kernels/
  kv_cache.py`` ``store_kv_cache_batched`` / ``store_kv_cache``
* :func:`silu_and_mul`    -- ``Qwen3MLP`` activation product (HF:81-83)
* :func:`paged_attention_decode` -- the reference's decode paged attention
  (server/model/kernels/paged_attention.py:8-192), in torch fp32 on the CPU
* :func:`varlen_attention` -- the reference's prefill varlen attention
  (server/model/kernels/varlen_attention.py:8-218), same blocking and
  rounding points, in torch on the CPU
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "lib", "liboracle_qwen3.so")
_lib = None

DTYPE_TAG = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p
c_int = ctypes.c_int
c_float = ctypes.c_float
I64x = ctypes.POINTER(ctypes.c_int64)


def build() -> str:
    """Compile the oracle with the committed Makefile; return the library path."""
    src = os.path.join(_HERE, "qwen3_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        sig = {
            "oracle_embedding": [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_int, c_vp, c_i64],
            "oracle_rmsnorm": [c_vp, c_i64, c_vp, c_i64, c_i64, c_float, c_int, c_vp, c_i64],
            "oracle_add_rmsnorm": [c_vp, c_vp, c_vp, c_i64, c_i64, c_float, c_int, c_vp, c_vp],
            "oracle_rope_cos_sin": [c_vp, c_i64, c_vp, c_i64, c_float, c_int, c_vp, c_vp],
            "oracle_qk_norm_rope_store": [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64,
                                          c_i64, c_vp, c_vp, c_float, c_vp, c_vp, c_i64, c_i64,
                                          c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp, c_vp,
                                          I64x, c_i64, c_i64, c_vp, c_vp, c_int],
            "oracle_kv_store_batched": [c_vp, I64x, c_vp, I64x, c_vp, c_vp, I64x, c_vp, c_vp,
                                        c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_int],
            "oracle_kv_store_seq": [c_i64, c_vp, c_i64, c_int, c_vp, I64x, c_vp, I64x, c_vp,
                                    c_vp, I64x, c_i64, c_i64, c_i64, c_i64, c_i64, c_int],
            "oracle_silu_and_mul": [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_int, c_vp, c_i64],
            "oracle_num_threads": [],
        }
        for name, argtypes in sig.items():
            fn = getattr(_lib, name)
            fn.argtypes = argtypes
            fn.restype = c_int
    return _lib


def num_threads() -> int:
    return lib().oracle_num_threads()


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _arr(vals) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def _cpu(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cpu":
        raise ValueError("oracle takes CPU tensors")
    return t


def _check(rc: int, what: str) -> None:
    if rc == 2:
        raise IndexError(f"oracle {what}: index out of range")
    if rc != 0:
        raise ValueError(f"oracle {what}: bad argument (rc={rc})")


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    ids = _cpu(ids).reshape(-1).to(torch.int64).contiguous()
    table = _cpu(table)
    assert table.stride(1) == 1
    V, H = table.shape
    out = torch.empty(ids.numel(), H, dtype=table.dtype)
    _check(lib().oracle_embedding(_p(ids), ids.numel(), _p(table), V, H, table.stride(0),
                                  DTYPE_TAG[table.dtype], _p(out), H), "embedding")
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = _cpu(x).contiguous()
    H = x.shape[-1]
    x2 = x.reshape(-1, H)
    w = w.to(x.dtype).contiguous()
    out = torch.empty_like(x2)
    _check(lib().oracle_rmsnorm(_p(x2), H, _p(w), x2.shape[0], H, eps, DTYPE_TAG[x.dtype],
                                _p(out), H), "rmsnorm")
    return out.reshape(x.shape)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Return (normed, new_residual) where new_residual = residual + x."""
    x = _cpu(x).contiguous()
    residual = _cpu(residual).contiguous()
    H = x.shape[-1]
    T = x.numel() // H
    w = w.to(x.dtype).contiguous()
    h = torch.empty_like(x)
    y = torch.empty_like(x)
    _check(lib().oracle_add_rmsnorm(_p(x), _p(residual), _p(w), T, H, eps, DTYPE_TAG[x.dtype],
                                    _p(h), _p(y)), "add_rmsnorm")
    return y, h


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """inv_freq exactly as compute_default_rope_parameters builds it (HF:125-132)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float)
                            / head_dim))


def rope_cos_sin(positions: torch.Tensor, inv_freq: torch.Tensor, head_dim: int,
                 dtype: torch.dtype, scaling: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    pos = _cpu(positions).reshape(-1).to(torch.int64).contiguous()
    inv = _cpu(inv_freq).to(torch.float32).contiguous()
    T = pos.numel()
    cos = torch.empty(T, head_dim, dtype=dtype)
    sin = torch.empty(T, head_dim, dtype=dtype)
    _check(lib().oracle_rope_cos_sin(_p(pos), T, _p(inv), head_dim, scaling, DTYPE_TAG[dtype],
                                     _p(cos), _p(sin)), "rope_cos_sin")
    return cos, sin


def qk_norm_rope_store(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor | None,
                       q_w: torch.Tensor | None, k_w: torch.Tensor | None, eps: float,
                       cos: torch.Tensor, sin: torch.Tensor,
                       k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                       block_mapping: torch.Tensor | None = None,
                       slot_mapping: torch.Tensor | None = None,
                       want_k_out: bool = True):
    """q: (T, Hq, D), k/v: (T, Hkv, D) (last dim contiguous), cos/sin: (T, D).

    Returns (q_out (T,Hq,D), k_out (T,Hkv,D) or None); mutates the caches.
    """
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    dt = q.dtype
    for t in (q, k) + ((v,) if v is not None else ()):
        _cpu(t)
        assert t.stride(2) == 1 and t.dtype == dt
    cos = cos.reshape(T, D).contiguous()
    sin = sin.reshape(T, D).contiguous()
    q_out = torch.empty(T, Hq, D, dtype=dt)
    k_out = torch.empty(T, Hkv, D, dtype=dt) if want_k_out else None
    qw = q_w.to(dt).contiguous() if q_w is not None else None
    kw = k_w.to(dt).contiguous() if k_w is not None else None
    if k_cache is not None:
        bm = block_mapping.contiguous()
        sm = slot_mapping.to(bm.dtype).contiguous()
        idx64 = int(bm.dtype == torch.int64)
        c = _arr(k_cache.stride())
        N, B = k_cache.shape[0], k_cache.shape[2]
        assert k_cache.stride() == v_cache.stride()
    else:
        bm = sm = None
        idx64 = 1
        c = _arr([0, 0, 0, 0])
        N = B = 0
    vv = v if v is not None else None
    _check(lib().oracle_qk_norm_rope_store(
        _p(q), q.stride(0), q.stride(1), _p(k), k.stride(0), k.stride(1),
        _p(vv), vv.stride(0) if vv is not None else 0, vv.stride(1) if vv is not None else 0,
        _p(qw), _p(kw), eps, _p(cos), _p(sin), D, T, Hq, Hkv, D, DTYPE_TAG[dt],
        _p(q_out), _p(k_out), _p(k_cache), _p(v_cache), c, N, B, _p(bm), _p(sm), idx64),
        "qk_norm_rope_store")
    return q_out, k_out


def kv_store_batched(k_src: torch.Tensor, v_src: torch.Tensor, k_cache: torch.Tensor,
                     v_cache: torch.Tensor, block_mapping: torch.Tensor,
                     slot_mapping: torch.Tensor) -> None:
    Hkv, T, D = k_src.shape
    assert k_cache.stride() == v_cache.stride()
    bm = _cpu(block_mapping).contiguous()
    sm = _cpu(slot_mapping).to(bm.dtype).contiguous()
    _check(lib().oracle_kv_store_batched(
        _p(k_src), _arr(k_src.stride()), _p(v_src), _arr(v_src.stride()), _p(k_cache),
        _p(v_cache), _arr(k_cache.stride()), _p(bm), _p(sm), int(bm.dtype == torch.int64),
        T, Hkv, D, k_cache.shape[0], k_cache.shape[2], k_src.element_size()),
        "kv_store_batched")


def kv_store_seq(start_position: int, block_table: torch.Tensor, k_src: torch.Tensor,
                 v_src: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    Hkv, T, D = k_src.shape
    bt = _cpu(block_table).contiguous()
    _check(lib().oracle_kv_store_seq(
        int(start_position), _p(bt), bt.numel(), int(bt.dtype == torch.int64), _p(k_src),
        _arr(k_src.stride()), _p(v_src), _arr(v_src.stride()), _p(k_cache), _p(v_cache),
        _arr(k_cache.stride()), T, Hkv, D, k_cache.shape[0], k_cache.shape[2],
        k_src.element_size()), "kv_store_seq")


def silu_and_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """gate, up: (T, I) views (row strides free, last dim contiguous)."""
    _cpu(gate)
    _cpu(up)
    T, I = gate.shape
    assert gate.stride(1) == 1 and up.stride(1) == 1 and gate.dtype == up.dtype
    out = torch.empty(T, I, dtype=gate.dtype)
    _check(lib().oracle_silu_and_mul(_p(gate), gate.stride(0), _p(up), up.stride(0), T, I,
                                     DTYPE_TAG[gate.dtype], _p(out), I), "silu_and_mul")
    return out


def paged_attention_decode(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, block_size: int,
                           seq_lens: torch.Tensor) -> torch.Tensor:
    """Decode paged attention as the reference defines it
    (server/model/kernels/paged_attention.py:8-121, wrapper :124-192): for
    sequence s and query head h, the first seq_lens[s] tokens of the sequence,
    token j at cache[block_tables[s, j // block_size], h // (Hq // Hkv),
    j % block_size], and out = softmax(q . K^T / sqrt(D)) @ V computed in
    fp32, stored in the query's dtype."""
    import math

    query, k_cache, v_cache = _cpu(query), _cpu(k_cache), _cpu(v_cache)
    block_tables, seq_lens = _cpu(block_tables), _cpu(seq_lens)
    S, Hq, D = query.shape
    Hkv = k_cache.shape[1]
    G = Hq // Hkv
    scale = 1.0 / math.sqrt(D)
    out = torch.empty_like(query)
    for s in range(S):
        L = int(seq_lens[s])
        nb = -(-L // block_size)
        blocks = block_tables[s, :nb].long()
        K = k_cache[blocks].permute(1, 0, 2, 3).reshape(Hkv, nb * block_size, D)[:, :L].float()
        V = v_cache[blocks].permute(1, 0, 2, 3).reshape(Hkv, nb * block_size, D)[:, :L].float()
        q = query[s].float().view(Hkv, G, D)
        w = torch.softmax(torch.einsum("hgd,hkd->hgk", q, K) * scale, dim=-1)
        out[s] = torch.einsum("hgk,hkd->hgd", w, V).reshape(Hq, D).to(query.dtype)
    return out


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, causal: bool,
                     softmax_scale: float | None = None, block_n: int = 32) -> torch.Tensor:
    """Prefill attention as the reference's Triton kernel computes it
    (server/model/kernels/varlen_attention.py:8-142): per sequence and query
    head, keys in blocks of ``block_n`` (BLOCK_N = 32, :190), fp32 scores
    scaled and masked (key beyond the sequence, or past the query when
    causal, :110-115), online softmax with the running row max, and the
    probabilities cast to the value dtype before the product with V (:121);
    the output cast to q's dtype.  The causal loop stops at the end of the
    query's 32-row block (:86-89), which never drops a key the mask keeps."""
    import math

    q, k, v = _cpu(q), _cpu(k), _cpu(v)
    cq, ck = _cpu(cu_seqlens_q).tolist(), _cpu(cu_seqlens_k).tolist()
    Tq, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    out = torch.empty_like(q)
    for b in range(len(cq) - 1):
        q0, q1, k0, k1 = cq[b], cq[b + 1], ck[b], ck[b + 1]
        nq, nk = q1 - q0, k1 - k0
        for h in range(Hq):
            Q = q[q0:q1, h].float()
            K = k[k0:k1, h // G].float()
            V = v[k0:k1, h // G]
            m = torch.full((nq,), float("-inf"))
            l = torch.zeros(nq)
            acc = torch.zeros(nq, D)
            qi = torch.arange(nq)
            for j0 in range(0, nk, block_n):
                kj = torch.arange(j0, min(nk, j0 + block_n))
                s = (Q @ K[kj].T) * scale
                if causal:
                    s = torch.where(qi[:, None] >= kj[None, :], s, float("-inf"))
                mn = torch.maximum(m, s.max(dim=1).values)
                p = torch.exp(s - mn[:, None])
                p = torch.where(torch.isnan(p), torch.zeros_like(p), p)
                corr = torch.exp(m - mn)
                corr = torch.where(torch.isnan(corr), torch.zeros_like(corr), corr)
                acc = acc * corr[:, None] + p.to(v.dtype).float() @ V[kj].float()
                l = l * corr + p.sum(dim=1)
                m = mn
            out[q0:q1, h] = (acc / l[:, None]).to(q.dtype)
    return out


# ---------------------------------------------------------------------------
# Sampling (server/model/sampling.py, server/model/determinism.py)

_MASK64 = (1 << 64) - 1


def mix64(seed: int, step: int) -> int:
    """splitmix64 of (seed, step) (determinism.py:30-41): seed times the
    golden-ratio increment plus step, then the two xor-shift-multiply rounds
    and a final xor-shift, all modulo 2^64."""
    x = ((seed & _MASK64) * 0x9E3779B97F4A7C15 + (step & _MASK64)) & _MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _MASK64
    return x ^ (x >> 31)


def uniform_from_hash(seed: int, step: int) -> float:
    """Top 53 bits of mix64 scaled by 2^-53, capped at 1 - 2^-24
    (determinism.py:44-51)."""
    return min((mix64(seed, step) >> 11) * 2.0 ** -53, 1.0 - 2.0 ** -24)


def uniforms_from_seeds(seeds, steps) -> torch.Tensor:
    """float32 [B] of uniform_from_hash per row (determinism.py:54-73)."""
    return torch.tensor([uniform_from_hash(int(s), int(t)) for s, t in zip(seeds, steps)],
                        dtype=torch.float32)


def sample_tokens(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                  top_p: torch.Tensor, uniforms: torch.Tensor) -> torch.Tensor:
    """The reference's batched sampler (sampling.py:118-194) in torch on the
    CPU, step for step: float32 logits over the clamped temperature, a
    stable descending sort, top-k as -inf past rank k, softmax, top-p
    dropping ranks whose mass before them exceeds top_p (rank 0 kept),
    inverse-CDF pick by searchsorted of u * total, greedy rows at rank 0."""
    logits, temperature, top_k, top_p, uniforms = (
        _cpu(t) for t in (logits, temperature, top_k, top_p, uniforms))
    B, V = logits.shape
    s = logits.float() / temperature.float().clamp(min=1e-5)[:, None]
    vals, order = torch.sort(s, dim=-1, descending=True, stable=True)
    keep = torch.where(top_k > 0, top_k, V)[:, None]
    vals = vals.masked_fill(torch.arange(V)[None, :] >= keep, float("-inf"))
    p = torch.softmax(vals, dim=-1)
    before = torch.cumsum(p, dim=-1) - p
    drop = before > top_p[:, None]
    drop[:, 0] = False
    cdf = torch.cumsum(p.masked_fill(drop, 0.0), dim=-1)
    target = (uniforms.float()[:, None] * cdf[:, -1:]).contiguous()
    rank = torch.searchsorted(cdf.contiguous(), target).clamp(max=V - 1)
    rank = torch.where(temperature[:, None] <= 0, torch.zeros_like(rank), rank)
    return order.gather(-1, rank).squeeze(-1)


def sample_margins(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                   top_p: torch.Tensor, uniforms: torch.Tensor):
    """The same decisions in float64 (exact order, exp and sums in double),
    with each row's distance from a decision boundary: the smaller of
    |mass before the first dropped rank - top_p|, |mass before the last kept
    rank - top_p| and the distance of u * total from the CDF values either
    side of the pick, all as fractions of the kept mass.  A row whose margin
    is below the float32 rounding of the reference's own softmax and cumsums
    can legitimately land on either neighbour.  Returns (tokens, margins,
    slack); greedy rows get margin inf.

    ``slack`` is, per row, how far the reference's own float32 arithmetic
    moves its decisions: |sum of its float32 softmax over the kept ranks - 1|
    (the reference never renormalises, so at top_p = 1.0 its top-p step drops
    the tail whose exclusive cumsum passes 1.0, and every threshold scales by
    that sum) plus 1e-6 for the float32 rounding of the cumsums.  Where a
    row's margin exceeds its slack the reference's token is the exact one."""
    import numpy as np

    logits, temperature, top_k, top_p, uniforms = (
        _cpu(t) for t in (logits, temperature, top_k, top_p, uniforms))
    B, V = logits.shape
    s32 = (logits.float() / temperature.float().clamp(min=1e-5)[:, None]).numpy()
    toks = np.zeros(B, dtype=np.int64)
    margins = np.full(B, np.inf)
    slack = np.full(B, 1e-6)
    for b in range(B):
        order = np.argsort(-s32[b].astype(np.float64), kind="stable")
        if float(temperature[b]) <= 0:
            toks[b] = order[0]
            continue
        k = int(top_k[b])
        k = k if 0 < k < V else V
        sv = s32[b][order[:k]].astype(np.float64)
        p32 = torch.softmax(torch.from_numpy(s32[b][order[:k]]), dim=-1)
        slack[b] += abs(float(p32.double().sum()) - 1.0)
        e = np.exp(sv - sv[0])
        p = e / e.sum()
        incl = np.cumsum(p)
        before = incl - p
        tp = float(top_p[b])
        later = np.nonzero(before[1:] > tp)[0]
        R = int(later[0]) + 1 if later.size else k
        margin = np.inf
        if tp < 1.0:  # at top_p >= 1 no rank is dropped in exact arithmetic
            if R < k:
                margin = min(margin, before[R] - tp)
            if R > 1:
                margin = min(margin, tp - before[R - 1])
        cdf = incl[:R]
        target = float(uniforms[b]) * cdf[-1]
        r = int(np.searchsorted(cdf, target, side="left"))
        r = min(r, R - 1)
        lo = cdf[r - 1] if r > 0 else 0.0
        margin = min(margin, target - lo if r > 0 else np.inf, cdf[r] - target)
        toks[b] = order[r]
        margins[b] = margin
    return torch.from_numpy(toks), torch.from_numpy(margins), torch.from_numpy(slack)
