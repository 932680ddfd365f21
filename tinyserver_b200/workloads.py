"""Seeded synthetic batches for the five benchmark configurations.

No public dataset or checkpoint is involved: every input is drawn from a
``torch.Generator`` seeded with ``1234 + config index`` (the seeding scheme of
the reference's scripts/bench_paged_attention.py:38, :167-205), with the
shapes and value distributions the configurations name:

====  ============================================================  =========
name  batch                                                         dtype
====  ============================================================  =========
c1    Qwen3-0.6B layer, 4 prefill sequences 37/64/128/255 (484)     float32
c2    Qwen3-1.7B layer, 16 prefill sequences, lengths U[128, 2048]  bfloat16
c3    Qwen3-8B layer, 256 decode tokens at positions U[1, 8191]     bfloat16
c4    Qwen3-8B layer, 32 x 192-token prefill chunks + 2048 decode   bfloat16
      tokens per GPU (8192), positions < 32768, 0.1% x50 outliers
c5    Qwen3-32B layer, 4 x 32768-token prefill per GPU (131072)     bfloat16
====  ============================================================  =========

The KV cache is a 6-D pool ``(2, 1, N, Hkv, B, D)`` whose ``[0, 0]``/``[1, 0]``
views are the per-layer caches, as the reference's qwen3_cache_allocator
builds them (server/model/patches/qwen3.py:49-62).  Every (sequence, logical
block) that the batch writes gets its own physical block from a seeded
permutation; the other block-table entries are seeded but may repeat (they
are never written).  The cache starts "poisoned" with random values so tests
can check that unwritten slots stay untouched.
"""

from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class LayerShape:
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1e6


QWEN3_06B = LayerShape(1024, 16, 8, 128, 3072)
QWEN3_17B = LayerShape(2048, 16, 8, 128, 6144)
QWEN3_8B = LayerShape(4096, 32, 8, 128, 12288)
QWEN3_32B = LayerShape(5120, 64, 8, 128, 25600)


@dataclasses.dataclass(frozen=True)
class Config:
    name: str
    index: int
    shape: LayerShape
    dtype: torch.dtype
    block_size: int
    num_blocks: int
    residual_std: float
    outliers: bool
    description: str


CONFIGS = {
    "c1": Config("c1", 0, QWEN3_06B, torch.float32, 16, 64, 1.0, False,
                 "Qwen3-0.6B layer, fp32, prefill 37/64/128/255 (484 tokens)"),
    "c2": Config("c2", 1, QWEN3_17B, torch.bfloat16, 16, 4096, 0.5, False,
                 "Qwen3-1.7B layer, bf16, 16 prefill sequences of U[128,2048] tokens"),
    "c3": Config("c3", 2, QWEN3_8B, torch.bfloat16, 16, 32768, 1.0, False,
                 "Qwen3-8B layer, bf16, decode step of 256 sequences"),
    "c4": Config("c4", 3, QWEN3_8B, torch.bfloat16, 16, 65536, 1.0, True,
                 "Qwen3-8B layer, bf16, mixed 32x192 prefill + 2048 decode = 8192 tokens/GPU"),
    "c5": Config("c5", 4, QWEN3_32B, torch.bfloat16, 16, 1_835_008, 1.0, False,
                 "Qwen3-32B layer, bf16, 4 x 32768-token prefill per GPU (131072 tokens)"),
}


def seed_of(cfg: Config, shard: int = 0) -> int:
    return 1234 + cfg.index + 1000 * shard


def sequences(cfg: Config, shard: int = 0) -> list[tuple[int, int]]:
    """(num_tokens, start_position) of every sequence of one GPU's batch."""
    g = torch.Generator().manual_seed(seed_of(cfg, shard))
    if cfg.name == "c1":
        return [(n, 0) for n in (37, 64, 128, 255)]
    if cfg.name == "c2":
        lens = torch.randint(128, 2049, (16,), generator=g).tolist()
        return [(n, 0) for n in lens]
    if cfg.name == "c3":
        pos = torch.randint(1, 8192, (256,), generator=g).tolist()
        return [(1, p) for p in pos]
    if cfg.name == "c4":
        starts = torch.randint(0, 32768 - 192 + 1, (32,), generator=g).tolist()
        pos = torch.randint(1, 32768, (2048,), generator=g).tolist()
        return [(192, s) for s in starts] + [(1, p) for p in pos]
    if cfg.name == "c5":
        return [(32768, 0)] * 4
    raise KeyError(cfg.name)


@dataclasses.dataclass
class Batch:
    """One GPU's batch: host-side index data plus (optionally) device tensors."""

    cfg: Config
    seqs: list
    num_tokens: int
    positions: torch.Tensor      # (T,) int64
    cu_seqlens: torch.Tensor     # (S+1,) int32
    block_tables: torch.Tensor   # (S, max_blocks) int32
    block_mapping: torch.Tensor  # (T,) int64
    slot_mapping: torch.Tensor   # (T,) int64
    tensors: dict = dataclasses.field(default_factory=dict)


def index_data(cfg: Config, shard: int = 0, num_blocks: int | None = None,
               max_tokens: int | None = None) -> Batch:
    """Positions, block tables and the (block, slot) mapping of one batch.

    ``max_tokens`` keeps a prefix of the batch (whole sequences first, the last
    one cut) for CPU-sized parity checks."""
    B = cfg.block_size
    N = num_blocks or cfg.num_blocks
    seqs = sequences(cfg, shard)
    if max_tokens is not None:
        kept, total = [], 0
        for n, p in seqs:
            if total >= max_tokens:
                break
            take = min(n, max_tokens - total)
            kept.append((take, p))
            total += take
        seqs = kept
    g = torch.Generator().manual_seed(seed_of(cfg, shard) + 17)
    max_blocks = max(math.ceil((p + n) / B) for n, p in seqs)
    tables = torch.randint(0, N, (len(seqs), max_blocks), generator=g, dtype=torch.int64)
    written = [(s, lb) for s, (n, p) in enumerate(seqs) for lb in range(p // B, (p + n - 1) // B + 1)]
    if len(written) > N:
        raise ValueError(f"{cfg.name}: batch writes {len(written)} blocks, cache has {N}")
    phys = torch.randperm(N, generator=g)[:len(written)]
    ws = torch.tensor([w[0] for w in written])
    wl = torch.tensor([w[1] for w in written])
    tables[ws, wl] = phys
    tables = tables.to(torch.int32)
    lens = torch.tensor([n for n, _ in seqs])
    starts = torch.tensor([p for _, p in seqs])
    T = int(lens.sum())
    seq_of_tok = torch.repeat_interleave(torch.arange(len(seqs)), lens)
    cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    positions = starts[seq_of_tok] + (torch.arange(T) - cu[:-1].long()[seq_of_tok])
    bm = tables.long()[seq_of_tok, positions // B]
    sm = positions % B
    return Batch(cfg, seqs, T, positions.long(), cu, tables, bm, sm)


def _normal(shape, g, device, dtype, std=1.0, mean=0.0):
    t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t.to(dtype)


def _with_outliers(t: torch.Tensor, g: torch.Generator, frac: float = 0.001,
                   scale: float = 50.0) -> torch.Tensor:
    mask = torch.rand(t.shape, generator=g, device=t.device) < frac
    return torch.where(mask, t.float() * scale, t.float()).to(t.dtype)


def make_batch(cfg: Config | str, device: str | torch.device = "cuda", shard: int = 0,
               num_blocks: int | None = None, max_tokens: int | None = None,
               with_table: bool = True, poison_cache: bool = True) -> Batch:
    """Index data plus every activation, weight and cache tensor on ``device``.

    Activations stand in for the GEMM outputs around the path: ``x_mlp`` (the
    previous layer's down_proj output), ``residual``, ``qkv`` (the merged
    q/k/v projection, (T, (Hq + 2 Hkv) * D)), ``attn_out`` (o_proj output) and
    ``gate_up`` (the merged gate/up projection, (T, 2I), gate first)."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    device = torch.device(device)
    b = index_data(cfg, shard, num_blocks, max_tokens)
    s = cfg.shape
    T, dt = b.num_tokens, cfg.dtype
    N = num_blocks or cfg.num_blocks
    g = torch.Generator(device=device).manual_seed(seed_of(cfg, shard) + 99)
    ten = {}
    ten["input_ids"] = torch.randint(0, s.vocab, (T,), generator=g, device=device)
    if with_table:
        ten["embed_weight"] = _normal((s.vocab, s.hidden), g, device, dt, std=0.02)
    for name in ("input_layernorm", "post_attention_layernorm"):
        ten[name] = _normal((s.hidden,), g, device, dt, std=0.02, mean=1.0)
    for name in ("q_norm", "k_norm"):
        ten[name] = _normal((s.head_dim,), g, device, dt, std=0.02, mean=1.0)
    ten["x_mlp"] = _normal((T, s.hidden), g, device, dt)
    ten["residual"] = _normal((T, s.hidden), g, device, dt, std=cfg.residual_std)
    ten["attn_out"] = _normal((T, s.hidden), g, device, dt)
    qkv_w = (s.num_q_heads + 2 * s.num_kv_heads) * s.head_dim
    ten["qkv"] = _normal((T, qkv_w), g, device, dt)
    ten["gate_up"] = _normal((T, 2 * s.intermediate), g, device, dt)
    if cfg.outliers:
        for name in ("x_mlp", "attn_out", "qkv", "gate_up"):
            ten[name] = _with_outliers(ten[name], g)
    pool_shape = (2, 1, N, s.num_kv_heads, cfg.block_size, s.head_dim)
    pool = torch.empty(pool_shape, dtype=dt, device=device)
    if poison_cache:
        pool.normal_(generator=g)
    ten["kv_pool"] = pool
    ten["k_cache"], ten["v_cache"] = pool[0, 0], pool[1, 0]
    ten["inv_freq"] = rope_inv_freq_cpu(s.head_dim, s.rope_theta).to(device)
    for name in ("positions", "block_mapping", "slot_mapping"):
        ten[name] = getattr(b, name).to(device)
    ten["cu_seqlens"] = b.cu_seqlens.to(device)
    ten["block_tables"] = b.block_tables.to(device)
    b.tensors = ten
    return b


def rope_inv_freq_cpu(head_dim: int, theta: float) -> torch.Tensor:
    """inv_freq as compute_default_rope_parameters builds it (fp32, on CPU)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float)
                            / head_dim))


def qkv_views(qkv: torch.Tensor, s: LayerShape):
    """(T, Hq, D), (T, Hkv, D), (T, Hkv, D) views of the merged projection,
    as the reference's .view() calls make them (qwen3.py:264-266)."""
    T = qkv.shape[0]
    D = s.head_dim
    q = qkv[:, : s.num_q_heads * D].view(T, s.num_q_heads, D)
    k = qkv[:, s.num_q_heads * D:(s.num_q_heads + s.num_kv_heads) * D].view(T, s.num_kv_heads, D)
    v = qkv[:, (s.num_q_heads + s.num_kv_heads) * D:].view(T, s.num_kv_heads, D)
    return q, k, v


def bytes_per_token(s: LayerShape, elem: int = 2) -> dict[str, int]:
    """Algorithmic HBM bytes per token of each kernel (what must move at least)."""
    D = s.head_dim
    return {
        "embedding": 2 * s.hidden * elem + 8,
        "add_rmsnorm": 4 * s.hidden * elem,
        "qk_norm_rope_store": (s.num_q_heads + 2 * s.num_kv_heads) * D * elem   # q, k, v in
        + s.num_q_heads * D * elem                                              # q out
        + 2 * s.num_kv_heads * D * elem                                         # k, v to cache
        + 24,                                                                   # pos, block, slot
        "silu_and_mul": 3 * s.intermediate * elem,
    }
