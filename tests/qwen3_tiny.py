"""A small random-initialised transformers Qwen3 model and the reference's
batch format, for the drop-in tests (no checkpoint: seeded weights).

The batch format is the reference's: a flattened (1, T) batch with
``position_ids`` restarting at 0 per prefill sequence
(server/model/prefill_helpers.py:16-33) and an inference context carrying
``mode`` and per-sequence ``num_tokens`` / ``block_table``
(server/model/inference_context.py:18-21).
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class Context:
    """Same fields as the reference's InferenceContext."""

    mode: str = "prefill"
    sequences: list[dict[str, Any]] = field(default_factory=list)


def tiny_config(**kw):
    from transformers import Qwen3Config

    args = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                rms_norm_eps=1e-6, rope_theta=1e6, max_position_embeddings=4096,
                hidden_act="silu", tie_word_embeddings=False)
    args.update(kw)
    cfg = Qwen3Config(**args)
    cfg._attn_implementation = "sdpa"
    return cfg


def tiny_model(dtype=torch.bfloat16, device="cpu", seed=7, **kw):
    """Seeded random weights; norm weights ~ 1 + N(0, 0.02) like the configs'."""
    from transformers import Qwen3ForCausalLM

    torch.manual_seed(seed)
    model = Qwen3ForCausalLM(tiny_config(**kw)).eval()
    with torch.no_grad():
        g = torch.Generator().manual_seed(seed + 1)
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):
                p.copy_(1.0 + 0.02 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(0.05 * torch.randn(p.shape, generator=g))
    return model.to(device=device, dtype=dtype)


def clone(model):
    return copy.deepcopy(model)


def block_tables(num_seqs: int, blocks_each: int, num_blocks: int, seed: int = 3):
    """Disjoint, randomly permuted physical blocks per sequence."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g)[: num_seqs * blocks_each]
    return [perm[i * blocks_each:(i + 1) * blocks_each].tolist() for i in range(num_seqs)]
