"""Prefill varlen attention on the GPU against the reference's own kernel
outputs (fp32 golden vectors) and the CPU oracle (16-bit types).

Tolerances: fp32 |a - e| <= 1e-4 + 1e-4 |e|; 16-bit outputs: the bf16/fp16
contract of tests/common.py.  The kernel rounds the probabilities to the value
dtype at the same point as the reference but with 64-key blocks where the
reference uses 32, so the running max they are rounded against differs
between the two and a small share of elements moves by one unit in the last
place.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from oracle import oracle
from tests.common import assert_close, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_reference_golden_cases_fp32():
    g = load_golden("varlen_attention.pt")
    for c in g["cases"]:
        cu = c["cu_seqlens"].to(DEV)
        out = tsb.flash_attn_varlen_func(c["q"].to(DEV), c["k"].to(DEV), c["v"].to(DEV), cu, cu,
                                         c["max_seqlen"], c["max_seqlen"], c["causal"])
        torch.testing.assert_close(out.cpu(), c["out"], atol=1e-4, rtol=1e-4, msg=c["name"])


def _packed(lens, hq, hkv, hd, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = torch.randn(T, hq, hd, generator=g).to(dtype)
    k = torch.randn(T, hkv, hd, generator=g).to(dtype)
    v = torch.randn(T, hkv, hd, generator=g).to(dtype)
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    return q, k, v, cu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 2), (16, 8), (32, 4)])
@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_16bit_against_oracle(dtype, hq, hkv, hd, causal):
    lens = [1, 7, 63, 64, 65, 130, 333]
    q, k, v, cu = _packed(lens, hq, hkv, hd, dtype, seed=hq * 10 + hd + causal)
    expected = oracle.varlen_attention(q, k, v, cu, cu, causal)
    out = tsb.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV), cu.to(DEV),
                                     max(lens), max(lens), causal)
    assert out.shape == q.shape and out.dtype == q.dtype
    assert_close(out, expected, f"{dtype} {hq}/{hkv} d{hd} causal={causal}", min_exact=0.9)


def test_views_of_a_merged_projection_at_qwen3_8b_heads():
    """q, k, v as strided head views of one (T, (Hq + 2 Hkv) * D) projection
    output, the layout the model produces (qwen3.py:264-266), one 192-token
    prefill chunk and a 1000-token sequence."""
    lens = [192, 1000]
    hq, hkv, hd = 32, 8, 128
    g = torch.Generator().manual_seed(3)
    T = sum(lens)
    qkv = torch.randn(T, (hq + 2 * hkv) * hd, generator=g).to(torch.bfloat16)
    q = qkv[:, :hq * hd].view(T, hq, hd)
    k = qkv[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd)
    v = qkv[:, (hq + hkv) * hd:].view(T, hkv, hd)
    cu = torch.tensor([0, 192, 1192], dtype=torch.int32)
    expected = oracle.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), cu, cu,
                                       True)
    d = qkv.to(DEV)
    out = tsb.flash_attn_varlen_func(d[:, :hq * hd].view(T, hq, hd),
                                     d[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd),
                                     d[:, (hq + hkv) * hd:].view(T, hkv, hd), cu.to(DEV),
                                     cu.to(DEV), 1000, 1000, True)
    assert_close(out, expected, "merged-projection views", min_exact=0.9)
