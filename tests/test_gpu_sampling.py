"""The batched sampler on the GPU against the reference's sample_tokens.

Parity bar.  Sampled token ids are integers, but the reference reaches them
through float32 softmax and cumsums, and its token on a row moves with that
rounding when the row's decision sits near a boundary.  The kernel does the
same decisions in exact integer arithmetic on fixed-point masses, so:

* against the float64 restatement of the algorithm (oracle.sample_margins):
  identical tokens on every row whose margin exceeds 1e-7 of the kept mass
  (the kernel's own precision: 2^-40 per element plus expf's last bit);
* against the reference's tokens (the oracle's float32 torch restatement,
  pinned to the reference's own outputs by tests/golden/sampling.pt):
  identical on every row whose margin exceeds that row's float32 slack --
  |sum of the reference's float32 softmax - 1| + 1e-6.  The reference never
  renormalises, so at top_p = 1.0 it still drops the tail whose exclusive
  cumsum passes 1.0, and every threshold moves with that sum.

The behavioural tests restate the reference's own test file
(tests/model/test_batch_sampling.py) against the CUDA path.
"""

import pytest
import torch

import tinyserver_b200 as tsb
from oracle import oracle
from tests.common import load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
EXACT_EPS = 1e-7


def _call(logit_rows, temperature, top_k, top_p, uniforms, dtype=torch.float32):
    return tsb.sample_tokens(
        torch.as_tensor(logit_rows, dtype=torch.float32).to(dtype).to(DEV),
        torch.as_tensor(temperature, dtype=torch.float32).to(DEV),
        torch.as_tensor(top_k, dtype=torch.int64).to(DEV),
        torch.as_tensor(top_p, dtype=torch.float32).to(DEV),
        torch.as_tensor(uniforms, dtype=torch.float32).to(DEV))


def _check_against(out, expected, args, what):
    """Exact tokens away from decision boundaries (see the module docstring);
    returns how many rows differ from the reference in total."""
    out = out.cpu()
    assert out.dtype == torch.int64 and out.shape == expected.shape
    exact, margins, slack = oracle.sample_margins(*args)
    bad = (out != exact) & (margins > EXACT_EPS)
    assert not bad.any(), (f"{what}: rows {bad.nonzero().flatten().tolist()[:8]} differ from "
                           f"exact arithmetic (got {out[bad][:8].tolist()}, "
                           f"want {exact[bad][:8].tolist()})")
    differ = out != expected
    bad = differ & (margins > slack)
    assert not bad.any(), (f"{what}: rows {bad.nonzero().flatten().tolist()[:8]} differ from "
                           f"the reference (got {out[bad][:8].tolist()}, "
                           f"want {expected[bad][:8].tolist()})")
    return int(differ.sum())


def test_reference_golden_cases():
    g = load_golden("sampling.pt")
    for c in g["cases"]:
        args = (c["logits"], c["temperature"], c["top_k"], c["top_p"], c["uniforms"])
        out = tsb.sample_tokens(*(t.to(DEV) for t in args))
        _check_against(out, c["out"], args, c["name"])


def test_uniforms_match_reference_hash_bit_exactly():
    h = load_golden("sampling.pt")["hash"]
    got = tsb.uniforms_from_seeds(h["seeds"], h["steps"])
    assert torch.equal(got.cpu(), h["uniforms_f32"])


def _random_case(B, V, dtype, seed, scale=3.0):
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(B, V, generator=g) * scale).to(dtype)
    temperature = torch.tensor([0.0, 0.5, 0.8, 1.0, 1.3, 2.0, 1e-6, 1.0])[
        torch.randint(0, 8, (B,), generator=g)]
    top_k = torch.tensor([0, 0, 1, 5, 50, 1000, V, V + 7])[torch.randint(0, 8, (B,), generator=g)]
    top_p = torch.tensor([1.0, 1.0, 0.9, 0.95, 0.5, 0.1, 0.0, 0.99])[
        torch.randint(0, 8, (B,), generator=g)]
    uniforms = oracle.uniforms_from_seeds(torch.randint(0, 2 ** 62, (B,), generator=g).tolist(),
                                          [seed] * B)
    return logits, temperature, top_k, top_p, uniforms


PATHS = ["cluster", "wide"]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("V", [1, 2, 7, 100, 4099, 32000])
def test_random_rows_against_oracle(dtype, V, path):
    args = _random_case(24, V, dtype, seed=V)
    expected = oracle.sample_tokens(*args)
    out = tsb.sample_tokens(*(t.to(DEV) for t in args), path=path)
    _check_against(out, expected, args, f"{dtype} V={V} {path}")


@pytest.mark.parametrize("path", PATHS)
def test_qwen3_vocab_decode_batch(path):
    """A c3-sized decode batch: 256 rows of Qwen3's 151936-token vocabulary."""
    args = _random_case(256, 151936, torch.bfloat16, seed=3, scale=4.0)
    expected = oracle.sample_tokens(*args)
    out = tsb.sample_tokens(*(t.to(DEV) for t in args), path=path)
    n = _check_against(out, expected, args, f"qwen3 vocab {path}")
    assert n <= 8, f"{n} boundary rows out of 256"


def _mixed_rows(B, V, seed, scale, dtype=torch.bfloat16):
    """Rows for both sampling paths: greedy rows, top-k cuts from 1 to far
    past the batch-wide path's candidate buffer, top-p and plain picks over
    peaked and flat logits, uniforms from 0 to just below 1."""
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(B, V, generator=g) * scale).to(dtype)
    pick = lambda vals: torch.tensor(vals)[torch.randint(0, len(vals), (B,), generator=g)]  # noqa
    temperature = pick([0.0, 0.6, 1.0, 1.3, 4.0])
    top_k = pick([0, 0, 0, 1, 50, 2048, 4096, 4097, 6000, 30000, V + 3])
    top_p = pick([1.0, 1.0, 0.5, 0.9, 0.95, 0.999, 0.0])
    uniforms = torch.rand(B, generator=g)
    uniforms[::7] = 1 - 2 ** -24
    uniforms[::11] = 0.0
    return logits, temperature, top_k, top_p, uniforms


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("B,V,scale", [(64, 151936, 4.0), (300, 151936, 0.5), (48, 4099, 1.0),
                                       (40, 32000, 8.0), (33, 37, 2.0)])
def test_wide_path_gives_the_cluster_kernels_tokens(B, V, scale, dtype):
    """The batch-wide passes compute the same integers as the per-row cluster
    kernel, so the tokens are identical on every row, boundary rows included;
    rows the batch-wide passes leave (candidate sets past the buffer, large
    top-k) go to the cluster kernel inside the same call."""
    args = [t.to(DEV) for t in _mixed_rows(B, V, seed=B + V, scale=scale, dtype=dtype)]
    wide = tsb.sample_tokens(*args, path="wide")
    cluster = tsb.sample_tokens(*args, path="cluster")
    assert torch.equal(wide, cluster), (wide != cluster).nonzero().flatten().tolist()[:8]
    assert torch.equal(tsb.sample_tokens(*args, path="wide"), wide)  # workspace reuse


def test_wide_path_against_oracle_with_rows_left_to_the_cluster_kernel():
    args = _mixed_rows(96, 151936, seed=5, scale=0.5)
    expected = oracle.sample_tokens(*args)
    out = tsb.sample_tokens(*(t.to(DEV) for t in args), path="wide")
    _check_against(out, expected, args, "wide, mixed rows")


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("scale", [1.0, 4.0])
def test_candidate_sets_on_both_sides_of_the_one_pass_limit(scale, path):
    """Rows whose filtered head (everything at or above the level-1 digit of
    the top-k cut, or of the top-p cut without top-k) holds from a few to
    thousands of elements, so the kernel takes its one-pass path on some and
    its select path on others; the tokens must match the oracle either way."""
    g = torch.Generator().manual_seed(int(scale * 7) + 40)
    B, V = 48, 151936
    logits = (torch.randn(B, V, generator=g) * scale).to(torch.bfloat16)
    temperature = torch.tensor([0.7, 1.0, 1.3] * 16)
    top_k = torch.tensor([20, 1500, 2000, 2048, 2049, 2600, 0, 0] * 6)
    top_p = torch.tensor([1.0, 0.95, 1.0, 0.9, 1.0, 0.8, 0.5, 0.99] * 6)
    uniforms = oracle.uniforms_from_seeds(torch.randint(0, 2 ** 62, (B,), generator=g).tolist(),
                                          [7] * B)
    args = (logits, temperature, top_k, top_p, uniforms)
    expected = oracle.sample_tokens(*args)
    out = tsb.sample_tokens(*(t.to(DEV) for t in args), path=path)
    _check_against(out, expected, args, f"one-pass limit scale={scale} {path}")


def test_strided_and_unaligned_rows():
    """Rows of a wider buffer (16-byte aligned row stride, vector loads) and
    rows at an odd bf16 stride (scalar loads) give the same tokens."""
    args = _random_case(16, 1000, torch.bfloat16, seed=11)
    logits = args[0]
    expected = oracle.sample_tokens(*args)
    rest = [t.to(DEV) for t in args[1:]]
    for width in (1024, 1001):
        wide = torch.zeros(16, width, dtype=logits.dtype)
        wide[:, :1000] = logits
        view = wide.to(DEV)[:, :1000]
        out = tsb.sample_tokens(view, *rest)
        _check_against(out, expected, args, f"row stride {width}")


@pytest.mark.parametrize("path", PATHS)
def test_ties_follow_index_order(path):
    """Long runs of equal logits: the stable sort puts equal values in index
    order, which decides both the top-k cut and the picked token."""
    g = torch.Generator().manual_seed(5)
    B, V = 64, 20000
    logits = torch.randint(-3, 4, (B, V), generator=g).float()
    temperature = torch.ones(B)
    top_k = torch.tensor([0, 1, 2, 3, 100, 5000, 12345, 0] * 8)
    top_p = torch.tensor([1.0, 1.0, 0.3, 1.0, 0.9, 1.0, 0.5, 0.01] * 8)
    uniforms = torch.linspace(0, 1 - 2 ** -24, B)
    args = (logits, temperature, top_k, top_p, uniforms)
    expected = oracle.sample_tokens(*args)
    out = tsb.sample_tokens(*(t.to(DEV) for t in args), path=path)
    _check_against(out, expected, args, f"ties {path}")


@pytest.mark.parametrize("path", PATHS)
def test_seeded_variant_equals_explicit_uniforms(path):
    args = _random_case(32, 5000, torch.bfloat16, seed=21)
    seeds = list(range(1000, 1032))
    steps = [3 * i for i in range(32)]
    u = tsb.uniforms_from_seeds(seeds, steps)
    a = tsb.sample_tokens(*(t.to(DEV) for t in args[:4]), u, path=path)
    b = tsb.sample_tokens_seeded(*(t.to(DEV) for t in args[:4]), seeds, steps, path=path)
    assert torch.equal(a, b)
    assert torch.equal(u.cpu(), oracle.uniforms_from_seeds(seeds, steps))


# ---------------------------------------------------------------------------
# The reference's behavioural tests, against the CUDA path

def test_identical_inputs_produce_identical_outputs():
    logits = torch.randn(6, 64).tolist()
    args = ([1.0] * 6, [0] * 6, [0.9] * 6, [0.1, 0.3, 0.5, 0.7, 0.9, 0.05])
    assert torch.equal(_call(logits, *args), _call(logits, *args))


def test_uniform_distribution_picks_by_hand_computed_cdf():
    result = _call([[0.0] * 4] * 4, [1.0] * 4, [0] * 4, [1.0] * 4, [0.1, 0.4, 0.6, 0.9])
    assert result.tolist() == [0, 1, 2, 3]


def test_returns_int64_of_batch_shape():
    result = _call(torch.randn(3, 10).tolist(), [1.0] * 3, [0] * 3, [1.0] * 3, [0.5] * 3)
    assert result.shape == (3,) and result.dtype == torch.int64
    assert result.device.type == "cuda"


def test_row_token_is_independent_of_batch_position():
    torch.manual_seed(0)
    target = torch.randn(128).tolist()
    others = torch.randn(15, 128).tolist()
    u = oracle.uniform_from_hash(1234, 9)
    alone = _call([target], [0.8], [40], [0.9], [u])
    rows = others[:7] + [target] + others[7:]
    us = [oracle.uniform_from_hash(i, 9) for i in range(16)]
    us[7] = u
    batched = _call(rows, [0.8] * 16, [40] * 16, [0.9] * 16, us)
    assert batched[7].item() == alone[0].item()


def test_batch_size_one_matches_row_in_larger_batch_for_every_row():
    torch.manual_seed(1)
    rows = torch.randn(8, 50).tolist()
    us = [oracle.uniform_from_hash(100 + i, 3) for i in range(8)]
    batched = _call(rows, [1.0] * 8, [10] * 8, [0.95] * 8, us)
    for i, row in enumerate(rows):
        assert _call([row], [1.0], [10], [0.95], [us[i]])[0].item() == batched[i].item()


def test_greedy_rows_match_argmax_when_mixed_with_sampled_rows():
    torch.manual_seed(2)
    logits = torch.randn(6, 40)
    temperature = [0.0, 1.0, 0.0, 0.7, 0.0, 1.2]
    result = _call(logits.tolist(), temperature, [0] * 6, [0.9] * 6,
                   [0.5, 0.5, 0.9, 0.9, 0.1, 0.1])
    greedy = logits.argmax(dim=-1)
    for i, t in enumerate(temperature):
        if t == 0.0:
            assert result[i].item() == greedy[i].item()


def test_greedy_breaks_ties_to_lowest_index_like_argmax():
    assert _call([[0.0, 5.0, 5.0, 1.0]], [0.0], [0], [1.0], [0.99]).tolist() == [1]


def test_greedy_ignores_uniform_value():
    torch.manual_seed(3)
    logits = torch.randn(2, 32).tolist()
    for u in (0.0, 0.25, 0.999):
        result = _call(logits, [0.0, 0.0], [0, 0], [1.0, 1.0], [u, u])
        assert result.tolist() == torch.tensor(logits).argmax(-1).tolist()


def _allowed_set(row, temperature, top_k, top_p):
    """Which token ids may be sampled (float64, plain Python over the order)."""
    scaled = row.double() / max(temperature, 1e-5)
    order = sorted(range(len(scaled)), key=lambda i: (-scaled[i].item(), i))
    if top_k > 0:
        order = order[:top_k]
    probs = torch.softmax(torch.tensor([scaled[i] for i in order], dtype=torch.float64), dim=-1)
    allowed, before = set(), 0.0
    for rank, tok in enumerate(order):
        if rank == 0 or before <= top_p:
            allowed.add(tok)
        before += probs[rank].item()
    return allowed


@pytest.mark.parametrize("top_k,top_p", [(0, 1.0), (5, 1.0), (0, 0.6), (5, 0.6), (1, 1.0),
                                         (1000, 1.0), (3, 0.3)])
def test_sampled_token_is_always_inside_allowed_set(top_k, top_p):
    torch.manual_seed(4)
    logits = torch.randn(4, 60)
    refs = [_allowed_set(logits[i], 0.9, top_k, top_p) for i in range(4)]
    for step in range(40):
        us = [(step * 4 + i) / 160.0 for i in range(4)]
        result = _call(logits.tolist(), [0.9] * 4, [top_k] * 4, [top_p] * 4, us)
        for i, tok in enumerate(result.tolist()):
            assert tok in refs[i], (i, tok, us[i])


def test_per_row_filters_are_honored_independently():
    row = [5.0, 4.0, 3.0, 2.0, 1.0, 0.0]
    assert _call([row] * 3, [1.0] * 3, [1, 2, 3], [1.0] * 3, [0.999] * 3).tolist() == [0, 1, 2]


def test_uniform_zero_picks_top_ranked_survivor():
    assert _call([[1.0, 9.0, 3.0, 7.0]], [1.0], [0], [1.0], [0.0]).tolist() == [1]


def test_top_k_one_is_argmax():
    torch.manual_seed(5)
    logits = torch.randn(4, 30)
    result = _call(logits.tolist(), [1.0] * 4, [1] * 4, [1.0] * 4, [0.0, 0.4, 0.8, 0.99])
    assert result.tolist() == logits.argmax(-1).tolist()


def test_tiny_top_p_returns_dominant_token():
    logits = [[-10.0] * 10 for _ in range(3)]
    logits[0][2], logits[1][7], logits[2][0] = 10.0, 10.0, 10.0
    assert _call(logits, [1.0] * 3, [0] * 3, [1e-6] * 3, [0.9] * 3).tolist() == [2, 7, 0]


def test_top_k_larger_than_vocab_is_a_no_op():
    torch.manual_seed(6)
    logits = torch.randn(3, 20).tolist()
    us = [0.15, 0.55, 0.85]
    assert torch.equal(_call(logits, [1.0] * 3, [0] * 3, [1.0] * 3, us),
                       _call(logits, [1.0] * 3, [999] * 3, [1.0] * 3, us))


_CRITICAL_AT_P999 = [10.83, 13.82, 16.27, 18.47, 20.52, 22.46, 24.32, 26.12, 27.88, 29.59,
                     31.26, 32.91, 34.53, 36.12, 37.70]


def test_distribution_matches_masked_reference_chi_square():
    """One row replicated 8000 times with distinct per-row noise: the counts
    follow the top-p-masked, renormalised distribution (chi-square, p=0.999)."""
    V, top_p, N = 20, 0.85, 8000
    w = torch.tensor([0.7 ** k for k in range(V)], dtype=torch.float64)
    target = w / w.sum()
    row = torch.log(target).float()
    allowed = _allowed_set(row, 1.0, 0, top_p)
    dist = torch.zeros(V, dtype=torch.float64)
    for t in allowed:
        dist[t] = target[t]
    dist /= dist.sum()
    expected = dist * N
    samples = _call(row[None].expand(N, V).tolist(), [1.0] * N, [0] * N, [top_p] * N,
                    [oracle.uniform_from_hash(s, 1) for s in range(N)])
    observed = torch.bincount(samples.cpu(), minlength=V).double()
    assert int(observed[dist == 0].sum()) == 0
    valid = expected >= 5
    chi = float(((observed[valid] - expected[valid]) ** 2 / expected[valid]).sum())
    df = int(valid.sum()) - 1
    assert chi < _CRITICAL_AT_P999[df - 1], (chi, df)


def test_empty_batch():
    out = tsb.sample_tokens(torch.zeros(0, 10, device=DEV), torch.zeros(0, device=DEV),
                            torch.zeros(0, dtype=torch.int64, device=DEV),
                            torch.zeros(0, device=DEV), torch.zeros(0, device=DEV))
    assert out.shape == (0,) and out.dtype == torch.int64
