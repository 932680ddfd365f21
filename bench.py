"""Benchmark of the fused Qwen3 decoder-layer memory-bound path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Workload: configuration c4 of BASELINE.json -- Qwen3-8B layer shapes (hidden
4096, 32 q / 8 kv heads, head_dim 128, intermediate 12288), bf16, a mixed
batch of 32 x 192-token prefill chunks + 2048 decode tokens = 8192 tokens per
GPU, positions < 32768, a 65536-block (16-token page) KV cache per GPU, seeded
synthetic inputs with 0.1% x50 outliers.  One step is one pass of the path
over the batch, in the decoder layer's order:

  embedding gather -> residual add + input RMSNorm ->
  q_norm/k_norm + RoPE (cos/sin computed in the kernel from the positions) +
  paged KV store -> residual add + post-attn RMSNorm -> SiLU-and-mul

(the GEMMs between them are outside the path; their outputs are seeded
inputs).  Ranks shard tokens (weak scaling, no collective on the timed path).
`value` is tokens/s over all ranks, timed with CUDA events (max over ranks);
`e2e` runs the same step through the public API from pinned host buffers with
the H2D copies of every per-step input and the D2H copies of every output
inside the timed region.

After the timed passes (never inside them):
  * `validation` -- every 64th token of the global batch: each rank's outputs
    and the K/V page rows it wrote are all-gathered to rank 0 (NCCL), which
    regenerates every rank's seeded inputs and checks them against the CPU
    oracle (the checker, not a measured leg);
  * `reference_gpu` (N=1) -- the reference's own GPU path on the same batch
    (its transformers modules on CUDA + its Triton KV store);
  * `rows` (N=1) -- the other configurations and the next rows of the path,
    each with its roofline, clocks, end-to-end, CPU baseline and reference-GPU
    figures: the c3 decode step (eager and CUDA graph), c5 at full size, the
    standalone KV store, decode and prefill attention and the sampler.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused-layer tokens/s and HBM GB/s (% of ~8 TB/s) per B200, Qwen3-8B shapes"
CONFIG = "c4"
FALLBACK_HBM_GBS = 6650.0
VALIDATE_EVERY = 64  # validation samples every 64th token of the global batch


# ----------------------------------------------------------------------------
def hbm_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def ncu_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            return float(json.load(f)[kernel]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML on a background thread."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int, interval: float = 0.02):
        self.samples: list[tuple[int, int]] = []
        self.interval = interval
        self._stop = threading.Event()
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self._nvml = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM)
                rs = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(self.interval)

    def start(self):
        if self.ok:
            self._t.start()
        return self

    def stop(self) -> dict:
        self._stop.set()
        if self.ok:
            self._t.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0, "note": "no NVML samples"}
        busy = [m for m, _ in self.samples]
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples)}


def timed(fn, steps: int, warmup: int, device_index: int) -> tuple[float, dict]:
    """Mean ms per call of ``fn`` over ``steps`` back-to-back calls between two
    CUDA events on the current stream (after ``warmup`` calls), with the SM
    clocks sampled meanwhile.  A timed region shorter than ~0.2 s is repeated
    until the clock sampler has seen it."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    sampler = ClockSampler(device_index).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total_ms, n, t_end = 0.0, 0, time.perf_counter() + 0.2
    while n == 0 or time.perf_counter() < t_end:
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        total_ms += e0.elapsed_time(e1)
        n += steps
    return total_ms / n, sampler.stop()


def event_loop(fn, steps: int, min_seconds: float = 0.0) -> tuple[float, int]:
    """Rounds of ``steps`` back-to-back calls between two CUDA events on the
    current stream, repeated until ``min_seconds`` have passed (so the clock
    sampler sees the timed region); returns (total ms, total calls)."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total_ms, n, t_end = 0.0, 0, time.perf_counter() + min_seconds
    while n == 0 or time.perf_counter() < t_end:
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        total_ms += e0.elapsed_time(e1)
        n += steps
    return total_ms, n


def roofline(bound: str, kernel: str, achieved: float, unit: str, traffic=None, **extra) -> dict:
    peak, kind = hbm_peak() if bound == "hbm" else tensor_peak()
    src = "hbm_gbs" if bound == "hbm" else "bf16_tflops (cuBLAS burst)"
    return {"bound": bound, "kernel": kernel, "achieved": round(achieved, 1), "peak": peak,
            "unit": unit, "frac": round(achieved / peak, 4),
            "peak_source": f"{kind} {src}" + (" of MEASURED_PEAKS.json" if kind == "measured"
                                               else " (fallback)"),
            "traffic": traffic, **extra}


# ----------------------------------------------------------------------------
class Step:
    """One fused-layer pass over one GPU's batch, through the public API."""

    KERNELS = ["embedding", "add_rmsnorm_in", "qk_norm_rope_store", "add_rmsnorm_post",
               "silu_and_mul"]

    def __init__(self, batch):
        import tinyserver_b200 as tsb
        from tinyserver_b200 import workloads as W

        self.tsb = tsb
        self.W = W
        self.b = batch
        self.s = batch.cfg.shape
        self.dt = batch.cfg.dtype

    def run(self, t: dict, events: list | None = None) -> dict:
        tsb, s = self.tsb, self.s
        ev = events
        if ev is not None:
            ev[0].record()
        x0 = tsb.embedding(t["input_ids"], t["embed_weight"])
        if ev is not None:
            ev[1].record()
        y1, h1 = tsb.fused_add_rms_norm(t["x_mlp"], x0, t["input_layernorm"], s.eps)
        if ev is not None:
            ev[2].record()
        q, k, v = self.W.qkv_views(t["qkv"], s)
        q_out, _ = tsb.qk_norm_rope_store(q, k, v, t["q_norm"], t["k_norm"], s.eps, None, None,
                                          t["k_cache"], t["v_cache"], t["block_mapping"],
                                          t["slot_mapping"], positions=t["positions"],
                                          inv_freq=t["inv_freq"], want_k_out=False)
        if ev is not None:
            ev[3].record()
        y2, h2 = tsb.fused_add_rms_norm(t["attn_out"], h1, t["post_attention_layernorm"], s.eps)
        if ev is not None:
            ev[4].record()
        act = tsb.silu_and_mul(t["gate_up"])
        if ev is not None:
            ev[5].record()
        return {"normed_in": y1, "q": q_out, "normed_post": y2, "residual": h2, "act": act}

    def runners(self, t: dict) -> dict:
        """Each kernel of the step as its own call, on the step's inputs (for
        timing the kernels one at a time)."""
        tsb, s = self.tsb, self.s
        x0 = tsb.embedding(t["input_ids"], t["embed_weight"])
        _, h1 = tsb.fused_add_rms_norm(t["x_mlp"], x0, t["input_layernorm"], s.eps)
        q, k, v = self.W.qkv_views(t["qkv"], s)
        return {
            "embedding": lambda: tsb.embedding(t["input_ids"], t["embed_weight"]),
            "add_rmsnorm_in": lambda: tsb.fused_add_rms_norm(t["x_mlp"], x0,
                                                             t["input_layernorm"], s.eps),
            "qk_norm_rope_store": lambda: tsb.qk_norm_rope_store(
                q, k, v, t["q_norm"], t["k_norm"], s.eps, None, None, t["k_cache"],
                t["v_cache"], t["block_mapping"], t["slot_mapping"], positions=t["positions"],
                inv_freq=t["inv_freq"], want_k_out=False),
            "add_rmsnorm_post": lambda: tsb.fused_add_rms_norm(
                t["attn_out"], h1, t["post_attention_layernorm"], s.eps),
            "silu_and_mul": lambda: tsb.silu_and_mul(t["gate_up"]),
        }

    def bytes_per_token(self) -> dict[str, int]:
        bpt = self.W.bytes_per_token(self.s)
        return {
            "embedding": bpt["embedding"],
            "add_rmsnorm_in": bpt["add_rmsnorm"],
            "qk_norm_rope_store": bpt["qk_norm_rope_store"],  # cos/sin computed, not read
            "add_rmsnorm_post": bpt["add_rmsnorm"],
            "silu_and_mul": bpt["silu_and_mul"],
        }


PER_STEP_INPUTS = ["input_ids", "positions", "block_mapping", "slot_mapping", "x_mlp",
                   "qkv", "attn_out", "gate_up"]


def measure_e2e(args, step: "Step", t: dict, dev: torch.device, world: int):
    """The step through the public API from pinned host buffers: every step
    copies its inputs host->device and every output device->host inside the
    timed region.  Copies run on their own streams, double-buffered, so step
    i+1's inputs go up and step i-1's outputs come down while step i computes
    (PCIe is full duplex); every step's bytes still cross.  Returns (max-over-
    ranks ms, steps, H2D bytes per step, D2H bytes per step)."""
    host_in = {k: t[k].to("cpu").pin_memory() for k in PER_STEP_INPUTS}
    dev_in = [{k: torch.empty_like(t[k]) for k in PER_STEP_INPUTS} for _ in range(2)]
    resident = {k: v for k, v in t.items() if k not in PER_STEP_INPUTS}
    outs = step.run(t)
    host_out = [{k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in outs.items()}
                for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    d2h = sum(v.numel() * v.element_size() for v in host_out[0].values())
    compute = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    n = max(3, min(args.steps, 50))

    def run(steps: int) -> None:
        uploaded = [torch.cuda.Event() for _ in range(steps)]
        consumed = [torch.cuda.Event() for _ in range(steps)]
        computed = [torch.cuda.Event() for _ in range(steps)]

        def upload(i):
            with torch.cuda.stream(up):
                if i >= 2:
                    up.wait_event(consumed[i - 2])  # step i-2 has read this buffer
                for k in PER_STEP_INPUTS:
                    dev_in[i % 2][k].copy_(host_in[k], non_blocking=True)
                uploaded[i].record(up)

        upload(0)
        for i in range(steps):
            if i + 1 < steps:
                upload(i + 1)
            compute.wait_event(uploaded[i])
            o = step.run({**resident, **dev_in[i % 2]})
            consumed[i].record(compute)
            computed[i].record(compute)
            with torch.cuda.stream(down):
                down.wait_event(computed[i])
                for k, v in o.items():
                    v.record_stream(down)  # keep the output alive until its copy is done
                    host_out[i % 2][k].copy_(v, non_blocking=True)
        compute.wait_stream(down)
        compute.wait_stream(up)

    run(2)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    up.wait_event(e0)
    down.wait_event(e0)
    run(n)
    e1.record(compute)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        m = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(m.item())
        torch.distributed.barrier()
    return e2e_ms, n, h2d, d2h


# ----------------------------------------------------------------------------
# validation of the outputs (after the timed passes)
def _within(actual: torch.Tensor, expected: torch.Tensor, exact: bool) -> dict:
    """The parity contract: bit-exact, or |a - e| <= 2e-2 + 1e-2 |e| (bf16)."""
    a, e = actual.float(), expected.float()
    err = (a - e).abs()
    as_int = {2: torch.int16, 4: torch.int32}[actual.element_size()]
    same = actual.reshape(-1).view(as_int) == expected.reshape(-1).view(as_int)
    ok = bool(same.all()) if exact else bool((err <= 2e-2 + 1e-2 * e.abs()).all()) and \
        bool(torch.isfinite(a).all())
    return {"ok": ok, "bit_exact": round(float(same.float().mean()), 6),
            "mismatched": int((~same).sum()),
            "max_abs_err": float(err.max()) if err.numel() else 0.0}


def _expected_rows(t: dict, rows: torch.Tensor, shape, dtype) -> dict:
    """Oracle outputs of the fused step for the token rows ``rows`` of a
    batch's tensors ``t`` (inputs sliced on the device, oracle on the CPU)."""
    from oracle import oracle
    from tinyserver_b200 import workloads as W

    s = shape
    cpu = lambda x: x[rows].cpu()  # noqa: E731
    x0 = t["embed_weight"][t["input_ids"][rows]].cpu()  # the row gather itself
    y1, h1 = oracle.add_rmsnorm(cpu(t["x_mlp"]), x0, t["input_layernorm"].cpu(), s.eps)
    q, k, v = W.qkv_views(cpu(t["qkv"]), s)
    cos, sin = oracle.rope_cos_sin(cpu(t["positions"]), t["inv_freq"].cpu(), s.head_dim, dtype)
    q_out, k_out = oracle.qk_norm_rope_store(q, k, None, t["q_norm"].cpu(), t["k_norm"].cpu(),
                                             s.eps, cos, sin)
    y2, h2 = oracle.add_rmsnorm(cpu(t["attn_out"]), h1, t["post_attention_layernorm"].cpu(),
                                s.eps)
    I = s.intermediate
    gu = cpu(t["gate_up"])
    act = oracle.silu_and_mul(gu[:, :I], gu[:, I:])
    return {"normed_in": y1, "q": q_out, "normed_post": y2, "residual": h2, "act": act,
            "k_page": k_out, "v_page": v}


_OUT_ORDER = ["normed_in", "q", "normed_post", "residual", "act", "k_page", "v_page"]
_EXACT = {"residual", "v_page"}  # one rounding of an add / a copy: bit-exact


def _sample_rows(outs: dict, t: dict, rows: torch.Tensor) -> torch.Tensor:
    """One bf16 row per sampled token: its outputs and the K/V page rows it wrote."""
    n = rows.numel()
    pages = t["kv_pool"][:, 0, t["block_mapping"][rows], :, t["slot_mapping"][rows], :]
    parts = [outs["normed_in"][rows], outs["q"][rows].reshape(n, -1), outs["normed_post"][rows],
             outs["residual"][rows], outs["act"][rows], pages[:, 0].reshape(n, -1),
             pages[:, 1].reshape(n, -1)]
    return torch.cat(parts, 1)


def validate_layer(step: "Step", t: dict, batch, dev, rank: int, world: int,
                   make_shard) -> dict | None:
    """Every VALIDATE_EVERY-th token of the global batch (the ranks' batches in
    rank order, rank r owning ``sharding.shard_range(world * T, world, r)``):
    each rank runs one more step, takes its sampled tokens' outputs and K/V
    page rows, and ``sharding.gather_rows`` (all-gather over NCCL) brings them
    to rank 0.  Rank 0 regenerates each rank's seeded inputs with
    ``make_shard(r)`` on its own GPU (the generator is the same on every
    device) and checks every gathered row against the CPU oracle.  Returns
    rank 0's summary (None on the other ranks)."""
    from tinyserver_b200 import sharding

    T = batch.num_tokens
    G = world * T
    glob = torch.arange(0, G, VALIDATE_EVERY)

    def local_rows(r):
        lo, hi = sharding.shard_range(G, world, r)
        return (glob[(glob >= lo) & (glob < hi)] - lo).to(dev)

    outs = step.run(t)
    mine = _sample_rows(outs, t, local_rows(rank))
    gathered = sharding.gather_rows(mine) if world > 1 else mine
    torch.cuda.synchronize()
    if rank != 0:
        return None
    res = guarded(_check_gathered, gathered, t, batch, rank, world, local_rows, make_shard)
    res.setdefault("validated", False)
    return res


def _check_gathered(gathered, t, batch, rank, world, local_rows, make_shard) -> dict:
    """Rank 0's half of validate_layer: every gathered row against the oracle."""
    s, dt = batch.cfg.shape, batch.cfg.dtype
    widths = [s.hidden, s.num_q_heads * s.head_dim, s.hidden, s.hidden, s.intermediate,
              s.num_kv_heads * s.head_dim, s.num_kv_heads * s.head_dim]
    got_all = gathered.cpu()
    checks = {name: {"ok": True, "bit_exact_min": 1.0, "max_abs_err": 0.0} for name in _OUT_ORDER}
    at = 0
    for r in range(world):
        rows = local_rows(r)
        tr = t if r == rank else make_shard(r).tensors
        exp = _expected_rows(tr, rows, s, dt)
        got = got_all[at:at + rows.numel()]
        at += rows.numel()
        col = 0
        for name, w in zip(_OUT_ORDER, widths):
            e = exp[name].reshape(rows.numel(), -1)
            c = _within(got[:, col:col + w], e, exact=name in _EXACT)
            col += w
            agg = checks[name]
            agg["ok"] = agg["ok"] and c["ok"]
            agg["bit_exact_min"] = min(agg["bit_exact_min"], c["bit_exact"])
            agg["max_abs_err"] = max(agg["max_abs_err"], c["max_abs_err"])
        if r != rank:
            del tr
            torch.cuda.empty_cache()
    return {"validated": all(c["ok"] for c in checks.values()), "rows_checked": int(at),
            "ranks": world, "every": VALIDATE_EVERY, "checks": checks,
            "how": "every 64th token of the global batch: outputs and written K/V page rows "
                   "all-gathered to rank 0 (sharding.gather_rows over NCCL when N>1), checked "
                   "against the CPU oracle on each rank's regenerated seeded inputs; residual "
                   "and V pages bit-exact, the rest within |a-e| <= 2e-2 + 1e-2|e|"}


# ----------------------------------------------------------------------------
# the reference's own GPU path (baseline/reference_gpu.py)
def reference_gpu_layer(batch, steps: int, ours_ms: float, local_rank: int,
                        ours_outs: dict | None = None) -> dict:
    """The reference's layer path (its transformers modules on CUDA and its
    Triton KV store) over the same batch, timed like the headline."""
    try:
        from baseline import reference_gpu as R

        t, s = batch.tensors, batch.cfg.shape
        weights = {k: t[k] for k in ("embed_weight", "input_layernorm",
                                     "post_attention_layernorm", "q_norm", "k_norm")}
        ref = R.ReferenceGpuLayer(s, batch.cfg.dtype, weights)
    except Exception as e:  # the reference or its Triton kernels are unavailable
        return {"unavailable": f"{type(e).__name__}: {e}"}
    args = (t["input_ids"], t["positions"], t["x_mlp"], t["qkv"], t["attn_out"], t["gate_up"],
            t["k_cache"], t["v_cache"], t["block_mapping"], t["slot_mapping"])
    ms, clocks = timed(lambda: ref.step(*args), max(3, min(steps, 50)), 3, local_rank)
    T = batch.num_tokens
    out = {"value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4),
           "speedup_of_ours": round(ms / ours_ms, 2), "clocks": clocks,
           "what": "the reference's path on this GPU: transformers 5.5.0 Qwen3 modules on CUDA "
                   "(embedding, RMSNorm, rotary, apply_rotary_pos_emb, SiLU*up, eager) and the "
                   "reference's Triton store_kv_cache_batched (server/model/kernels/kv_cache.py) "
                   "with device mappings, from baseline/_ref"}
    if ours_outs is not None:  # the two paths agree on this batch
        normed, q, normed2, hidden, act = ref.step(*args)
        T_ = q.shape[2]
        mine = {"normed_in": normed[0], "q": q[0].transpose(0, 1).reshape(T_, -1, q.shape[-1]),
                "normed_post": normed2[0], "residual": hidden[0], "act": act[0]}
        agree = {k: _within(ours_outs[k].reshape(mine[k].shape), mine[k], exact=(k == "residual"))
                 for k in mine}
        out["agrees_with_ours"] = all(v["ok"] for v in agree.values())
        out["agreement"] = {k: {"bit_exact": v["bit_exact"], "max_abs_err": v["max_abs_err"]}
                            for k, v in agree.items()}
    return out


def _ref_timed(get_fn, call, steps: int, local_rank: int, ours_ms: float, unit_value) -> dict:
    """Time one of the reference's GPU functions (``call(fn)`` per step)."""
    try:
        fn = get_fn()
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {e}"}
    ms, clocks = timed(lambda: call(fn), steps, 3, local_rank)
    v, unit = unit_value(ms)
    return {"value": round(v, 1), "unit": unit, "ms_per_step": round(ms, 4),
            "speedup_of_ours": round(ms / ours_ms, 2), "clocks": clocks}


# ----------------------------------------------------------------------------
def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    from tinyserver_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    make = lambda r: W.make_batch(CONFIG, dev, shard=r, max_tokens=args.max_tokens,  # noqa
                                  num_blocks=args.num_blocks)
    batch = make(rank)
    t = batch.tensors
    T = batch.num_tokens
    step = Step(batch)
    bpt = step.bytes_per_token()
    step_bytes = sum(bpt.values()) * T

    import tinyserver_b200 as tsb
    tsb.load_library()

    # ---- device-resident timing: the headline --------------------------------
    # The step's five launches are captured once, through the public API, as a
    # CUDA graph (the way a serving loop runs a step), and each step is one
    # replay.  Launched eagerly from Python the step costs ~170 us of host time
    # against ~235 us of GPU time, so any host-side hiccup (the clock sampler's
    # thread taking the GIL) can leave the GPU idle between launches; a replay
    # costs a few us.  Programmatic dependent launch carries into the graph.
    # W warm-up replays run right before the timed ones, so the GPU is busy
    # (and at its working clocks) up to the start of the timed region; then K
    # replays back to back between two events.  The clocks are sampled every
    # 2 ms over the whole stretch.
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # uncaptured calls on the capture stream first
        for _ in range(3):
            step.run(t)
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step.run(t)

    def headline(fn) -> float:
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(max(args.warmup, 3)):
            fn()
        tsb.check_errors(dev)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            fn()
        stop.record()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        ms = start.elapsed_time(stop)
        tsb.check_errors(dev)
        if world > 1:
            m = torch.tensor([ms], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
            ms = float(m.item())
        return ms

    sampler = ClockSampler(local_rank, interval=0.002).start()
    elapsed_ms = headline(graph.replay)
    clocks = sampler.stop()
    # the same K steps launched eagerly from Python, reported beside it
    eager_ms = headline(lambda: step.run(t))
    del graph

    # ---- per-kernel attribution: a second timed pass with an event between
    # every two kernels (on the launch stream); these events serialise the
    # launches, so this pass runs a little slower than the headline pass.
    nk = len(Step.KERNELS)
    kb = max(50, min(args.steps, 200))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] for _ in range(kb)]
    for _ in range(3):
        step.run(t)
    torch.cuda.synchronize()
    for i in range(kb):
        step.run(t, evs[i])
    torch.cuda.synchronize()
    per_kernel_us = {}  # the median over the steps: one disturbed step does not move it
    for j, name in enumerate(Step.KERNELS):
        per_kernel_us[name] = 1e3 * statistics.median(e[j].elapsed_time(e[j + 1]) for e in evs)
    tsb.check_errors(dev)

    # ---- each kernel alone: a 256 MB read between launches evicts L2, so every
    # launch reads its inputs from HBM; its own writes may still sit in L2 when
    # its stop event fires (the next kernel in a real step pays that write-back).
    iso_us = {}
    flush = torch.ones(64 * 2 ** 20, dtype=torch.float32, device=dev)
    for name, fn in step.runners(t).items():
        ts = []
        for i in range(25):
            flush.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= 5:
                ts.append(1e3 * e0.elapsed_time(e1))
        iso_us[name] = statistics.median(ts)
    del flush
    tsb.check_errors(dev)

    # ---- outputs checked against the oracle (all ranks, outside the timing) --
    validation = None
    if not args.no_validate:
        validation = validate_layer(step, t, batch, dev, rank, world, make)
        if world > 1:
            torch.distributed.barrier()

    # ---- end to end from pinned host buffers ----------------------------------
    e2e = None if args.no_e2e else measure_e2e(args, step, t, dev, world)

    if rank != 0:
        return None

    peak, peak_kind = hbm_peak()
    ms_per_step = elapsed_ms / args.steps
    value = world * T * args.steps / (elapsed_ms / 1e3)
    kernels = {}
    for name in Step.KERNELS:
        us = per_kernel_us[name]
        gbs = bpt[name] * T / (us * 1e-6) / 1e9
        kernels[name] = {"us": round(us, 2), "bytes_per_token": bpt[name],
                         "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
    kernels_isolated = {}
    for name in Step.KERNELS:
        us = iso_us[name]
        gbs = bpt[name] * T / (us * 1e-6) / 1e9
        kernels_isolated[name] = {"us": round(us, 2), "gbs": round(gbs, 1),
                                  "frac": round(gbs / peak, 4)}
    attributed_ms = sum(per_kernel_us.values()) / 1e3
    dom = max(Step.KERNELS, key=lambda n: per_kernel_us[n])
    dom_gbs = bpt[dom] * T / (per_kernel_us[dom] * 1e-6) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded torch.Generator inputs of config c4's shapes and "
                "distributions (no dataset or checkpoint)",
        "config": layer_config(world, T, step_bytes),
        "hbm_gbs": round(step_bytes / (ms_per_step * 1e-3) / 1e9, 1),
        "hbm_frac": round(step_bytes / (ms_per_step * 1e-3) / 1e9 / peak, 4),
        "hbm_peak_gbs": peak,
        "hbm_peak_kind": peak_kind,
        "kernels": kernels,
        "kernels_note": "per-kernel CUDA-event times from a second pass with an event between "
                        f"every two launches (median over {kb} steps; the medians sum to "
                        f"{attributed_ms:.4f} ms); the headline is the pass without them",
        "kernels_isolated": kernels_isolated,
        "kernels_isolated_note": "each kernel alone on the step's inputs, median of 20 launches, "
                                 "a 256 MB read between launches so its inputs come from HBM; "
                                 "its own writes may end in L2 (in the step, the next kernel "
                                 "pays that write-back)",
        "roofline": roofline("hbm", dom, dom_gbs, "GB/s", ncu_traffic(dom),
                             algorithmic_bytes_per_launch=bpt[dom] * T),
        "gpu_launches": nk * args.steps,
        "pdl": "programmatic dependent launch between the step's kernels",
        "launch": {"headline": "one CUDA graph of the step (its five launches captured through "
                               "the public API), replayed once per step",
                   "eager_ms_per_step": round(eager_ms / args.steps, 4),
                   "eager_note": "the same K steps launched from Python, timed the same way"},
        "clocks": clocks,
        "e2e": None,
        "validation": validation,
    }
    if e2e is not None:
        e2e_ms, e2e_steps, h2d, d2h = e2e
        line["e2e"] = {"value": round(world * T * e2e_steps / (e2e_ms / 1e3), 1),
                       "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                       "note": "public API from pinned host buffers; every per-step input H2D "
                               "and every output D2H inside the timed region; copies on their "
                               "own streams, double-buffered, overlapping the neighbouring "
                               "steps' compute"}
    if args.max_tokens is not None or args.num_blocks is not None:
        line["config"]["workload"] = (f"c4 prefix of {T} tokens, {batch.tensors['k_cache'].shape[0]}"
                                      "-block cache (a profiling case, not the benchmark workload)")
    if world == 1 and not args.no_reference_gpu:
        line["reference_gpu"] = guarded(reference_gpu_layer, batch, args.steps, ms_per_step,
                                        local_rank, step.run(t))
    if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
        line["cpu_baseline"] = guarded(cpu_baseline, batch, budget_s=args.cpu_seconds)
    if world == 1 and not args.no_rows:
        del step, t, batch
        guarded(torch.cuda.empty_cache)
        line["rows"] = run_rows(args, local_rank)
    return line


def layer_config(world: int, T: int, step_bytes: int) -> dict:
    return {
        "workload": "c4: Qwen3-8B layer, mixed 32x192 prefill + 2048 decode = "
                    "8192 tokens/GPU, 16-token pages, 65536 blocks/GPU",
        "tokens_per_gpu": T, "global_tokens": world * T, "hidden": 4096,
        "num_q_heads": 32, "num_kv_heads": 8, "head_dim": 128, "intermediate": 12288,
        "block_size": 16, "num_blocks": 65536,
        "parallelism": f"token-sharded x{world}, no collective on the timed path",
        "l2": f"inputs larger than L2: {step_bytes / 1e9:.2f} GB moved per step per GPU",
    }


# ----------------------------------------------------------------------------
# rows: the other configurations and the next rows of the path (N=1)
def _compact(line: dict) -> dict:
    keep = ("metric", "value", "unit", "ms_per_step", "us_per_step", "steps", "config",
            "roofline", "clocks", "e2e", "cpu_baseline", "reference_gpu", "validation",
            "graph", "kv_store", "path", "gpu_launches", "dtype", "e2e_note", "error")
    return {k: line[k] for k in keep if k in line}


def guarded(fn, *args, **kw):
    """fn(*args, **kw), or {"error": ...} if it raises: an optional leg of the
    bench never keeps the headline line from being printed."""
    try:
        return fn(*args, **kw)
    except Exception as e:  # noqa: BLE001 -- recorded in the JSON line
        return {"error": f"{type(e).__name__}: {e}"[:500]}


def run_rows(args, local_rank: int) -> dict:
    """Each row in turn on this GPU, its memory freed before the next; a row
    that fails records its error and the others still run."""
    rows = {}
    for name, fn in (("c3_decode_step", row_c3_step), ("decode_attention", run_attention),
                     ("prefill_attention", run_prefill), ("sampler", run_sample),
                     ("c5_long_prefill", row_c5)):
        def one():
            line = fn(args, 0, 1, local_rank, as_row=True)
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            return _compact(line) if line is not None else None

        rows[name] = guarded(one)
    return rows


def row_c3_step(args, rank: int, world: int, local_rank: int, as_row: bool = False) -> dict:
    """The fused-layer step on config c3: a continuous-batching decode step of
    256 sequences (one token each, Qwen3-8B shapes, 32768-block cache).  Too
    small to fill the GPU, so it is launch-bound: timed eagerly and as one
    CUDA-graph replay per step (the way a serving loop would run it)."""
    import tinyserver_b200 as tsb
    from tinyserver_b200 import workloads as W

    dev = torch.device("cuda", local_rank)
    batch = W.make_batch("c3", dev, poison_cache=False)
    t, T = batch.tensors, batch.num_tokens
    step = Step(batch)
    step_bytes = sum(step.bytes_per_token().values()) * T
    n = 200
    eager_ms, _ = timed(lambda: step.run(t), n, 5, local_rank)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            step.run(t)
    torch.cuda.current_stream(dev).wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = step.run(t)
    graph_ms, clocks = timed(g.replay, n, 5, local_rank)
    tsb.check_errors(dev)
    # every token of the step against the oracle
    rows = torch.arange(T, device=dev)
    exp = _expected_rows(t, rows, batch.cfg.shape, batch.cfg.dtype)
    got = _sample_rows(outs, t, rows).cpu()
    s = batch.cfg.shape
    widths = [s.hidden, s.num_q_heads * s.head_dim, s.hidden, s.hidden, s.intermediate,
              s.num_kv_heads * s.head_dim, s.num_kv_heads * s.head_dim]
    col, checks = 0, {}
    for name, w in zip(_OUT_ORDER, widths):
        checks[name] = _within(got[:, col:col + w], exp[name].reshape(T, -1), name in _EXACT)
        col += w
    peak, _ = hbm_peak()
    gbs = step_bytes / (graph_ms * 1e-3) / 1e9
    ref = None
    if not args.no_reference_gpu:
        ref = reference_gpu_layer(batch, n, graph_ms, local_rank)
    del g
    e2e = None
    if not args.no_e2e:  # eager, through the public API, host buffers every step
        e2e_ms, e2e_steps, h2d, d2h = measure_e2e(args, step, t, dev, 1)
        e2e = {"value": round(T * e2e_steps / (e2e_ms / 1e3), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps}
    cpu = None if args.no_cpu_baseline else cpu_baseline(batch, budget_s=min(args.cpu_seconds, 3.0))
    return {
        "metric": "fused-layer decode step tokens/s per B200 (c3, Qwen3-8B shapes)",
        "value": round(T / (graph_ms * 1e-3), 1), "unit": "tokens/s",
        "ms_per_step": round(graph_ms, 5), "us_per_step": round(1e3 * graph_ms, 2),
        "steps": n, "dtype": "bf16",
        "config": {"workload": "c3: 256 decode tokens, positions U[1, 8191], Qwen3-8B layer, "
                               "32768-block cache", "tokens": T,
                   "l2": f"{step_bytes / 1e6:.0f} MB per step: the step fits in L2 "
                         "(decode steps are launch- and latency-bound)"},
        "graph": {"us_per_step": round(1e3 * graph_ms, 2),
                  "eager_us_per_step": round(1e3 * eager_ms, 2),
                  "note": "value is the CUDA-graph replay of the five launches; eager is the "
                          "same step launched from Python"},
        "roofline": roofline("hbm", "whole step (5 kernels)", gbs, "GB/s",
                             algorithmic_bytes_per_launch=step_bytes),
        "clocks": clocks, "reference_gpu": ref, "e2e": e2e, "cpu_baseline": cpu,
        "validation": {"validated": all(c["ok"] for c in checks.values()), "rows_checked": T,
                       "checks": checks},
        "gpu_launches": 5 * n,
    }


def row_c5(args, rank: int, world: int, local_rank: int, as_row: bool = False) -> dict:
    """Config c5 at its full token count on one GPU: Qwen3-32B layer shapes,
    4 x 32768-token prefill (131072 tokens), with the paged cache as large as
    the GPU holds next to the step's tensors (up to the configuration's 1.835 M
    blocks, 120 GB).  Also times the standalone KV store (this library's and
    the reference's Triton kernel) into that cache."""
    import tinyserver_b200 as tsb
    from tinyserver_b200 import workloads as W

    dev = torch.device("cuda", local_rank)
    cfg = W.CONFIGS["c5"]
    s = cfg.shape
    T = 4 * 32768
    elem = 2
    inputs = (T * (3 * s.hidden + (s.num_q_heads + 2 * s.num_kv_heads) * s.head_dim
                   + 2 * s.intermediate) + s.vocab * s.hidden) * elem
    outputs = T * (5 * s.hidden + s.num_q_heads * s.head_dim + s.intermediate) * elem
    block_bytes = 2 * s.num_kv_heads * cfg.block_size * s.head_dim * elem
    free = torch.cuda.mem_get_info(dev)[0]
    margin = 12 * 2 ** 30  # store sources, allocator slack, the oracle's sampled rows
    blocks = int(min(cfg.num_blocks, (free - inputs - outputs - margin) // block_bytes))
    if blocks < 8192 * 2:
        raise MemoryError(f"c5: only {free / 1e9:.0f} GB free")
    batch = W.make_batch(cfg, dev, num_blocks=blocks, poison_cache=False)
    t = batch.tensors
    step = Step(batch)
    bpt = step.bytes_per_token()
    step_bytes = sum(bpt.values()) * T
    ms, clocks = timed(lambda: step.run(t), max(3, min(args.steps, 10)), 2, local_rank)
    tsb.check_errors(dev)
    # sampled rows against the oracle
    rows = torch.arange(0, T, 512, device=dev)
    exp = _expected_rows(t, rows, s, cfg.dtype)
    got = _sample_rows(step.run(t), t, rows).cpu()
    widths = [s.hidden, s.num_q_heads * s.head_dim, s.hidden, s.hidden, s.intermediate,
              s.num_kv_heads * s.head_dim, s.num_kv_heads * s.head_dim]
    col, checks = 0, {}
    for name, w in zip(_OUT_ORDER, widths):
        checks[name] = _within(got[:, col:col + w], exp[name].reshape(rows.numel(), -1),
                               name in _EXACT)
        col += w
    del exp, got
    # the standalone store (store_kv_cache_batched) into the same cache: K/V
    # sources as the reference's caller makes them, (Hkv, T, D) contiguous
    _, k, v = W.qkv_views(t["qkv"], s)
    k_src, v_src = k.transpose(0, 1).contiguous(), v.transpose(0, 1).contiguous()
    bm, sm = t["block_mapping"], t["slot_mapping"]
    store_bytes = 4 * T * s.num_kv_heads * s.head_dim * elem + 16 * T
    st_ms, st_clocks = timed(lambda: tsb.store_kv_cache_batched(k_src, v_src, t["k_cache"],
                                                                 t["v_cache"], bm, sm),
                             10, 3, local_rank)
    tsb.check_errors(dev)
    from baseline import reference_gpu as R
    ref_store = _ref_timed(R.kv_store_batched,
                           lambda fn: fn(k_src, v_src, t["k_cache"], t["v_cache"], bm, sm),
                           10, local_rank, st_ms,
                           lambda m: (store_bytes / (m * 1e-3) / 1e9, "GB/s"))
    kv_store = {
        "metric": "standalone store_kv_cache_batched GB/s (c5 K/V into the c5 cache)",
        "us": round(1e3 * st_ms, 2),
        "roofline": roofline("hbm", "kv_store_batched", store_bytes / (st_ms * 1e-3) / 1e9,
                             "GB/s", algorithmic_bytes_per_launch=store_bytes),
        "clocks": st_clocks, "reference_gpu": ref_store,
        "note": "sources 2 x 268 MB (> L2), rows scattered over the whole cache; the "
                "reference's Triton kernel gets the same tensors"}
    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_baseline(batch, budget_s=min(args.cpu_seconds, 3.0), max_tokens=2048,
                           compact_cache=True)
    gbs = step_bytes / (ms * 1e-3) / 1e9
    return {
        "metric": "fused-layer tokens/s and HBM GB/s per B200 (c5, Qwen3-32B shapes)",
        "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 4),
        "dtype": "bf16",
        "config": {"workload": "c5: 4 x 32768-token prefill (131072 tokens) on one GPU, "
                               f"Qwen3-32B layer, {blocks}-block cache "
                               f"({blocks * block_bytes / 1e9:.0f} GB"
                               + ("" if blocks == cfg.num_blocks else
                                  f"; the configuration's {cfg.num_blocks} blocks do not fit "
                                  "beside the step's tensors") + ")",
                   "tokens": T, "num_blocks": blocks,
                   "l2": f"{step_bytes / 1e9:.1f} GB moved per step (> L2)"},
        "roofline": roofline("hbm", "whole step (5 kernels)", gbs, "GB/s",
                             algorithmic_bytes_per_launch=step_bytes),
        "clocks": clocks,
        "validation": {"validated": all(c["ok"] for c in checks.values()),
                       "rows_checked": int(rows.numel()), "every": 512, "checks": checks},
        "kv_store": kv_store, "gpu_launches": 5, "cpu_baseline": cpu,
        "e2e_note": "no end-to-end leg at c5: a step's host buffers would be ~34 GB",
    }


# ----------------------------------------------------------------------------
def _reference_inputs(batch, n_tokens: int, device="cpu"):
    """The first n_tokens of the batch (CPU copies) for the reference CPU path."""
    t = batch.tensors
    sl = slice(0, n_tokens)
    keys = ["input_ids", "positions", "x_mlp", "residual", "qkv", "attn_out", "gate_up",
            "block_mapping", "slot_mapping"]
    out = {k: t[k][sl].to(device) for k in keys}
    return out


def _cpu_cache(batch, dtype, num_blocks: int | None = None):
    """K and V caches of the batch's full geometry (65536 blocks at c4) on the
    host, left unfilled: the store touches only its rows, as on the GPU."""
    s = batch.cfg.shape
    N = num_blocks or (batch.tensors["k_cache"].shape[0] if "k_cache" in batch.tensors
                       else batch.cfg.num_blocks)
    kc = torch.empty(N, s.num_kv_heads, batch.cfg.block_size, s.head_dim, dtype=dtype)
    return kc, torch.empty_like(kc)


def cpu_baseline(batch, budget_s: float = 10.0, threads: int | None = None,
                 max_tokens: int | None = None, compact_cache: bool = False) -> dict:
    """Time the reference's CPU path (transformers modules + index_put store) on
    the batch (or its first ``max_tokens`` tokens) for about ``budget_s``
    seconds; returns tokens/s.  The whole batch by default: a small sample
    would sit in the host caches and flatter the CPU.  ``compact_cache``
    stores into a cache of only the sample's blocks (for caches too large for
    host memory, c5's 120 GB)."""
    from oracle.ref_torch_cpu import ReferenceLayerPath

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    t = batch.tensors
    s = batch.cfg.shape
    weights = {"embed_weight": t["embed_weight"].to("cpu")}
    for k in ("input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"):
        weights[k] = t[k].to("cpu")
    ref = ReferenceLayerPath(s, batch.cfg.dtype, weights)
    n = batch.num_tokens if max_tokens is None else min(max_tokens, batch.num_tokens)
    inp = _reference_inputs(batch, n)
    bm = inp.pop("block_mapping")
    sm = inp.pop("slot_mapping")
    if compact_cache:
        uniq, bm = torch.unique(bm, return_inverse=True)
        kc, vc = _cpu_cache(batch, batch.cfg.dtype, num_blocks=len(uniq))
    else:
        kc, vc = _cpu_cache(batch, batch.cfg.dtype)

    def once():
        ref.step(inp["input_ids"], inp["positions"], inp["x_mlp"], inp["residual"], inp["qkv"],
                 inp["attn_out"], inp["gate_up"], kc, vc, bm, sm)

    once()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        once()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    cache = (f"a {kc.shape[0]}-block cache of only the sample's blocks" if compact_cache
             else f"the full {kc.shape[0]}-block cache")
    return {"value": round(n / med, 1), "unit": "tokens/s", "cores": threads,
            "kind": "reference",
            "sample": f"{n} tokens of {batch.cfg.name} per step, median of {len(times)} steps "
                      f"({sum(times):.1f} s); transformers {__import__('transformers').__version__}"
                      f" Qwen3 modules + torch index_put KV store into {cache}, bf16, "
                      f"torch.set_num_threads({threads})"}


def run_reference(args, rank: int) -> dict | None:
    """--impl reference: the reference's torch CPU path on the host cores."""
    if rank != 0:
        return None
    from tinyserver_b200 import workloads as W

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    batch = W.make_batch(CONFIG, "cpu", poison_cache=False)
    from oracle.ref_torch_cpu import ReferenceLayerPath

    t = batch.tensors
    s = batch.cfg.shape
    weights = {k: t[k] for k in ("embed_weight", "input_layernorm", "post_attention_layernorm",
                                 "q_norm", "k_norm")}
    ref = ReferenceLayerPath(s, batch.cfg.dtype, weights)
    kc, vc = t["k_cache"], t["v_cache"]  # the batch's own 65536-block cache

    def make(n):
        inp = _reference_inputs(batch, n)
        bm = inp.pop("block_mapping")
        sm = inp.pop("slot_mapping")
        return inp, bm, sm

    def run(pack):
        inp, bm, sm = pack
        ref.step(inp["input_ids"], inp["positions"], inp["x_mlp"], inp["residual"], inp["qkv"],
                 inp["attn_out"], inp["gate_up"], kc, vc, bm, sm)

    # size the per-step sample so the whole run stays near args.cpu_total seconds
    probe = make(64)
    run(probe)
    t0 = time.perf_counter()
    run(probe)
    per_tok = (time.perf_counter() - t0) / 64
    budget = args.cpu_total / max(1, args.steps + args.warmup)
    n = int(max(16, min(batch.num_tokens, budget / per_tok)))
    pack = make(n)
    for _ in range(args.warmup):
        run(pack)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run(pack)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = n * args.steps / total
    bpt = W.bytes_per_token(s)
    step_bytes = (sum(bpt.values()) + bpt["add_rmsnorm"]) * batch.num_tokens  # two add+norms
    config = layer_config(1, batch.num_tokens, step_bytes)
    config.pop("l2")
    config.update({"workload": "c4: Qwen3-8B layer, mixed 32x192 prefill + 2048 decode = "
                               f"8192 tokens/GPU; each step a {n}-token sample of that batch",
                   "tokens_per_step": n, "parallelism": "host CPU, rank 0 only"})
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded torch.Generator inputs of config c4",
        "config": config,
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": threads,
                         "kind": "reference",
                         "sample": f"{n} tokens of c4 per step on the host CPU: transformers "
                                   "Qwen3 modules + torch index_put KV store into the full "
                                   f"{kc.shape[0]}-block cache (the reference's Triton store "
                                   "has no CPU path)"},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    return line


# ----------------------------------------------------------------------------
def decode_attention_batch(dev, rank: int = 0):
    """Config c3's decode attention step with every sequence's context in
    blocks of its own: 256 sequences, one new token each at positions
    U[1, 8191] (context = position + 1), Qwen3-8B heads, 16-token pages.  The
    cache has exactly the blocks the contexts need (a seeded permutation of
    them), so no two sequences share a block and every K/V byte comes from
    HBM once."""
    from tinyserver_b200 import workloads as W

    cfg = W.CONFIGS["c3"]
    s = cfg.shape
    B = cfg.block_size
    pos = torch.tensor([p for _, p in W.sequences(cfg, rank)])
    lens = (pos + 1).to(torch.int32)
    per = ((lens + B - 1) // B).tolist()
    N = sum(per)
    g = torch.Generator().manual_seed(W.seed_of(cfg, rank) + 23)
    perm = torch.randperm(N, generator=g).to(torch.int32)
    bt = torch.zeros(len(per), max(per), dtype=torch.int32)
    at = 0
    for i, n in enumerate(per):
        bt[i, :n] = perm[at:at + n]
        at += n
    gd = torch.Generator(device=dev).manual_seed(W.seed_of(cfg, rank) + 5)
    pool = torch.randn(2, N, s.num_kv_heads, B, s.head_dim, generator=gd, device=dev,
                       dtype=torch.float32).to(cfg.dtype)
    q = torch.randn(len(per), s.num_q_heads, s.head_dim, generator=gd, device=dev,
                    dtype=torch.float32).to(cfg.dtype)
    return cfg, q, pool, bt.to(dev), lens


def run_attention(args, rank: int, world: int, local_rank: int, as_row: bool = False) -> dict | None:
    """--workload attn: decode paged attention (the next row after the fused
    path) on config c3's decode step with disjoint blocks (see
    decode_attention_batch).  Algorithmic bytes: every context token's K and V
    row of every kv head once, plus q, out and the block tables."""
    import tinyserver_b200 as tsb

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg, q, pool, bt, lens = decode_attention_batch(dev, rank)
    s = cfg.shape
    S, Hq, Hkv, D, B = q.shape[0], s.num_q_heads, s.num_kv_heads, s.head_dim, cfg.block_size
    sl = lens.to(dev)
    ws = torch.empty(tsb.paged_attention_workspace_bytes(S, Hq, D, bt.shape[1] * B) // 4 + 1,
                     dtype=torch.float32, device=dev)
    steps = min(args.steps, 50) if as_row else args.steps

    def once():
        return tsb.paged_attention_forward(q, pool[0], pool[1], bt, B, sl, workspace=ws)

    for _ in range(max(args.warmup, 3)):
        once()
    tsb.check_errors(dev)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank).start()
    ms, steps = event_loop(once, steps, 0.25 if as_row else 0.0)
    clocks = sampler.stop()
    tsb.check_errors(dev)
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        ms = float(m.item())
    per_ms = ms / steps

    # end to end: the step's queries, block tables and lengths from pinned host
    # memory, the output back; the KV cache is device state, as in the engine
    e2e = None
    if not args.no_e2e:
        hq_, hbt, hsl = q.cpu().pin_memory(), bt.cpu().pin_memory(), sl.cpu().pin_memory()
        dq, dbt, dsl = torch.empty_like(q), torch.empty_like(bt), torch.empty_like(sl)
        out_h = torch.empty(S, Hq, D, dtype=cfg.dtype).pin_memory()

        def e2e_once():
            for d, h in ((dq, hq_), (dbt, hbt), (dsl, hsl)):
                d.copy_(h, non_blocking=True)
            out_h.copy_(tsb.paged_attention_forward(dq, pool[0], pool[1], dbt, B, dsl,
                                                    workspace=ws), non_blocking=True)

        for _ in range(3):
            e2e_once()
        torch.cuda.synchronize()
        n_e2e = max(10, min(steps, 50))
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(n_e2e):
            e2e_once()
        a1.record()
        torch.cuda.synchronize()
        e2e_ms = a0.elapsed_time(a1) / n_e2e
        e2e = {"value": round(world * S / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
               "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": int(q.numel() * 2 + bt.numel() * bt.element_size()
                                         + sl.numel() * 4),
               "d2h_bytes_per_step": S * Hq * D * 2}
    if rank != 0:
        return None
    ctx = int(lens.sum())
    nbytes = ctx * Hkv * D * 2 * 2 + 2 * S * Hq * D * 2 + S * (bt.shape[1] + 1) * 4

    # CPU baseline: the restated reference kernel on the host cores over
    # groups of 8 sequences for a bounded time, scaled to the batch by
    # context tokens (the work is one K and V row per context token)
    cpu = None
    if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
        from oracle import oracle
        kc, vc, qh, bth = pool[0].cpu(), pool[1].cpu(), q.cpu(), bt.cpu()
        budget = min(args.cpu_seconds, 3.0 if as_row else 10.0)
        done, c0, i = 0, time.perf_counter(), 0
        while True:
            lo = (8 * i) % S
            oracle.paged_attention_decode(qh[lo:lo + 8], kc, vc, bth[lo:lo + 8], B,
                                          lens[lo:lo + 8])
            done += int(lens[lo:lo + 8].sum())
            i += 1
            secs = time.perf_counter() - c0
            if secs > budget:
                break
        rate = done / secs
        cpu = {"value": round(S / (ctx / rate), 1), "unit": "tokens/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{8 * i} sequences of the batch in groups of 8 ({done} context tokens "
                         f"in {secs:.1f} s), scaled to the batch's {ctx} context tokens; the "
                         "reference kernel's algorithm restated in torch on the host cores"}
    ref = None
    if world == 1 and not args.no_reference_gpu:
        from baseline import reference_gpu as R
        ref = _ref_timed(R.paged_attention_forward,
                         lambda fn: fn(q, pool[0], pool[1], bt, B, sl), 20, local_rank, per_ms,
                         lambda m: (S / (m * 1e-3), "tokens/s"))
        ref["what"] = ("the reference's Triton paged_attention_forward "
                       "(server/model/kernels/paged_attention.py) on the same batch")
    gbs = nbytes / (per_ms * 1e-3) / 1e9
    return {
        "metric": "decode paged attention tokens/s and HBM GB/s per B200, Qwen3-8B heads",
        "value": round(world * S / (per_ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded positions and cache contents of config c3",
        "config": {"workload": "c3 decode attention: 256 sequences x 1 token, context "
                               f"{ctx} tokens in all, every sequence in blocks of its own "
                               f"({pool.shape[1]} blocks of 16 tokens)",
                   "context_tokens": ctx, "num_blocks": int(pool.shape[1]),
                   "l2": f"{nbytes / 1e9:.2f} GB read per step (> L2), no block shared"},
        "roofline": roofline("hbm", "paged_decode_mma_kernel + merge", gbs, "GB/s",
                             ncu_traffic("paged_attention_disjoint"),
                             algorithmic_bytes_per_launch=nbytes),
        "cpu_baseline": cpu, "e2e": e2e, "reference_gpu": ref, "gpu_launches": 2 * steps,
        "clocks": clocks,
    }


def run_prefill(args, rank: int, world: int, local_rank: int, as_row: bool = False) -> dict | None:
    """--workload prefill: causal varlen prefill attention on config c2: 16
    packed sequences of U[128, 2048] tokens, Qwen3-1.7B heads (16 q / 8 kv,
    head_dim 128), bf16.  A contraction, so the roofline is the tensor-core
    one: FLOPs = sum over sequences and query heads of 4 * D * L(L+1)/2
    (QK^T and PV over the causal half) against the measured bf16 peak."""
    import tinyserver_b200 as tsb
    from tinyserver_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = W.CONFIGS["c2"]
    s = cfg.shape
    lens = [n for n, _ in W.sequences(cfg, rank)]
    T, Hq, Hkv, D = sum(lens), s.num_q_heads, s.num_kv_heads, s.head_dim
    g = torch.Generator(device=dev).manual_seed(W.seed_of(cfg, rank) + 9)
    # two input sets alternate (q/k/v 120 MB each, 240 MB together, more than
    # the 126 MB L2), so a step's inputs were last touched two steps earlier
    sets = []
    for _ in range(2):
        q = torch.randn(T, Hq, D, generator=g, device=dev).to(cfg.dtype)
        k = torch.randn(T, Hkv, D, generator=g, device=dev).to(cfg.dtype)
        v = torch.randn(T, Hkv, D, generator=g, device=dev).to(cfg.dtype)
        sets.append((q, k, v))
    in_mb = sum(t.numel() * t.element_size() for t in sets[0]) / 1e6
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    cu = cu.to(dev)
    L = max(lens)
    step = [0]
    steps = min(args.steps, 50) if as_row else args.steps

    def once():
        q, k, v = sets[step[0] % 2]
        step[0] += 1
        return tsb.flash_attn_varlen_func(q, k, v, cu, cu, L, L, causal=True)

    for _ in range(max(args.warmup, 3)):
        once()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank).start()
    ms, steps = event_loop(once, steps, 0.25 if as_row else 0.0)
    clocks = sampler.stop()
    tsb.check_errors(dev)
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        ms = float(m.item())
    flops = sum(4 * D * n * (n + 1) // 2 for n in lens) * Hq
    per_ms = ms / steps

    # end to end: q, k, v and cu_seqlens from pinned host memory, the output
    # back to pinned host memory, every step
    e2e = None
    if not args.no_e2e:
        hq_, hk_, hv_ = (t.cpu().pin_memory() for t in sets[0])
        hcu = cu.cpu().pin_memory()
        dq, dk, dv, dcu = (torch.empty_like(t) for t in (*sets[0], cu))
        out_h = torch.empty(T, Hq, D, dtype=cfg.dtype).pin_memory()

        def e2e_once():
            for d, h in ((dq, hq_), (dk, hk_), (dv, hv_), (dcu, hcu)):
                d.copy_(h, non_blocking=True)
            out_h.copy_(tsb.flash_attn_varlen_func(dq, dk, dv, dcu, dcu, L, L, causal=True),
                        non_blocking=True)

        for _ in range(3):
            e2e_once()
        torch.cuda.synchronize()
        n_e2e = max(10, min(steps, 20))
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(n_e2e):
            e2e_once()
        a1.record()
        torch.cuda.synchronize()
        e2e_ms = a0.elapsed_time(a1) / n_e2e
        e2e = {"value": round(world * T / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
               "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": int(sum(t.numel() * t.element_size() for t in sets[0])
                                         + cu.numel() * 4),
               "d2h_bytes_per_step": T * Hq * D * 2}
    if rank != 0:
        return None

    # CPU baseline: whole sequences of the batch, in order, through the
    # restatement of the reference's kernel (32-key blocks, torch on the host
    # cores) for a bounded time; FLOP rate scaled to the batch
    cpu = None
    if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
        from oracle import oracle
        cq_h, ck_h, cv_h = (t.cpu() for t in sets[0])
        offs = [0]
        for n in lens:
            offs.append(offs[-1] + n)
        budget = min(args.cpu_seconds, 3.0 if as_row else 10.0)
        done, c0, i = 0, time.perf_counter(), 0
        while True:
            n, o = lens[i % len(lens)], offs[i % len(lens)]
            c1 = torch.tensor([0, n], dtype=torch.int32)
            oracle.varlen_attention(cq_h[o:o + n], ck_h[o:o + n], cv_h[o:o + n], c1, c1, True)
            done += 4 * D * n * (n + 1) // 2 * Hq
            i += 1
            secs = time.perf_counter() - c0
            if secs > budget:
                break
        rate = done / secs
        cpu = {"value": round(T / (flops / rate), 1), "unit": "tokens/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{i} whole sequences of the batch in order ({done / 1e9:.1f} GFLOP in "
                         f"{secs:.1f} s, {rate / 1e9:.2f} GFLOP/s), scaled to the batch's "
                         f"{flops / 1e9:.0f} GFLOP; the reference kernel's algorithm restated "
                         "in torch on the host cores"}
    ref = None
    if world == 1 and not args.no_reference_gpu:
        from baseline import reference_gpu as R
        q0, k0, v0 = sets[0]
        ref = _ref_timed(R.flash_attn_varlen_func,
                         lambda fn: fn(q0, k0, v0, cu, cu, L, L, True), 10, local_rank, per_ms,
                         lambda m: (T / (m * 1e-3), "tokens/s"))
        if "ms_per_step" in ref:
            ref["tflops"] = round(flops / (ref["ms_per_step"] * 1e-3) / 1e12, 1)
        ref["what"] = ("the reference's Triton flash_attn_varlen_func "
                       "(server/model/kernels/varlen_attention.py) on the same batch")
    tf = flops / (per_ms * 1e-3) / 1e12
    return {
        "metric": "prefill varlen attention tokens/s and TFLOP/s per B200, Qwen3-1.7B heads",
        "value": round(world * T / (per_ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded lengths and activations of config c2",
        "config": {"workload": f"c2 prefill attention: {len(lens)} sequences, {T} tokens, causal",
                   "tokens": T, "max_seqlen": L,
                   "l2": f"two input sets alternate: {2 * in_mb:.0f} MB of q/k/v between reuses "
                         f"> 126 MB L2"},
        "roofline": roofline("tensor", "varlen_attn_tc_kernel", tf, "TFLOP/s",
                             ncu_traffic("varlen_attn_tc_kernel"), flops_per_launch=flops),
        "cpu_baseline": cpu, "e2e": e2e, "reference_gpu": ref, "gpu_launches": steps,
        "clocks": clocks,
    }


SAMPLE_ROWS, SAMPLE_VOCAB = 256, 151936


def _sample_inputs(B: int, V: int, seed: int, device) -> tuple:
    """One decode step's sampling inputs: bf16 logits N(0, 4^2) (a spread LM
    distribution), per-row mixed settings -- 1 in 8 rows greedy, temperature
    0.6..1.2, top-k off/20/50/1000, top-p off/0.9/0.95 -- and counter-hash
    uniforms."""
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(B, V, generator=g) * 4.0).to(torch.bfloat16)
    pick = lambda vals: torch.tensor(vals)[torch.randint(0, len(vals), (B,), generator=g)]  # noqa
    temperature = pick([0.0, 0.6, 0.7, 0.8, 0.9, 1.0, 1.0, 1.2]).float()
    top_k = pick([0, 0, 20, 50, 1000]).long()
    top_p = pick([1.0, 0.9, 0.95, 0.95]).float()
    seeds = torch.randint(0, 2 ** 62, (B,), generator=g)
    return (logits.to(device), temperature.to(device), top_k.to(device), top_p.to(device),
            seeds.to(device), torch.full((B,), seed, dtype=torch.int64, device=device))


def run_sample(args, rank: int, world: int, local_rank: int, as_row: bool = False) -> dict | None:
    """--workload sample: the batched sampler after lm_head on a c3-sized
    decode step: 256 rows of Qwen3's 151936-token vocabulary, bf16 logits,
    mixed greedy / temperature / top-k / top-p rows, counter-hash noise fused
    into the launch.  Three logits buffers (233 MB together, larger than L2)
    rotate so every step reads its logits from HBM.  Roofline: HBM, on the
    logits bytes read once per launch."""
    import tinyserver_b200 as tsb

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    B, V = args.sample_rows, SAMPLE_VOCAB
    sets = [_sample_inputs(B, V, 1000 * rank + i, dev) for i in range(3)]
    steps = min(args.steps, 50) if as_row else args.steps

    from tinyserver_b200.kernels import sampling as S
    path = "wide" if S.WIDE_MIN_ROWS <= B <= S.WIDE_MAX_ROWS else "cluster"

    def once(i, how="auto"):
        x, t, k, p, sd, st = sets[i % 3]
        return tsb.sample_tokens_seeded(x, t, k, p, sd, st, path=how)

    for i in range(max(args.warmup, 3)):
        once(i)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    sampler = ClockSampler(local_rank).start()
    counter = [0]

    def next_step():
        once(counter[0])
        counter[0] += 1

    ms, steps = event_loop(next_step, steps, 0.25 if as_row else 0.0)
    clocks = sampler.stop()
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        ms = float(m.item())
    per_ms = ms / steps
    # the other path on the same batches, for comparison (not the value)
    other = "cluster" if path == "wide" else "wide"
    for i in range(3):
        once(i, other)
    torch.cuda.synchronize()
    counter[0] = 0
    ms_o, steps_o = event_loop(lambda: (once(counter[0], other),
                                        counter.__setitem__(0, counter[0] + 1)), steps)
    other_ms = ms_o / steps_o

    # end to end: logits from pinned host memory, tokens back to the host
    e2e = None
    if not args.no_e2e:
        host = [s[0].cpu().pin_memory() for s in sets[:2]]
        dbuf = [torch.empty_like(s[0]) for s in sets[:2]]
        out_h = torch.empty(B, dtype=torch.int64).pin_memory()
        n_e2e = max(10, min(steps, 50))
        _, t, k, p, sd, st = sets[0]
        for i in range(3):
            dbuf[i % 2].copy_(host[i % 2], non_blocking=True)
            out_h.copy_(tsb.sample_tokens_seeded(dbuf[i % 2], t, k, p, sd, st), non_blocking=True)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for i in range(n_e2e):
            dbuf[i % 2].copy_(host[i % 2], non_blocking=True)
            out_h.copy_(tsb.sample_tokens_seeded(dbuf[i % 2], t, k, p, sd, st), non_blocking=True)
        a1.record()
        torch.cuda.synchronize()
        e2e_ms = a0.elapsed_time(a1) / n_e2e
        e2e = {"value": round(world * B / (e2e_ms * 1e-3), 1), "unit": "rows/s",
               "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": B * V * 2,
               "d2h_bytes_per_step": B * 8}
    if rank != 0:
        return None

    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle
        x, t, k, p, sd, st = (s.cpu() for s in sets[0])
        n = 32
        u = oracle.uniforms_from_seeds(sd[:n].tolist(), st[:n].tolist())
        oracle.sample_tokens(x[:4], t[:4], k[:4], p[:4], u[:4])
        budget = min(args.cpu_seconds, 3.0 if as_row else 10.0)
        c0 = time.perf_counter()
        reps = 0
        while True:
            oracle.sample_tokens(x[:n], t[:n], k[:n], p[:n], u)
            reps += 1
            if time.perf_counter() - c0 > budget:
                break
        cs = (time.perf_counter() - c0) / reps
        cpu = {"value": round(n / cs, 1), "unit": "rows/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"{n} rows of the same batch, {reps} repetitions, the "
                                         "reference's sort-based sample_tokens restated in torch "
                                         "on the host cores"}
    ref = None
    if world == 1 and not args.no_reference_gpu:
        from baseline import reference_gpu as R
        x, t, k, p, sd, st = sets[0]
        u = tsb.uniforms_from_seeds(sd, st)
        ref = _ref_timed(R.sample_tokens, lambda fn: fn(x, t, k, p, u), 20, local_rank, per_ms,
                         lambda m: (B / (m * 1e-3), "rows/s"))
        ref["what"] = ("the reference's sample_tokens (server/model/sampling.py, torch sort, "
                       "softmax and cumsum on the GPU) on the same logits and uniforms")
    nbytes = B * V * 2 + B * (4 + 8 + 4 + 8 + 8 + 8)
    gbs = nbytes / (per_ms * 1e-3) / 1e9
    return {
        "metric": "sampled rows/s per B200 (Qwen3 vocabulary, top-k/top-p/temperature mix)",
        "value": round(world * B / (per_ms * 1e-3), 1), "unit": "rows/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded bf16 logits N(0, 16), mixed per-row sampling settings",
        "config": {"workload": f"c3 decode step sampling: {B} rows x {V} vocab, bf16 logits"
                               + ("" if B == SAMPLE_ROWS else " (a profiling case, not the benchmark)"),
                   "rows": B, "vocab": V, "l2": "3 rotating logits buffers (233 MB > L2)"},
        "roofline": roofline("hbm", "batch-wide sampler (5 kernels + cluster kernel for the rows "
                             "it leaves)" if path == "wide" else "sample_kernel", gbs, "GB/s",
                             ncu_traffic("sampler_batch_wide" if path == "wide" else "sample_kernel"),
                             bytes_per_launch=nbytes),
        "path": {"taken": path, "ms_per_step": {path: round(per_ms, 4),
                                                other: round(other_ms, 4)},
                 "note": "both paths give identical tokens; value is the taken path"},
        "cpu_baseline": cpu, "e2e": e2e, "reference_gpu": ref,
        "gpu_launches": steps * (6 if path == "wide" else 1),
        "clocks": clocks,
    }


# ----------------------------------------------------------------------------
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-validate", action="store_true",
                    help="skip the check of sampled outputs against the oracle")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU code")
    ap.add_argument("--no-rows", action="store_true",
                    help="skip the other configurations and rows (N=1 only)")
    ap.add_argument("--max-tokens", type=int, default=None,
                    help="keep a prefix of the batch (small profiling cases only)")
    ap.add_argument("--num-blocks", type=int, default=None,
                    help="KV-cache blocks per GPU (small profiling cases only)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline timing budget (ours arm)")
    ap.add_argument("--cpu-total", type=float, default=90.0,
                    help="total CPU time budget of the --impl reference run")
    ap.add_argument("--sample-rows", type=int, default=SAMPLE_ROWS,
                    help="rows of --workload sample (small profiling cases only)")
    ap.add_argument("--workload", choices=["layer", "attn", "prefill", "sample", "c3", "c5"],
                    default="layer",
                    help="layer: the fused-layer step (the headline); attn: decode attention; "
                         "prefill: varlen prefill attention; sample: the batched sampler; "
                         "c3 / c5: the fused step on those configurations")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        fn = {"attn": run_attention, "prefill": run_prefill, "sample": run_sample,
              "c3": row_c3_step, "c5": row_c5}.get(args.workload)
        if fn is None:
            line = run_ours(args, rank, world, local_rank)
        elif args.workload in ("c3", "c5"):
            torch.cuda.set_device(local_rank)
            line = fn(args, rank, world, local_rank) if rank == 0 else None
        else:
            line = fn(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
