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


# ----------------------------------------------------------------------------
def hbm_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


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
def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    from tinyserver_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    batch = W.make_batch(CONFIG, dev, shard=rank, max_tokens=args.max_tokens,
                         num_blocks=args.num_blocks)
    t = batch.tensors
    T = batch.num_tokens
    step = Step(batch)
    bpt = step.bytes_per_token()
    step_bytes = sum(bpt.values()) * T

    import tinyserver_b200 as tsb
    tsb.load_library()
    for _ in range(max(args.warmup, 3)):
        step.run(t)
    tsb.check_errors(dev)
    torch.cuda.synchronize()

    # ---- device-resident timing: the headline --------------------------------
    # K steps back to back between two events; nothing is recorded between
    # the kernels, so consecutive launches keep their programmatic-dependent-
    # launch overlap.
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank).start()
    time.sleep(0.05)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start.record()
    for _ in range(args.steps):
        step.run(t)
    stop.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(stop)
    tsb.check_errors(dev)
    if world > 1:
        m = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        elapsed_ms = float(m.item())

    # ---- per-kernel attribution: a second timed pass with an event between
    # every two kernels (on the launch stream); these events serialise the
    # launches, so this pass runs a little slower than the headline pass.
    nk = len(Step.KERNELS)
    kb = min(args.steps, 200)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] for _ in range(kb)]
    torch.cuda.synchronize()
    for i in range(kb):
        step.run(t, evs[i])
    torch.cuda.synchronize()
    per_kernel_us = {}
    for j, name in enumerate(Step.KERNELS):
        per_kernel_us[name] = 1e3 * sum(e[j].elapsed_time(e[j + 1]) for e in evs) / kb
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
    traffic = ncu_traffic(dom)
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
        "config": {
            "workload": "c4: Qwen3-8B layer, mixed 32x192 prefill + 2048 decode = "
                        "8192 tokens/GPU, 16-token pages, 65536 blocks/GPU",
            "tokens_per_gpu": T, "global_tokens": world * T, "hidden": 4096,
            "num_q_heads": 32, "num_kv_heads": 8, "head_dim": 128, "intermediate": 12288,
            "parallelism": f"token-sharded x{world}, no collective on the timed path",
            "l2": f"inputs larger than L2: {step_bytes / 1e9:.2f} GB moved per step per GPU",
        },
        "hbm_gbs": round(step_bytes / (ms_per_step * 1e-3) / 1e9, 1),
        "hbm_frac": round(step_bytes / (ms_per_step * 1e-3) / 1e9 / peak, 4),
        "hbm_peak_gbs": peak,
        "hbm_peak_kind": peak_kind,
        "kernels": kernels,
        "kernels_note": "per-kernel CUDA-event times from a second pass with an event between "
                        f"every two launches ({kb} steps, {attributed_ms:.4f} ms per step); "
                        "the headline is the pass without them",
        "kernels_isolated": kernels_isolated,
        "kernels_isolated_note": "each kernel alone on the step's inputs, median of 20 launches, "
                                 "a 256 MB read between launches so its inputs come from HBM; "
                                 "its own writes may end in L2 (in the step, the next kernel "
                                 "pays that write-back)",
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(dom_gbs, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(dom_gbs / peak, 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6650 GB/s",
                     "algorithmic_bytes_per_launch": bpt[dom] * T,
                     "traffic": traffic},
        "gpu_launches": nk * args.steps,
        "pdl": "programmatic dependent launch between the step's kernels",
        "clocks": clocks,
        "e2e": None,
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
    if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
        line["cpu_baseline"] = cpu_baseline(batch, budget_s=args.cpu_seconds)
    return line


# ----------------------------------------------------------------------------
def _reference_inputs(batch, n_tokens: int, device="cpu"):
    """The first n_tokens of the batch (CPU copies) for the reference CPU path."""
    t = batch.tensors
    sl = slice(0, n_tokens)
    keys = ["input_ids", "positions", "x_mlp", "residual", "qkv", "attn_out", "gate_up",
            "block_mapping", "slot_mapping"]
    out = {k: t[k][sl].to(device) for k in keys}
    return out


def cpu_baseline(batch, budget_s: float = 10.0, threads: int | None = None,
                 max_tokens: int | None = None) -> dict:
    """Time the reference's CPU path (transformers modules + index_put store) on
    the batch (or its first ``max_tokens`` tokens) for about ``budget_s``
    seconds; returns tokens/s.  The whole batch by default: a small sample
    would sit in the host caches and flatter the CPU."""
    from oracle.ref_torch_cpu import ReferenceLayerPath

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    t = batch.tensors
    s = batch.cfg.shape
    weights = {"embed_weight": t["embed_weight"].to("cpu")}
    for k in ("input_layernorm", "post_attention_layernorm", "q_norm", "k_norm"):
        weights[k] = t[k].to("cpu")
    ref = ReferenceLayerPath(s, batch.cfg.dtype, weights)
    # a CPU cache large enough for the sample's slots (same page geometry)
    n = batch.num_tokens if max_tokens is None else min(max_tokens, batch.num_tokens)
    inp = _reference_inputs(batch, n)
    bm = inp.pop("block_mapping")
    sm = inp.pop("slot_mapping")
    uniq, bm_local = torch.unique(bm, return_inverse=True)
    kc = torch.zeros(len(uniq), s.num_kv_heads, batch.cfg.block_size, s.head_dim,
                     dtype=batch.cfg.dtype)
    vc = torch.zeros_like(kc)

    def once():
        ref.step(inp["input_ids"], inp["positions"], inp["x_mlp"], inp["residual"], inp["qkv"],
                 inp["attn_out"], inp["gate_up"], kc, vc, bm_local, sm)

    once()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        once()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": round(n / med, 1), "unit": "tokens/s", "cores": threads,
            "kind": "reference",
            "sample": f"{n} tokens of c4 per step, median of {len(times)} steps "
                      f"({sum(times):.1f} s); transformers {__import__('transformers').__version__}"
                      " Qwen3 modules + torch index_put KV store, bf16, "
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

    def make(n):
        inp = _reference_inputs(batch, n)
        bm = inp.pop("block_mapping")
        sm = inp.pop("slot_mapping")
        uniq, bm_local = torch.unique(bm, return_inverse=True)
        kc = torch.zeros(len(uniq), s.num_kv_heads, batch.cfg.block_size, s.head_dim,
                         dtype=batch.cfg.dtype)
        return inp, kc, torch.zeros_like(kc), bm_local, sm

    def run(pack):
        inp, kc, vc, bm, sm = pack
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
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded torch.Generator inputs of config c4",
        "config": {"workload": "c4: Qwen3-8B layer, mixed prefill+decode batch; each step a "
                               f"{n}-token sample of the 8192-token batch",
                   "tokens_per_step": n},
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": threads,
                         "kind": "reference",
                         "sample": f"{n} tokens of c4 per step on the host CPU: transformers "
                                   "Qwen3 modules + torch index_put KV store (the reference's "
                                   "Triton store has no CPU path)"},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    return line


# ----------------------------------------------------------------------------
def run_attention(args, rank: int, world: int, local_rank: int) -> dict | None:
    """--workload attn: decode paged attention (the next row after the fused
    path) on config c3: 256 sequences, one new token each at positions
    U[1, 8191] (context = position + 1), Qwen3-8B heads (32 q / 8 kv,
    head_dim 128), 16-token pages in a 32768-block cache, bf16.  Algorithmic
    bytes: every context token's K and V row of every kv head once, plus q
    and out."""
    import tinyserver_b200 as tsb
    from tinyserver_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = W.CONFIGS["c3"]
    s = cfg.shape
    b = W.index_data(cfg, shard=rank)
    lens = (b.positions + 1).to(torch.int32)  # each sequence's one token attends to 0..pos
    S, Hq, Hkv, D, B = len(b.seqs), s.num_q_heads, s.num_kv_heads, s.head_dim, cfg.block_size
    g = torch.Generator(device=dev).manual_seed(W.seed_of(cfg, rank) + 5)
    pool = torch.randn(2, cfg.num_blocks, Hkv, B, D, generator=g, device=dev,
                       dtype=torch.float32).to(cfg.dtype)
    q = torch.randn(S, Hq, D, generator=g, device=dev, dtype=torch.float32).to(cfg.dtype)
    bt = b.block_tables.to(dev)
    sl = lens.to(dev)
    ws = torch.empty(tsb.paged_attention_workspace_bytes(S, Hq, D, bt.shape[1] * B) // 4 + 1,
                     dtype=torch.float32, device=dev)

    def once():
        return tsb.paged_attention_forward(q, pool[0], pool[1], bt, B, sl, workspace=ws)

    for _ in range(max(args.warmup, 3)):
        once()
    tsb.check_errors(dev)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank).start()
    e0.record()
    for _ in range(args.steps):
        once()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    tsb.check_errors(dev)
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        ms = float(m.item())

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
        n_e2e = max(10, min(args.steps, 50))
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

    # CPU baseline: the restated reference kernel on the host cores over
    # groups of 8 sequences for about ten seconds, scaled to the batch by
    # context tokens (the work is one K and V row per context token)
    cpu = None
    if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
        from oracle import oracle
        kc, vc, qh, bth = pool[0].cpu(), pool[1].cpu(), q.cpu(), bt.cpu()
        done, c0, i = 0, time.perf_counter(), 0
        while True:
            lo = (8 * i) % S
            oracle.paged_attention_decode(qh[lo:lo + 8], kc, vc, bth[lo:lo + 8], B,
                                          lens[lo:lo + 8])
            done += int(lens[lo:lo + 8].sum())
            i += 1
            secs = time.perf_counter() - c0
            if secs > min(args.cpu_seconds, 10.0):
                break
        rate = done / secs
        cpu = {"value": round(S / (ctx / rate), 1), "unit": "tokens/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{8 * i} sequences of the batch in groups of 8 ({done} context tokens "
                         f"in {secs:.1f} s), scaled to the batch's {ctx} context tokens; the "
                         "reference kernel's algorithm restated in torch on the host cores"}
    peak, peak_kind = hbm_peak()
    nbytes = ctx * Hkv * D * 2 * 2 + 2 * S * Hq * D * 2 + S * (bt.shape[1] + 1) * 4
    per_ms = ms / args.steps
    gbs = nbytes / (per_ms * 1e-3) / 1e9
    return {
        "metric": "decode paged attention tokens/s and HBM GB/s per B200, Qwen3-8B heads",
        "value": round(world * S / (per_ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded positions and cache contents of config c3",
        "config": {"workload": "c3 decode attention: 256 sequences x 1 token, context "
                               f"{ctx} tokens in all, 16-token pages, 32768 blocks",
                   "context_tokens": ctx, "l2": f"{nbytes / 1e9:.2f} GB read per step (> L2)"},
        "roofline": {"bound": "hbm", "kernel": "paged_decode_mma_kernel + merge",
                     "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "algorithmic_bytes_per_launch": nbytes,
                     "traffic": ncu_traffic("paged_attention")},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": 2 * args.steps, "clocks": clocks,
    }


def tensor_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def run_prefill(args, rank: int, world: int, local_rank: int) -> dict | None:
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

    def once():
        q, k, v = sets[step[0] % 2]
        step[0] += 1
        return tsb.flash_attn_varlen_func(q, k, v, cu, cu, L, L, causal=True)

    for _ in range(max(args.warmup, 3)):
        once()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank).start()
    e0.record()
    for _ in range(args.steps):
        once()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        ms = float(m.item())
    flops = sum(4 * D * n * (n + 1) // 2 for n in lens) * Hq

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
        n_e2e = max(10, min(args.steps, 20))
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
    # cores) for about ten seconds; FLOP rate scaled to the batch
    cpu = None
    if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
        from oracle import oracle
        cq_h, ck_h, cv_h = (t.cpu() for t in sets[0])
        offs = [0]
        for n in lens:
            offs.append(offs[-1] + n)
        done, c0, i = 0, time.perf_counter(), 0
        while True:
            n, o = lens[i % len(lens)], offs[i % len(lens)]
            c1 = torch.tensor([0, n], dtype=torch.int32)
            oracle.varlen_attention(cq_h[o:o + n], ck_h[o:o + n], cv_h[o:o + n], c1, c1, True)
            done += 4 * D * n * (n + 1) // 2 * Hq
            i += 1
            secs = time.perf_counter() - c0
            if secs > min(args.cpu_seconds, 10.0):
                break
        rate = done / secs
        cpu = {"value": round(T / (flops / rate), 1), "unit": "tokens/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{i} whole sequences of the batch in order ({done / 1e9:.1f} GFLOP in "
                         f"{secs:.1f} s, {rate / 1e9:.2f} GFLOP/s), scaled to the batch's "
                         f"{flops / 1e9:.0f} GFLOP; the reference kernel's algorithm restated "
                         "in torch on the host cores"}
    per_ms = ms / args.steps
    tf = flops / (per_ms * 1e-3) / 1e12
    peak, kind = tensor_peak()
    return {
        "metric": "prefill varlen attention tokens/s and TFLOP/s per B200, Qwen3-1.7B heads",
        "value": round(world * T / (per_ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded lengths and activations of config c2",
        "config": {"workload": f"c2 prefill attention: {len(lens)} sequences, {T} tokens, causal",
                   "tokens": T, "max_seqlen": L,
                   "l2": f"two input sets alternate: {2 * in_mb:.0f} MB of q/k/v between reuses "
                         f"> 126 MB L2"},
        "roofline": {"bound": "tensor", "kernel": "varlen_attn_tc_kernel", "achieved": round(tf, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(tf / peak, 4),
                     "peak_source": f"{kind} bf16_tflops (cuBLAS burst)", "flops_per_launch": flops,
                     "traffic": ncu_traffic("varlen_attn_tc_kernel")},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks,
    }


SAMPLE_ROWS, SAMPLE_VOCAB = 256, 151936


def _sample_inputs(B: int, V: int, seed: int, device) -> tuple:
    """One decode step's sampling inputs: bf16 logits N(0, 4^2) (a spread LM
    distribution), per-row mixed settings -- 1 in 8 rows greedy, temperature
    0.6..1.2, top-k off/20/50/1000, top-p off/0.9/0.95 -- and counter-hash
    uniforms."""
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(B, V, generator=g) * 4.0).to(torch.bfloat16)
    pick = lambda vals: torch.tensor(vals)[torch.randint(0, len(vals), (B,), generator=g)]
    temperature = pick([0.0, 0.6, 0.7, 0.8, 0.9, 1.0, 1.0, 1.2]).float()
    top_k = pick([0, 0, 20, 50, 1000]).long()
    top_p = pick([1.0, 0.9, 0.95, 0.95]).float()
    seeds = torch.randint(0, 2 ** 62, (B,), generator=g)
    return (logits.to(device), temperature.to(device), top_k.to(device), top_p.to(device),
            seeds.to(device), torch.full((B,), seed, dtype=torch.int64, device=device))


def run_sample(args, rank: int, world: int, local_rank: int) -> dict | None:
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

    def once(i):
        x, t, k, p, sd, st = sets[i % 3]
        return tsb.sample_tokens_seeded(x, t, k, p, sd, st)

    for i in range(max(args.warmup, 3)):
        once(i)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank).start()
    e0.record()
    for i in range(args.steps):
        once(i)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        m = torch.tensor([ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(m, op=torch.distributed.ReduceOp.MAX)
        ms = float(m.item())

    # end to end: logits from pinned host memory, tokens back to the host
    e2e = None
    if not args.no_e2e:
        host = [s[0].cpu().pin_memory() for s in sets[:2]]
        dbuf = [torch.empty_like(s[0]) for s in sets[:2]]
        out_h = torch.empty(B, dtype=torch.int64).pin_memory()
        n_e2e = max(10, min(args.steps, 50))
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
        c0 = time.perf_counter()
        reps = 0
        while True:
            oracle.sample_tokens(x[:n], t[:n], k[:n], p[:n], u)
            reps += 1
            if time.perf_counter() - c0 > min(args.cpu_seconds, 10.0):
                break
        cs = (time.perf_counter() - c0) / reps
        cpu = {"value": round(n / cs, 1), "unit": "rows/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"{n} rows of the same batch, {reps} repetitions, the "
                                         "reference's sort-based sample_tokens restated in torch "
                                         "on the host cores"}

    per_ms = ms / args.steps
    nbytes = B * V * 2 + B * (4 + 8 + 4 + 8 + 8 + 8)
    gbs = nbytes / (per_ms * 1e-3) / 1e9
    peak, kind = hbm_peak()
    return {
        "metric": "sampled rows/s per B200 (Qwen3 vocabulary, top-k/top-p/temperature mix)",
        "value": round(world * B / (per_ms * 1e-3), 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded bf16 logits N(0, 16), mixed per-row sampling settings",
        "config": {"workload": f"c3 decode step sampling: {B} rows x {V} vocab, bf16 logits"
                               + ("" if B == SAMPLE_ROWS else " (a profiling case, not the benchmark)"),
                   "rows": B, "vocab": V, "l2": "3 rotating logits buffers (233 MB > L2)"},
        "roofline": {"bound": "hbm", "kernel": "sample_kernel", "achieved": round(gbs, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                     "peak_source": f"{kind} hbm_gbs", "bytes_per_launch": nbytes,
                     "traffic": ncu_traffic("sample_kernel")},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks,
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
    ap.add_argument("--workload", choices=["layer", "attn", "prefill", "sample"],
                    default="layer",
                    help="layer: the fused-layer step (the headline); attn: decode attention; "
                         "prefill: varlen prefill attention; sample: the batched sampler")
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
        if args.workload == "attn":
            line = run_attention(args, rank, world, local_rank)
        elif args.workload == "prefill":
            line = run_prefill(args, rank, world, local_rank)
        elif args.workload == "sample":
            line = run_sample(args, rank, world, local_rank)
        else:
            line = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
