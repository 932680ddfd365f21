"""bench.py's host-side helpers (no GPU): the parity check its validation
leg applies, the guard around its optional legs, and the compact row form."""

import torch

import bench


def test_within_exact_and_tolerance():
    e = torch.tensor([1.0, -2.0, 0.5, 100.0]).to(torch.bfloat16)
    assert bench._within(e.clone(), e, exact=True)["ok"]
    a = e.clone()
    a[3] = 101.0  # within 2e-2 + 1e-2 * 100
    r = bench._within(a, e, exact=False)
    assert r["ok"] and r["mismatched"] == 1 and r["bit_exact"] == 0.75
    assert not bench._within(a, e, exact=True)["ok"]
    a[0] = 1.5  # outside 2e-2 + 1e-2 * 1
    assert not bench._within(a, e, exact=False)["ok"]
    a[0] = float("nan")
    assert not bench._within(a, e, exact=False)["ok"]


def test_guarded_records_the_error_instead_of_raising():
    def boom():
        raise RuntimeError("no Triton here")

    assert bench.guarded(lambda x: x + 1, 1) == 2
    r = bench.guarded(boom)
    assert r == {"error": "RuntimeError: no Triton here"}


def test_compact_row_keeps_the_reported_fields():
    line = {"metric": "m", "value": 1.0, "unit": "u", "roofline": {"frac": 0.5}, "clocks": {},
            "n_gpus": 1, "vs_baseline": None, "kv_store": {"us": 2}}
    c = bench._compact(line)
    assert c == {"metric": "m", "value": 1.0, "unit": "u", "roofline": {"frac": 0.5},
                 "clocks": {}, "kv_store": {"us": 2}}


def test_layer_config_names_the_workload():
    cfg = bench.layer_config(2, 8192, 1_477_000_000)
    assert cfg["global_tokens"] == 16384 and cfg["num_blocks"] == 65536
    assert "token-sharded x2" in cfg["parallelism"]
