"""bench.py's roofline bookkeeping on CPU: the dominant operator, its achieved rate against the
measured peak, and the per-launch DRAM traffic it takes from the committed capture summary."""

from __future__ import annotations

import importlib.util
import json
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
M, H, I, E = 98304, 2880, 2880, 32  # cfg3
PEAKS = {"hbm_gbs": 6545.0, "bf16_tflops": 1635.7, "bf16_tflops_sustained": 1355.9}


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ops(**ms):
    return {k: {"avg_ms": v, "total_ms": 20 * v, "launches": 20} for k, v in ms.items()}


def test_dominant_operator_and_rate(bench):
    ops = _ops(up_swiglu_fwd=2.68, down_fwd=1.41, up_wgrad_bias=2.61)
    e = bench.roofline_entry(ops, M, H, I, PEAKS, "measured", steps=20)
    assert e["kernel"] == "up_swiglu_fwd"
    flop = 4.0 * M * H * I
    assert e["algorithmic_flop_per_launch"] == pytest.approx(flop)
    assert e["achieved"] == pytest.approx(flop / 2.68e-3 / 1e12)
    assert e["frac"] == pytest.approx(e["achieved"] / PEAKS["bf16_tflops"])
    assert e["frac_of_sustained"] == pytest.approx(e["achieved"] / PEAKS["bf16_tflops_sustained"])
    assert set(e["ops"]) == set(ops)


def test_traffic_comes_from_the_dominant_operators_capture(bench):
    cap = json.loads((REPO / "profiles" / "launch_traffic_cfg3.json").read_text())
    for name in ("up_swiglu_fwd", "up_wgrad_bias", "down_dgrad_swiglu_bwd"):
        ops = _ops(**{name: 3.0, "down_fwd": 1.0})
        e = bench.roofline_entry(ops, M, H, I, PEAKS, "measured", steps=20)
        assert e["kernel"] == name
        assert e["traffic"] == cap["ops"][name]["bytes_per_launch"]
        assert "MB read" in e["traffic_source"]
    # the e4m3 line has no captured traffic; its peak is the e4m3 burst measured on the GPU, the
    # nominal dense figure only when none was measured
    e = bench.roofline_entry(_ops(up_swiglu_fwd=1.5), M, H, I, PEAKS, "measured", fp8=True, steps=20,
                             fp8_peak=3040.0)
    assert e["traffic"] is None and e["peak"] == 3040.0 and e["frac"] == pytest.approx(e["achieved"] / 3040.0)
    e = bench.roofline_entry(_ops(up_swiglu_fwd=1.5), M, H, I, PEAKS, "measured", fp8=True, steps=20)
    assert e["peak"] == 4500.0


def test_traffic_summary_is_consistent_with_its_algorithmic_bytes():
    cap = json.loads((REPO / "profiles" / "launch_traffic_cfg3.json").read_text())
    alg = {
        "up_swiglu_fwd": M * H + 2 * E * H * I + 3 * M * I,
        "down_fwd": M * I + E * I * H + M * H,
        "down_wgrad_bias": M * I + M * H + E * I * H,
        "down_dgrad_swiglu_bwd": M * H + E * I * H + 4 * M * I,
        "up_dgrad": 2 * M * I + 2 * E * H * I + M * H,
        "up_wgrad_bias": M * H + 2 * M * I + 2 * E * H * I,
    }
    assert set(cap["ops"]) == set(alg)
    for name, entry in cap["ops"].items():
        assert entry["cfg3_algorithmic_bytes"] == 2 * alg[name]
        captured = entry["captured_read_bytes"] + entry["captured_write_bytes"]
        ratio = captured / entry["captured_algorithmic_bytes"]
        assert ratio == pytest.approx(entry["ratio_to_algorithmic"], abs=1e-3)
        assert entry["bytes_per_launch"] == pytest.approx(ratio * entry["cfg3_algorithmic_bytes"], rel=1e-6)
