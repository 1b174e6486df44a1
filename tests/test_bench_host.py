"""bench.py's host-side logic on the CPU: the config-4 utterance set and its
partition over 1-8 ranks, the roofline arithmetic of its JSON line, and the
utterance the CPU legs time."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_config4_set_has_the_baseline_shape():
    _, specs = bench.batched_set()
    assert len(specs) == 64
    frames = np.array([s[2] for s in specs])
    assert frames.min() >= 50 and frames.max() <= 750
    assert all(text == int(round(0.4 * f)) for text, _, f in specs)
    refs = [ref for _, ref, _ in specs if ref]
    assert len(refs) == 32 and min(refs) >= 125 and max(refs) <= 250


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config4_partition_covers_every_utterance_once(native, world):
    shares, audio = [], set()
    for rank in range(world):
        desc, inputs, seeds, total_audio, scaling, extra = bench.make_workload("c4", rank, world)
        assert scaling == "strong" and inputs and len(inputs) == len(seeds)
        assert 1.0 <= extra["imbalance_max_over_mean"] < 1.05
        shares.append(seeds)
        audio.add(total_audio)
    flat = sorted(s for share in shares for s in share)
    assert flat == [1000 + i for i in range(64)]
    assert len(audio) == 1  # every rank reports the whole job's audio


def test_single_utterance_workloads_scale_weakly(native):
    one = bench.make_workload("c2", 0, 1)
    eight = bench.make_workload("c2", 3, 8)
    assert one[4] == "weak" and eight[3] == pytest.approx(8 * one[3])
    assert one[3] == pytest.approx(250 / 25.0)


def _prof():
    return [
        {"name": "rmsnorm", "ms": 4.0, "launches": 55, "flops": 0.0, "bytes": 55 * 458.2e6},
        {"name": "attention", "ms": 20.0, "launches": 28, "flops": 28 * 438.5e9, "bytes": 0.0},
        {"name": "gemm_gate_up_swiglu", "ms": 19.0, "launches": 28, "flops": 28 * 938.4e9,
         "bytes": 0.0},
    ]


def test_roofline_takes_the_dominant_class_and_the_power_capped_peak():
    import json
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    capped = {"reasons": ["sw_power_cap"]}
    r = bench.roofline(_prof(), "c4", capped, 28 * 938.4e9, 19.0)
    assert r["kernel"] == "attention" and r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert r["achieved"] == pytest.approx(438.5e9 / (20.0e-3 / 28) / 1e12)
    assert r["peak"] == peaks["bf16_tflops_sustained"]
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"])
    assert r["traffic"] == bench.NCU_TRAFFIC[("c4", "attention")]
    burst = bench.roofline(_prof(), "c4", {"reasons": []}, 1.0, 1.0)
    assert burst["peak"] == peaks["bf16_tflops"]


def test_roofline_of_a_memory_bound_class():
    prof = _prof()[:1]
    r = bench.roofline(prof, "c1", {"reasons": []}, 0.0, 0.0)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert r["achieved"] == pytest.approx(458.2e6 / (4.0e-3 / 55) / 1e9)
    assert r["traffic"] is None and r["all_gemms_tflops"] is None


def test_cpu_sample_is_the_median_cost_utterance(native):
    _, inputs, _, _, _, extra = bench.make_workload("c4", 0, 1)
    from omnivoice_b200.scheduler import utterance_cost
    i = bench.cpu_sample(inputs)
    costs = sorted(utterance_cost(x.length, x.target_frames) for x in inputs)
    assert utterance_cost(inputs[i].length, inputs[i].target_frames) == costs[len(costs) // 2]
