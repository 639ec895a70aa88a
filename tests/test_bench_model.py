"""bench.py's accounting, checked on the CPU: the algorithmic bytes behind
every roofline fraction it prints, and the clock record that decides
whether a run stands."""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from titania_b200 import synth  # noqa: E402


def test_qwen3_0_6b_step_bytes():
    """Linear 440 401 920 + lm_head 155 582 464 + norms 65 536 parameters in
    bf16 = 1 192 099 840 B, plus the 2 048-byte embedding row; K/V per
    context position 28 layers x 1024 x (K, V) x 4 B (f32) or 2 B (bf16)."""
    weights, kv = bench.model_bytes(synth.QWEN3_0_6B)
    assert weights == 1_192_099_840 + 2048
    assert kv == 28 * 1024 * 2 * 4
    assert bench.model_bytes(synth.QWEN3_0_6B, kv_bytes=2)[1] == 114_688


def test_qwen3_4b_step_bytes():
    """Linear 3 633 315 840 + lm_head 388 956 160 parameters (+ norms) in bf16,
    and 2048 x 36 x 4096 B of bf16 K/V at context 2048."""
    weights, kv = bench.model_bytes(synth.QWEN3_4B, kv_bytes=2)
    c = synth.QWEN3_4B
    norms = (c["num_hidden_layers"] * (2 * c["hidden_size"] + 2 * 128) + c["hidden_size"]) * 2
    assert weights == (3_633_315_840 + 388_956_160) * 2 + norms + 2 * c["hidden_size"]
    assert 2048 * kv == 2048 * 36 * 4096


def test_peaks_reads_the_measured_file():
    p, kind = bench.peaks()
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            assert (p, kind) == (float(json.load(fh)["hbm_gbs"]), "measured")
    else:
        assert kind == "fallback"


def _clocks(lines):
    c = bench.Clocks(0)
    c.lines = lines
    return c.summary()


def test_clock_summary_median_and_reasons():
    ok = "0, 1965, 1965, 700.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"
    capped = "0, 1800, 1965, 999.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
    hot = "0, 1500, 1965, 990.0, 0x0000000000000020, Not Active, Not Active, Active, Not Active"
    s = _clocks([ok, ok, capped])
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    s = _clocks([ok, hot, "garbage line", ""])
    assert s["reasons"] == ["sw_thermal_slowdown"] and s["samples"] == 2
    assert _clocks([])["sm_mhz"] is None


def test_step_timeline_segments_add_up_to_the_step():
    """bench.timeline: consecutive segments ordered by each unit's last DONE
    sum to the traced step, per op summed over layers."""
    import numpy as np

    import bench

    dt = np.dtype([("tag", "<u4"), ("cta", "<u4"), ("event", "<u4"), ("sm", "<u4"), ("ns", "<u8")])
    recs = []
    t = 1000
    for layer in range(3):
        for op in (32, 33, 34, 35):
            for cta in range(4):
                recs.append(((op << 16) | layer, cta, 2, 0, t + 10 * cta))        # INPUT
                recs.append(((op << 16) | layer, cta, 4, 0, t + 100 + 10 * cta))  # DONE
            t += 200
    recs.append((37 << 16, 0, 0, 0, 900))  # START, the step's first record
    tr = np.array(recs, dtype=dt)
    tl = bench.timeline(tr, bench.PERSIST_NAMES)
    assert abs(sum(tl["segments_us"].values()) - tl["step_us"]) < 1e-6
    assert tl["step_us"] == (t - 200 + 130 - 900) / 1e3
    assert tl["own_work_us_per_launch"]["q|k|v"] == 0.1
