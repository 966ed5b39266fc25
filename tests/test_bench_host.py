"""Host-side pieces of bench.py that shape the reported roofline (no GPU needed):
the dominant kernel's denominator follows how its launches were timed."""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from chunkkv_b200.engine.weights import SHAPES  # noqa: E402

PEAKS = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1300.0}


class _Ev:
    def __init__(self, t_ms: float):
        self.t = t_ms

    def elapsed_time(self, other: "_Ev") -> float:
        return other.t - self.t


class _Timer:
    """Stand-in for ops.LaunchTimer: records of (name, flops, bytes, start, end)."""

    def __init__(self, gate_cycles: int, launches: list[tuple[str, float, float]]):
        self.gate_cycles = gate_cycles
        self.records = [(name, flops, 0.0, _Ev(0.0), _Ev(ms)) for name, flops, ms in launches]


def _swiglu_flops(shape, rows: int) -> float:
    return 4.0 * shape.inter * shape.hidden * rows


def test_roofline_uses_the_burst_peak_for_launches_timed_alone():
    shape = SHAPES["qwen2.5-7b"]
    f938, f5248 = _swiglu_flops(shape, 938), _swiglu_flops(shape, 5248)
    # 27 launches at the selected-row shape and one layer-0 launch: the roofline takes the
    # most frequent shape, M = 938, and its mean time
    launches = [("ckv_linear_swiglu", f938, 0.2)] * 27 + [("ckv_linear_swiglu", f5248, 1.0),
                                                          ("ckv_qkv_rope", 1e9, 0.05)]
    gated = bench.dominant_roofline(_Timer(98250, launches), PEAKS, "measured", shape)
    achieved = f938 / 0.2e-3 / 1e12
    assert gated["rows"] == 938 and gated["launches"] == 27
    assert abs(gated["achieved"] - round(achieved, 1)) < 1e-6
    assert gated["peak"] == PEAKS["bf16_tflops"] and gated["peak_source"] == "measured bf16_tflops"
    assert abs(gated["frac"] - round(achieved / 1600.0, 4)) < 1e-9
    assert abs(gated["frac_sustained"] - round(achieved / 1300.0, 4)) < 1e-9
    assert gated["traffic"] == bench.SWIGLU_M938_TRAFFIC

    plain = bench.dominant_roofline(_Timer(0, launches), PEAKS, "measured", shape)
    assert plain["peak"] == PEAKS["bf16_tflops_sustained"]
    assert plain["frac"] == plain["frac_sustained"]


def test_roofline_without_swiglu_launches_reports_zero():
    out = bench.dominant_roofline(_Timer(0, [("ckv_qkv_rope", 1e9, 0.05)]), PEAKS, "measured",
                                  SHAPES["qwen2.5-7b"])
    assert out["achieved"] == 0.0 and out["frac"] == 0.0
