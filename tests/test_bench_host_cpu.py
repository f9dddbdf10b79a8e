"""Host-side pieces of bench.py, on CPU: the clock-record parser that decides
whether a run is kept (throttle reasons, median SM clock), the peak lookup,
and the benchmark shapes against the 2B architecture."""
from __future__ import annotations

import bench
from bitnetrs_b200 import bitnet_2b_config


class _FakeProc:
    def __init__(self, text):
        self.text = text

    def terminate(self):
        pass

    def communicate(self, timeout=None):
        return self.text, ""


def _clocks(lines):
    c = bench.Clocks(0)
    c.proc = _FakeProc("\n".join(lines))
    return c.stop()


def test_clock_record_clean_run():
    row = "0, {sm}, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active"
    r = _clocks([row.format(sm=s) for s in (1965, 1965, 1950, 1965, 345)])
    assert r["sm_mhz"] == 1965 and r["sm_max_mhz"] == 1965 and r["reasons"] == [] and r["samples"] == 5


def test_clock_record_reports_throttle_reasons():
    ok = "0, 1965, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active"
    hot = "0, 1500, 1965, 990.0, 0x20, Active, Not Active, Active, Active"
    r = _clocks([ok, hot, "garbage", "0, N/A, 1965, 1, 0, a, b, c, d"])
    assert r["reasons"] == ["hw_slowdown", "sw_power_cap", "sw_thermal_slowdown"]
    assert r["samples"] == 2


def test_clock_record_without_nvidia_smi():
    c = bench.Clocks(0)
    c.proc = None
    assert c.stop()["reasons"] == ["nvidia-smi unavailable"]


def test_peaks_reads_measured_or_falls_back(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.peaks() == (6650.0, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text('{"hbm_gbs": 6552.0}')
    assert bench.peaks() == (6552.0, "measured")


def test_shapes_follow_the_2b_architecture():
    c = bitnet_2b_config()
    H, F, qd, kvd = c.hidden_size, c.intermediate_size, c.q_dim(), c.kv_dim()
    assert dict((n, (a, b)) for n, a, b in bench.GEMV_SHAPES) == {
        "qkv": (qd + 2 * kvd, H), "o": (H, qd), "gate_up": (2 * F, H), "down": (H, F)}
    assert dict((n, (a, b)) for n, a, b in bench.C2_SHAPES) == {
        "q/o": (H, H), "k/v": (kvd, H), "gate/up": (F, H), "down": (H, F)}
    assert bench.C2_M == [1, 8, 64, 512, 4096]
    # ternary weights of the 2B model: 69,468,160 per layer, two ops each
    per_layer = (qd + 2 * kvd) * H + H * qd + 2 * F * H + H * F
    assert per_layer == 69_468_160
    assert bench.TERNARY_OPS_PER_TOKEN == 2 * per_layer * c.num_hidden_layers
