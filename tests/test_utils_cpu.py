"""Measurement utilities on CPU: the clock-sample parser that guards every benchmark number
(throttle reasons, median SM clock), the launch counter behind `gpu_launches`, and the perf log."""

import json

from hetero_cp_ringattn_b200.utils import launches
from hetero_cp_ringattn_b200.utils.perf import ClockSampler, PerfLog, max_over_ranks


def test_clock_summary_reports_median_and_reasons():
    s = ClockSampler()
    s.lines = ["0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
               "0, 1800, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active",
               "0, 1350, 1965, 999.0, 0x4, Not Active, Not Active, Not Active, Active",
               "garbage line", "0, [N/A], 1965, 1, x, Active, Not Active, Not Active, Not Active"]
    out = s.summary()
    assert out == {"sm_mhz": 1800.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 3}
    s.lines.append("0, 900, 1965, 500, 0x8, Active, Active, Not Active, Not Active")
    assert s.summary()["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap"]
    assert ClockSampler().summary()["sm_mhz"] is None


def test_launch_counter_counts_graph_replays():
    launches.reset()
    launches.count(3)
    with launches.capture() as cap:
        launches.count(5)          # recorded into the graph, not launched
        launches.count(2)
    assert cap.launches == 7 and launches.total() == 3
    launches.count(cap.launches)   # one replay
    assert launches.total() == 10
    launches.reset()
    assert launches.total() == 0


def test_perf_log_lines_and_single_process_max(tmp_path):
    p = tmp_path / "perf.jsonl"
    log = PerfLog(str(p))
    assert log.enabled and not PerfLog(None).enabled
    log.emit("ring_attention", layer=1, total_ms=2.5)
    ev = json.loads(p.read_text())
    assert ev["event"] == "ring_attention" and ev["layer"] == 1 and "ts" in ev
    assert max_over_ranks(4.5) == 4.5
