"""Per-layer / per-request performance events (JSONL), CUDA-event timing and clock sampling.

Parity: the reference's `HCP_PERF_LOG` JSONL events (rust/src/model/attention/ring.rs:822-844,
1376-1395: `ring_attention` per layer with total/compute/recv/send ms and byte counters;
`ring_decode` ring.rs:801-815; `stationary_decode` worker_sdk/tch_backend.rs:859-880). The
reference times with host wall clocks around libtorch calls; here device time comes from CUDA
events on the launching stream, and multi-rank numbers are reduced as the max over ranks.
"""

from __future__ import annotations

import json
import os
import subprocess
import threading
import time
from typing import Optional


class PerfLog:
    def __init__(self, path: Optional[str]):
        self.path = path
        self._lock = threading.Lock()

    @property
    def enabled(self) -> bool:
        return bool(self.path)

    @classmethod
    def from_env(cls, env=None) -> "PerfLog":
        path = getattr(env, "perf_log", None) if env is not None else os.environ.get("HCP_PERF_LOG")
        return cls(path)

    def emit(self, event: str, **fields) -> None:
        if not self.path:
            return
        rec = {"ts": time.time(), "event": event, **fields}
        line = json.dumps(rec)
        with self._lock:
            with open(self.path, "a") as f:
                f.write(line + "\n")


_PEAK = None


def peak_bf16_tflops() -> float:
    """bf16 tensor throughput that perf events report roofline fractions against: the
    HCP_PEAK_BF16_TFLOPS override, else the sustained cuBLAS bf16 figure of a MEASURED_PEAKS.json
    beside the package (written by the benchmark driver on the target GPUs), else 1400 (a B200
    under its 1 kW power cap)."""
    global _PEAK
    if _PEAK is None:
        env = os.environ.get("HCP_PEAK_BF16_TFLOPS")
        if env:
            _PEAK = float(env)
        else:
            path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(
                os.path.abspath(__file__)))), "MEASURED_PEAKS.json")
            try:
                with open(path) as f:
                    p = json.load(f)
                _PEAK = float(p.get("bf16_tflops_sustained", p["bf16_tflops"]))
            except (OSError, KeyError, ValueError):
                _PEAK = 1400.0
    return _PEAK


class CudaTimer:
    """Device time between two points of the current stream (milliseconds)."""

    def __init__(self):
        import torch
        self.start = torch.cuda.Event(enable_timing=True)
        self.stop = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        self.start.record()
        return self

    def __exit__(self, *exc):
        self.stop.record()
        return False

    def ms(self) -> float:
        self.stop.synchronize()
        return self.start.elapsed_time(self.stop)


def max_over_ranks(value: float, group=None) -> float:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """Samples `nvidia-smi` clocks and throttle reasons in the background (read-only query)."""

    def __init__(self, gpu_index: int = 0, period_ms: int = 200):
        self.gpu = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.lines: list = []
        self._thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", str(self.period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread = threading.Thread(target=self._reader, daemon=True)
            self._thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _reader(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._thread is not None:
                self._thread.join(timeout=2)
        return False

    def summary(self) -> dict:
        mhz, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for i, n in enumerate(names):
                if parts[5 + i].lower() == "active":
                    reasons.add(n)
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None,
                "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(mhz)}
