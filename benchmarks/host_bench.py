"""Host-side costs on the serving path (CPU only): control-frame encode + decode of a Prefill
command for long prompts (the native binary codec against a JSON encoding of the same message),
the KV-growth owner table of a request, and capacity chunking.

    python benchmarks/host_bench.py            # prints one JSON line

Wall-clock medians over repeated calls (`time.perf_counter`), after one warm-up call.
"""

from __future__ import annotations

import dataclasses
import json
import os
import statistics
import sys
import time

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from hetero_cp_ringattn_b200.parallel.capacity import allocate_by_capacity  # noqa: E402
from hetero_cp_ringattn_b200.parallel.schedule import assignee_table  # noqa: E402
from hetero_cp_ringattn_b200.serve import protocol as P  # noqa: E402


def median_ms(fn, reps: int) -> float:
    fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(ts)


def main() -> int:
    out = {"metric": "host-side serving costs (ms, median)"}
    rng = np.random.default_rng(0)
    for n in (32768, 131072):
        ids = rng.integers(0, 128256, n).tolist()
        cmd = P.Prefill(1, ids, [n // 8] * 8, "zigzag", 256, [1] * 8, False)
        native = median_ms(lambda: P.decode(P.encode(cmd)), 20)

        def as_json():
            body = json.dumps({"type": "Prefill", "body": dataclasses.asdict(cmd)}).encode()
            obj = json.loads(body.decode())
            return P.Prefill(**obj["body"])

        js = median_ms(as_json, 5)
        out[f"prefill_frame_{n // 1024}k"] = {"native_ms": round(native, 3), "json_ms": round(js, 3),
                                              "bytes": len(P.encode(cmd))}
    out["assignee_table_8ranks_256x32"] = round(
        median_ms(lambda: assignee_table([5, 5, 5, 5, 2, 2, 1, 1], 7, 256, 32), 50), 4)
    out["allocate_by_capacity_131072_8ranks"] = round(
        median_ms(lambda: allocate_by_capacity(131072, [5, 5, 5, 5, 2, 2, 1, 1]), 200), 5)
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
