"""Serving benchmark client for the `/v1/completions` API: TTFT, TPOT and output tokens/s.

The same workload shape as the reference's serving baselines (docs/PHASE3_N2_PERF_BASELINE.md,
measured there with `vllm bench serve`): random prompts of `--input-len` tokens, `--output-len`
generated tokens with EOS ignored, either Poisson arrivals at `--request-rate` requests/s or
closed-loop at `--max-concurrency` requests in flight. Every request streams (SSE): TTFT is the
time to the first token chunk, TPOT the mean gap between the following chunks.

    python -m hetero_cp_ringattn_b200 serve ... --http-addr 127.0.0.1:8000 &
    python benchmarks/serve_bench.py --url http://127.0.0.1:8000 --num-prompts 32 \\
        --input-len 32 --output-len 16 --request-rate 1          # the reference's L1
    python benchmarks/serve_bench.py ... --max-concurrency 4      # L3

Prints one JSON line. Wall-clock host timing: this measures the serving stack end to end
(HTTP, tokenizer, coordinator, control plane and the engine), not device time.
"""

from __future__ import annotations

import argparse
import json
import random
import string
import threading
import time
import urllib.request
from typing import List, Optional


def _pct(v: List[float], q: float) -> Optional[float]:
    if not v:
        return None
    s = sorted(v)
    k = min(len(s) - 1, max(0, int(round(q / 100.0 * (len(s) - 1)))))
    return s[k]


def _stats(name: str, v: List[float]) -> dict:
    return {f"mean_{name}": (sum(v) / len(v)) if v else None, f"median_{name}": _pct(v, 50),
            f"p99_{name}": _pct(v, 99)}


def random_prompt(rng: random.Random, n_chars: int) -> str:
    """Random printable text; the byte tokenizer maps one character to one token."""
    alphabet = string.ascii_letters + string.digits + "     "
    return "".join(rng.choice(alphabet) for _ in range(n_chars))


def one_request(url: str, prompt, max_tokens: int, timeout: float) -> dict:
    body = {"prompt": prompt, "max_tokens": max_tokens, "stream": True, "ignore_eos": True}
    req = urllib.request.Request(url.rstrip("/") + "/v1/completions",
                                 data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    t0 = time.perf_counter()
    stamps: List[float] = []
    err = None
    try:
        with urllib.request.urlopen(req, timeout=timeout) as r:
            for raw in r:
                line = raw.decode().strip()
                if not line.startswith("data: "):
                    continue
                data = line[6:]
                if data == "[DONE]":
                    break
                obj = json.loads(data)
                if "error" in obj:
                    err = obj["error"]
                    break
                stamps.append(time.perf_counter())
    except OSError as e:
        err = str(e)
    t1 = time.perf_counter()
    out = {"ok": err is None and bool(stamps), "error": err, "tokens": len(stamps),
           "latency_s": t1 - t0}
    if stamps:
        out["ttft_ms"] = (stamps[0] - t0) * 1e3
        if len(stamps) > 1:
            out["tpot_ms"] = (stamps[-1] - stamps[0]) / (len(stamps) - 1) * 1e3
    return out


def run(url: str, num_prompts: int, input_len: int, output_len: int,
        request_rate: float = float("inf"), max_concurrency: Optional[int] = None, seed: int = 0,
        timeout: float = 600.0, token_ids_below: int = 0) -> dict:
    """`token_ids_below` > 0 sends each prompt as `input_len` random token ids below that bound
    (exact prompt lengths with any tokenizer) instead of random text."""
    rng = random.Random(seed)
    if token_ids_below > 0:
        prompts = [[rng.randrange(token_ids_below) for _ in range(input_len)]
                   for _ in range(num_prompts)]
    else:
        prompts = [random_prompt(rng, input_len) for _ in range(num_prompts)]
    gaps = [rng.expovariate(request_rate) if request_rate != float("inf") else 0.0
            for _ in range(num_prompts)]
    sem = threading.Semaphore(max_concurrency) if max_concurrency else None
    results: List[dict] = [None] * num_prompts  # type: ignore[list-item]

    def worker(i: int) -> None:
        try:
            results[i] = one_request(url, prompts[i], output_len, timeout)
        finally:
            if sem is not None:
                sem.release()

    threads = []
    t0 = time.perf_counter()
    for i in range(num_prompts):
        if gaps[i] > 0:
            time.sleep(gaps[i])
        if sem is not None:
            sem.acquire()
        th = threading.Thread(target=worker, args=(i,), daemon=True)
        th.start()
        threads.append(th)
    for th in threads:
        th.join(timeout)
    dur = time.perf_counter() - t0
    ok = [r for r in results if r is not None and r["ok"]]
    out_tokens = sum(r["tokens"] for r in ok)
    res = {"metric": "serve TTFT / TPOT / output tok/s", "num_prompts": num_prompts,
           "completed": len(ok), "failed": num_prompts - len(ok), "input_len": input_len,
           "output_len": output_len,
           "request_rate": None if request_rate == float("inf") else request_rate,
           "max_concurrency": max_concurrency, "duration_s": dur,
           "request_throughput": len(ok) / dur if dur > 0 else None,
           "output_throughput": out_tokens / dur if dur > 0 else None,
           **_stats("ttft_ms", [r["ttft_ms"] for r in ok if "ttft_ms" in r]),
           **_stats("tpot_ms", [r["tpot_ms"] for r in ok if "tpot_ms" in r]),
           **_stats("latency_s", [r["latency_s"] for r in ok])}
    errs = [r["error"] for r in results if r is not None and not r["ok"]]
    if errs:
        res["first_error"] = errs[0]
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--num-prompts", type=int, default=32)
    ap.add_argument("--input-len", type=int, default=32)
    ap.add_argument("--output-len", type=int, default=16)
    ap.add_argument("--request-rate", type=float, default=float("inf"))
    ap.add_argument("--max-concurrency", type=int, default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--timeout", type=float, default=600.0)
    ap.add_argument("--token-ids", type=int, default=0, metavar="VOCAB",
                    help="send prompts as random token ids below VOCAB (exact input lengths)")
    a = ap.parse_args(argv)
    res = run(a.url, a.num_prompts, a.input_len, a.output_len, a.request_rate, a.max_concurrency,
              a.seed, a.timeout, a.token_ids)
    print(json.dumps(res))
    return 0 if res["failed"] == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
