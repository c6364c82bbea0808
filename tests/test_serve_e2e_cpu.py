"""Local multi-process serving end to end: `serve` under torchrun with two CPU (gloo) ranks, an HF
directory of random weights, an uneven 3:1 capacity ratio and the zigzag layout; completions over
HTTP, concurrent requests, health and metrics, then a shutdown on SIGINT without rank tracebacks.

Parity: the reference's local multi-process drivers (scripts/test_http_api_local.sh,
test_http_api_concurrent_local.sh: coordinator + 2 workers on one host, curl /v1/completions,
/health, /metrics).
"""

import json
import os
import signal
import socket
import subprocess
import sys
import threading
import time
import urllib.error
import urllib.request

import pytest
import torch

from hetero_cp_ringattn_b200.config import preset
from hetero_cp_ringattn_b200.models import reference_model
from hetero_cp_ringattn_b200.models.weights import ModelWeights
from hetero_cp_ringattn_b200.serve.tokenizer import ByteTokenizer

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _get(port, path):
    with urllib.request.urlopen(f"http://127.0.0.1:{port}{path}", timeout=30) as r:
        return json.loads(r.read())


def _complete(port, prompt, n):
    req = urllib.request.Request(f"http://127.0.0.1:{port}/v1/completions",
                                 data=json.dumps({"prompt": prompt, "max_tokens": n}).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=120) as r:
        return json.loads(r.read())


@pytest.fixture(scope="module")
def server(tmp_path_factory):
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=5, dtype=torch.float32, std=0.2)
    mdir = tmp_path_factory.mktemp("model")
    w.save(str(mdir))
    http = _port()
    env = dict(os.environ, HCP_QUIC_TIMEOUT_SECS="60", PYTHONPATH=REPO, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "-m", "hetero_cp_ringattn_b200", "serve", "--model-dir", str(mdir), "--device", "cpu",
           "--max-context", "512", "--ratio", "3:1", "--ring-strategy", "zigzag",
           "--http-addr", f"127.0.0.1:{http}"]
    log = open(mdir / "serve.log", "w")
    proc = subprocess.Popen(cmd, cwd=REPO, env=env, stdout=log, stderr=subprocess.STDOUT,
                            start_new_session=True)
    try:
        deadline = time.time() + 420
        while True:
            try:
                health = _get(http, "/health")
                break
            except OSError:
                if proc.poll() is not None or time.time() > deadline:
                    log.flush()
                    raise RuntimeError("serve did not come up:\n" + (mdir / "serve.log").read_text()[-3000:])
                time.sleep(0.5)
        yield w, http, health, proc, mdir / "serve.log"
    finally:
        if proc.poll() is None:
            proc.send_signal(signal.SIGINT)
            try:
                proc.wait(timeout=60)
            except subprocess.TimeoutExpired:
                os.killpg(proc.pid, signal.SIGKILL)  # the group this fixture started
                proc.wait(timeout=30)
        log.close()


def _expected(w, prompt, n):
    tok = ByteTokenizer(w.cfg.vocab_size)
    ids = tok.encode(prompt)
    ref, _ = reference_model.greedy_generate(w, torch.tensor(ids), n - 1)
    return tok.decode(ref), len(ids)


def test_two_rank_server_health_and_completion(server):
    w, port, health, _, _ = server
    assert health == {"status": "ok", "workers_connected": 2, "num_domains": 2}
    text, n_prompt = _expected(w, "heterogeneous context parallel ring", 6)
    res = _complete(port, "heterogeneous context parallel ring", 6)
    assert res["choices"][0]["text"] == text
    assert res["usage"] == {"prompt_tokens": n_prompt, "completion_tokens": 6,
                            "total_tokens": n_prompt + 6}


def test_two_rank_server_concurrent_requests(server):
    w, port, _, _, _ = server
    prompts = ["ab", "two ranks share one prompt", "zigzag layout, uneven 3:1 split", "xyz"]
    out = {}

    def go(i, p):
        out[i] = _complete(port, p, 4)

    ts = [threading.Thread(target=go, args=(i, p)) for i, p in enumerate(prompts)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=180)
    for i, p in enumerate(prompts):
        assert out[i]["choices"][0]["text"] == _expected(w, p, 4)[0]
    m = _get(port, "/metrics")
    assert m["completed_requests"] >= len(prompts) + 1
    assert m["active_requests"] == 0 and m["failed_requests"] == 0


def _post(port, body):
    req = urllib.request.Request(f"http://127.0.0.1:{port}/v1/completions",
                                 data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=120) as r:
        return json.loads(r.read())


def test_two_rank_server_session_keep_kv_then_append(server):
    """A keep_kv request leaves its KV sharded over both ranks; the append continues it; the
    texts equal the dense oracle on the whole context."""
    w, port, _, _, _ = server
    tok = ByteTokenizer(w.cfg.vocab_size)
    p1, p2 = "first turn of a session", " and the second turn"
    r1 = _post(port, {"prompt": p1, "max_tokens": 4, "session_id": "conv", "keep_kv": True})
    ids1 = tok.encode(p1)
    g1, _ = reference_model.greedy_generate(w, torch.tensor(ids1), 3)
    assert r1["choices"][0]["text"] == tok.decode(g1)
    r2 = _post(port, {"prompt": p2, "max_tokens": 3, "session_id": "conv", "append": True})
    g2, _ = reference_model.greedy_generate(w, torch.tensor(ids1 + g1 + tok.encode(p2)), 2)
    assert r2["choices"][0]["text"] == tok.decode(g2)
    with pytest.raises(urllib.error.HTTPError) as ei:   # the append without keep_kv ended it
        _post(port, {"prompt": "x y", "max_tokens": 1, "session_id": "conv", "append": True})
    assert ei.value.code == 400


def test_two_rank_server_rejects_prompt_shorter_than_ranks(server):
    _, port, _, _, _ = server
    with pytest.raises(urllib.error.HTTPError) as ei:
        _complete(port, "a", 2)
    assert ei.value.code == 400
    assert "must be >= num_domains (2)" in ei.value.read().decode()


def test_two_rank_continuation_e2e_cli(tmp_path):
    """`serve --continuation-segment` under torchrun with two ranks and uneven tickets: the
    generated ids and the three logits dumps match the dense oracle."""
    import numpy as np
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=6, dtype=torch.float32, std=0.2)
    mdir = tmp_path / "model"
    w.save(str(mdir))
    dump = tmp_path / "dump"
    prompt = list(range(3, 24))
    seg = [40, 41, 42, 43, 44]
    env = dict(os.environ, HCP_QUIC_TIMEOUT_SECS="60", PYTHONPATH=REPO, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "-m", "hetero_cp_ringattn_b200", "serve", "--model-dir", str(mdir), "--device", "cpu",
           "--max-context", "256", "--num-domains", "2", "--max-tokens", "4",
           "--prompt-token-ids", ",".join(map(str, prompt)),
           "--continuation-segment", ",".join(map(str, seg)),
           "--continuation-request-id", "9", "--continuation-capacity-tickets", "3,1",
           "--export-logits", str(dump)]
    out = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    line = [ln for ln in out.stdout.splitlines() if ln.startswith('{"continuation_e2e"')][0]
    meta = json.loads(line)["continuation_e2e"]
    t0 = meta["decode_token"]
    ref_more, _ = reference_model.greedy_generate(w, torch.tensor(prompt + [t0] + seg), 2)
    assert meta["generated_ids"] == [t0] + ref_more
    assert meta["prefix_splits"] == [11, 10] and meta["capacity_tickets"] == [3, 1]
    assert meta["continuation_offsets_by_domain"] == [[0, 1, 2, 3], [4]]
    for name, ids in (("prefill_last_logits", prompt), ("decode_logits", prompt + [t0]),
                      ("continuation_last_logits", prompt + [t0] + seg)):
        got = np.fromfile(str(dump / f"{name}.f32le"), dtype="<f4")
        ref = reference_model.forward(w, torch.tensor(ids), last_only=True)[0].numpy()
        assert np.abs(got - ref).max() < 1e-3, name


def test_infer_under_torchrun_matches_single_process(tmp_path):
    """`infer` on two ranks (zigzag, 3:1) exports the same logits and tokens as on one rank, so
    `compare-logits` passes between a distributed and a single-device run."""
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=8, dtype=torch.float32, std=0.2)
    mdir = tmp_path / "model"
    w.save(str(mdir))
    env = dict(os.environ, PYTHONPATH=REPO, OMP_NUM_THREADS="2")
    base = ["-m", "hetero_cp_ringattn_b200", "infer", "--model-dir", str(mdir), "--device", "cpu",
            "--prompt", "distributed logits export check", "--max-tokens", "5"]
    one = subprocess.run([sys.executable] + base + ["--export-logits", str(tmp_path / "a.bin")],
                         cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert one.returncode == 0, one.stderr[-3000:]
    two = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                          "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                          "--master-port", str(_port())] + base +
                         ["--export-logits", str(tmp_path / "b.bin"), "--ratio", "3:1",
                          "--ring-strategy", "zigzag", "--num-domains", "2"],
                         cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert two.returncode == 0, two.stdout[-2000:] + two.stderr[-3000:]
    r1 = json.loads(one.stdout.strip().splitlines()[-1])
    r2 = json.loads([ln for ln in two.stdout.splitlines() if ln.startswith("{")][-1])
    assert r2["world"] == 2 and r2["chunks"][0] > r2["chunks"][1]
    assert r1["tokens"] == r2["tokens"]
    cmp_ = subprocess.run([sys.executable, "-m", "hetero_cp_ringattn_b200", "compare-logits",
                           str(tmp_path / "a.bin"), str(tmp_path / "b.bin"), "--tolerance", "1e-3"],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=120)
    assert cmp_.returncode == 0 and json.loads(cmp_.stdout)["passed"], cmp_.stdout


def test_serve_bench_client_against_two_ranks(server):
    """benchmarks/serve_bench.py (the reference's serving baseline shape: random prompts,
    fixed output length with EOS ignored, closed-loop concurrency) completes every request and
    reports TTFT / TPOT / throughput."""
    sys.path.insert(0, os.path.join(REPO, "benchmarks"))
    try:
        import serve_bench
    finally:
        sys.path.pop(0)
    _, port, _, _, _ = server
    res = serve_bench.run(f"http://127.0.0.1:{port}", num_prompts=6, input_len=12, output_len=5,
                          max_concurrency=2, seed=1)
    assert res["completed"] == 6 and res["failed"] == 0
    assert res["output_throughput"] > 0 and res["mean_ttft_ms"] > 0 and res["mean_tpot_ms"] > 0
    assert res["median_ttft_ms"] <= res["p99_ttft_ms"]
    ids = serve_bench.run(f"http://127.0.0.1:{port}", num_prompts=3, input_len=9, output_len=3,
                          max_concurrency=3, seed=2, token_ids_below=100)
    assert ids["completed"] == 3 and ids["failed"] == 0


def test_two_rank_chunked_prefill_cli(tmp_path):
    """`serve --prefill-chunk-tokens` under torchrun on two ranks (zigzag, 3:1): the prompt is
    prefilled in pieces (ring layout for the first, continuation segments after) and the tokens
    equal the oracle's."""
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=7, dtype=torch.float32, std=0.2)
    mdir = tmp_path / "model"
    w.save(str(mdir))
    prompt = [(13 * j + 1) % cfg.vocab_size for j in range(90)]
    env = dict(os.environ, HCP_QUIC_TIMEOUT_SECS="60", PYTHONPATH=REPO, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "-m", "hetero_cp_ringattn_b200", "serve", "--model-dir", str(mdir), "--device", "cpu",
           "--max-context", "256", "--ratio", "3:1", "--ring-strategy", "zigzag",
           "--prefill-chunk-tokens", "20", "--max-tokens", "5",
           "--prompt-token-ids", ",".join(map(str, prompt))]
    out = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    res = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith('{"prompt_token_ids"')][0])
    ref, _ = reference_model.greedy_generate(w, torch.tensor(prompt), 4)
    assert res["tokens"] == ref


# stops the module's server: keep it the last test that uses the fixture
def test_two_rank_server_exits_on_interrupt(server):
    """Ctrl-C reaches every rank through torchrun; each rank leaves its loop without a
    traceback (torchrun itself still reports the signal in its own exit status)."""
    _, _, _, proc, log = server
    proc.send_signal(signal.SIGINT)
    proc.wait(timeout=60)
    text = log.read_text()
    assert "[rank0]: Traceback" not in text and "[rank1]: Traceback" not in text, text[-3000:]
