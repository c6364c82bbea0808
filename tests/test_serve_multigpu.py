"""Serving on several GPUs end to end: `serve` under torchrun with one process per GPU (NCCL for
the bootstrap, gloo for the control plane, CUDA-IPC peer memory for the KV ring and the decode
exchange), an uneven 3:1 capacity ratio and the zigzag layout; health, completions (plain,
streamed, concurrent), metrics, then a shutdown on SIGINT.

The prefill's logits are the same bits at any CP degree, so the logits the server dumps for a
request (`serve --export-logits`) must equal a single-GPU engine's for the same weights and
prompt, bit for bit, and the first generated token is their argmax.
Skipped when fewer than two GPUs are visible.

Parity: the reference's two-worker HTTP deployment (docs/PHASE3_N2_PERF_BASELINE.md: coordinator
+ 2 workers, `/v1/completions`, `/health`, `/metrics`; rust/src/api/server.rs:39-205).
"""

import json
import os
import signal
import socket
import subprocess
import sys
import threading
import time
import urllib.request

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

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


def _post(port, body, raw=False):
    req = urllib.request.Request(f"http://127.0.0.1:{port}/v1/completions",
                                 data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=300) as r:
        data = r.read()
    return data.decode() if raw else json.loads(data)


@pytest.fixture(scope="module")
def server(tmp_path_factory):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models.weights import ModelWeights
    cfg = preset("tiny-gpu")
    w = ModelWeights.random_init(cfg, seed=3, dtype=torch.bfloat16)
    mdir = tmp_path_factory.mktemp("model")
    w.save(str(mdir))
    http = _port()
    env = dict(os.environ, HCP_QUIC_TIMEOUT_SECS="120", PYTHONPATH=REPO)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "-m", "hetero_cp_ringattn_b200", "serve", "--model-dir", str(mdir), "--device", "cuda",
           "--max-context", "4096", "--ratio", "3:1", "--ring-strategy", "zigzag",
           "--http-addr", f"127.0.0.1:{http}", "--export-logits", str(mdir / "dumps")]
    log = open(mdir / "serve.log", "w")
    proc = subprocess.Popen(cmd, cwd=REPO, env=env, stdout=log, stderr=subprocess.STDOUT,
                            start_new_session=True)
    try:
        deadline = time.time() + 600
        while True:
            try:
                health = _get(http, "/health")
                break
            except OSError:
                if proc.poll() is not None or time.time() > deadline:
                    log.flush()
                    raise RuntimeError("serve did not come up:\n" + (mdir / "serve.log").read_text()[-4000:])
                time.sleep(0.5)
        yield mdir, http, health, proc, mdir / "serve.log"
    finally:
        if proc.poll() is None:
            proc.send_signal(signal.SIGINT)
            try:
                proc.wait(timeout=90)
            except subprocess.TimeoutExpired:
                os.killpg(proc.pid, signal.SIGKILL)  # the process group this fixture started
                proc.wait(timeout=30)
        log.close()


def _single_gpu_prefill_logits(mdir, ids):
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    dev = torch.device("cuda", 0)
    hf = ModelWeights.from_dir(str(mdir), device=dev)
    eng = LlamaCPEngine(hf.cfg, PreparedWeights.from_weights(hf), device=dev, max_context=4096,
                        max_batch=1, decode_reserve=16)
    _, logits = eng.prefill(1, torch.tensor(ids), [len(ids)], decode_horizon=2, return_logits=True)
    out = logits.float().cpu().numpy()
    eng.release(1)
    eng.close()
    return out


def test_two_gpu_server_health_and_bit_identical_prefill(server):
    from hetero_cp_ringattn_b200.serve.logits_dump import read_raw_logits
    from hetero_cp_ringattn_b200.serve.tokenizer import load_tokenizer
    mdir, port, health, _, _ = server
    assert health["status"] == "ok" and health["workers_connected"] == 2
    tok = load_tokenizer(str(mdir), 1024)
    g = torch.Generator().manual_seed(11)
    for n in (700, 1500):      # several KV tiles per rank, split 3:1 in the zigzag layout
        ids = torch.randint(0, 1024, (n,), generator=g).tolist()
        res = _post(port, {"prompt": ids, "max_tokens": 1})
        assert res["usage"]["prompt_tokens"] == n and res["usage"]["completion_tokens"] == 1
        rid = res["id"].rsplit("-", 1)[1]
        got = read_raw_logits(str(mdir / "dumps" / f"request_{rid}" / "prefill_last_logits.f32le"))
        want = _single_gpu_prefill_logits(mdir, ids)
        assert got.shape == want.shape and (got == want).all(), \
            f"max diff {abs(got - want).max()}"
        assert res["choices"][0]["text"] == tok.decode([int(want.argmax())])


def test_two_gpu_server_stream_and_concurrency(server):
    _, port, _, _, _ = server
    sse = _post(port, {"prompt": "two gpus, one ring", "max_tokens": 8, "stream": True,
                       "ignore_eos": True}, raw=True)
    events = [ln[6:] for ln in sse.split("\n") if ln.startswith("data: ")]
    assert events[-1] == "[DONE]" and len(events) == 9
    out = {}

    def go(i):
        out[i] = _post(port, {"prompt": f"request {i} " * (20 + 30 * i), "max_tokens": 6,
                              "ignore_eos": True})

    ts = [threading.Thread(target=go, args=(i,)) for i in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=300)
    assert all(out[i]["usage"]["completion_tokens"] == 6 for i in range(4))
    m = _get(port, "/metrics")
    assert m["failed_requests"] == 0 and m["active_requests"] == 0
    assert m["completed_requests"] >= 5
