"""Failure detection on CPU ranks (gloo): nothing here faults, traps or hangs a GPU.

Parity with the reference's failure handling: bounded control-plane timeouts
(protocol.rs:348-353, HCP_QUIC_TIMEOUT_SECS), errors returned as `Error` responses without killing
the worker (runtime.rs:275,310), reservation rollback on a failed prefill (coordinator.rs:855-871),
rejection of truncated frames (tcp.rs partial-frame tests).
"""

import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hetero_cp_ringattn_b200.config import preset
from hetero_cp_ringattn_b200.errors import ProtocolError
from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
from hetero_cp_ringattn_b200.serve import protocol as P
from hetero_cp_ringattn_b200.serve.worker import Worker


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _never_joins(rank, port, q):
    if rank == 1:
        return  # this rank dies before joining the process group
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=timedelta(seconds=3))
        q.put(("joined", time.time() - t0))
    except Exception as e:  # expected: rendezvous times out
        q.put(("error", time.time() - t0, type(e).__name__))


def test_rank_that_never_joins_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_never_joins, args=(r, free_port() if r == 0 else 0, q)) for r in (0, 1)]
    port = free_port()
    procs = [ctx.Process(target=_never_joins, args=(r, port, q)) for r in (0, 1)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "error" and res[1] < 60


def _dies_between_steps(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=5))
    cp = P.ControlPlane(dist.group.WORLD, rank, 2)
    cmd = cp.broadcast(P.ReleaseRequest(1) if rank == 0 else None)
    assert isinstance(cmd, P.ReleaseRequest)
    cp.gather(P.Ack(1))
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    t0 = time.time()
    try:
        cp.broadcast(P.ReleaseRequest(2))
        cp.gather(P.Ack(2))
        q.put(("no-error", time.time() - t0))
    except Exception as e:
        q.put(("error", time.time() - t0, type(e).__name__))


def test_rank_that_leaves_between_steps_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_dies_between_steps, args=(r, port, q)) for r in (0, 1)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0] == "error" and res[1] < 60


def test_truncated_and_unknown_frames_are_rejected():
    frame = P.encode(P.DecodeBatch([[1, 2]]))
    for bad in (frame[:3], frame[:-2], b"\x00\x00\x00\x02{}"):
        with pytest.raises(ProtocolError):
            P.decode(bad)
    with pytest.raises(ProtocolError):
        P.encode(object())
    with pytest.raises(ProtocolError):
        P.unpack_handshake(b"\x00" * 15)


def test_errors_become_responses_and_the_worker_keeps_serving():
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=0, dtype=torch.float32, std=0.2)
    eng = LlamaCPEngine(cfg, PreparedWeights.from_weights(w, dtype=torch.float32),
                        device=torch.device("cpu"), max_context=64)
    worker = Worker(eng, P.ControlPlane())
    # context longer than the engine's capacity -> Error, not an exception
    r = worker.execute(P.Prefill(1, list(range(100)), [100], "vanilla", 4))
    assert isinstance(r, P.Error) and "capacity" in r.message
    # unknown request -> Error
    r = worker.execute(P.DecodeBatch([[77, 3]]))
    assert isinstance(r, P.Error)
    # invalid stationary decode plan -> Error
    r = worker.execute(P.StationaryDecode(1, 3, 10, [0], 0, 0, 4))
    assert isinstance(r, P.Error)
    # the worker still serves a valid request afterwards
    r = worker.execute(P.Prefill(2, [1, 2, 3, 4], [4], "vanilla", 4))
    assert isinstance(r, P.PrefillDone)
    r = worker.execute(P.StationaryDecode(2, r.token, 4, [1], 0, 0, 4))
    assert isinstance(r, P.DecodeDone)
    assert isinstance(worker.execute(P.ReleaseRequest(2)), P.Ack)


def test_broken_control_group_fails_requests_and_health():
    """A control-group failure (here a fake whose collectives raise, as a dead rank's gloo
    connection does) fails the request with a 500, and /health turns 503 so an orchestrator can
    restart the job; rank-level errors keep /health ok."""
    import json
    import urllib.error
    import urllib.request
    from hetero_cp_ringattn_b200.serve.coordinator import Coordinator, CoordinatorArgs
    from hetero_cp_ringattn_b200.serve.http_server import ApiServer, ApiState
    from hetero_cp_ringattn_b200.serve.tokenizer import ByteTokenizer

    class BrokenControl(P.ControlPlane):
        def __init__(self):
            super().__init__(None, 0, 1)
            self.broken = False

        def broadcast(self, cmd=None):
            if self.broken:
                raise RuntimeError("Connection closed by peer [127.0.0.1]:1234")
            return cmd

        def gather(self, resp):
            return [resp]

    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=0, dtype=torch.float32, std=0.2)
    eng = LlamaCPEngine(cfg, PreparedWeights.from_weights(w, dtype=torch.float32),
                        device=torch.device("cpu"), max_context=64)
    control = BrokenControl()
    tok = ByteTokenizer(cfg.vocab_size)
    coord = Coordinator(Worker(eng, control), control, tok, cfg, CoordinatorArgs())
    srv = ApiServer(ApiState(coord, tok, "tiny", 1)).start()

    def health():
        try:
            with urllib.request.urlopen(f"http://127.0.0.1:{srv.port}/health", timeout=10) as r:
                return r.status, json.loads(r.read())
        except urllib.error.HTTPError as e:
            return e.code, json.loads(e.read())

    try:
        ok = coord.generate(tok.encode("fine"), max_tokens=2)
        assert "error" not in ok and health()[0] == 200
        control.broken = True
        bad = coord.generate(tok.encode("broken"), max_tokens=2)
        assert bad.get("status") == 500 and "Connection closed" in bad["error"]
        code, body = health()
        assert code == 503 and body["status"] == "unhealthy" and "Connection closed" in body["error"]
    finally:
        srv.stop()
