"""Control protocol, scheduler, coordinator and HTTP API on a single CPU rank.

Parity: rust/src/distributed/protocol.rs:555-763 (validators, frames), scheduler.rs:171-420,
api/server.rs:211-438 (API contract incl. SSE [DONE], /health, /metrics), api/types.rs:159-214
(session field validation), worker_sdk/tch_backend.rs:1765 (decode after release fails).
"""

import json
import threading
import urllib.error
import urllib.request

import pytest
import torch

from hetero_cp_ringattn_b200.config import preset
from hetero_cp_ringattn_b200.errors import ProtocolError
from hetero_cp_ringattn_b200.models import reference_model
from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
from hetero_cp_ringattn_b200.serve import protocol as P
from hetero_cp_ringattn_b200.serve.coordinator import Coordinator, CoordinatorArgs
from hetero_cp_ringattn_b200.serve.http_server import ApiServer, ApiState
from hetero_cp_ringattn_b200.serve.scheduler import BatchScheduler, Job
from hetero_cp_ringattn_b200.serve.tokenizer import ByteTokenizer
from hetero_cp_ringattn_b200.serve.worker import Worker


def test_protocol_roundtrip_and_partial_frames():
    for msg in [P.Prefill(1, [1, 2, 3], [2, 1], "zigzag", 8, [5, 1], True), P.Decode(3, 7),
                P.DecodeBatch([[1, 2], [3, 4]]), P.StationaryDecode(1, 2, 3, [1, 1], 0, 0, 4),
                P.ReleaseRequest(9), P.Shutdown(), P.PrefillDone(1, 5, 3), P.Error(1, "x")]:
        frame = P.encode(msg)
        assert P.as_plain(P.decode(frame)) == P.as_plain(msg)
        with pytest.raises(ProtocolError):
            P.decode(frame[:-1])
        with pytest.raises(ProtocolError):
            P.decode(frame + b"\x00")
    with pytest.raises(ProtocolError):
        P.decode(b"\x00\x00\x00\x05{\"ty")
    # the wire layout: [u32 payload][u8 version][u8 type][fields], token arrays as raw int64
    f = P.encode(P.Prefill(7, [1, 2, 3], [3], "vanilla", 4, None, False))
    assert f[4] == 1 and f[5] == 1 and int.from_bytes(f[:4], "little") == len(f) - 4
    bad = bytearray(f)
    bad[4] = 9
    with pytest.raises(ProtocolError, match="version"):
        P.decode(bytes(bad))
    bad[4], bad[5] = 1, 200
    with pytest.raises(ProtocolError, match="unknown message type"):
        P.decode(bytes(bad))
    big = P.decode(P.encode(P.Prefill(1, list(range(70000)), [70000], "zigzag", 4, [1], True)))
    assert big.prompt.dtype.name == "int64" and int(big.prompt[-1]) == 69999
    assert big.chunks == [70000] and big.capacity_tickets == [1] and big.keep_kv is True
    hs = P.pack_handshake(3, 4096)
    assert len(hs) == 16 and P.unpack_handshake(hs) == (3, 4096)


def test_validators():
    P.validate_stationary_decode(2, [1, 1], 1, 0, 4)
    for args in [(0, [], 0, 0, 1), (2, [1], 0, 0, 1), (2, [0, 0], 0, 0, 1), (2, [1, 1], 2, 0, 1),
                 (2, [1, 1], 0, 0, 0), (2, [1, 1], 0, 4, 4)]:
        with pytest.raises(ProtocolError):
            P.validate_stationary_decode(*args)
    P.validate_stationary_continuation(2, [1, 2], [5, 6], [1, 1], 0)
    for args in [(2, [], [], [1, 1], 0), (2, [1], [1, 2], [1, 1], 0), (2, [1], [1], [1], 0),
                 (2, [1], [1], [0, 0], 0), (2, [1], [1], [1, 1], 3)]:
        with pytest.raises(ProtocolError):
            P.validate_stationary_continuation(*args)


def test_scheduler_fifo_and_capacity():
    s = BatchScheduler(max_batch_size=2)
    for i in range(3):
        s.enqueue(Job(request_id=i, prompt_ids=[1]))
    from hetero_cp_ringattn_b200.serve.scheduler import ActiveRequest
    a = s.pop_pending()
    s.activate(ActiveRequest(job=a, chunks=[1]))
    b = s.pop_pending()
    s.activate(ActiveRequest(job=b, chunks=[1]))
    assert (a.request_id, b.request_id) == (0, 1)
    assert s.pop_pending() is None  # full
    s.complete(0)
    assert s.pop_pending().request_id == 2
    with pytest.raises(ValueError):
        BatchScheduler(0)


@pytest.fixture(scope="module")
def stack():
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=0, dtype=torch.float32, std=0.2)
    pw = PreparedWeights.from_weights(w, dtype=torch.float32)
    eng = LlamaCPEngine(cfg, pw, device=torch.device("cpu"), max_context=512)
    control = P.ControlPlane()
    worker = Worker(eng, control)
    tok = ByteTokenizer(cfg.vocab_size)
    coord = Coordinator(worker, control, tok, cfg, CoordinatorArgs(max_batch_size=4))
    return cfg, w, eng, coord, tok


def test_coordinator_generate_matches_reference(stack):
    cfg, w, eng, coord, tok = stack
    ids = tok.encode("hello heterogeneous ring")
    res = coord.generate(ids, max_tokens=5)
    ref_tokens, _ = reference_model.greedy_generate(w, torch.tensor(ids), 4)
    assert res["tokens"] == ref_tokens
    assert res["finish_reason"] == "length"
    assert not eng.reqs  # released


def test_coordinator_batches_concurrent_requests(stack):
    cfg, w, eng, coord, tok = stack
    outs = {}
    jobs = []
    for i, text in enumerate(["abc", "a much longer prompt here", "xyz!"]):
        ids = tok.encode(text)
        jobs.append((ids, i))
        coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=ids, max_tokens=4,
                         done=lambda r, i=i: outs.__setitem__(i, r)))
    while len(outs) < 3:
        coord.iteration()
    for ids, i in jobs:
        ref_tokens, _ = reference_model.greedy_generate(w, torch.tensor(ids), 3)
        assert outs[i]["tokens"] == ref_tokens


def test_decode_after_release_fails(stack):
    cfg, w, eng, coord, tok = stack
    r = coord.worker.execute(P.Prefill(999, [1, 2, 3], [3], "vanilla", 4))
    assert isinstance(r, P.PrefillDone)
    assert isinstance(coord.worker.execute(P.ReleaseRequest(999)), P.Ack)
    r = coord.worker.execute(P.DecodeBatch([[999, r.token]]))
    assert isinstance(r, P.Error)


def _post(port, body, raw=False):
    req = urllib.request.Request(f"http://127.0.0.1:{port}/v1/completions",
                                 data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=60) as r:
        data = r.read().decode()
    return data if raw else json.loads(data)


def test_http_api(stack):
    cfg, w, eng, coord, tok = stack
    stop = threading.Event()
    loop = threading.Thread(target=lambda: [coord.iteration() or stop.wait(0.005) for _ in iter(stop.is_set, True)],
                            daemon=True)
    loop.start()
    srv = ApiServer(ApiState(coord, tok, "tiny", 1)).start()
    try:
        with urllib.request.urlopen(f"http://127.0.0.1:{srv.port}/health", timeout=10) as r:
            h = json.loads(r.read())
        assert h == {"status": "ok", "workers_connected": 1, "num_domains": 1}
        with urllib.request.urlopen(f"http://127.0.0.1:{srv.port}/v1/models", timeout=10) as r:
            assert json.loads(r.read())["data"][0]["id"] == "tiny"
        ids_prompt = tok.encode("token ids")
        by_ids = _post(srv.port, {"prompt": ids_prompt, "max_tokens": 3})
        ref_ids, _ = reference_model.greedy_generate(w, torch.tensor(ids_prompt), 2)
        assert by_ids["choices"][0]["text"] == tok.decode(ref_ids)
        assert by_ids["usage"]["prompt_tokens"] == len(ids_prompt)
        for bad in ({"prompt": [1, "a"]}, {"prompt": []}, {"prompt": [cfg.vocab_size]}):
            with pytest.raises(urllib.error.HTTPError) as ei:
                _post(srv.port, bad)
            assert ei.value.code == 422
        res = _post(srv.port, {"prompt": "ring attention", "max_tokens": 4})
        assert res["object"] == "text_completion"
        assert res["usage"]["completion_tokens"] == 4
        assert res["usage"]["total_tokens"] == res["usage"]["prompt_tokens"] + 4
        ids = tok.encode("ring attention")
        ref_tokens, _ = reference_model.greedy_generate(w, torch.tensor(ids), 3)
        assert res["choices"][0]["text"] == tok.decode(ref_tokens)
        sse = _post(srv.port, {"prompt": "ring attention", "max_tokens": 3, "stream": True}, raw=True)
        events = [ln[6:] for ln in sse.split("\n") if ln.startswith("data: ")]
        assert events[-1] == "[DONE]"
        chunks = [json.loads(e) for e in events[:-1]]
        assert len(chunks) == 3 and chunks[-1]["choices"][0]["finish_reason"] == "length"
        with pytest.raises(urllib.error.HTTPError) as ei:
            _post(srv.port, {"prompt": "x", "append": True})
        assert ei.value.code == 400
        for bad in ({"prompt": "x", "max_tokens": "5"}, {"prompt": "x", "max_tokens": 0},
                    {"prompt": "x", "temperature": -1}, {"prompt": "x", "top_p": 0},
                    {"prompt": "x", "stream": "yes"}, {"prompt": "x", "stop": [1]},
                    {"prompt": "x", "max_tokens": True}, {"prompt": 3}):
            with pytest.raises(urllib.error.HTTPError) as ei:
                _post(srv.port, bad)
            assert ei.value.code == 422, bad
        import http.client
        conn = http.client.HTTPConnection("127.0.0.1", srv.port, timeout=10)
        conn.putrequest("POST", "/v1/completions")
        conn.putheader("Content-Length", str(1 << 40))
        conn.endheaders()
        assert conn.getresponse().status == 413
        conn.close()
        with pytest.raises(urllib.error.HTTPError) as ei:
            _post(srv.port, {"prompt": "x", "keep_kv": True})
        assert ei.value.code == 400
        with urllib.request.urlopen(f"http://127.0.0.1:{srv.port}/metrics", timeout=10) as r:
            m = json.loads(r.read())
        assert m["completed_requests"] >= 2 and m["failed_requests"] >= 2
        assert set(m) == {"total_requests", "completed_requests", "failed_requests",
                          "queued_requests", "active_requests"}
        with urllib.request.urlopen(f"http://127.0.0.1:{srv.port}/metrics/prometheus",
                                    timeout=10) as r:
            prom = r.read().decode()
        lines = dict(ln.rsplit(" ", 1) for ln in prom.splitlines() if not ln.startswith("#"))
        assert int(lines["hcp_requests_completed_total"]) == m["completed_requests"]
        assert int(lines["hcp_generated_tokens_total"]) >= 7
        assert int(lines['hcp_ttft_seconds_bucket{le="+Inf"}']) == int(lines["hcp_ttft_seconds_count"])
        assert int(lines["hcp_ttft_seconds_count"]) >= 2
        parser = pytest.importorskip("prometheus_client.parser")
        fams = {f.name: f for f in parser.text_string_to_metric_families(prom)}
        assert fams["hcp_ttft_seconds"].type == "histogram"
        assert fams["hcp_requests_active"].type == "gauge"
    finally:
        srv.stop()
        stop.set()
        loop.join(timeout=5)


def test_continuation_e2e_and_logits_dumps(stack, tmp_path):
    """The reference's experimental continuation run (coordinator.rs:1973-2245) on one rank:
    prefill, one decode, a continuation segment right after it, greedy decode; the three logits
    dumps equal the dense oracle's last-row logits of the matching prefixes."""
    from hetero_cp_ringattn_b200.serve.logits_dump import read_raw_logits
    cfg, w, eng, coord, tok = stack
    coord.args.export_logits_dir = str(tmp_path / "cont")
    try:
        prompt = tok.encode("stationary continuation")
        seg = tok.encode(" and more")
        meta = coord.continuation_e2e(77, prompt, seg, max_tokens=4, tickets=[1])
        t0 = meta["decode_token"]
        ref_more, _ = reference_model.greedy_generate(w, torch.tensor(prompt + [t0] + seg), 2)
        assert meta["generated_ids"] == [t0] + ref_more
        d = tmp_path / "cont"
        for name, ids in (("prefill_last_logits", prompt), ("decode_logits", prompt + [t0]),
                          ("continuation_last_logits", prompt + [t0] + seg)):
            got = read_raw_logits(str(d / f"{name}.f32le"))
            ref = reference_model.forward(w, torch.tensor(ids), last_only=True)[0]
            assert got.shape == (cfg.vocab_size,)
            assert abs(got - ref.numpy()).max() < 1e-3, name
        m = json.loads((d / "meta.json").read_text())
        assert m["generated_ids"] == meta["generated_ids"] and m["prefix_splits"] == [len(prompt)]
        assert m["continuation_offsets_by_domain"] == [list(range(len(seg)))]
        assert 77 not in eng.reqs  # released
        # the service path dumps per request
        res = coord.generate(prompt, max_tokens=2)
        pd = tmp_path / "cont" / f"request_{res['request_id']}"
        assert (pd / "prefill_last_logits.f32le").exists()
        assert json.loads((pd / "meta.json").read_text())["prefill_argmax"] == res["tokens"][0]
    finally:
        coord.args.export_logits_dir = None


def test_session_lifecycle_matches_reference_rules(stack):
    """keep_kv registers a session; append (+keep_kv) continues and advances it; an append
    without keep_kv ends it and frees its KV; a keep_kv id that already holds KV and an unknown
    session are rejected; a failed append drops its session (coordinator.rs:1743-1810,
    2630-2830). Every phase's tokens equal the dense oracle on the whole context."""
    cfg, w, eng, coord, tok = stack
    free0 = coord.ledger.free_bytes()
    prompt = tok.encode("session prompt")
    r1 = coord.generate(prompt, max_tokens=3, session_id="s", keep_kv=True)
    ref1, _ = reference_model.greedy_generate(w, torch.tensor(prompt), 2)
    assert r1["tokens"] == ref1 and "s" in coord.sessions
    with pytest.raises(P.ProtocolError):
        coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=[1, 2], session_id="s",
                         keep_kv=True))
    with pytest.raises(P.ProtocolError):
        coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=[1, 2], session_id="nope",
                         append=True))
    seg1 = tok.encode(" more")
    r2 = coord.generate(seg1, max_tokens=3, session_id="s", append=True, keep_kv=True)
    ctx = prompt + ref1 + seg1
    ref2, _ = reference_model.greedy_generate(w, torch.tensor(ctx), 2)
    assert r2["tokens"] == ref2
    seg2 = tok.encode(" end")
    r3 = coord.generate(seg2, max_tokens=2, session_id="s", append=True)
    ref3, _ = reference_model.greedy_generate(w, torch.tensor(ctx + ref2 + seg2), 1)
    assert r3["tokens"] == ref3
    assert "s" not in coord.sessions and not eng.reqs and coord.ledger.free_bytes() == free0
    # a failed append (segment past the engine's context) drops the session and its KV
    coord.generate(prompt, max_tokens=2, session_id="t", keep_kv=True)
    bad = coord.generate([5] * 600, max_tokens=2, session_id="t", append=True)
    assert "error" in bad and "t" not in coord.sessions and not eng.reqs
    assert coord.ledger.free_bytes() == free0


def test_kv_capacity_wall_queues_instead_of_failing(stack):
    """More concurrent long prompts than the KV byte budget holds (the reference's KV-wall scan,
    docs/PHASE3_KV_WALL_SCAN.md): admission keeps the ledger within budget, requests that do not
    fit wait for KV to be released, every request completes with the oracle's tokens; a request
    larger than the whole budget fails alone with a capacity error."""
    from hetero_cp_ringattn_b200.parallel.capacity import KvLedger
    cfg, w, eng, coord, tok = stack
    saved = coord.ledger
    per_req = (150 + 8) * cfg.num_layers * coord.bytes_per_token_layer
    budget = int(2.5 * per_req)
    coord.ledger = KvLedger([budget])
    try:
        outs, peak = {}, [0]
        prompts = [[(7 * i + j) % cfg.vocab_size for j in range(140)] for i in range(5)]
        for i, ids in enumerate(prompts):
            coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=ids, max_tokens=4,
                             done=lambda r, i=i: outs.__setitem__(i, r)))
        while len(outs) < len(prompts):
            coord.iteration()
            peak[0] = max(peak[0], coord.ledger.used[0])
            assert len(coord.sched.active) <= 2
        assert peak[0] <= budget
        for i, ids in enumerate(prompts):
            ref_tokens, _ = reference_model.greedy_generate(w, torch.tensor(ids), 3)
            assert outs[i].get("tokens") == ref_tokens, outs[i]
        huge = coord.generate([1] * 400, max_tokens=2)
        assert "error" in huge and huge["status"] == 400
        assert coord.ledger.used == [0] and not eng.reqs
    finally:
        coord.ledger = saved


def test_sse_streams_whole_characters():
    """Streamed deltas are incremental detokenizations: a multi-byte UTF-8 character split over
    tokens arrives whole, and the concatenated deltas equal the decoded completion."""
    from hetero_cp_ringattn_b200.serve.coordinator import Metrics
    from hetero_cp_ringattn_b200.serve.http_server import ApiServer, ApiState

    tok = ByteTokenizer(512)
    text = "héllo ✓ \U0001F600!"
    gen = tok.encode(text)                       # one token per UTF-8 byte

    class StubCoordinator:
        metrics = Metrics()

        def next_request_id(self):
            return 1

        def submit(self, job):
            for i, t in enumerate(gen):
                job.on_token(t, "length" if i == len(gen) - 1 else None)
            job.done({"request_id": 1, "tokens": gen, "prompt_tokens": 1,
                      "finish_reason": "length"})

    srv = ApiServer(ApiState(StubCoordinator(), tok, "stub", 1)).start()
    try:
        sse = _post(srv.port, {"prompt": "x", "max_tokens": len(gen), "stream": True}, raw=True)
    finally:
        srv.stop()
    events = [ln[6:] for ln in sse.split("\n") if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    deltas = [json.loads(e)["choices"][0]["text"] for e in events[:-1]]
    assert len(deltas) == len(gen) and "".join(deltas) == text
    assert all("�" not in d for d in deltas)


def test_stream_client_disconnect_aborts_generation(stack, tmp_path):
    """A streaming client that goes away stops its generation: the request finishes with
    finish_reason "abort" long before max_tokens and its KV is released."""
    from hetero_cp_ringattn_b200.serve.coordinator import TraceSink
    cfg, w, eng, coord, tok = stack
    saved = coord.trace
    coord.trace = TraceSink(str(tmp_path / "trace.jsonl"))
    stop = threading.Event()
    loop = threading.Thread(target=lambda: [coord.iteration() or stop.wait(0.002)
                                            for _ in iter(stop.is_set, True)], daemon=True)
    loop.start()
    srv = ApiServer(ApiState(coord, tok, "tiny", 1)).start()
    try:
        req = urllib.request.Request(
            f"http://127.0.0.1:{srv.port}/v1/completions",
            data=json.dumps({"prompt": "abc", "max_tokens": 450, "stream": True,
                             "ignore_eos": True}).encode(),
            headers={"Content-Type": "application/json"})
        r = urllib.request.urlopen(req, timeout=30)
        assert r.readline().startswith(b"data: ")
        r.close()
        done = None
        for _ in range(500):
            evs = [json.loads(l) for l in open(tmp_path / "trace.jsonl")]
            done = [e for e in evs if e["event"] == "completed"]
            if done:
                break
            stop.wait(0.02)
        assert done and done[0]["finish_reason"] == "abort"
        assert done[0]["completion_tokens"] < 450
        for _ in range(100):
            if not eng.reqs:
                break
            stop.wait(0.02)
        assert not eng.reqs and not coord.sched.active
    finally:
        srv.stop()
        stop.set()
        loop.join(timeout=5)
        coord.trace = saved


def test_session_append_longer_than_default_horizon(stack):
    """An append may generate more tokens than the default continuation horizon: the horizon
    travels with the continuation command."""
    cfg, w, eng, coord, tok = stack
    p1 = tok.encode("long")
    r1 = coord.generate(p1, max_tokens=2, session_id="long", keep_kv=True)
    seg = tok.encode(" tail")
    r2 = coord.generate(seg, max_tokens=150, session_id="long", append=True)
    assert "error" not in r2 and len(r2["tokens"]) == 150
    ref, _ = reference_model.greedy_generate(w, torch.tensor(p1 + r1["tokens"] + seg), 149)
    assert r2["tokens"] == ref


def test_chunked_prefill_interleaves_with_decode(stack):
    """With prefill_chunk_tokens a long prompt is prefilled piece by piece while an active
    request keeps decoding between the pieces; both outputs equal the oracle's, and a keep_kv
    session built by a chunked prefill continues correctly."""
    cfg, w, eng, coord, tok = stack
    coord.args.prefill_chunk_tokens = 16
    try:
        events = []
        outs = {}
        short = tok.encode("short one")
        long_ = [(11 * j + 5) % cfg.vocab_size for j in range(100)]
        for name, ids, n in (("short", short, 12), ("long", long_, 4)):
            coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=ids, max_tokens=n,
                             on_token=lambda t, fr, name=name: events.append(name),
                             done=lambda r, name=name: outs.__setitem__(name, r)))
        while len(outs) < 2:
            coord.iteration()
        for name, ids, n in (("short", short, 12), ("long", long_, 4)):
            ref, _ = reference_model.greedy_generate(w, torch.tensor(ids), n - 1)
            assert outs[name]["tokens"] == ref
        # the short request emitted tokens while the long prompt was still being prefilled
        assert events.index("long") >= 5 and events[:5] == ["short"] * 5
        r1 = coord.generate(long_, max_tokens=3, session_id="chunked", keep_kv=True)
        seg = tok.encode(" next")
        r2 = coord.generate(seg, max_tokens=3, session_id="chunked", append=True)
        ref2, _ = reference_model.greedy_generate(w, torch.tensor(long_ + r1["tokens"] + seg), 2)
        assert r2["tokens"] == ref2 and not eng.reqs
    finally:
        coord.args.prefill_chunk_tokens = 0


def test_session_requests_survive_a_capacity_wait(stack):
    """keep_kv and append jobs that wait for KV (ledger full while another request runs) are
    admitted later and keep their session semantics."""
    from hetero_cp_ringattn_b200.parallel.capacity import KvLedger
    cfg, w, eng, coord, tok = stack
    saved = coord.ledger
    per_req = (60 + 40) * cfg.num_layers * coord.bytes_per_token_layer
    coord.ledger = KvLedger([int(1.5 * per_req)])
    try:
        outs = {}
        blocker = [(3 * j + 2) % cfg.vocab_size for j in range(60)]
        p1 = [(5 * j + 1) % cfg.vocab_size for j in range(60)]
        coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=blocker, max_tokens=6,
                         done=lambda r: outs.__setitem__("blocker", r)))
        coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=p1, max_tokens=3,
                         session_id="wait", keep_kv=True, done=lambda r: outs.__setitem__("s", r)))
        while len(outs) < 2:
            coord.iteration()
        assert "error" not in outs["s"] and "wait" in coord.sessions
        ref1, _ = reference_model.greedy_generate(w, torch.tensor(p1), 2)
        assert outs["s"]["tokens"] == ref1
        seg = tok.encode(" go")
        r2 = coord.generate(seg, max_tokens=2, session_id="wait", append=True)
        ref2, _ = reference_model.greedy_generate(w, torch.tensor(p1 + ref1 + seg), 1)
        assert r2["tokens"] == ref2 and not eng.reqs
    finally:
        coord.ledger = saved


def test_queue_limit_answers_503(stack):
    cfg, w, eng, coord, tok = stack
    from hetero_cp_ringattn_b200.errors import Overloaded
    from hetero_cp_ringattn_b200.serve.http_server import ApiServer, ApiState
    coord.args.max_queue = 2
    srv = ApiServer(ApiState(coord, tok, "tiny", 1)).start()
    try:
        jobs = [Job(request_id=coord.next_request_id(), prompt_ids=[1, 2, 3], max_tokens=2)
                for _ in range(2)]
        for j in jobs:
            coord.submit(j)
        with pytest.raises(Overloaded):
            coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=[1, 2], max_tokens=1))
        with pytest.raises(urllib.error.HTTPError) as ei:
            _post(srv.port, {"prompt": "over the limit", "max_tokens": 1})
        assert ei.value.code == 503
        while coord.sched.queued or coord.sched.active:
            coord.iteration()
    finally:
        srv.stop()
        coord.args.max_queue = 0


def test_stop_strings_cut_the_completion(stack):
    """`stop` ends generation once the text contains a stop string and the string is not
    returned, in plain and streamed responses (no part of it is ever streamed)."""
    cfg, w, eng, coord, tok = stack
    from hetero_cp_ringattn_b200.serve.http_server import ApiServer, ApiState
    prompt = "stop sequences"
    ref_tokens, _ = reference_model.greedy_generate(w, torch.tensor(tok.encode(prompt)), 15)
    full = tok.decode(ref_tokens)
    stop = full[6:8]
    expected = full[:full.find(stop)]
    stopper = threading.Event()
    loop = threading.Thread(target=lambda: [coord.iteration() or stopper.wait(0.002)
                                            for _ in iter(stopper.is_set, True)], daemon=True)
    loop.start()
    srv = ApiServer(ApiState(coord, tok, "tiny", 1)).start()
    try:
        res = _post(srv.port, {"prompt": prompt, "max_tokens": 16, "stop": [stop, "never-there"]})
        assert res["choices"][0]["text"] == expected
        assert res["choices"][0]["finish_reason"] == "stop"
        assert res["usage"]["completion_tokens"] < 16
        sse = _post(srv.port, {"prompt": prompt, "max_tokens": 16, "stop": stop, "stream": True},
                    raw=True)
        events = [ln[6:] for ln in sse.split("\n") if ln.startswith("data: ")]
        deltas = [json.loads(e)["choices"][0]["text"] for e in events[:-1]]
        assert "".join(deltas) == expected
        assert json.loads(events[-2])["choices"][0]["finish_reason"] == "stop"
    finally:
        srv.stop()
        stopper.set()
        loop.join(timeout=5)


def test_streaming_with_a_byte_level_bpe_tokenizer(tmp_path):
    """HF tokenizer.json (a byte-level BPE trained here offline): load_tokenizer picks it up,
    and the streamed deltas of a text with spaces and multi-byte characters, decoded through the
    sliding window, concatenate to the full decode."""
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers import decoders, models, pre_tokenizers, trainers
    from hetero_cp_ringattn_b200.serve.coordinator import Metrics
    from hetero_cp_ringattn_b200.serve.http_server import ApiServer, ApiState
    from hetero_cp_ringattn_b200.serve.tokenizer import HfTokenizer, load_tokenizer

    bpe = tokenizers.Tokenizer(models.BPE())
    bpe.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    bpe.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=400, initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    bpe.train_from_iterator(["hello world, ring attention over many ranks", "héllo wörld ✓ 😀"] * 20,
                            trainer)
    bpe.save(str(tmp_path / "tokenizer.json"))
    tok = load_tokenizer(str(tmp_path), 512)
    assert isinstance(tok, HfTokenizer)
    text = "hello wörld, ring ✓ over ranks 😀!"
    gen = tok.encode(text)
    assert tok.decode(gen) == text

    class StubCoordinator:
        metrics = Metrics()

        def next_request_id(self):
            return 1

        def submit(self, job):
            for i, t in enumerate(gen):
                job.on_token(t, "length" if i == len(gen) - 1 else None)
            job.done({"request_id": 1, "tokens": gen, "prompt_tokens": 1,
                      "finish_reason": "length"})

    srv = ApiServer(ApiState(StubCoordinator(), tok, "bpe", 1)).start()
    try:
        sse = _post(srv.port, {"prompt": "x", "max_tokens": len(gen), "stream": True}, raw=True)
    finally:
        srv.stop()
    events = [ln[6:] for ln in sse.split("\n") if ln.startswith("data: ")]
    deltas = [json.loads(e)["choices"][0]["text"] for e in events[:-1]]
    assert "".join(deltas) == text and all("�" not in d for d in deltas)


def test_more_active_requests_than_one_engine_decode_batch(stack):
    """Six concurrent requests with an engine decode batch of 4: each iteration decodes them in
    two engine steps; every output equals the oracle's."""
    cfg, w, eng, coord, tok = stack
    saved = (coord.sched, coord.args.decode_batch_limit)
    from hetero_cp_ringattn_b200.serve.scheduler import BatchScheduler
    coord.sched = BatchScheduler(6)
    coord.args.decode_batch_limit = 4
    seen = []
    orig = coord.run_command

    def spy(cmd):
        if isinstance(cmd, P.DecodeBatch):
            seen.append(len(cmd.request_tokens))
        return orig(cmd)

    coord.run_command = spy
    try:
        outs = {}
        prompts = [tok.encode(f"request {i} " + "x" * i) for i in range(6)]
        for i, ids in enumerate(prompts):
            coord.submit(Job(request_id=coord.next_request_id(), prompt_ids=ids, max_tokens=5,
                             done=lambda r, i=i: outs.__setitem__(i, r)))
        while len(outs) < 6:
            coord.iteration()
        assert max(seen) == 4 and 2 in seen
        for i, ids in enumerate(prompts):
            ref, _ = reference_model.greedy_generate(w, torch.tensor(ids), 4)
            assert outs[i]["tokens"] == ref
    finally:
        del coord.run_command
        coord.sched, coord.args.decode_batch_limit = saved


def test_ledger_follows_the_kv_arena_in_pages():
    """With the ranks' KV arena sizes the ledger budget is the smaller of free memory and arena
    bytes, and each rank's rows are rounded up to whole pages; a rank's own capacity error
    ("CapacityError: ...") takes the capacity path (wait for KV, else 400), not a 500."""
    from hetero_cp_ringattn_b200.serve.coordinator import Coordinator, CoordinatorArgs

    class Fake:
        last_logits = None
        fail = False

        def execute(self, cmd):
            if isinstance(cmd, P.Prefill):
                if self.fail:
                    return P.Error(cmd.request_id, "CapacityError: KV arena out of pages")
                return P.PrefillDone(cmd.request_id, 7, len(cmd.prompt))
            return P.Ack(getattr(cmd, "request_id", -1))

    cfg = preset("tiny")
    bpt = cfg.kv_bytes_per_token_per_layer(2) * cfg.num_layers
    fake = Fake()
    coord = Coordinator(fake, P.ControlPlane(), ByteTokenizer(cfg.vocab_size), cfg,
                        CoordinatorArgs(kv_page_tokens=16, activation_reserve_mb=0),
                        capacities_mb=[1024], kv_budget_bytes=[10 * 16 * bpt])
    assert coord.ledger.budgets == [10 * 16 * bpt]
    per = coord._reserve(1, [20], 3)          # 20 rows + 4 growth -> 2 pages
    assert per == [2 * 16 * bpt]
    fake.fail = True
    res = coord.generate([1, 2, 3], max_tokens=2)
    assert res["status"] == 400 and "CapacityError" in res["error"]


def test_idle_sessions_expire_with_a_ttl(stack):
    cfg, w, eng, coord, tok = stack
    free0 = coord.ledger.free_bytes()
    coord.args.session_ttl_s = 0.05
    try:
        coord.generate(tok.encode("ttl"), max_tokens=2, session_id="idle", keep_kv=True)
        assert "idle" in coord.sessions and eng.reqs
        import time
        time.sleep(0.1)
        coord.iteration()
        assert "idle" not in coord.sessions and not eng.reqs
        assert coord.ledger.free_bytes() == free0
        with pytest.raises(ProtocolError, match="unknown or expired"):
            coord.generate(tok.encode("x"), max_tokens=1, session_id="idle", append=True)
    finally:
        coord.args.session_ttl_s = 0.0


def test_worker_backend_interface_drives_the_control_plane():
    """Any `WorkerBackend` implementation can sit under the worker: a scripted backend serves a
    request through the coordinator; an incomplete implementation cannot be instantiated."""
    from hetero_cp_ringattn_b200.serve.backend import WorkerBackend
    from hetero_cp_ringattn_b200.serve.coordinator import Coordinator, CoordinatorArgs

    class Counting(WorkerBackend):
        def __init__(self):
            self.reqs = {}

        def prefill(self, request_id, prompt, chunks, strategy, decode_horizon, tickets, keep_kv,
                    want_logits=True):
            self.reqs[request_id] = [len(prompt), 0]
            return 10, None

        def decode_batch(self, request_ids, tokens, want_logits=True):
            for r in request_ids:
                self.reqs[r][0] += 1
                self.reqs[r][1] += 1
            return [t + 1 for t in tokens], None

        def continuation(self, request_id, tokens, position_ids, tickets, horizon,
                         want_logits=True):
            self.reqs[request_id][0] += len(tokens)
            return 99, None

        def release(self, request_id):
            return self.reqs.pop(request_id, None) is not None

        def context_len(self, request_id):
            return self.reqs[request_id][0] if request_id in self.reqs else None

        def decode_offset(self, request_id):
            return self.reqs[request_id][1] if request_id in self.reqs else None

        world = property(lambda self: 1)
        rank = property(lambda self: 0)

        def capacity_mb(self):
            return 1024

        def num_layers(self):
            return 2

        def device(self):
            return "scripted"

    backend = Counting()
    worker = Worker(backend, P.ControlPlane())
    cfg = preset("tiny")
    coord = Coordinator(worker, P.ControlPlane(), ByteTokenizer(cfg.vocab_size), cfg,
                        CoordinatorArgs())
    res = coord.generate([1, 2, 3], max_tokens=4)
    assert res["tokens"] == [10, 11, 12, 13] and not backend.reqs
    assert worker.handshake() == P.pack_handshake(0, 1024) and worker.device() == "scripted"

    class Incomplete(WorkerBackend):
        pass

    with pytest.raises(TypeError):
        Incomplete()


def test_prefill_ships_logits_only_when_read(stack):
    """Greedy requests do not move the first token's logits to the ranks; sampling does."""
    cfg, w, eng, coord, tok = stack
    seen = []
    orig = coord.run_command

    def spy(cmd):
        if isinstance(cmd, P.Prefill):
            seen.append(cmd.want_logits)
        return orig(cmd)

    coord.run_command = spy
    try:
        g = coord.generate(tok.encode("greedy"), max_tokens=3)
        ref, _ = reference_model.greedy_generate(w, torch.tensor(tok.encode("greedy")), 2)
        assert g["tokens"] == ref
        s = coord.generate(tok.encode("sampled"), max_tokens=3, temperature=0.8)
        assert len(s["tokens"]) == 3 and all(0 <= t < cfg.vocab_size for t in s["tokens"])
        assert seen == [False, True]
    finally:
        del coord.run_command


def test_single_token_generations_on_every_path(stack):
    """max_tokens=1 finishes at the first token on the plain, chunked-prefill and session paths,
    and an EOS as the first token ends the request with finish_reason "stop"; no KV is left."""
    cfg, w, eng, coord, tok = stack
    ids = [(7 * j + 3) % cfg.vocab_size for j in range(40)]
    ref, _ = reference_model.greedy_generate(w, torch.tensor(ids), 0)
    r = coord.generate(ids, max_tokens=1)
    assert r["tokens"] == ref[:1] and r["finish_reason"] == "length"
    coord.args.prefill_chunk_tokens = 8
    try:
        r = coord.generate(ids, max_tokens=1)
        assert r["tokens"] == ref[:1]
    finally:
        coord.args.prefill_chunk_tokens = 0
    r = coord.generate(ids, max_tokens=1, session_id="one", keep_kv=True)
    seg = [5, 6, 7]
    r2 = coord.generate(seg, max_tokens=1, session_id="one", append=True)
    ref2, _ = reference_model.greedy_generate(w, torch.tensor(ids + ref[:1] + seg), 0)
    assert r2["tokens"] == ref2[:1]
    saved = coord.args.eos_ids
    coord.args.eos_ids = [ref[0]]
    try:
        r = coord.generate(ids, max_tokens=5)
        assert r["tokens"] == ref[:1] and r["finish_reason"] == "stop"
    finally:
        coord.args.eos_ids = saved
    assert not eng.reqs and not coord.sched.active and not coord._prefilling


def test_plain_client_disconnect_aborts_generation(stack, tmp_path):
    """A non-streaming client that closes its connection while it waits also stops its
    generation: the handler sees the close, the request finishes with "abort", KV released."""
    import socket
    from hetero_cp_ringattn_b200.serve.coordinator import TraceSink
    cfg, w, eng, coord, tok = stack
    saved = coord.trace
    coord.trace = TraceSink(str(tmp_path / "trace.jsonl"))
    stop = threading.Event()
    loop = threading.Thread(target=lambda: [coord.iteration() or stop.wait(0.002)
                                            for _ in iter(stop.is_set, True)], daemon=True)
    loop.start()
    aborted0 = coord.metrics.aborted
    srv = ApiServer(ApiState(coord, tok, "tiny", 1)).start()
    try:
        body = json.dumps({"prompt": "abc", "max_tokens": 450, "ignore_eos": True}).encode()
        s = socket.create_connection(("127.0.0.1", srv.port), timeout=30)
        s.sendall(b"POST /v1/completions HTTP/1.1\r\nHost: x\r\nContent-Type: application/json\r\n"
                  + f"Content-Length: {len(body)}\r\n\r\n".encode() + body)
        trace = tmp_path / "trace.jsonl"

        def events():
            return [json.loads(l) for l in open(trace)] if trace.exists() else []

        done = None
        for _ in range(500):
            evs = events()
            if any(e["event"] in ("prefill_accepted", "token") for e in evs):
                break
            stop.wait(0.01)
        s.close()
        for _ in range(500):
            evs = events()
            done = [e for e in evs if e["event"] == "completed"]
            if done:
                break
            stop.wait(0.02)
        assert done and done[0]["finish_reason"] == "abort"
        assert done[0]["completion_tokens"] < 450
        assert coord.metrics.aborted == aborted0 + 1
        assert f"hcp_requests_aborted_total {aborted0 + 1}" in coord.metrics.prometheus(0, 0)
        for _ in range(100):
            if not eng.reqs:
                break
            stop.wait(0.02)
        assert not eng.reqs and not coord.sched.active
    finally:
        srv.stop()
        stop.set()
        loop.join(5)
        coord.trace = saved


def test_peer_closed_handles_descriptors_above_fd_setsize():
    """The disconnect probe works for socket descriptors above FD_SETSIZE (1024), which a busy
    server reaches: an open idle socket is not closed, pending (pipelined) bytes are not a close,
    and an orderly shutdown by the peer is."""
    import os
    import resource
    import socket
    from hetero_cp_ringattn_b200.serve.http_server import _peer_closed
    target = 1500
    soft, hard = resource.getrlimit(resource.RLIMIT_NOFILE)
    if hard != resource.RLIM_INFINITY and hard <= target + 8:
        pytest.skip(f"RLIMIT_NOFILE hard limit {hard} is too low for descriptor {target}")
    if soft <= target + 8:
        resource.setrlimit(resource.RLIMIT_NOFILE, (target + 64, hard))
    a, b = socket.socketpair()
    hi = None
    try:
        hi = socket.socket(fileno=os.dup2(a.fileno(), target))
        a.close()
        assert hi.fileno() == target
        assert not _peer_closed(hi)
        b.sendall(b"x")
        assert not _peer_closed(hi)          # a pipelined byte is data, not a close
        assert hi.recv(1) == b"x"
        b.close()
        assert _peer_closed(hi)
    finally:
        if hi is not None:
            hi.close()
        b.close()
        resource.setrlimit(resource.RLIMIT_NOFILE, (soft, hard))
