"""Engine equivalence on CPU ranks: N-rank context parallelism == single-device reference.

Parity: rust/src/model/model.rs:765-1559 (2-domain prefill logits == 1-domain reference, decode and
multi-step decode equivalence) and worker_sdk/tch_backend.rs tests (request isolation, release),
run here as real OS processes over a gloo process group instead of a single-process mock ring.
"""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hetero_cp_ringattn_b200.config import preset
from hetero_cp_ringattn_b200.models import reference_model
from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights


def tiny_weights(seed=0):
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=seed, dtype=torch.float32, std=0.2)
    return cfg, w


def test_single_rank_prefill_and_decode_match_reference():
    cfg, w = tiny_weights()
    pw = PreparedWeights.from_weights(w, dtype=torch.float32)
    eng = LlamaCPEngine(cfg, pw, device=torch.device("cpu"), max_context=256)
    prompt = torch.randint(0, cfg.vocab_size, (37,), generator=torch.Generator().manual_seed(1))
    tok, logits = eng.prefill(1, prompt, [37], "vanilla", decode_horizon=8, return_logits=True)
    ref_logits = reference_model.forward(w, prompt, last_only=True)[0]
    assert (logits - ref_logits).abs().max() < 1e-4
    ref_tokens, _ = reference_model.greedy_generate(w, prompt, 6)
    toks = [int(tok)]
    cur = tok
    for _ in range(6):
        cur = eng.decode_step([1], cur)
        toks.append(int(cur))
    assert toks == ref_tokens
    assert eng.release(1)
    assert not eng.release(1)


def test_qwen2_bias_path_matches_reference():
    cfg = preset("tiny")
    cfg.attention_bias = True
    w = ModelWeights.random_init(cfg, seed=3, dtype=torch.float32, std=0.2)
    pw = PreparedWeights.from_weights(w, dtype=torch.float32)
    eng = LlamaCPEngine(cfg, pw, device=torch.device("cpu"), max_context=128)
    prompt = torch.randint(0, cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(2))
    _, logits = eng.prefill(7, prompt, [20], decode_horizon=2, return_logits=True)
    ref_logits = reference_model.forward(w, prompt, last_only=True)[0]
    assert (logits - ref_logits).abs().max() < 1e-4


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, chunks, strategy, steps, out_path, tickets):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w = tiny_weights()
        pw = PreparedWeights.from_weights(w, dtype=torch.float32)
        eng = LlamaCPEngine(cfg, pw, rank=rank, world=world, device=torch.device("cpu"),
                            max_context=256)
        L = sum(chunks)
        prompt = torch.randint(0, cfg.vocab_size, (L,), generator=torch.Generator().manual_seed(1))
        tok, logits = eng.prefill(5, prompt, chunks, strategy, decode_horizon=steps + 1,
                                  return_logits=True, tickets=tickets)
        toks = [int(tok)]
        cur = tok
        for _ in range(steps):
            cur = eng.decode_step([5], cur)
            toks.append(int(cur))
        if rank == 0:
            torch.save({"tokens": toks, "logits": logits}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("chunks,strategy,tickets", [
    ([20, 17], "vanilla", None),
    ([20, 17], "zigzag", None),
    ([25, 25, 5], "vanilla", [5, 5, 1]),
    ([25, 25, 5], "striped", [5, 5, 1]),
    # a rank holding a single token whose peers hold only future (or only past) positions
    # (the reference's single-token causal prefill with future peer KV, tch_backend.rs:1809)
    ([1, 12], "vanilla", None),
    ([12, 1], "zigzag", [1, 1]),
])
def test_gloo_ranks_match_single_device(chunks, strategy, tickets):
    world = len(chunks)
    steps = 6
    cfg, w = tiny_weights()
    L = sum(chunks)
    prompt = torch.randint(0, cfg.vocab_size, (L,), generator=torch.Generator().manual_seed(1))
    ref_tokens, ref_logits = reference_model.greedy_generate(w, prompt, steps)
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.pt")
        mp.start_processes(_worker, args=(world, free_port(), chunks, strategy, steps, out, tickets),
                           nprocs=world, join=True, start_method="spawn")
        res = torch.load(out)
    assert (res["logits"] - ref_logits[0]).abs().max() < 1e-4
    assert res["tokens"] == ref_tokens


def _session_worker(rank, world, port, out_path):
    if world > 1:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w = tiny_weights()
        pw = PreparedWeights.from_weights(w, dtype=torch.float32)
        eng = LlamaCPEngine(cfg, pw, rank=rank, world=world, device=torch.device("cpu"), max_context=256)
        g = torch.Generator().manual_seed(11)
        a = torch.randint(0, cfg.vocab_size, (23,), generator=g)
        b = torch.randint(0, cfg.vocab_size, (9,), generator=g)
        chunks = [12, 11][:world] if world > 1 else [23]
        tok, _ = eng.prefill(3, a, chunks, "vanilla", decode_horizon=4, keep_kv=True)
        toks = [int(tok)]
        cur = tok
        for _ in range(3):
            cur = eng.decode_step([3], cur)
            toks.append(int(cur))
        seg = torch.tensor([toks[-1]] + b.tolist())
        L0 = eng.reqs[3].context_len
        tok2, _ = eng.append(3, seg, list(range(L0, L0 + seg.numel())), [1] * world)
        more = [int(tok2)]
        cur = tok2
        for _ in range(3):
            cur = eng.decode_step([3], cur)
            more.append(int(cur))
        if rank == 0:
            torch.save({"a": a, "b": b, "toks": toks, "more": more}, out_path)
        if world > 1:
            dist.barrier()
    finally:
        if world > 1:
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_session_append_matches_reference(world):
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "s.pt")
        if world == 1:
            _session_worker(0, 1, 0, out)
        else:
            mp.start_processes(_session_worker, args=(world, free_port(), out), nprocs=world,
                               join=True, start_method="spawn")
        r = torch.load(out)
    cfg, w = tiny_weights()
    ref_first, _ = reference_model.greedy_generate(w, r["a"], 3)
    assert r["toks"] == ref_first
    full = torch.cat([r["a"], torch.tensor(r["toks"]), r["b"]])
    ref_more, _ = reference_model.greedy_generate(w, full, 3)
    assert r["more"] == ref_more


def _route_worker(rank, world, port, out_dir, env_kwargs):
    from hetero_cp_ringattn_b200.config import EnvConfig
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w = tiny_weights()
        pw = PreparedWeights.from_weights(w, dtype=torch.float32)
        eng = LlamaCPEngine(cfg, pw, rank=rank, world=world, device=torch.device("cpu"),
                            max_context=256, env=EnvConfig(**env_kwargs))
        g = torch.Generator().manual_seed(11)
        a = torch.randint(0, cfg.vocab_size, (29,), generator=g)
        b = torch.randint(0, cfg.vocab_size, (7,), generator=g)
        chunks = [12, 11, 6][:world]
        tok, _ = eng.prefill(4, a, chunks, "zigzag", decode_horizon=5, keep_kv=True,
                             tickets=[2, 2, 1][:world])
        toks = [int(tok)]
        cur = tok
        for _ in range(4):
            cur = eng.decode_step([4], cur)
            toks.append(int(cur))
        # rows stored on this rank after decoding: (own rows, replicated rows, decoded positions)
        kv0 = eng.reqs[4].host_kv[0]
        mine = [int(p) for p, s in zip(kv0[2], kv0[3]) if s and int(p) >= 29]
        replicated = [int(p) for p, s in zip(kv0[2], kv0[3]) if not s]
        seg = torch.tensor([toks[-1]] + b.tolist())
        L0 = eng.reqs[4].context_len
        tok2, _ = eng.append(4, seg, list(range(L0, L0 + seg.numel())), [1] * world)
        more = [int(tok2)]
        cur = tok2
        for _ in range(3):
            cur = eng.decode_step([4], cur)
            more.append(int(cur))
        torch.save({"a": a, "b": b, "toks": toks, "more": more, "mine": mine,
                    "replicated": replicated}, os.path.join(out_dir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("env_kwargs", [
    {"decode_sd": False, "micro_kv_block_size": 7},   # Q-ring placement: position % N
    {"decode_ring": False},                           # legacy KV re-send decode
])
def test_decode_routes_match_reference(env_kwargs):
    """The reference's selectable decode routes (HCP_RING_DECODE_SD=0, HCP_RING_DECODE_RING=0;
    ring.rs:682-818, :982-997, :1934) give the single-device tokens, before and after a session
    continuation, with their own KV placement."""
    world = 3
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_route_worker, args=(world, free_port(), d, env_kwargs), nprocs=world,
                           join=True, start_method="spawn")
        res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    cfg, w = tiny_weights()
    r0 = res[0]
    ref_first, _ = reference_model.greedy_generate(w, r0["a"], 4)
    full = torch.cat([r0["a"], torch.tensor(r0["toks"]), r0["b"]])
    ref_more, _ = reference_model.greedy_generate(w, full, 3)
    decoded = list(range(29, 33))  # positions of the 4 decoded tokens with KV before the append
    for r, out in enumerate(res):
        assert out["toks"] == ref_first and out["more"] == ref_more
        if env_kwargs.get("decode_ring") is False:
            assert out["mine"] == [] and out["replicated"] == decoded
        else:
            assert out["replicated"] == [] and out["mine"] == [p for p in decoded if p % world == r]


def test_page_size_from_environment():
    from hetero_cp_ringattn_b200.config import EnvConfig
    from hetero_cp_ringattn_b200.errors import CapacityError
    cfg, w = tiny_weights()
    pw = PreparedWeights.from_weights(w, dtype=torch.float32)
    eng = LlamaCPEngine(cfg, pw, device=torch.device("cpu"), max_context=256,
                        env=EnvConfig(kv_block_size=384))
    assert eng.page_size == 384 and eng.kv.page_size == 384
    assert LlamaCPEngine(cfg, pw, device=torch.device("cpu"), max_context=256, page_size=128,
                         env=EnvConfig(kv_block_size=384)).page_size == 128
    with pytest.raises(CapacityError):
        LlamaCPEngine(cfg, pw, device=torch.device("cpu"), env=EnvConfig(kv_block_size=0))


def _perf_worker(rank, world, port, out_dir):
    from hetero_cp_ringattn_b200.utils.perf import PerfLog
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w = tiny_weights()
        pw = PreparedWeights.from_weights(w, dtype=torch.float32)
        eng = LlamaCPEngine(cfg, pw, rank=rank, world=world, device=torch.device("cpu"),
                            max_context=256,
                            perf_log=PerfLog(os.path.join(out_dir, f"perf{rank}.jsonl")))
        tok, _ = eng.prefill(2, torch.arange(3, 30), [14, 13], decode_horizon=4)
        for _ in range(3):
            tok = eng.decode_step([2], tok)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_decode_perf_events_two_ranks(tmp_path):
    """HCP_PERF_LOG decode events in the reference's `stationary_decode` shape: one per step and
    rank, with the (O, LSE) exchange's message count and bytes."""
    import json
    world = 2
    mp.start_processes(_perf_worker, args=(world, free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    cfg = preset("tiny")
    part = cfg.num_heads * (cfg.head_dim + 1) * 4
    for r in range(world):
        evs = [json.loads(l) for l in open(tmp_path / f"perf{r}.jsonl")]
        dec = [e for e in evs if e["event"] == "stationary_decode"]
        assert [e["position"] for e in dec] == [27, 28, 29]
        assert [e["token_offset"] for e in dec] == [0, 1, 2]
        for e in dec:
            assert e["domain"] == r and e["domains"] == 2 and e["route"] == "o_lse_exchange"
            assert e["sends"] == cfg.num_layers and e["wire_sent_bytes"] == cfg.num_layers * part
            assert e["total_ms"] > 0 and e["decode_horizon"] == 4
        assert sum(1 for e in evs if e["event"] == "prefill") == 1
    # across ranks, every (token, layer) KV row is appended exactly once
    rows = [sum(e["kv_rows_appended"] for e in map(json.loads, open(tmp_path / f"perf{r}.jsonl"))
                if e["event"] == "stationary_decode") for r in range(world)]
    assert sum(rows) == 3 * cfg.num_layers


def test_warmup_leaves_no_state():
    cfg, w = tiny_weights()
    pw = PreparedWeights.from_weights(w, dtype=torch.float32)
    eng = LlamaCPEngine(cfg, pw, device=torch.device("cpu"), max_context=128, max_batch=4)
    free = eng.kv.alloc.free_pages
    eng.warmup()
    assert not eng.reqs and eng.kv.alloc.free_pages == free
    prompt = torch.randint(0, cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(3))
    ref_tokens, _ = reference_model.greedy_generate(w, prompt, 3)
    assert [int(t) for t in eng.generate_batch([prompt], 4)[0]] == ref_tokens
