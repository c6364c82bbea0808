"""Command-line entry points.

Parity: the reference's single binary with modes (rust/src/cli.rs:14-165, lib.rs:211-634):
  * `correctness` - the ring-vs-dense oracle suite with tolerance tiers and a JSON report
    (`--report-path`, `--tolerance-tier`, `--stress-test`; lib.rs:107-199);
  * `infer` - single-node inference with `--export-logits` in the reference's binary layout
    ([vocab u64 LE][steps u64 LE] then f32 rows; rust/src/infer.rs:74-79);
  * `serve` - coordinator + workers: one torchrun job, rank 0 coordinates and serves the HTTP API
    (`/v1/completions`, `/health`, `/metrics`), every rank runs the worker command loop
    (coordinator.rs:76-273 and worker.rs:77-143 flags that still apply on one NVSwitch box:
    --model-dir, --prompt/--prompt-file/--prompts-file, --max-tokens, --temperature, --top-p,
    --chunk-sizes, --capacity-aware, --ring-strategy, --trace-jsonl, --max-batch-size,
    --activation-reserve-mb, --session-continuation-tokens, --http-addr);
  * `gen-prompt` - an exact-N-token random prompt (rust/src/bin/gen_prompt.rs).

  python -m hetero_cp_ringattn_b200 correctness --report-path reports/ring.json
  torchrun --nproc-per-node 8 -m hetero_cp_ringattn_b200 serve --model-preset llama-3.2-1b --http-addr 127.0.0.1:8000
"""

from __future__ import annotations

import argparse
import json
import logging
import os
import signal
import struct
import sys
from typing import List, Optional

import torch


def _add_model_args(ap):
    ap.add_argument("--model-dir", default=None, help="HF directory (config.json + *.safetensors)")
    ap.add_argument("--model-preset", default="tiny-gpu", help="random-init shape when no model dir")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--max-context", type=int, default=32768)
    ap.add_argument("--max-batch-size", type=int, default=4)
    ap.add_argument("--device", default=None, help="cuda|cuda:N|cpu (HCP_TORCH_DEVICE)")


def _load_model(args, device):
    from .config import ModelConfig, preset
    from .models.weights import ModelWeights, PreparedWeights
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    if args.model_dir:
        cfg = ModelConfig.from_file(os.path.join(args.model_dir, "config.json"))
        w = ModelWeights.from_dir(args.model_dir, device="cpu", dtype=dtype, cfg=cfg)
        return cfg, PreparedWeights.from_weights(w, device=device, dtype=dtype, free_source=True)
    cfg = preset(args.model_preset)
    if device.type == "cuda":
        return cfg, PreparedWeights.random(cfg, seed=args.seed, device=device, dtype=dtype)
    w = ModelWeights.random_init(cfg, seed=args.seed, dtype=dtype)
    return cfg, PreparedWeights.from_weights(w, dtype=dtype)


def _device(args) -> torch.device:
    name = args.device or os.environ.get("HCP_TORCH_DEVICE") or os.environ.get("HCP_TCH_DEVICE")
    if not name:
        name = "cuda" if torch.cuda.is_available() else "cpu"
    if name == "cuda":
        name = f"cuda:{int(os.environ.get('LOCAL_RANK', '0'))}"
    return torch.device(name)


def cmd_correctness(args) -> int:
    from .config import RingAttnConfig
    from .correctness import case_from_ring_config, run_suite, write_report
    from .errors import ToleranceTier
    tier = ToleranceTier.parse(args.tolerance_tier)
    extra = [(os.path.basename(p), case_from_ring_config(RingAttnConfig.from_file(p)))
             for p in (args.config or [])]
    rep = run_suite(tier, stress_seeds=args.stress_test, extra_cases=extra, oracle=args.oracle)
    for c in rep["cases"]:
        w = c["worst_seed"]
        print(f"[{'PASS' if c['passed'] else 'FAIL'}] {c['name']}: out max_abs={w['output']['max_abs_err']:.3e} "
              f"lse max_abs={w['lse']['max_abs_err']:.3e}")
    if args.report_path:
        os.makedirs(os.path.dirname(os.path.abspath(args.report_path)), exist_ok=True)
        write_report(rep, args.report_path)
    print("overall:", "PASS" if rep["passed"] else "FAIL")
    return 0 if rep["passed"] else 1


def write_logits(path: str, rows: List[torch.Tensor]) -> None:
    """[vocab u64 LE][steps u64 LE] + f32 LE rows (prefill row first, then one per decode step)."""
    vocab = rows[0].numel()
    with open(path, "wb") as f:
        f.write(struct.pack("<QQ", vocab, len(rows) - 1))
        for r in rows:
            f.write(r.detach().float().cpu().numpy().astype("<f4").tobytes())


def read_logits(path: str):
    import numpy as np
    with open(path, "rb") as f:
        vocab, steps = struct.unpack("<QQ", f.read(16))
        data = np.frombuffer(f.read(), dtype="<f4").reshape(steps + 1, vocab)
    return vocab, steps, data


def _debug_exports(args, dev, ids) -> int:
    """--export-hidden-states / --prefill-debug: float32 oracle intermediates on the same weights."""
    from .config import ModelConfig, preset
    from .debug_export import export_hidden_states, prefill_debug_layer0
    from .models.weights import ModelWeights
    if args.model_dir:
        cfg = ModelConfig.from_file(os.path.join(args.model_dir, "config.json"))
        w = ModelWeights.from_dir(args.model_dir, device=dev, dtype=torch.float32, cfg=cfg)
    else:
        cfg = preset(args.model_preset)
        w = ModelWeights.random_init(cfg, seed=args.seed, dtype=torch.float32, device=dev)
    ids = ids.to(dev)
    out = {"prompt_tokens": ids.numel()}
    if args.prefill_debug:
        prefill_debug_layer0(w, ids, args.prefill_debug, args.qk_inject)
        out["prefill_debug"] = args.prefill_debug
    if args.export_hidden_states:
        out["first_token"] = export_hidden_states(w, ids, args.export_hidden_states)
        out["export_hidden_states"] = args.export_hidden_states
    print(json.dumps(out))
    return 0


def cmd_infer(args) -> int:
    from .models.llama import LlamaCPEngine
    from .serve.tokenizer import load_tokenizer
    dev = _device(args)
    if args.export_hidden_states or args.prefill_debug:
        from .config import ModelConfig, preset
        cfg0 = (ModelConfig.from_file(os.path.join(args.model_dir, "config.json")) if args.model_dir
                else preset(args.model_preset))
        tok0 = load_tokenizer(args.model_dir, cfg0.vocab_size)
        text = open(args.prompt_file).read() if args.prompt_file else (args.prompt or "hello")
        return _debug_exports(args, dev, torch.tensor(tok0.encode(text), dtype=torch.int64))
    import torch.distributed as dist
    from .models.sampling import sample_token
    from .parallel.capacity import chunk_sizes
    rank, world, group = _init_ranks(dev, args.num_domains)
    cfg, w = _load_model(args, dev)
    tok = load_tokenizer(args.model_dir, cfg.vocab_size)
    prompt = args.prompt
    if args.prompt_file:
        prompt = open(args.prompt_file).read()
    ids = torch.tensor(tok.encode(prompt or "hello"), dtype=torch.int64)
    ratio = [int(x) for x in args.ratio.split(":")] if args.ratio else None
    chunks = chunk_sizes(ids.numel(), world, ratio=ratio,
                         explicit=[int(x) for x in args.chunk_sizes.split(",")] if args.chunk_sizes else None)
    eng = LlamaCPEngine(cfg, w, rank=rank, world=world, device=dev, group=group,
                        max_context=max(args.max_context, ids.numel()), max_batch=1,
                        decode_reserve=args.max_tokens + 8)
    gen = torch.Generator().manual_seed(args.seed)

    def pick(argmax_tok, logits):
        """Greedy uses the engine's (identical on every rank) argmax; sampling happens on rank 0
        and the token is broadcast so every rank feeds the same one."""
        if args.temperature <= 0:
            return int(argmax_tok)
        t = torch.tensor([sample_token(logits.float().cpu(), args.temperature, args.top_p, gen)
                          if rank == 0 else 0])
        if world > 1:
            dist.broadcast(t, src=0, group=group)
        return int(t[0])

    try:
        first, logits = eng.prefill(1, ids, chunks, args.ring_strategy,
                                    decode_horizon=max(1, args.max_tokens), return_logits=True,
                                    tickets=ratio)
        rows = [logits.float().cpu()]
        out = [pick(first, logits)]
        for _ in range(args.max_tokens - 1):
            cur = torch.tensor([out[-1]], dtype=torch.int64, device=dev)
            nxt = eng.decode_step([1], cur)
            lg = eng.last_logits(1)[0]
            if args.export_logits:
                rows.append(lg.float().cpu())
            out.append(pick(nxt.view(-1)[0], lg))
        if rank == 0:
            if args.export_logits:
                write_logits(args.export_logits, rows)
            print(json.dumps({"prompt_tokens": ids.numel(), "tokens": out, "text": tok.decode(out),
                              "chunks": chunks, "world": world}))
    finally:
        eng.close()
        if world > 1:
            dist.destroy_process_group()
    return 0


def _init_ranks(dev: torch.device, num_domains: Optional[int] = None):
    """(rank, world, gloo control group or None) from the torchrun environment. Multi-rank runs
    get an NCCL (GPU) or gloo (CPU) default group plus a gloo group for host control messages,
    with HCP_QUIC_TIMEOUT_SECS as the timeout of both."""
    import torch.distributed as dist
    from datetime import timedelta
    from .config import EnvConfig
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if num_domains is not None and num_domains != world:
        raise SystemExit(f"--num-domains {num_domains} but WORLD_SIZE is {world} "
                         f"(launch one process per domain with torchrun)")
    if world == 1:
        return rank, world, None
    timeout = timedelta(seconds=EnvConfig.from_env().control_timeout_s)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", device_id=dev, timeout=timeout)
    else:
        dist.init_process_group("gloo", timeout=timeout)
    return rank, world, dist.new_group(backend="gloo", timeout=timeout)


def _raise_interrupt(signum, frame):
    raise KeyboardInterrupt


def cmd_serve(args) -> int:
    from .config import EnvConfig
    from .errors import RingError
    from .models.llama import LlamaCPEngine
    from .parallel.capacity import query_device_capacity_mb
    from .serve import protocol as P
    from .serve.coordinator import Coordinator, CoordinatorArgs
    from .serve.http_server import ApiServer, ApiState
    from .serve.tokenizer import load_tokenizer
    from .serve.worker import Worker
    dev = _device(args)
    rank, world, group = _init_ranks(dev, args.num_domains)
    cfg, w = _load_model(args, dev)
    # the engine decodes at most 8 rows per step on CUDA; more concurrent requests are decoded
    # in several engine steps per coordinator iteration
    eng_batch = min(args.max_batch_size, 8) if dev.type == "cuda" else args.max_batch_size
    page = EnvConfig.from_env().kv_block_size
    kv_pages = -(-args.max_context // page) + args.max_batch_size * -(-512 // page) + 2
    eng = LlamaCPEngine(cfg, w, rank=rank, world=world, device=dev, group=group,
                        max_context=args.max_context, max_batch=eng_batch, kv_pages=kv_pages)
    control = P.ControlPlane(group, rank, world)
    worker = Worker(eng, control)
    if not args.no_warmup:
        eng.warmup()   # decode graphs captured before the first request (every rank)
    caps = control.all_gather(query_device_capacity_mb(str(dev)))  # the handshake
    arenas = control.all_gather(eng.kv_capacity_bytes())
    # torchrun forwards SIGINT / SIGTERM to every rank: both end the serve loop the same way
    signal.signal(signal.SIGTERM, _raise_interrupt)
    if rank != 0:
        try:
            worker.loop()
        except KeyboardInterrupt:
            eng.close(sync=False)  # the other ranks are stopping too: no barrier
            return 0
        eng.close()
        return 0
    tok = load_tokenizer(args.model_dir, cfg.vocab_size)
    ca = CoordinatorArgs(strategy=args.ring_strategy,
                         chunk_sizes=[int(x) for x in args.chunk_sizes.split(",")] if args.chunk_sizes else None,
                         capacity_aware=args.capacity_aware,
                         ratio=[int(x) for x in args.ratio.split(":")] if args.ratio else None,
                         max_batch_size=args.max_batch_size,
                         activation_reserve_mb=args.activation_reserve_mb,
                         session_continuation_tokens=args.session_continuation_tokens,
                         trace_jsonl=args.trace_jsonl, eos_ids=cfg.eos_token_id,
                         export_logits_dir=args.export_logits,
                         prefill_chunk_tokens=args.prefill_chunk_tokens,
                         max_queue=args.max_queue, decode_batch_limit=eng_batch,
                         session_ttl_s=args.session_ttl_s,
                         kv_page_tokens=eng.page_size if dev.type == "cuda" else 1)
    coord = Coordinator(worker, control, tok, cfg, ca, capacities_mb=caps,
                        kv_budget_bytes=arenas if all(a is not None for a in arenas) else None)
    prompts = []
    if args.prompt:
        prompts.append(args.prompt)
    if args.prompt_file:
        prompts.append(open(args.prompt_file).read())
    if args.prompts_file:
        prompts += [ln.rstrip("\n") for ln in open(args.prompts_file) if ln.strip()]
    ints = (lambda v: [int(x) for x in v.split(",") if x.strip()] if v else None)
    status = 0
    try:
        if args.continuation_segment:
            ids = ints(args.prompt_token_ids) or tok.encode(prompts[0] if prompts else "hello")
            try:
                meta = coord.continuation_e2e(args.continuation_request_id, ids,
                                              ints(args.continuation_segment), args.max_tokens,
                                              ints(args.continuation_capacity_tickets))
            except RingError as e:
                print(json.dumps({"continuation_e2e_failed": str(e)}), flush=True)
                status = 1
            else:
                print(json.dumps({"continuation_e2e": meta}), flush=True)
        elif args.prompt_token_ids and not args.http_addr:
            r = coord.generate(ints(args.prompt_token_ids), args.max_tokens, args.temperature,
                               args.top_p)
            print(json.dumps({"prompt_token_ids": ints(args.prompt_token_ids),
                              "text": tok.decode(r.get("tokens", [])), **r}), flush=True)
        elif prompts and not args.http_addr:
            for p in prompts:
                r = coord.generate(tok.encode(p), args.max_tokens, args.temperature, args.top_p)
                print(json.dumps({"prompt": p, "text": tok.decode(r.get("tokens", [])), **r}), flush=True)
        else:
            host, port = (args.http_addr or "127.0.0.1:8000").rsplit(":", 1)
            srv = ApiServer(ApiState(coord, tok, args.model_dir or cfg.name, world), host, int(port)).start()
            print(f"[coordinator] serving on http://{host}:{srv.port}", flush=True)
            coord.run_forever()
    except KeyboardInterrupt:
        pass
    finally:
        # the workers reached Shutdown: they close after a barrier, so close with one too
        workers_stopped_cleanly = coord.shutdown()
    eng.close(sync=workers_stopped_cleanly)
    return status


def cmd_compare_logits(args) -> int:
    """Compare two logits exports (the reference's scripts/compare_logits.py): per-step max/mean
    absolute difference and argmax agreement."""
    import numpy as np
    va, sa, a = read_logits(args.a)
    vb, sb, b = read_logits(args.b)
    if va != vb:
        print(json.dumps({"error": f"vocab mismatch {va} vs {vb}"}))
        return 1
    n = min(sa, sb) + 1
    rows = []
    for i in range(n):
        d = np.abs(a[i].astype(np.float64) - b[i].astype(np.float64))
        rows.append({"step": i, "max_abs": float(d.max()), "mean_abs": float(d.mean()),
                     "argmax_match": bool(int(a[i].argmax()) == int(b[i].argmax()))})
    worst = max(r["max_abs"] for r in rows)
    ok = worst <= args.tolerance and all(r["argmax_match"] for r in rows)
    print(json.dumps({"steps": n, "worst_max_abs": worst, "passed": ok, "per_step": rows}))
    return 0 if ok else 1


def cmd_compare_hidden(args) -> int:
    """Compare two tensor-dump directories (--export-hidden-states / --prefill-debug outputs, or
    the reference's dumps; the reference's scripts/compare_hidden_states.py): every file name
    present in both, shape check, max / mean absolute and max relative difference."""
    from .debug_export import read_tensor_bin
    names = sorted(set(f for f in os.listdir(args.a) if f.endswith(".bin") and f != "logits.bin") &
                   set(f for f in os.listdir(args.b) if f.endswith(".bin")))
    rows, ok = [], True
    for n in names:
        ta = read_tensor_bin(os.path.join(args.a, n)).double()
        tb = read_tensor_bin(os.path.join(args.b, n)).double()
        if ta.shape != tb.shape:
            rows.append({"file": n, "error": f"shape {tuple(ta.shape)} vs {tuple(tb.shape)}"})
            ok = False
            continue
        d = (ta - tb).abs()
        rel = float((d / tb.abs().clamp_min(1e-6)).max()) if d.numel() else 0.0
        r = {"file": n, "max_abs": float(d.max()) if d.numel() else 0.0,
             "mean_abs": float(d.mean()) if d.numel() else 0.0, "max_rel": rel}
        ok = ok and r["max_abs"] <= args.tolerance
        rows.append(r)
    print(json.dumps({"files": len(names), "passed": ok and bool(names), "per_file": rows}))
    return 0 if ok and names else 1


def cmd_perf_summary(args) -> int:
    """Aggregate HCP_PERF_LOG JSONL files per event (the reference's parse_worker_perf.py): the
    mean of every numeric field; `--ledger` adds the KV transport ledger of the reference's
    kv_transport_ledger.py, total bytes sent / received per event and rank (`domain`)."""
    import collections
    agg = collections.defaultdict(lambda: collections.defaultdict(float))
    counts = collections.Counter()
    ledger = collections.defaultdict(lambda: collections.defaultdict(float))
    byte_fields = ("kv_sent_bytes", "kv_recv_bytes", "wire_sent_bytes", "wire_recv_bytes")
    for path in args.path:
        for line in open(path):
            try:
                ev = json.loads(line)
            except json.JSONDecodeError:
                continue
            name = ev.get("event", "?")
            counts[name] += 1
            for k, v in ev.items():
                if isinstance(v, (int, float)) and not isinstance(v, bool) and \
                        k not in ("ts", "layer", "domain"):
                    agg[name][k] += v
            if args.ledger:
                key = f"{name}/domain-{ev.get('domain', '?')}"
                for k in byte_fields:
                    v = ev.get(k)
                    if isinstance(v, (int, float)) and v >= 0:
                        ledger[key][k] += v
                ledger[key]["events"] += 1
    out = {name: {"count": counts[name], **{k: v / counts[name] for k, v in fields.items()}}
           for name, fields in agg.items()}
    if getattr(args, "by_domain", False):
        # per rank: the mean of every numeric field of each event, and per field the spread
        # between the slowest and the fastest rank (max - min of the per-rank means)
        per = collections.defaultdict(lambda: collections.defaultdict(float))
        cnt = collections.Counter()
        for path in args.path:
            for line in open(path):
                try:
                    ev = json.loads(line)
                except json.JSONDecodeError:
                    continue
                key = (ev.get("event", "?"), ev.get("domain", ev.get("rank", "?")))
                cnt[key] += 1
                for k, v in ev.items():
                    if isinstance(v, (int, float)) and not isinstance(v, bool) and \
                            k not in ("ts", "layer", "domain", "rank"):
                        per[key][k] += v
        by = collections.defaultdict(dict)
        for (name, dom), fields in sorted(per.items(), key=lambda kv: (kv[0][0], str(kv[0][1]))):
            by[name][str(dom)] = {"count": cnt[(name, dom)],
                                  **{k: v / cnt[(name, dom)] for k, v in fields.items()}}
        for name, doms in by.items():
            fields = {k for d in doms.values() for k in d if k != "count"}
            out.setdefault(name, {})["rank_spread"] = {
                k: max(d.get(k, 0.0) for d in doms.values()) - min(d.get(k, 0.0) for d in doms.values())
                for k in sorted(fields)}
        out["by_domain"] = dict(by)
    if args.ledger:
        out["kv_transport_ledger"] = {k: dict(v) for k, v in sorted(ledger.items())}
    print(json.dumps(out, indent=2))
    return 0


def cmd_gen_prompt(args) -> int:
    g = torch.Generator().manual_seed(args.seed)
    ids = torch.randint(0, args.vocab, (args.tokens,), generator=g)
    print(json.dumps(ids.tolist()))
    return 0


def main(argv: Optional[List[str]] = None) -> int:
    # every line names its rank (the reference prefixes [coordinator] / [worker N])
    role = "coordinator" if os.environ.get("RANK", "0") == "0" else f"worker {os.environ['RANK']}"
    logging.basicConfig(level=os.environ.get("HCP_LOG", "WARNING"),
                        format=f"%(asctime)s [{role}] %(name)s %(levelname)s: %(message)s")
    args = build_parser().parse_args(argv)
    return args.fn(args)


def build_parser() -> argparse.ArgumentParser:
    """The `hcp` command line: one sub-command per tool, each bound to its `cmd_*` function."""
    ap = argparse.ArgumentParser(prog="hcp")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("correctness")
    c.add_argument("--report-path", default=None)
    c.add_argument("--tolerance-tier", default="strict")
    c.add_argument("--stress-test", type=int, default=5)
    c.add_argument("--oracle", choices=["python", "native"], default="python",
                   help="float64 oracle: torch (python) or the C++ host library (native)")
    c.add_argument("--config", action="append", default=None,
                   help="domain layout JSON (global_seq_len, heads, domains[seq_chunk_len, block_size])")
    c.set_defaults(fn=cmd_correctness)
    i = sub.add_parser("infer")
    _add_model_args(i)
    i.add_argument("--prompt", default=None)
    i.add_argument("--prompt-file", default=None)
    i.add_argument("--max-tokens", type=int, default=10)
    i.add_argument("--export-logits", default=None)
    i.add_argument("--temperature", type=float, default=0.0)
    i.add_argument("--top-p", type=float, default=1.0)
    i.add_argument("--num-domains", type=int, default=None,
                   help="expected number of ranks (checked against WORLD_SIZE)")
    i.add_argument("--chunk-sizes", default=None)
    i.add_argument("--ratio", default=None, help="capacity ratio, e.g. 5:5:1")
    i.add_argument("--ring-strategy", default="vanilla", choices=["vanilla", "striped", "zigzag"])
    i.add_argument("--export-hidden-states", default=None, metavar="DIR",
                   help="per-layer K/V after prefill + first decode step hidden states (f32 oracle)")
    i.add_argument("--prefill-debug", default=None, metavar="DIR",
                   help="layer-0 prefill intermediates + every layer's K/V (f32 oracle)")
    i.add_argument("--qk-inject", default=None, metavar="DIR",
                   help="with --prefill-debug: read layer 0's q/k projections from DIR")
    i.set_defaults(fn=cmd_infer)
    s = sub.add_parser("serve", aliases=["coordinator", "worker"])
    _add_model_args(s)
    s.add_argument("--prompt", default=None)
    s.add_argument("--prompts-file", default=None)
    s.add_argument("--max-tokens", type=int, default=20)
    s.add_argument("--temperature", type=float, default=0.0)
    s.add_argument("--top-p", type=float, default=1.0)
    s.add_argument("--chunk-sizes", default=None)
    s.add_argument("--capacity-aware", action="store_true")
    s.add_argument("--ratio", default=None, help="capacity ratio override, e.g. 5:5:1")
    s.add_argument("--ring-strategy", default="vanilla", choices=["vanilla", "striped", "zigzag"])
    s.add_argument("--trace-jsonl", default=None)
    s.add_argument("--activation-reserve-mb", type=int, default=1536)
    s.add_argument("--session-continuation-tokens", type=int, default=64)
    s.add_argument("--http-addr", default=None)
    s.add_argument("--prompt-file", default=None, help="one prompt: the whole file")
    s.add_argument("--session-ttl-s", type=float, default=0.0,
                   help="release keep_kv sessions idle this many seconds (0: keep until ended)")
    s.add_argument("--max-queue", type=int, default=0,
                   help="reject requests with 503 while this many are queued (0: no limit)")
    s.add_argument("--prefill-chunk-tokens", type=int, default=0,
                   help="prefill prompts longer than this in pieces, decoding the active "
                        "requests between pieces (0: one prefill per prompt)")
    s.add_argument("--no-warmup", action="store_true",
                   help="skip the start-up dummy requests that capture the decode graphs")
    s.add_argument("--num-domains", type=int, default=None,
                   help="expected number of ranks (checked against WORLD_SIZE)")
    s.add_argument("--export-logits", default=None, metavar="DIR",
                   help="per-request logits dumps: DIR/request_<id>/<name>.f32le + meta.json")
    s.add_argument("--prompt-token-ids", default=None, help="comma-separated prompt token ids")
    s.add_argument("--continuation-segment", default=None,
                   help="comma-separated token ids: run the continuation end-to-end check")
    s.add_argument("--continuation-request-id", type=int, default=1)
    s.add_argument("--continuation-capacity-tickets", default=None,
                   help="comma-separated tickets per rank (default: the handshake capacities)")
    s.set_defaults(fn=cmd_serve)
    ch = sub.add_parser("compare-hidden")
    ch.add_argument("a")
    ch.add_argument("b")
    ch.add_argument("--tolerance", type=float, default=2e-2)
    ch.set_defaults(fn=cmd_compare_hidden)
    cl = sub.add_parser("compare-logits")
    cl.add_argument("a")
    cl.add_argument("b")
    cl.add_argument("--tolerance", type=float, default=2e-2)
    cl.set_defaults(fn=cmd_compare_logits)
    ps = sub.add_parser("perf-summary")
    ps.add_argument("path", nargs="+", help="HCP_PERF_LOG JSONL file(s), e.g. one per rank")
    ps.add_argument("--ledger", action="store_true",
                    help="add total KV bytes sent / received per event and rank")
    ps.add_argument("--by-domain", action="store_true",
                    help="add per-rank means of every field and the spread between the ranks")
    ps.set_defaults(fn=cmd_perf_summary)
    g = sub.add_parser("gen-prompt")
    g.add_argument("--tokens", type=int, required=True)
    g.add_argument("--vocab", type=int, default=128256)
    g.add_argument("--seed", type=int, default=0)
    g.set_defaults(fn=cmd_gen_prompt)
    return ap


if __name__ == "__main__":
    sys.exit(main())
