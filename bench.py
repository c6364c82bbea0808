"""Headline benchmark: long-context prefill tok/s + TTFT and decode tok/s, CP = N ranks on one node.

Config: Llama-3.2-1B-shaped decoder (16 layers, hidden 2048, 32 heads,
8 KV heads, head_dim 64, SwiGLU 8192, vocab 128256, RoPE theta 5e5), bf16, random-init weights
N(0, 0.02), a 32768-token prompt of uniform-random token ids, then 128 greedy tokens; equal chunks
(zigzag layout for N > 1 so every rank carries the same causal work). One "step" is one full
request: prefill of the whole prompt + 127 decode steps.

  python bench.py --gpus N --steps K --warmup W          (N > 1: launched under torchrun)
  python bench.py --impl reference ...                   (the reference's own code path)

Rank 0 prints one JSON line. `value` is prefill tokens/s for the whole job (prompt tokens divided
by the device-timed prefill time, max over ranks). Weights (~2.5 GB) and activations are far
larger than the 126 MB L2, so no explicit L2 flush is done between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

BASELINE_PREFILL_TOK_S = None  # no published same-metric number of the reference to divide by

CONFIGS = {
    "llama-3.2-1b-32k": dict(model="llama-3.2-1b", prompt=32768, new_tokens=128),
    "qwen2.5-3b-64k": dict(model="qwen2.5-3b", prompt=65536, new_tokens=128),
    "llama-3-8b-128k": dict(model="llama-3-8b", prompt=131072, new_tokens=256),
    "tiny": dict(model="tiny-gpu", prompt=4096, new_tokens=16),
}


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="hcp", choices=["hcp", "reference", "torch-restatement"],
                    help="hcp: this framework; reference: the unmodified reference (unavailable "
                         "here); torch-restatement: the reference's algorithm restated in stock "
                         "PyTorch (benchmarks/ref_ring_torch.py), for a same-box comparison")
    ap.add_argument("--restatement-decode", type=int, default=32,
                    help="decode steps timed for the torch restatement")
    ap.add_argument("--config", default="llama-3.2-1b-32k", choices=sorted(CONFIGS))
    ap.add_argument("--strategy", default=None, help="vanilla|striped|zigzag (default: zigzag for N>1)")
    ap.add_argument("--ratio", default=None, help="capacity ratio override, e.g. 5:5:1")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--decode-batch", type=int, default=1,
                    help="also time batched decode of B requests that share the prompt length")
    return ap.parse_args(argv)


def reference_unavailable(args) -> None:
    """The reference is a Rust/tch-rs + QUIC program: it has no Python packaging (no setup.py or
    pyproject.toml, so the offline pip install into baseline/_ref fails) and needs cargo/rustc and
    crates.io, which this image does not have."""
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({
            "impl": "reference",
            "unavailable": "stark-sim/hetero-cp-ringattn is a Rust (cargo + tch-rs + quinn) project "
                           "with no Python package: pip install into baseline/_ref fails ('Neither "
                           "setup.py nor pyproject.toml found') and no cargo/rustc/crates are available "
                           "offline to build it",
            "n_gpus": args.gpus,
        }), flush=True)


def run_restatement(args) -> int:
    """Time the PyTorch restatement of the reference's algorithm on the same config."""
    import torch.distributed as dist
    from benchmarks.ref_ring_torch import RefRingModel, hf_random_weights
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.parallel.capacity import equal_chunks
    from hetero_cp_ringattn_b200.utils.perf import max_over_ranks
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=900))
    spec = CONFIGS[args.config]
    cfg = preset(spec["model"])
    Lp = spec["prompt"]
    chunks = equal_chunks(Lp, world)
    model = RefRingModel(cfg, hf_random_weights(cfg, dev), rank, world, dev)
    prompt = torch.randint(0, cfg.vocab_size, (Lp,), generator=torch.Generator().manual_seed(1234))
    steps_dec = max(1, args.restatement_decode)

    def one():
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        tok = model.prefill(prompt, chunks)
        e1.record()
        for _ in range(steps_dec):
            tok = model.decode_step(tok)
        e2.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1), e1.elapsed_time(e2)

    for _ in range(max(1, args.warmup)):
        one()
    pre, dec = [], []
    for _ in range(args.steps):
        p, d = one()
        pre.append(p)
        dec.append(d)
    prefill_ms = max_over_ranks(sum(pre) / len(pre))
    decode_ms = max_over_ranks(sum(dec) / len(dec))
    if rank == 0:
        print(json.dumps({
            "impl": "torch-restatement",
            "note": "stock-PyTorch restatement of the reference's ring algorithm "
                    "(benchmarks/ref_ring_torch.py); not the reference itself",
            "metric": "prefill tok/s & TTFT @32k and decode tok/s (CP=N B200, max over ranks)",
            "value": Lp / (prefill_ms / 1e3), "unit": "prompt tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ttft_ms": prefill_ms,
            "decode_ms_per_token": decode_ms / steps_dec,
            "decode_tok_s": steps_dec / (decode_ms / 1e3), "dtype": "bf16",
            "config": {"model": spec["model"], "seq_len": Lp, "chunks": chunks,
                       "strategy": "vanilla", "parallelism": f"cp{world}"},
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        reference_unavailable(args)
        return 0
    if args.impl == "torch-restatement":
        return run_restatement(args)

    from hetero_cp_ringattn_b200.config import preset, parse_ratio
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import PreparedWeights
    from hetero_cp_ringattn_b200.parallel.capacity import chunks_from_ratio, equal_chunks
    from hetero_cp_ringattn_b200.utils import launches
    from hetero_cp_ringattn_b200.utils.perf import ClockSampler, max_over_ranks
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torchrun --nproc-per-node N")
        raise SystemExit(f"WORLD_SIZE={world} but --gpus={args.gpus}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=600))
        group = dist.new_group(backend="gloo", timeout=timedelta(seconds=600))

    spec = CONFIGS[args.config]
    cfg = preset(spec["model"])
    Lp, new_tokens = spec["prompt"], spec["new_tokens"]
    strategy = args.strategy or ("zigzag" if world > 1 else "vanilla")
    if args.ratio:
        chunks = chunks_from_ratio(Lp, parse_ratio(args.ratio))
    else:
        chunks = equal_chunks(Lp, world)

    weights = PreparedWeights.random(cfg, seed=0, device=dev)
    B = max(1, args.decode_batch)
    page = 256
    kv_pages = B * (-(-max(chunks) // page) + -(-(new_tokens + 8) // page)) + 2
    eng = LlamaCPEngine(cfg, weights, rank=rank, world=world, device=dev, group=group,
                        max_context=Lp, max_batch=B, decode_reserve=new_tokens + 8,
                        kv_pages=kv_pages, use_graphs=not args.no_graphs)
    gen = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, cfg.vocab_size, (Lp,), generator=gen, dtype=torch.int64).pin_memory()
    prompt_dev = prompt.to(dev)

    def barrier():
        if world > 1:
            dist.barrier(group=group)
        torch.cuda.synchronize()

    req = [100]

    def one_request(dev_prompt):
        """Device-timed request: prefill (events) + decode (events). Returns (prefill_ms, decode_ms)."""
        req[0] += 1
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        tok, _ = eng.prefill(req[0], dev_prompt, chunks, strategy, decode_horizon=new_tokens)
        e1.record()
        cur = tok
        for _ in range(new_tokens - 1):
            cur = eng.decode_step([req[0]], cur)
        e2.record()
        eng.release(req[0])
        torch.cuda.synchronize()
        return e0.elapsed_time(e1), e1.elapsed_time(e2), cur

    for _ in range(args.warmup):
        one_request(prompt_dev)
    barrier()
    launches.reset()
    pre_ms, dec_ms = [], []
    with ClockSampler(local_rank) as clocks:
        barrier()
        t_all0 = torch.cuda.Event(enable_timing=True)
        t_all1 = torch.cuda.Event(enable_timing=True)
        t_all0.record()
        for _ in range(args.steps):
            p, d, _ = one_request(prompt_dev)
            pre_ms.append(p)
            dec_ms.append(d)
        t_all1.record()
        barrier()
    n_launch = launches.total() // max(1, args.steps)
    total_ms = max_over_ranks(t_all0.elapsed_time(t_all1) / args.steps, group)
    prefill_ms = max_over_ranks(sum(pre_ms) / len(pre_ms), group)
    decode_ms = max_over_ranks(sum(dec_ms) / len(dec_ms), group)
    eng.check_device()

    # ---------------------------------------------------------------- end to end (public API)
    e2e = None
    if not args.no_e2e:
        h2d = int(len(prompt)) * prompt.element_size()
        ttfts, totals = [], []
        for i in range(max(1, min(args.steps, 3)) + 1):
            barrier()
            t0 = time.perf_counter()
            req[0] += 1
            tok, _ = eng.prefill(req[0], prompt, chunks, strategy, decode_horizon=new_tokens)
            first = int(tok.item())  # device -> host read of the first token (TTFT)
            t1 = time.perf_counter()
            cur = tok
            outs = [tok]
            for _ in range(new_tokens - 1):
                cur = eng.decode_step([req[0]], cur)
                outs.append(cur.view(1))
            gen_ids = torch.cat(outs).cpu()  # device -> host read of the generated tokens
            t2 = time.perf_counter()
            eng.release(req[0])
            if i > 0:  # first iteration is a warm-up of the host path
                ttfts.append(t1 - t0)
                totals.append(t2 - t0)
        ttft = max_over_ranks(sum(ttfts) / len(ttfts), group)
        total = max_over_ranks(sum(totals) / len(totals), group)
        e2e = {"value": Lp / ttft, "unit": "prompt tokens/s (end to end: pinned prompt H2D, "
               "prefill, first-token D2H)", "ttft_ms": ttft * 1e3, "request_ms": total * 1e3,
               "decode_tok_s": (new_tokens - 1) / max(1e-9, total - ttft),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8 + new_tokens * 8}

    # ---------------------------------------------------------------- batched decode (B requests)
    batch = None
    if B > 1:
        ids = []
        toks = []
        for b in range(B):
            req[0] += 1
            tok, _ = eng.prefill(req[0], prompt_dev, chunks, strategy, decode_horizon=new_tokens)
            ids.append(req[0])
            toks.append(tok.view(1))
        cur = torch.cat(toks)
        for _ in range(3):
            cur = eng.decode_step(ids, cur)
        barrier()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_dec = new_tokens - 4
        b0.record()
        for _ in range(n_dec):
            cur = eng.decode_step(ids, cur)
        b1.record()
        barrier()
        bms = max_over_ranks(b0.elapsed_time(b1) / n_dec, group)
        for i in ids:
            eng.release(i)
        batch = {"batch": B, "context": Lp, "decode_ms_per_step": bms,
                 "decode_tok_s": B * 1e3 / bms, "steps_timed": n_dec}

    clk = clocks.summary()
    value = Lp / (prefill_ms / 1e3)
    if rank == 0:
        out = {
            "metric": "prefill tok/s & TTFT @32k and decode tok/s (CP=N B200, max over ranks)",
            "value": value,
            "unit": "prompt tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": (value / BASELINE_PREFILL_TOK_S) if BASELINE_PREFILL_TOK_S else None,
            "dtype": "bf16",
            "data": "synthetic: uniform-random prompt token ids, random-init N(0,0.02) weights",
            "ttft_ms": prefill_ms,
            "decode_ms_per_token": decode_ms / max(1, new_tokens - 1),
            "decode_tok_s": (new_tokens - 1) / (decode_ms / 1e3),
            "gpu_launches": n_launch,
            "config": {"model": spec["model"], "global_batch": 1, "seq_len": Lp,
                       "new_tokens": new_tokens, "parallelism": f"cp{world}",
                       "chunks": chunks, "strategy": strategy,
                       "l2": "no flush: weights + activations (>2.5 GB) exceed the 126 MB L2",
                       "step": "one request = prefill of the prompt + 127 decode steps"},
            "clocks": clk,
            "e2e": e2e,
        }
        if batch is not None:
            out["decode_batch"] = batch
        print(json.dumps(out), flush=True)
    eng.close()
    if world > 1:
        dist.barrier(group=group)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
