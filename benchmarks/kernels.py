"""Kernel microbenchmarks, roofline fractions and the ring-attention sweep (no model).

Single GPU (one kernel family per call; ``--small`` picks a case sized for an ncu capture):

    python benchmarks/kernels.py gemm  [--small]      # tcgen05 GEMMs at the model's shapes vs cuBLAS
    python benchmarks/kernels.py attn  [--small]      # causal flash attention vs torch SDPA
    python benchmarks/kernels.py gemv  [--small]      # decode GEMVs (fused RMSNorm / SwiGLU / argmax)
    python benchmarks/kernels.py norm  [--small]      # RMSNorm and embedding gather
    python benchmarks/kernels.py decode [--small]     # one decode step (graph) at a 32k context

Ring-attention sweep (the kernel-sweep shape: 32 query heads, 8 KV heads, head_dim 128, causal),
one process per GPU, every number device-timed as the max over ranks:

    torchrun --nproc-per-node N benchmarks/kernels.py ring --seq 32768 --ratio 4:1

``ring`` times one ring-attention layer of this framework (K/V push into every rank's staging
buffer over NVLink + flash attention on the local staging buffer, the two launches of
``DomainRuntime::RunRingAttentionLayer``) and, with ``--compare``, the same layer in the
reference's style (f32 K/V blocks rotated with NCCL send/recv, GQA-expanded, ATen ops; the
restatement in ``benchmarks/ref_ring_torch.py``). Roofline for the fused ring:
max(FLOPs_rank / measured bf16 peak, bytes pushed over NVLink by the rank / 770 GB/s).

Every line printed is one JSON object. Peaks come from ``MEASURED_PEAKS.json`` at the repo root
(fallback 6.65 TB/s, 1.59 PFLOP/s).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

NVLINK_GBS = 770.0          # measured peer copy, GB/s per direction per GPU


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "tflops": float(p["bf16_tflops"]),
                "tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


def timed(fn, iters: int, warmup: int = 3, flush: torch.Tensor = None) -> float:
    """Mean device ms per call (CUDA events on the current stream, L2 flushed between calls)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def emit(**kw):
    print(json.dumps(kw), flush=True)


def l2_flush_buffer(dev):
    return torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # 256 MB > 126 MB L2


# ----------------------------------------------------------------------------- GEMM
def bench_gemm(args, dev, pk):
    from hetero_cp_ringattn_b200.ops import kernels as K
    T = 4096 if args.small else args.tokens
    shapes = [("qkv", 3072, 2048, "store"), ("o", 2048, 2048, "residual"),
              ("gate_up", 16384, 2048, "swiglu"), ("down", 2048, 8192, "residual"),
              ("qkv_8b", 6144, 4096, "store"), ("gate_up_8b", 28672, 4096, "swiglu"),
              ("down_8b", 4096, 14336, "residual")]
    if args.small:
        shapes = shapes[2:3]
    flush = l2_flush_buffer(dev)
    for name, n, k, epi in shapes:
        a = torch.randn(T, k, device=dev, dtype=torch.bfloat16)
        w = torch.randn(n, k, device=dev, dtype=torch.bfloat16) * 0.02
        res = torch.randn(T, n, device=dev, dtype=torch.bfloat16) if epi == "residual" else None
        out = torch.empty(T, n // 2 if epi == "swiglu" else n, device=dev, dtype=torch.bfloat16)
        fl = 2.0 * T * n * k
        ms_cublas = timed(lambda: torch.matmul(a, w.t()), args.iters, flush=flush)
        for gv in args.gemm_variants:
            ms = timed(lambda: K.gemm(a, w, epi, residual=res, out=out, variant=gv), args.iters,
                       flush=flush)
            emit(kernel="gemm_sm100", shape=name, M=T, N=n, K=k, epilogue=epi, variant=gv,
                 ms=round(ms, 4), tflops=round(fl / ms / 1e9, 1),
                 frac_of_measured=round(fl / ms / 1e9 / pk["tflops"], 3),
                 cublas_tflops=round(fl / ms_cublas / 1e9, 1), vs_cublas=round(ms_cublas / ms, 3),
                 peaks=pk["source"])


# ----------------------------------------------------------------------------- attention
def causal_flops(Lq: int, Lk: int, H: int, D: int) -> float:
    """QK^T and PV FLOPs of causal attention with the queries at the end of the key range."""
    pairs = Lq * (Lk - Lq) + Lq * (Lq + 1) / 2.0
    return 4.0 * pairs * H * D


def bench_attn(args, dev, pk):
    from hetero_cp_ringattn_b200.ops import kernels as K
    import torch.nn.functional as F
    cases = [(8192, args.head_dim)] if args.small else [(s, d) for d in (64, 128) for s in args.seqs]
    H, Hkv = 32, 8
    for L, D in cases:
        k = torch.randn(Hkv, L, D, device=dev, dtype=torch.bfloat16)
        v = torch.randn_like(k)
        if args.cp > 1:
            # one context-parallel rank's rows (zigzag, equal chunks) against the whole key range
            from hetero_cp_ringattn_b200.parallel.capacity import equal_chunks
            from hetero_cp_ringattn_b200.parallel.strategy import layout_positions
            pos_np = layout_positions(equal_chunks(L, args.cp), args.strategy)[args.rank]
            pos = torch.as_tensor(pos_np, device=dev).int()
            fl = 4.0 * H * D * float((pos_np + 1).sum())
        else:
            pos = torch.arange(L, device=dev, dtype=torch.int32)
            fl = causal_flops(L, L, H, D)
        T = int(pos.numel())
        q = torch.randn(T, H, D, device=dev, dtype=torch.bfloat16)
        iters = max(2, args.iters if L <= 32768 else 3)
        variants = [(vv, o) for vv in (args.variants if D == 64 else [0]) for o in args.orders]
        # kernel variants / CTA orders timed in alternation (--variants 0,3 --orders 0,1), best of
        # the repetitions
        best = {}
        for _ in range(args.reps):
            for vv, o in variants:
                t = timed(lambda: K.attention(q, k, v, pos, L, causal=True, variant=vv, order=o), iters)
                best[(vv, o)] = min(best.get((vv, o), t), t)
        base = dict(kernel="attn_fwd_sm100", L=L, T=T, H=H, Hkv=Hkv, D=D, causal=True)
        if args.cp > 1:
            base.update(cp=args.cp, rank=args.rank, strategy=args.strategy)
        for vv, o in variants[:-1]:
            emit(**base, variant=vv, order=o, ms=round(best[(vv, o)], 3),
                 tflops=round(fl / best[(vv, o)] / 1e9, 1),
                 frac_of_measured=round(fl / best[(vv, o)] / 1e9 / pk["tflops"], 3), peaks=pk["source"])
        ms = best[variants[-1]]
        row = dict(**base, variant=variants[-1][0], order=variants[-1][1], ms=round(ms, 3),
                   tflops=round(fl / ms / 1e9, 1),
                   frac_of_measured=round(fl / ms / 1e9 / pk["tflops"], 3), peaks=pk["source"])
        if not args.small and L <= 65536 and args.cp == 1:
            qs = q.transpose(0, 1).unsqueeze(0)
            ks, vs = k.unsqueeze(0), v.unsqueeze(0)
            ms_s = timed(lambda: F.scaled_dot_product_attention(qs, ks, vs, is_causal=True,
                                                                enable_gqa=True), iters)
            row.update(sdpa_tflops=round(fl / ms_s / 1e9, 1), vs_sdpa=round(ms_s / ms, 3))
        emit(**row)


# ----------------------------------------------------------------------------- GEMV / norm
def bench_gemv(args, dev, pk):
    from hetero_cp_ringattn_b200.ops import kernels as K
    flush = l2_flush_buffer(dev)
    hid = 2048
    nw = torch.ones(hid, device=dev, dtype=torch.bfloat16)
    cases = [("qkv+norm", 3072, hid, "f32"), ("gate_up+norm+swiglu", 16384, hid, "swiglu"),
             ("down+residual", 2048, 8192, "residual"), ("lm_head+norm+argmax", 128256, hid, "argmax"),
             ("8b gate_up+swiglu", 28672, 4096, "swiglu"), ("8b down+residual", 4096, 14336, "residual")]
    if args.small:
        cases = cases[1:2]
    nw = torch.ones(4096, device=dev, dtype=torch.bfloat16)
    for B in args.batches:
        for name, n, k, epi in cases:
            xx = torch.randn(B, k, device=dev, dtype=torch.bfloat16)
            w = torch.randn(n, k, device=dev, dtype=torch.bfloat16) * 0.02
            y32 = torch.empty(B, n, device=dev, dtype=torch.float32)
            yb = torch.zeros(B, n // 2 if epi == "swiglu" else n, device=dev, dtype=torch.bfloat16)
            am = torch.zeros(B, dtype=torch.int64, device=dev)
            norm = nw[:k] if epi != "residual" else None
            kw = dict(y_f32=y32 if epi in ("f32",) else None,
                      y_bf16=yb if epi in ("swiglu", "residual") else None,
                      argmax=am if epi == "argmax" else None, norm_w=norm)
            ms = timed(lambda: K.gemv(xx, w, epi, **kw), args.iters, flush=flush)
            byts = n * k * 2.0
            emit(kernel="gemv_sm100", shape=name, B=B, N=n, K=k, epilogue=epi, us=round(ms * 1e3, 2),
                 gbs=round(byts / ms / 1e6, 1),
                 frac_of_measured_hbm=round(byts / ms / 1e6 / pk["hbm_gbs"], 3), peaks=pk["source"])


def bench_norm(args, dev, pk):
    from hetero_cp_ringattn_b200.ops import kernels as K
    T = 8192 if args.small else args.tokens
    hid = 2048
    x = torch.randn(T, hid, device=dev, dtype=torch.bfloat16)
    w = torch.randn(hid, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(x)
    ms = timed(lambda: K.rmsnorm(x, w, 1e-5, out=out), args.iters)
    byts = 2.0 * T * hid * 2
    emit(kernel="rmsnorm", T=T, hidden=hid, us=round(ms * 1e3, 2), gbs=round(byts / ms / 1e6, 1),
         frac_of_measured_hbm=round(byts / ms / 1e6 / pk["hbm_gbs"], 3), peaks=pk["source"])
    emb = torch.randn(128256, hid, device=dev, dtype=torch.bfloat16)
    ids = torch.randint(0, 128256, (T,), device=dev, dtype=torch.int32)
    ms = timed(lambda: K.embedding(ids, emb, out=out), args.iters)
    emit(kernel="embedding", T=T, hidden=hid, us=round(ms * 1e3, 2), gbs=round(byts / ms / 1e6, 1),
         frac_of_measured_hbm=round(byts / ms / 1e6 / pk["hbm_gbs"], 3), peaks=pk["source"])


def bench_decode(args, dev, pk):
    """Decode step of a model preset (``--model``) over a prefilled ``--seq`` context, for each
    batch size of ``--batches`` (that many requests of the same context decoded together).

    The step is the captured CUDA graph the engine replays per token; ``--small`` uses 2 layers."""
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import PreparedWeights
    cfg = preset(args.model)
    cfg.num_layers = 2 if args.small else (args.layers or cfg.num_layers)
    ctx = args.seq
    w = PreparedWeights.random(cfg, seed=0, device=dev)
    bmax = max(args.batches)
    page = 256
    pages = bmax * (-(-ctx // page) + -(-(args.iters + 16) // page) + 1) + 2  # every request's KV
    eng = LlamaCPEngine(cfg, w, device=dev, max_context=ctx, max_batch=bmax,
                        decode_reserve=args.iters + 16, page_size=page, kv_pages=pages)
    prompt = torch.randint(0, cfg.vocab_size, (ctx,), dtype=torch.int64)
    per_layer_w = (cfg.hidden_size * (cfg.num_heads + 2 * cfg.kv_heads) * cfg.head_dim
                   + cfg.num_heads * cfg.head_dim * cfg.hidden_size + 3 * cfg.hidden_size * cfg.intermediate_size) * 2
    for B in args.batches:
        ids = list(range(1, B + 1))
        toks = [eng.prefill(r, prompt, [ctx], decode_horizon=args.iters + 8)[0].view(1) for r in ids]
        cur = torch.cat(toks)
        for _ in range(3):
            cur = eng.decode_step(ids, cur, logits=False)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = args.iters
        s.record()
        for _ in range(n):
            cur = eng.decode_step(ids, cur, logits=False)
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e) / n
        eng.check_device()
        kv = B * ctx * 2 * cfg.kv_heads * cfg.head_dim * 2
        byts = cfg.num_layers * (per_layer_w + kv) + cfg.vocab_size * cfg.hidden_size * 2
        emit(kernel="decode_step", model=args.model, layers=cfg.num_layers, context=ctx, batch=B,
             ms_per_token=round(ms, 4), tok_s=round(B * 1e3 / ms, 1), gbs=round(byts / ms / 1e6, 1),
             frac_of_measured_hbm=round(byts / ms / 1e6 / pk["hbm_gbs"], 3), peaks=pk["source"])
        for r in ids:
            eng.release(r)
    eng.close()


def bench_chunked(args, dev, pk):
    """Prefill of a ``--seq``-token prompt in one call against the chunked prefill of
    ``serve --prefill-chunk-tokens P`` for each P of ``--pieces``: the first P tokens through
    ``prefill`` (ring layout, session kept), the rest as continuation segments of P tokens
    through ``append`` (each attends to every stored row of the session). One rank; ms per
    prompt, CUDA events around the whole prompt (host work included, as in serving)."""
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import PreparedWeights
    cfg = preset(args.model)
    cfg.num_layers = 2 if args.small else (args.layers or cfg.num_layers)
    ctx = 8192 if args.small else args.seq
    w = PreparedWeights.random(cfg, seed=0, device=dev)
    eng = LlamaCPEngine(cfg, w, device=dev, max_context=ctx, max_batch=1, decode_reserve=16)
    prompt = torch.randint(0, cfg.vocab_size, (ctx,), dtype=torch.int64)

    def whole():
        tok, _ = eng.prefill(1, prompt, [ctx], decode_horizon=8)
        eng.release(1)
        return tok

    def pieces(p):
        tok, _ = eng.prefill(1, prompt[:p], [p], decode_horizon=8, keep_kv=True)
        done = p
        while done < ctx:
            end = min(ctx, done + p)
            tok, _ = eng.append(1, prompt[done:end], list(range(done, end)), [1])
            done = end
        eng.release(1)
        return tok

    def time_it(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(max(1, args.iters)):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            tok = fn()
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        return best, int(tok)

    ms_whole, tok_whole = time_it(whole)
    for p in args.pieces:
        if p >= ctx:
            continue
        ms, tok = time_it(lambda: pieces(p))
        emit(kernel="chunked_prefill", model=args.model, layers=cfg.num_layers, prompt=ctx, piece=p,
             segments=-(-ctx // p), ms=round(ms, 2), ms_whole=round(ms_whole, 2),
             ratio=round(ms / ms_whole, 3), same_token=tok == tok_whole)
    eng.close()


# ----------------------------------------------------------------------------- ring sweep
def parse_ratio(text: str, n: int) -> list:
    """'1:1' -> equal; 'a:b' with n > 2 -> first half of the ranks weight a, second half b."""
    parts = [int(p) for p in text.split(":")]
    if len(parts) == n:
        return parts
    if len(parts) == 2:
        return [parts[0]] * (n - n // 2) + [parts[1]] * (n // 2) if n > 1 else [1]
    raise SystemExit(f"ratio {text!r} does not fit {n} ranks")


def bench_ring(args, pk):
    import torch.distributed as dist
    from hetero_cp_ringattn_b200.ops._ext import native
    from hetero_cp_ringattn_b200.ops import reference as ref
    from hetero_cp_ringattn_b200.parallel.capacity import chunks_from_ratio
    from hetero_cp_ringattn_b200.parallel.strategy import build_assignment, build_domain_positions
    from hetero_cp_ringattn_b200.utils.perf import max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    H, Hkv, D = args.heads, args.kv_heads, args.head_dim
    L = args.seq
    chunks = chunks_from_ratio(L, parse_ratio(args.ratio, world))
    assignment = build_assignment(chunks, args.strategy)
    positions = build_domain_positions(assignment, world)
    my_pos = positions[rank]
    T = len(my_pos)
    page = 256
    pages = -(-T // page) + 1
    rt = native().Runtime(rank, world, local, 1, pages, page, Hkv, D, H, L, 1, 5000)
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, rt.export_handle())
        rt.open_peers(handles)
        dist.barrier()
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    qkv = torch.randn(T, (H + 2 * Hkv) * D, device=dev, dtype=torch.bfloat16, generator=g)
    pos = torch.from_numpy(my_pos.astype("int32")).to(dev)
    cos, sin = ref.rope_cos_sin(torch.arange(L + 8, device=dev), D, 1e6)
    cos, sin = cos.contiguous(), sin.contiguous()
    pt = torch.arange(pages, dtype=torch.int32, device=dev)
    q_buf = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
    o_buf = torch.empty_like(q_buf)
    scale = 1.0 / math.sqrt(D)
    epoch = [0]
    ring = {}
    if world > 1 and not args.serial:
        # overlapped ring: local projection, the attention kernel pushes and waits per tile
        from hetero_cp_ringattn_b200.models.llama import ring_plan
        src, push = ring_plan(positions, rank, L)
        ring = dict(tile_src=torch.from_numpy(src).to(dev), push_tiles=torch.from_numpy(push).to(dev))

    def layer():
        epoch[0] += 1
        a = (qkv, pos, cos, sin, 0, pt, 0, L, scale, True, q_buf, o_buf, None, epoch[0])
        rt.push_layer(*a, **ring)
        rt.attend_layer(*a, **ring)

    iters = args.iters
    for _ in range(3):
        layer()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        layer()
    e.record()
    e.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / iters)
    rt.check()
    # work per rank: this rank's queries against every earlier position; the slowest rank bounds
    fl_rank = sum(4.0 * (int(p) + 1) * H * D for p in my_pos)
    fl_max = max_over_ranks(fl_rank)
    fl_total = sum(4.0 * (p + 1) * H * D for p in range(L))
    push_bytes = T * 2 * Hkv * D * 2.0 * (world - 1)         # own rows into every peer's staging
    push_max = max_over_ranks(push_bytes)
    t_compute = fl_max / (pk["tflops"] * 1e9)
    t_link = push_max / (NVLINK_GBS * 1e6)
    roof = max(t_compute, t_link)
    row = dict(kernel="ring_attention_layer", cp=world, seq=L, chunks=chunks, strategy=args.strategy,
               ring="serial" if (args.serial or world == 1) else "overlapped",
               H=H, Hkv=Hkv, D=D, ms=round(ms, 3), tflops_total=round(fl_total / ms / 1e9, 1),
               tflops_per_gpu=round(fl_total / ms / 1e9 / world, 1),
               nvlink_gbs_per_gpu=round(push_max / ms / 1e6, 1),
               roofline_ms=round(roof, 3), frac_of_roofline=round(roof / ms, 3),
               bound="compute" if t_compute >= t_link else "nvlink", peaks=pk["source"])
    if args.compare and L <= args.compare_max_seq:
        from benchmarks.ref_ring_torch import RefRingModel

        class _Cfg:
            num_heads, kv_heads, head_dim, rope_theta = H, Hkv, D, 1e6
        m = RefRingModel(_Cfg(), {}, rank, world, dev)
        qq = qkv[:, :H * D].view(T, H, D)
        kk = qkv[:, H * D:(H + Hkv) * D].view(T, Hkv, D)
        vv = qkv[:, (H + Hkv) * D:].view(T, Hkv, D)
        plong = pos.long()
        m._ring_attention(qq, kk, vv, plong)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        n_ref = max(1, min(iters, 3))
        s.record()
        for _ in range(n_ref):
            m._ring_attention(qq, kk, vv, plong)
        e.record()
        e.synchronize()
        ms_ref = max_over_ranks(s.elapsed_time(e) / n_ref)
        row.update(ref_ring_ms=round(ms_ref, 3), ref_tflops_total=round(fl_total / ms_ref / 1e9, 1),
                   speedup_vs_ref_ring=round(ms_ref / ms, 2))
    if rank == 0:
        emit(**row)
    if world > 1:
        dist.barrier()
    rt.shutdown()
    if world > 1:
        dist.destroy_process_group()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("what", choices=["gemm", "attn", "gemv", "norm", "decode", "ring", "chunked"])
    ap.add_argument("--small", action="store_true", help="one small case (sized for an ncu capture)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--seqs", type=lambda s: [int(x) for x in s.split(",")], default=[8192, 32768])
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--pieces", type=lambda s: [int(x) for x in s.split(",")], default=[4096, 8192],
                    help="chunked: prefill piece sizes")
    ap.add_argument("--layers", type=int, default=0, help="decode: layers (0 = the model's)")
    ap.add_argument("--model", default="llama-3.2-1b", help="decode: model preset")
    ap.add_argument("--ratio", default="1:1")
    ap.add_argument("--strategy", default="zigzag")
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--variants", type=lambda s: [int(x) for x in s.split(",")], default=[0],
                    help="attn: head_dim-64 kernel variants to time (0 default, 1, 2, 3 pipelined)")
    ap.add_argument("--reps", type=int, default=1, help="attn: alternating repetitions")
    ap.add_argument("--batches", type=lambda s: [int(x) for x in s.split(",")], default=[1],
                    help="gemv: decode rows (1, 2, 4, 8)")
    ap.add_argument("--gemm-variants", type=lambda s: [int(x) for x in s.split(",")], default=[0],
                    help="gemm: kernels to time (0 default, 1 one CTA per tile, 2 CTA pairs)")
    ap.add_argument("--orders", type=lambda s: [int(x) for x in s.split(",")], default=[-1],
                    help="attn: CTA orders to time (-1 kernel's choice, 0 KV-head major, 1 pair major)")
    ap.add_argument("--cp", type=int, default=1, help="attn: time one rank's rows of this CP degree")
    ap.add_argument("--rank", type=int, default=0, help="attn: the rank for --cp")
    ap.add_argument("--compare", action="store_true", help="also time the NCCL send/recv ring restatement")
    ap.add_argument("--serial", action="store_true",
                    help="ring: the serial ring (push, wait for every rank, attend) instead of the "
                         "overlapped ring inside the attention kernel")
    ap.add_argument("--compare-max-seq", type=int, default=131072)
    args = ap.parse_args(argv)
    pk = peaks()
    if args.what == "ring":
        return bench_ring(args, pk)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    {"gemm": bench_gemm, "attn": bench_attn, "gemv": bench_gemv, "norm": bench_norm,
     "decode": bench_decode, "chunked": bench_chunked}[args.what](args, dev, pk)


if __name__ == "__main__":
    main()
