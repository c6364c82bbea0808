"""Ring-attention correctness suite (oracle vs. ring model, optionally vs. the device kernels).

Parity: the reference's correctness orchestrator and runner (rust/src/lib.rs:107-199,
rust/src/smoke/correctness.rs:5-176): seven default cases with uneven chunks and blocks, five
stress seeds for small cases, worst-seed reporting and a JSON report. Case geometry
(chunks, block sizes, heads, head_dim) is kept identical to `default_cases()` so the two suites
measure the same configurations. Extensions: causal masking on global positions, GQA, LSE
comparison, and the benchmark plumbing case (1024/512 split, 16 query heads, 4 KV heads, D=64).
"""

from __future__ import annotations

import dataclasses
import json
import time
from typing import Optional, Sequence

import torch

from .errors import ToleranceTier
from .ops import reference as ref
from .parallel.strategy import layout_positions


@dataclasses.dataclass
class CaseConfig:
    chunks: list
    block_sizes: list
    num_heads: int
    head_dim: int
    num_kv_heads: Optional[int] = None
    causal: bool = False
    strategy: str = "vanilla"

    @property
    def global_seq_len(self) -> int:
        return sum(self.chunks)

    @property
    def domains(self) -> int:
        return len(self.chunks)


def default_cases() -> list:
    """The reference's seven cases (non-causal MHA, as in reference_algo.rs)."""
    return [
        ("2domain_uneven_chunks", CaseConfig([80, 48], [16, 12], 4, 16)),
        ("3domain_uneven_blocks", CaseConfig([64, 40, 56], [32, 10, 14], 3, 24)),
        ("4domain_small_tail_blocks", CaseConfig([32, 64, 48, 48], [7, 16, 11, 13], 2, 32)),
        ("3domain_large_seq", CaseConfig([512, 256, 256], [128, 64, 64], 8, 64)),
        ("1domain_single_block", CaseConfig([64], [64], 4, 16)),
        ("2domain_unit_blocks", CaseConfig([16, 16], [1, 1], 2, 8)),
        ("1domain_medium", CaseConfig([128], [32], 4, 16)),
    ]


def extended_cases() -> list:
    """Causal / GQA / strategy cases added for the B200 build."""
    return [
        ("baseline_2domain_1024_512_gqa_causal",
         CaseConfig([1024, 512], [1024, 512], 16, 64, num_kv_heads=4, causal=True)),
        ("3domain_551_zigzag_gqa_causal",
         CaseConfig([250, 250, 50], [64, 64, 64], 8, 32, num_kv_heads=2, causal=True,
                    strategy="zigzag")),
        ("4domain_striped_causal",
         CaseConfig([64, 32, 48, 16], [16, 8, 16, 4], 4, 16, num_kv_heads=1, causal=True,
                    strategy="striped")),
    ]


def _metrics(a: torch.Tensor, b: torch.Tensor) -> dict:
    fin = torch.isfinite(a) & torch.isfinite(b)
    same_inf = (~torch.isfinite(a)) & (a == b)
    bad = ~(fin | same_inf)
    diff = (a - b).abs().where(fin, torch.zeros_like(a))
    denom = b.abs().where(fin, torch.ones_like(b)).clamp_min(1e-6)
    return {
        "max_abs_err": float(diff.max()) if diff.numel() else 0.0,
        "mean_abs_err": float(diff.mean()) if diff.numel() else 0.0,
        "max_rel_err": float((diff / denom).max()) if diff.numel() else 0.0,
        "nonfinite_mismatch": int(bad.sum()),
    }


def make_case_tensors(cfg: CaseConfig, seed: int, dtype=torch.float64, device="cpu"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    L = cfg.global_seq_len
    hkv = cfg.num_kv_heads or cfg.num_heads
    q = torch.randn(L, cfg.num_heads, cfg.head_dim, generator=g, dtype=torch.float64)
    k = torch.randn(L, hkv, cfg.head_dim, generator=g, dtype=torch.float64)
    v = torch.randn(L, hkv, cfg.head_dim, generator=g, dtype=torch.float64)
    return q.to(device=device, dtype=dtype), k.to(device=device, dtype=dtype), \
        v.to(device=device, dtype=dtype)


def run_case_single_seed(cfg: CaseConfig, seed: int, dtype=torch.float64,
                         oracle: str = "python") -> dict:
    q, k, v = make_case_tensors(cfg, seed, dtype)
    L = cfg.global_seq_len
    if oracle == "native":
        # the C++ float64 oracle of the host library (both the ring and the full attention)
        from .host import lib
        qn, kn, vn = (t.double().numpy() for t in (q, k, v))
        pos = layout_positions(cfg.chunks, cfg.strategy)
        fo, fl = lib().attention_f64(qn, kn, vn, cfg.causal)
        ro, rl = lib().ring_attention_f64(qn, kn, vn, list(pos), list(cfg.block_sizes), cfg.causal)
        return {"seed": seed, "output": _metrics(torch.from_numpy(ro), torch.from_numpy(fo)),
                "lse": _metrics(torch.from_numpy(rl), torch.from_numpy(fl))}
    pos_all = torch.arange(L)
    full_o, full_lse = ref.full_attention(q, k, v, pos_all, pos_all, causal=cfg.causal)
    positions = [torch.as_tensor(p) for p in layout_positions(cfg.chunks, cfg.strategy)]
    qc = [q[p] for p in positions]
    kc = [k[p] for p in positions]
    vc = [v[p] for p in positions]
    outs = ref.ring_attention_model(qc, kc, vc, positions, cfg.block_sizes, causal=cfg.causal)
    ring_o = torch.empty_like(full_o)
    ring_lse = torch.empty_like(full_lse)
    for p, (o, lse) in zip(positions, outs):
        ring_o[p] = o
        ring_lse[:, p] = lse
    m_o = _metrics(ring_o, full_o)
    m_l = _metrics(ring_lse, full_lse)
    return {"seed": seed, "output": m_o, "lse": m_l}


def run_case(name: str, cfg: CaseConfig, seeds: Sequence[int], tier: ToleranceTier,
             dtype=torch.float64, oracle: str = "python") -> dict:
    per_seed = [run_case_single_seed(cfg, s, dtype, oracle) for s in seeds]
    worst = max(per_seed, key=lambda r: max(r["output"]["max_abs_err"], r["lse"]["max_abs_err"]))
    tol = tier.tolerance()
    passed = all(
        r[key]["max_abs_err"] <= tol.max_abs_err and r[key]["mean_abs_err"] <= tol.mean_abs_err
        and r[key]["nonfinite_mismatch"] == 0
        for r in per_seed for key in ("output", "lse"))
    rep = {"name": name, "config": dataclasses.asdict(cfg), "seeds": list(seeds),
           "worst_seed": worst, "passed": passed, "tolerance_tier": tier.value, "oracle": oracle}
    # the reference's report keys for the same case (rust/src/report.rs: status, seed,
    # tolerance, metrics, config with per-domain entries, ring trace summary)
    rep.update({
        "status": "pass" if passed else "fail",
        "seed": worst["seed"],
        "tolerance": {"max_abs_err": tol.max_abs_err, "mean_abs_err": tol.mean_abs_err},
        "metrics": {k: max(worst["output"][k], worst["lse"][k])
                    for k in ("max_abs_err", "mean_abs_err")},
    })
    rep["config"].update({
        "global_seq_len": cfg.global_seq_len, "dtype": str(dtype).replace("torch.", ""),
        "domains": [{"domain_id": f"domain-{d}", "seq_chunk_len": c, "block_size": b,
                     "device": "model"} for d, (c, b) in enumerate(zip(cfg.chunks, cfg.block_sizes))]})
    rep["ring_trace_summary"] = ring_trace_summary(cfg)
    return rep


def ring_trace_summary(cfg: CaseConfig, first: int = 4) -> list:
    """Per domain: its positions, how many KV blocks it folds and the first `first` of them in
    fold order (own chunk first, then the ring's other sources), as ring_attention_model walks
    them. Blocks index each source's local rows; with the vanilla layout those are global
    positions."""
    n = cfg.domains
    offs = [sum(cfg.chunks[:d]) for d in range(n)]
    out = []
    for t in range(n):
        blocks = []
        for step in range(n):
            src = (t + step) % n
            bs = max(1, int(cfg.block_sizes[src]))
            for b0 in range(0, cfg.chunks[src], bs):
                b1 = min(cfg.chunks[src], b0 + bs)
                blocks.append({"source_domain": f"domain-{src}", "block_start": offs[src] + b0,
                               "block_stop": offs[src] + b1, "block_len": b1 - b0})
        out.append({"domain_id": f"domain-{t}", "seq_offset": offs[t], "seq_chunk_len": cfg.chunks[t],
                    "block_visits": len(blocks), "first_blocks": blocks[:first]})
    return out


def case_from_ring_config(cfg) -> CaseConfig:
    """A domain layout file (config.RingAttnConfig: chunks, block sizes, heads) as a causal case."""
    return CaseConfig(cfg.chunks, cfg.block_sizes, cfg.num_heads, cfg.head_dim,
                      num_kv_heads=cfg.num_kv_heads, causal=True)


def run_suite(tier: ToleranceTier = ToleranceTier.STRICT, stress_seeds: int = 5,
              include_extended: bool = True, dtype=torch.float64, extra_cases=(),
              oracle: str = "python") -> dict:
    t0 = time.time()
    cases = default_cases() + (extended_cases() if include_extended else []) + list(extra_cases)
    reports = []
    for name, cfg in cases:
        small = cfg.global_seq_len <= 256
        seeds = list(range(stress_seeds)) if small else [0]
        reports.append(run_case(name, cfg, seeds, tier, dtype, oracle))
    n_pass = sum(1 for r in reports if r["passed"])
    return {"suite": "ring_attention_correctness", "tolerance": dataclasses.asdict(tier.tolerance()),
            "passed": n_pass == len(reports), "cases": reports, "elapsed_s": time.time() - t0,
            # the reference's top-level keys
            "status": "pass" if n_pass == len(reports) else "fail",
            "summary": {"cases": len(reports), "passed": n_pass, "failed": len(reports) - n_pass}}


def write_report(report: dict, path: str) -> None:
    with open(path, "w") as f:
        json.dump(report, f, indent=2)
