"""Ring-attention oracle suite on CPU: the reference's seven cases (non-causal MHA, uneven chunks and
blocks, 1-4 domains) plus causal / GQA / zigzag / striped extensions and the benchmark plumbing case
(1024/512 split, 16 query heads, 4 KV heads, D=64, fp32, tolerance 1e-4 on O and LSE)."""

import json

import pytest
import torch

from hetero_cp_ringattn_b200 import correctness as C
from hetero_cp_ringattn_b200.cli import main as cli_main
from hetero_cp_ringattn_b200.errors import ToleranceTier


@pytest.mark.parametrize("name,cfg", C.default_cases() + C.extended_cases(), ids=lambda x: x if isinstance(x, str) else "")
def test_ring_model_matches_full_attention_f64(name, cfg):
    rep = C.run_case(name, cfg, seeds=[0, 1] if cfg.global_seq_len <= 256 else [0],
                     tier=ToleranceTier.STRICT)
    assert rep["passed"], rep["worst_seed"]


def test_baseline_plumbing_case_fp32():
    cfg = C.CaseConfig([1024, 512], [1024, 512], 16, 64, num_kv_heads=4, causal=True)
    r = C.run_case_single_seed(cfg, seed=0, dtype=torch.float32)
    assert r["output"]["max_abs_err"] < 1e-4
    assert r["lse"]["max_abs_err"] < 1e-4


def test_merge_partials_is_exact():
    from hetero_cp_ringattn_b200.ops import reference as ref
    torch.manual_seed(0)
    q = torch.randn(7, 4, 16, dtype=torch.float64)
    k = torch.randn(30, 2, 16, dtype=torch.float64)
    v = torch.randn(30, 2, 16, dtype=torch.float64)
    o, lse = ref.full_attention(q, k, v, causal=False)
    parts = [ref.full_attention(q, k[a:b], v[a:b], causal=False) for a, b in [(0, 11), (11, 12), (12, 30)]]
    om, lm = ref.merge_partials([p[0] for p in parts], [p[1] for p in parts])
    assert (om - o).abs().max() < 1e-12 and (lm - lse).abs().max() < 1e-12
    # an empty shard (lse = -inf) contributes nothing
    e = (torch.zeros_like(o), torch.full_like(lse, float("-inf")))
    om2, lm2 = ref.merge_partials([e[0], o], [e[1], lse])
    assert (om2 - o).abs().max() < 1e-12 and (lm2 - lse).abs().max() < 1e-12


def test_cli_correctness_report(tmp_path):
    path = tmp_path / "ring.json"
    assert cli_main(["correctness", "--report-path", str(path), "--stress-test", "1"]) == 0
    rep = json.loads(path.read_text())
    assert rep["passed"] and len(rep["cases"]) == 10


def test_domain_layout_files_run_as_cases(tmp_path):
    """The shipped domain layout files (configs/*.json) parse, validate and pass as causal ring
    cases; the CLI takes them with --config."""
    import glob
    import json
    import os
    import subprocess
    import sys
    from hetero_cp_ringattn_b200.config import RingAttnConfig
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    files = sorted(glob.glob(os.path.join(root, "configs", "*.json")))
    assert files
    for p in files:
        cfg = RingAttnConfig.from_file(p)
        rep = C.run_case(os.path.basename(p), C.case_from_ring_config(cfg), seeds=[0],
                         tier=ToleranceTier.STRICT)
        assert rep["passed"], rep["worst_seed"]
    out = tmp_path / "r.json"
    r = subprocess.run([sys.executable, "-m", "hetero_cp_ringattn_b200", "correctness", "--stress-test", "1",
                        "--config", files[0], "--report-path", str(out)],
                       capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    names = [c["name"] for c in json.load(open(out))["cases"]]
    assert os.path.basename(files[0]) in names


def test_report_carries_the_reference_schema(tmp_path):
    """Reports also carry the reference's keys (reports/ringattn_correctness.json: status,
    summary, per case status / seed / tolerance / metrics / domains / ring_trace_summary); the
    trace of the 2-domain uneven case equals the reference report's."""
    from hetero_cp_ringattn_b200.correctness import default_cases, run_case
    from hetero_cp_ringattn_b200.errors import ToleranceTier
    name, cfg = default_cases()[0]
    rep = run_case(name, cfg, [42], ToleranceTier.STRICT)
    assert rep["status"] == "pass" and rep["seed"] == 42
    assert set(rep["tolerance"]) == {"max_abs_err", "mean_abs_err"}
    assert rep["metrics"]["max_abs_err"] < 1e-12
    assert rep["config"]["global_seq_len"] == 128
    assert [d["seq_chunk_len"] for d in rep["config"]["domains"]] == [80, 48]
    t0, t1 = rep["ring_trace_summary"]
    assert (t0["seq_offset"], t0["block_visits"], t1["seq_offset"], t1["block_visits"]) == (0, 9, 80, 9)
    assert [(b["block_start"], b["block_stop"]) for b in t0["first_blocks"]] == \
        [(0, 16), (16, 32), (32, 48), (48, 64)]
    assert [(b["source_domain"], b["block_start"], b["block_len"]) for b in t1["first_blocks"][:1]] == \
        [("domain-1", 80, 12)]


@pytest.mark.parametrize("name,cfg", C.default_cases()[:4] + C.extended_cases()[1:],
                         ids=lambda x: x if isinstance(x, str) else "")
def test_native_oracle_matches_python_oracle(name, cfg):
    """The C++ float64 oracle (host library) and the Python one agree on ring and full attention
    to rounding level, for the reference's cases and causal GQA zigzag / striped layouts."""
    import numpy as np
    from hetero_cp_ringattn_b200.host import lib
    from hetero_cp_ringattn_b200.ops import reference as ref
    from hetero_cp_ringattn_b200.parallel.strategy import layout_positions
    q, k, v = C.make_case_tensors(cfg, seed=3)
    pos = layout_positions(cfg.chunks, cfg.strategy)
    o_n, l_n = lib().ring_attention_f64(q.numpy(), k.numpy(), v.numpy(), list(pos),
                                        list(cfg.block_sizes), cfg.causal)
    f_n, fl_n = lib().attention_f64(q.numpy(), k.numpy(), v.numpy(), cfg.causal)
    L = cfg.global_seq_len
    all_pos = torch.arange(L)
    f_p, fl_p = ref.full_attention(q, k, v, all_pos, all_pos, causal=cfg.causal)
    assert np.abs(f_n - f_p.numpy()).max() < 1e-12 and np.abs(fl_n - fl_p.numpy()).max() < 1e-12
    assert np.abs(o_n - f_p.numpy()).max() < 1e-10 and np.abs(l_n - fl_p.numpy()).max() < 1e-10


def test_cli_correctness_with_native_oracle(tmp_path):
    out = tmp_path / "native.json"
    assert cli_main(["correctness", "--oracle", "native", "--stress-test", "2",
                     "--report-path", str(out)]) == 0
    rep = json.loads(out.read_text())
    assert rep["status"] == "pass" and rep["summary"]["failed"] == 0
    assert all(c["oracle"] == "native" for c in rep["cases"])


def test_query_chunked_dense_attention_matches():
    """The float32 oracle's long-context mode (queries in chunks) gives every row the same result
    as the one-shot dense attention, causal on positions and not."""
    import torch
    from hetero_cp_ringattn_b200.ops import reference as ref
    g = torch.Generator().manual_seed(3)
    q = torch.randn(37, 8, 16, generator=g)
    k = torch.randn(50, 2, 16, generator=g)
    v = torch.randn(50, 2, 16, generator=g)
    qp = torch.arange(13, 50)
    for causal in (True, False):
        o1, l1 = ref.full_attention(q, k, v, qp, None, causal=causal)
        o2, l2 = ref.full_attention(q, k, v, qp, None, causal=causal, q_chunk=5)
        assert torch.allclose(o1, o2, atol=1e-6) and torch.allclose(l1, l2, atol=1e-6)
