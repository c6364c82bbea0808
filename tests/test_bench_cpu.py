"""Host-side pieces of the benchmark entry points (no GPU): the configs name existing model shapes
of the benchmark table, `--impl reference` prints its one-line JSON and exits 0, and the kernel
bench's ratio / FLOP helpers."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_bench_configs_are_known_shapes():
    import bench
    from hetero_cp_ringattn_b200.config import preset
    assert bench.CONFIGS["llama-3.2-1b-32k"]["prompt"] == 32768
    for name, spec in bench.CONFIGS.items():
        cfg = preset(spec["model"])
        assert cfg.max_position_embeddings >= spec["prompt"] + spec["new_tokens"], name


def test_reference_arm_reports_unavailable():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference"], cwd=ROOT,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


def test_kernel_bench_helpers():
    from benchmarks import kernels as kb
    assert kb.parse_ratio("1:1", 2) == [1, 1]
    assert kb.parse_ratio("4:1", 8) == [4, 4, 4, 4, 1, 1, 1, 1]
    assert kb.parse_ratio("5:5:1", 3) == [5, 5, 1]
    # causal FLOPs of an L-token prefill: 4 * H * D * L (L + 1) / 2
    assert kb.causal_flops(8, 8, 2, 4) == 4.0 * 2 * 4 * 36
    p = kb.peaks()
    assert p["hbm_gbs"] > 0 and p["tflops"] > 0


def test_host_bench_reports_native_and_json_costs(capsys):
    import importlib.util
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "benchmarks", "host_bench.py")
    spec = importlib.util.spec_from_file_location("host_bench", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.main() == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    f = out["prefill_frame_32k"]
    assert f["native_ms"] > 0 and f["json_ms"] > 0 and f["bytes"] > 32768 * 8


def test_bench_secondary_configs_per_n():
    """Besides the headline, every N also measures BASELINE config #3 (the uneven
    5:5:5:5:2:2:1:1 split at 8 ranks, equal chunks otherwise) and N=8 config #4 with batch-1 and
    batch-8 decode; the CP output check runs by default."""
    import bench
    assert [c[0] for c in bench.secondary_configs(1)] == ["#3"]
    assert [c[0] for c in bench.secondary_configs(8)] == ["#3", "#4"]
    c3 = bench.secondary_configs(8)[0]
    assert c3[1] == "qwen2.5-3b-64k" and c3[2] == "5:5:5:5:2:2:1:1"
    c4 = bench.secondary_configs(8)[1]
    assert c4[1] == "llama-3-8b-128k" and c4[3] == [1, 8]
    a = bench.parse([])
    assert not a.no_check and not a.no_secondary
