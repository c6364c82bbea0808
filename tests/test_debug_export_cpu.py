"""Debug exports (hidden states, layer-0 prefill intermediates, q/k injection) on CPU: file layout
[ndims u64][dims u64...][f32], shapes, agreement with the oracle's logits, and that injecting the
exported q/k reproduces the same intermediates."""

import os
import struct

import torch

from hetero_cp_ringattn_b200.config import preset
from hetero_cp_ringattn_b200.debug_export import (export_hidden_states, prefill_debug_layer0,
                                                  read_tensor_bin, write_tensor_bin)
from hetero_cp_ringattn_b200.models import reference_model
from hetero_cp_ringattn_b200.models.weights import ModelWeights


def _model():
    cfg = preset("tiny")
    return cfg, ModelWeights.random_init(cfg, seed=3, dtype=torch.float32)


def test_tensor_file_roundtrip(tmp_path):
    t = torch.randn(2, 3, 5)
    p = str(tmp_path / "t.bin")
    write_tensor_bin(t, p)
    with open(p, "rb") as f:
        assert struct.unpack("<Q", f.read(8))[0] == 3
        assert struct.unpack("<QQQ", f.read(24)) == (2, 3, 5)
    assert torch.equal(read_tensor_bin(p), t)


def test_export_hidden_states(tmp_path):
    cfg, w = _model()
    ids = torch.randint(0, cfg.vocab_size, (23,), generator=torch.Generator().manual_seed(1))
    d = str(tmp_path / "hs")
    first = export_hidden_states(w, ids, d)
    logits = reference_model.forward(w, ids, last_only=True)[0]
    assert first == int(torch.argmax(logits))
    for i in range(cfg.num_layers):
        k = read_tensor_bin(os.path.join(d, f"prefill_k_layer_{i}.bin"))
        v = read_tensor_bin(os.path.join(d, f"prefill_v_layer_{i}.bin"))
        assert tuple(k.shape) == (1, cfg.kv_heads, 23, cfg.head_dim) == tuple(v.shape)
        hs = read_tensor_bin(os.path.join(d, f"layer_{i}.bin"))
        assert tuple(hs.shape) == (1, 1, cfg.hidden_size)
    fn = read_tensor_bin(os.path.join(d, "final_norm.bin"))
    assert tuple(fn.shape) == (1, 1, cfg.hidden_size)
    with open(os.path.join(d, "logits.bin"), "rb") as f:
        vocab, rows = struct.unpack("<QQ", f.read(16))
        assert (vocab, rows) == (cfg.vocab_size, 1)
    # the exported decode-step logits are the oracle's logits for prompt + first token
    ids1 = torch.cat([ids, torch.tensor([first])])
    ref1 = reference_model.forward(w, ids1, last_only=True)[0]
    import numpy as np
    got = np.fromfile(os.path.join(d, "logits.bin"), dtype="<f4", offset=16)
    assert np.allclose(got, ref1.numpy(), atol=1e-5)


def test_prefill_debug_and_qk_injection(tmp_path):
    cfg, w = _model()
    ids = torch.randint(0, cfg.vocab_size, (17,), generator=torch.Generator().manual_seed(2))
    d1, d2 = str(tmp_path / "a"), str(tmp_path / "b")
    prefill_debug_layer0(w, ids, d1)
    names = ["embedding_output", "layer_0_input_norm", "q_proj_layer_0", "k_proj_layer_0",
             "v_proj_layer_0", "layer_0_post_attn", "layer_0_post_mlp"]
    for n in names:
        t = read_tensor_bin(os.path.join(d1, n + ".bin"))
        assert t.shape[0] == 1 and t.shape[1] == 17
    # injecting the exported q/k gives the same downstream intermediates
    prefill_debug_layer0(w, ids, d2, qk_inject_dir=d1)
    for n in ["layer_0_post_attn", "layer_0_post_mlp", "prefill_k_layer_1"]:
        a = read_tensor_bin(os.path.join(d1, n + ".bin"))
        b = read_tensor_bin(os.path.join(d2, n + ".bin"))
        assert torch.allclose(a, b, atol=1e-6)
    # and injecting zeros changes them
    z = str(tmp_path / "z")
    os.makedirs(z)
    q = read_tensor_bin(os.path.join(d1, "q_proj_layer_0.bin"))
    write_tensor_bin(torch.zeros_like(q), os.path.join(z, "q_proj_layer_0.bin"))
    write_tensor_bin(read_tensor_bin(os.path.join(d1, "k_proj_layer_0.bin")), os.path.join(z, "k_proj_layer_0.bin"))
    d3 = str(tmp_path / "c")
    prefill_debug_layer0(w, ids, d3, qk_inject_dir=z)
    a = read_tensor_bin(os.path.join(d1, "layer_0_post_attn.bin"))
    c = read_tensor_bin(os.path.join(d3, "layer_0_post_attn.bin"))
    assert not torch.allclose(a, c)


def test_compare_hidden_cli(tmp_path):
    import json
    import subprocess
    import sys
    cfg, w = _model()
    ids = torch.randint(0, cfg.vocab_size, (9,), generator=torch.Generator().manual_seed(4))
    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    prefill_debug_layer0(w, ids, a)
    prefill_debug_layer0(w, ids, b)
    r = subprocess.run([sys.executable, "-m", "hetero_cp_ringattn_b200", "compare-hidden", a, b],
                       capture_output=True, text=True, timeout=120)
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 0 and out["passed"] and out["files"] >= 7
    # perturb one file: the comparison fails and names it
    t = read_tensor_bin(os.path.join(b, "layer_0_post_attn.bin"))
    write_tensor_bin(t + 1.0, os.path.join(b, "layer_0_post_attn.bin"))
    r = subprocess.run([sys.executable, "-m", "hetero_cp_ringattn_b200", "compare-hidden", a, b],
                       capture_output=True, text=True, timeout=120)
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 1 and not out["passed"]
    bad = [x for x in out["per_file"] if x["max_abs"] > 0.5]
    assert [x["file"] for x in bad] == ["layer_0_post_attn.bin"]
