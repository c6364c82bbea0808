"""Parity with HF transformers (the implementation the reference validates its logits against:
scripts/export_python_logits.py, compare_logits.py) on tiny random Llama / Qwen2 models, float32
on the CPU.

The checkpoint is written by this framework (`ModelWeights.save`, HF file layout), loaded by
`transformers.AutoModelForCausalLM`, and compared with (a) the framework's model oracle, which
every GPU kernel test uses as its reference, and (b) the engine's own path: prefill logits and
greedy tokens. RoPE variants: none, linear, llama3 (Llama 3.1 / 3.2 checkpoints) and YaRN.
"""

import pytest
import torch

transformers = pytest.importorskip("transformers")

from hetero_cp_ringattn_b200.config import preset  # noqa: E402
from hetero_cp_ringattn_b200.models import reference_model  # noqa: E402
from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine  # noqa: E402
from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights  # noqa: E402
from hetero_cp_ringattn_b200.ops import reference as ref  # noqa: E402

LLAMA3 = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 64}
YARN = {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 64}
LINEAR = {"rope_type": "linear", "factor": 2.0}
CASES = [("llama", False, None), ("llama-llama3", False, LLAMA3), ("llama-linear", False, LINEAR),
         ("qwen2", True, None), ("qwen2-yarn", True, YARN)]


def _model(tmp_path, name, bias, scaling):
    cfg = preset("tiny")
    cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads = 64, 4, 2
    cfg.intermediate_size, cfg.vocab_size = 128, 256
    cfg.attention_bias, cfg.rope_scaling, cfg.rope_theta = bias, scaling, 10000.0
    cfg.architectures = None
    cfg.max_position_embeddings = 256
    w = ModelWeights.random_init(cfg, seed=1, dtype=torch.float32, std=0.2)
    d = tmp_path / name
    w.save(str(d))
    hf = transformers.AutoModelForCausalLM.from_pretrained(str(d), dtype=torch.float32).eval()
    return cfg, w, hf


@pytest.mark.parametrize("name,bias,scaling", CASES)
def test_oracle_and_engine_match_transformers(tmp_path, name, bias, scaling):
    cfg, w, hf = _model(tmp_path, name, bias, scaling)
    assert type(hf).__name__ == ("Qwen2ForCausalLM" if bias else "LlamaForCausalLM")
    ids = torch.randint(0, cfg.vocab_size, (150,), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        want = hf(ids[None]).logits[0]
        gen = hf.generate(ids[None], max_new_tokens=5, do_sample=False,
                          attention_mask=torch.ones(1, ids.numel(), dtype=torch.long))
    assert (reference_model.forward(w, ids) - want).abs().max() < 2e-4
    eng = LlamaCPEngine(cfg, PreparedWeights.from_weights(w, dtype=torch.float32),
                        device=torch.device("cpu"), max_context=200)
    tok, logits = eng.prefill(1, ids, [ids.numel()], decode_horizon=6, return_logits=True)
    assert (logits - want[-1]).abs().max() < 2e-4
    toks = [int(tok)]
    for _ in range(4):
        tok = eng.decode_step([1], tok)
        toks.append(int(tok))
    assert toks == gen[0, ids.numel():].tolist()


@pytest.mark.parametrize("scaling", [LLAMA3, YARN, LINEAR])
def test_rope_frequencies_match_transformers(scaling):
    from transformers import LlamaConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    hcfg = LlamaConfig(hidden_size=2048, num_attention_heads=16, num_key_value_heads=4,
                       rope_theta=500000.0, max_position_embeddings=int(64 * scaling["factor"]),
                       rope_scaling=dict(scaling))
    inv_hf, amp_hf = ROPE_INIT_FUNCTIONS[scaling["rope_type"]](hcfg, "cpu")
    inv, amp = ref.rope_inv_freq(128, 500000.0, scaling)
    assert torch.allclose(inv.float(), inv_hf.float(), rtol=1e-5, atol=0)
    assert abs(amp - float(amp_hf)) < 1e-6


def test_rope_scaling_config_round_trip_and_unsupported_types():
    from hetero_cp_ringattn_b200.config import ModelConfig
    from hetero_cp_ringattn_b200.errors import RingError
    d = preset("llama-3.2-1b").to_hf_dict()
    d["rope_scaling"] = dict(LLAMA3)
    cfg = ModelConfig.from_dict(d)
    assert cfg.rope_scaling == LLAMA3 and cfg.to_hf_dict()["rope_scaling"] == LLAMA3
    d["rope_scaling"] = {"rope_type": "dynamic", "factor": 2.0}
    with pytest.raises(RingError, match="unsupported rope_scaling"):
        ModelConfig.from_dict(d)


def test_unsupported_checkpoint_options_fail_loudly(tmp_path, caplog):
    from hetero_cp_ringattn_b200.config import ModelConfig
    from hetero_cp_ringattn_b200.errors import RingError
    d = preset("llama-3.2-1b").to_hf_dict()
    with pytest.raises(RingError, match="mlp_bias"):
        ModelConfig.from_dict(dict(d, mlp_bias=True))
    cfg, w, _ = _model(tmp_path, "bias-check", False, None)
    w.tensors["model.layers.0.self_attn.o_proj.bias"] = torch.zeros(cfg.hidden_size)
    with pytest.raises(RingError, match="o_proj.bias"):
        w.validate()
    with caplog.at_level("WARNING"):
        ModelConfig.from_dict(dict(d, use_sliding_window=True, sliding_window=4096))
    assert "sliding" in caplog.text
