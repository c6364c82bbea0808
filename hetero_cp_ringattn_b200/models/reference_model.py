"""Dense single-device Llama/Qwen2 forward in plain PyTorch (fp32 by default): the logits oracle.

Parity: rust/src/model/model.rs:195-343 (embedding -> decoder layers -> final norm -> LM head),
rust/src/model/layers/mod.rs:59-90 (pre-norm, attention, residual, pre-norm, MLP, residual),
rust/src/model/layers/attention.rs:81-171 (QKV (+bias), RoPE at absolute positions, dense
causal softmax attention, O projection) and mlp.rs:42-67 (SwiGLU). Used only by tests and the
logits-export tool, never on the GPU hot path.
"""

from __future__ import annotations

from typing import Optional

import torch

from ..ops import reference as ref
from .weights import ModelWeights


@torch.no_grad()
def forward(w: ModelWeights, ids: torch.Tensor, positions: Optional[torch.Tensor] = None,
            dtype=torch.float32, last_only: bool = False) -> torch.Tensor:
    """Full causal forward over `ids` [L]; returns logits [L, vocab] (or [1, vocab])."""
    cfg = w.cfg
    dev = ids.device
    L = ids.numel()
    pos = positions if positions is not None else torch.arange(L, device=dev)
    H, Hkv, D = cfg.num_heads, cfg.kv_heads, cfg.head_dim

    def t(name):
        return w[name].to(device=dev, dtype=dtype)

    x = t("model.embed_tokens.weight")[ids.long()]
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        h = ref.rmsnorm(x, t(p + "input_layernorm.weight"), cfg.rms_norm_eps)
        q = ref.linear(h, t(p + "self_attn.q_proj.weight"),
                       t(p + "self_attn.q_proj.bias") if cfg.attention_bias else None)
        k = ref.linear(h, t(p + "self_attn.k_proj.weight"),
                       t(p + "self_attn.k_proj.bias") if cfg.attention_bias else None)
        v = ref.linear(h, t(p + "self_attn.v_proj.weight"),
                       t(p + "self_attn.v_proj.bias") if cfg.attention_bias else None)
        q = ref.apply_rope(q.view(L, H, D), pos, cfg.rope_theta)
        k = ref.apply_rope(k.view(L, Hkv, D), pos, cfg.rope_theta)
        o, _ = ref.full_attention(q, k, v.view(L, Hkv, D), pos, pos, causal=True)
        x = x + ref.linear(o.reshape(L, H * D), t(p + "self_attn.o_proj.weight"))
        h = ref.rmsnorm(x, t(p + "post_attention_layernorm.weight"), cfg.rms_norm_eps)
        g = ref.linear(h, t(p + "mlp.gate_proj.weight"))
        u = ref.linear(h, t(p + "mlp.up_proj.weight"))
        x = x + ref.linear(ref.swiglu(g, u), t(p + "mlp.down_proj.weight"))
    if last_only:
        x = x[-1:]
    x = ref.rmsnorm(x, t("model.norm.weight"), cfg.rms_norm_eps)
    return ref.linear(x, w.lm_head().to(device=dev, dtype=dtype))


@torch.no_grad()
def greedy_generate(w: ModelWeights, prompt: torch.Tensor, steps: int, dtype=torch.float32):
    """Greedy decoding by full recomputation (small models only). Returns (tokens, logits list)."""
    ids = prompt.clone().long()
    out, logits_all = [], []
    for _ in range(steps + 1):
        logits = forward(w, ids, dtype=dtype, last_only=True)[0]
        logits_all.append(logits)
        tok = int(torch.argmax(logits))
        out.append(tok)
        ids = torch.cat([ids, torch.tensor([tok], device=ids.device)])
    return out[:steps + 1], logits_all
