"""Dense single-device Llama/Qwen2 forward in plain PyTorch (fp32 by default): the logits oracle.

Parity: rust/src/model/model.rs:195-343 (embedding -> decoder layers -> final norm -> LM head),
rust/src/model/layers/mod.rs:59-90 (pre-norm, attention, residual, pre-norm, MLP, residual),
rust/src/model/layers/attention.rs:81-171 (QKV (+bias), RoPE at absolute positions, dense
causal softmax attention, O projection) and mlp.rs:42-67 (SwiGLU). Used only by tests and the
logits-export tool, never on the GPU hot path.
"""

from __future__ import annotations

from typing import Callable, Dict, Optional

import torch

from ..ops import reference as ref
from .weights import ModelWeights


@torch.no_grad()
def forward(w: ModelWeights, ids: torch.Tensor, positions: Optional[torch.Tensor] = None,
            dtype=torch.float32, last_only: bool = False,
            tap: Optional[Callable[[str, torch.Tensor], None]] = None,
            inject: Optional[Dict[str, torch.Tensor]] = None) -> torch.Tensor:
    """Full causal forward over `ids` [L]; returns logits [L, vocab] (or [1, vocab]).

    `tap(name, tensor)` receives the intermediates the debug exports write (embedding_output,
    layer_{i}_input_norm, {q,k,v}_proj_layer_{i} before RoPE, prefill_{k,v}_layer_{i} as cached,
    layer_{i}_post_attn, layer_{i} (= post-MLP hidden), final_norm); `inject` replaces
    q_proj_layer_{i} / k_proj_layer_{i} ([L, heads * D]) before RoPE."""
    cfg = w.cfg
    tap = tap or (lambda name, t: None)
    inject = inject or {}
    dev = ids.device
    L = ids.numel()
    pos = positions if positions is not None else torch.arange(L, device=dev)
    H, Hkv, D = cfg.num_heads, cfg.kv_heads, cfg.head_dim

    def t(name):
        return w[name].to(device=dev, dtype=dtype)

    x = t("model.embed_tokens.weight")[ids.long()]
    tap("embedding_output", x)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        h = ref.rmsnorm(x, t(p + "input_layernorm.weight"), cfg.rms_norm_eps)
        tap(f"layer_{i}_input_norm", h)
        q = ref.linear(h, t(p + "self_attn.q_proj.weight"),
                       t(p + "self_attn.q_proj.bias") if cfg.attention_bias else None)
        k = ref.linear(h, t(p + "self_attn.k_proj.weight"),
                       t(p + "self_attn.k_proj.bias") if cfg.attention_bias else None)
        v = ref.linear(h, t(p + "self_attn.v_proj.weight"),
                       t(p + "self_attn.v_proj.bias") if cfg.attention_bias else None)
        q = inject.get(f"q_proj_layer_{i}", q).to(device=dev, dtype=dtype)
        k = inject.get(f"k_proj_layer_{i}", k).to(device=dev, dtype=dtype)
        tap(f"q_proj_layer_{i}", q)
        tap(f"k_proj_layer_{i}", k)
        tap(f"v_proj_layer_{i}", v)
        q = ref.apply_rope(q.reshape(L, H, D), pos, cfg.rope_theta, cfg.rope_scaling)
        k = ref.apply_rope(k.reshape(L, Hkv, D), pos, cfg.rope_theta, cfg.rope_scaling)
        tap(f"prefill_k_layer_{i}", k.transpose(0, 1).unsqueeze(0))
        tap(f"prefill_v_layer_{i}", v.view(L, Hkv, D).transpose(0, 1).unsqueeze(0))
        # queries in chunks whose [H, chunk, L] score matrix stays near 4 GB (long contexts)
        chunk = max(1, (1 << 30) // max(1, H * L))
        o, _ = ref.full_attention(q, k, v.view(L, Hkv, D), pos, pos, causal=True, q_chunk=chunk)
        x = x + ref.linear(o.reshape(L, H * D), t(p + "self_attn.o_proj.weight"))
        tap(f"layer_{i}_post_attn", x)
        h = ref.rmsnorm(x, t(p + "post_attention_layernorm.weight"), cfg.rms_norm_eps)
        g = ref.linear(h, t(p + "mlp.gate_proj.weight"))
        u = ref.linear(h, t(p + "mlp.up_proj.weight"))
        x = x + ref.linear(ref.swiglu(g, u), t(p + "mlp.down_proj.weight"))
        tap(f"layer_{i}", x)
    if last_only:
        x = x[-1:]
    x = ref.rmsnorm(x, t("model.norm.weight"), cfg.rms_norm_eps)
    tap("final_norm", x)
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
