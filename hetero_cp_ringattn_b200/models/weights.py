"""HF-layout weights: safetensors loading/saving, random init, and the kernel-ready layout.

Parity: rust/src/model/weights.rs:17-224 (load every `*.safetensors` in a directory in sorted
order; F32/F16/BF16; HF names `model.embed_tokens.weight`,
`model.layers.{i}.self_attn.{q,k,v,o}_proj.{weight,bias}`, `mlp.{gate,up,down}_proj.weight`,
`{input,post_attention}_layernorm.weight`, `model.norm.weight`, `lm_head.weight` falling back to
the embedding when tied). Unlike the reference (which decodes through f32 and re-casts), tensors
are read straight into the compute dtype on the target device.

`PreparedWeights` builds the layouts the sm_100a kernels consume: one fused QKV weight (+ fused
bias for Qwen2), gate||up interleaved in 128-row blocks for the SwiGLU epilogue (intermediate
padded to a multiple of 128 with zeros), and the down projection padded to match.
"""

from __future__ import annotations

import dataclasses
import json
import os
from pathlib import Path
from typing import Dict, Optional

import torch

from ..config import ModelConfig
from ..errors import RingError
from ..ops.kernels import interleave_gate_up, pad_down_proj


def layer_names(i: int, bias: bool) -> list:
    p = f"model.layers.{i}."
    names = [p + f"self_attn.{x}_proj.weight" for x in "qkvo"]
    if bias:
        names += [p + f"self_attn.{x}_proj.bias" for x in "qkv"]
    names += [p + f"mlp.{x}_proj.weight" for x in ("gate", "up", "down")]
    names += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight"]
    return names


def expected_shapes(cfg: ModelConfig) -> Dict[str, tuple]:
    h, d = cfg.hidden_size, cfg.head_dim
    shapes = {"model.embed_tokens.weight": (cfg.vocab_size, h), "model.norm.weight": (h,)}
    if not cfg.tie_word_embeddings:
        shapes["lm_head.weight"] = (cfg.vocab_size, h)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        shapes[p + "self_attn.q_proj.weight"] = (cfg.num_heads * d, h)
        shapes[p + "self_attn.k_proj.weight"] = (cfg.kv_heads * d, h)
        shapes[p + "self_attn.v_proj.weight"] = (cfg.kv_heads * d, h)
        shapes[p + "self_attn.o_proj.weight"] = (h, cfg.num_heads * d)
        if cfg.attention_bias:
            shapes[p + "self_attn.q_proj.bias"] = (cfg.num_heads * d,)
            shapes[p + "self_attn.k_proj.bias"] = (cfg.kv_heads * d,)
            shapes[p + "self_attn.v_proj.bias"] = (cfg.kv_heads * d,)
        shapes[p + "mlp.gate_proj.weight"] = (cfg.intermediate_size, h)
        shapes[p + "mlp.up_proj.weight"] = (cfg.intermediate_size, h)
        shapes[p + "mlp.down_proj.weight"] = (h, cfg.intermediate_size)
        shapes[p + "input_layernorm.weight"] = (h,)
        shapes[p + "post_attention_layernorm.weight"] = (h,)
    return shapes


class ModelWeights:
    """Name -> tensor map in HF layout."""

    def __init__(self, cfg: ModelConfig, tensors: Dict[str, torch.Tensor]):
        self.cfg = cfg
        self.tensors = tensors

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.tensors[name]

    def lm_head(self) -> torch.Tensor:
        if "lm_head.weight" in self.tensors:
            return self.tensors["lm_head.weight"]
        return self.tensors["model.embed_tokens.weight"]

    def validate(self) -> None:
        # biases this engine does not apply must not be silently dropped (HF Llama puts one on
        # o_proj when attention_bias is set; mlp_bias puts them on the MLP)
        ignored = [n for n in self.tensors if n.endswith(("o_proj.bias", "gate_proj.bias",
                                                           "up_proj.bias", "down_proj.bias"))]
        if ignored:
            raise RingError(f"checkpoint has {ignored[0]} (and {len(ignored) - 1} more): biases on "
                            "the output projection or the MLP are not supported")
        for name, shape in expected_shapes(self.cfg).items():
            if name not in self.tensors:
                raise RingError(f"missing weight {name}")
            if tuple(self.tensors[name].shape) != tuple(shape):
                raise RingError(f"weight {name} has shape {tuple(self.tensors[name].shape)}, "
                                f"expected {shape}")

    # ------------------------------------------------------------------ io
    @classmethod
    def from_dir(cls, model_dir: str | Path, device="cpu", dtype=torch.bfloat16,
                 cfg: Optional[ModelConfig] = None) -> "ModelWeights":
        from safetensors.torch import load_file
        model_dir = Path(model_dir)
        cfg = cfg or ModelConfig.from_file(model_dir / "config.json")
        files = sorted(model_dir.glob("*.safetensors"))
        if not files:
            raise RingError(f"no *.safetensors files in {model_dir}")
        tensors: Dict[str, torch.Tensor] = {}
        dev = str(device)
        for f in files:
            for k, v in load_file(str(f), device=dev).items():
                tensors[k] = v.to(dtype) if v.is_floating_point() else v
        w = cls(cfg, tensors)
        w.validate()
        return w

    def save(self, model_dir: str | Path, shard_bytes: int = 4 << 30) -> None:
        from safetensors.torch import save_file
        model_dir = Path(model_dir)
        model_dir.mkdir(parents=True, exist_ok=True)
        with open(model_dir / "config.json", "w") as f:
            json.dump(self.cfg.to_hf_dict(), f, indent=2)
        # HF layout: one `model.safetensors`, or `model-0000i-of-0000n.safetensors` shards plus
        # `model.safetensors.index.json` (transformers and this loader read either)
        shards: list = [{}]
        size = 0
        total = 0
        for n in sorted(self.tensors):
            t = self.tensors[n].detach().contiguous().cpu()
            nb = t.numel() * t.element_size()
            if size + nb > shard_bytes and shards[-1]:
                shards.append({})
                size = 0
            shards[-1][n] = t
            size += nb
            total += nb
        if len(shards) == 1:
            save_file(shards[0], str(model_dir / "model.safetensors"), metadata={"format": "pt"})
            return
        weight_map = {}
        for i, shard in enumerate(shards):
            fname = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
            save_file(shard, str(model_dir / fname), metadata={"format": "pt"})
            weight_map.update({n: fname for n in shard})
        with open(model_dir / "model.safetensors.index.json", "w") as f:
            json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)

    @classmethod
    def random_init(cls, cfg: ModelConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                    std: float = 0.02) -> "ModelWeights":
        """N(0, std) projections/embeddings, unit norms (zero biases drawn N(0, std) too)."""
        g = torch.Generator(device=str(device) if str(device).startswith("cuda") else "cpu")
        g.manual_seed(seed)
        tensors = {}
        for name, shape in expected_shapes(cfg).items():
            if name.endswith("norm.weight"):
                t = torch.ones(shape, dtype=dtype, device=device)
            else:
                t = torch.empty(shape, dtype=torch.float32, device=device)
                t.normal_(0.0, std, generator=g)
                t = t.to(dtype)
            tensors[name] = t
        return cls(cfg, tensors)


@dataclasses.dataclass
class LayerWeights:
    in_norm: torch.Tensor
    wqkv: torch.Tensor
    bqkv: Optional[torch.Tensor]
    wo: torch.Tensor
    post_norm: torch.Tensor
    wgu: torch.Tensor        # interleaved gate||up, [2 * I_pad, hidden]
    wd: torch.Tensor         # [hidden, I_pad]


@dataclasses.dataclass
class PreparedWeights:
    cfg: ModelConfig
    embed: torch.Tensor
    final_norm: torch.Tensor
    lm_head: torch.Tensor
    layers: list
    intermediate_padded: int

    @classmethod
    def from_weights(cls, w: ModelWeights, device=None, dtype=torch.bfloat16,
                     free_source: bool = False) -> "PreparedWeights":
        cfg = w.cfg
        dev = device if device is not None else w["model.embed_tokens.weight"].device

        def get(name):
            t = w[name].to(device=dev, dtype=dtype)
            if free_source:
                w.tensors[name] = t
            return t

        layers = []
        ip = None
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            wq, wk, wv = (get(p + f"self_attn.{x}_proj.weight") for x in "qkv")
            wqkv = torch.cat([wq, wk, wv]).contiguous()
            bqkv = None
            if cfg.attention_bias:
                bqkv = torch.cat([get(p + f"self_attn.{x}_proj.bias") for x in "qkv"]).contiguous()
            wgu = interleave_gate_up(get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight"))
            wd = pad_down_proj(get(p + "mlp.down_proj.weight"))
            ip = wd.shape[1]
            layers.append(LayerWeights(
                in_norm=get(p + "input_layernorm.weight").contiguous(),
                wqkv=wqkv, bqkv=bqkv, wo=get(p + "self_attn.o_proj.weight").contiguous(),
                post_norm=get(p + "post_attention_layernorm.weight").contiguous(),
                wgu=wgu, wd=wd))
            if free_source:
                for n in layer_names(i, cfg.attention_bias):
                    w.tensors.pop(n, None)
        embed = get("model.embed_tokens.weight").contiguous()
        lm = embed if cfg.tie_word_embeddings or "lm_head.weight" not in w.tensors else get("lm_head.weight").contiguous()
        return cls(cfg=cfg, embed=embed, final_norm=get("model.norm.weight").contiguous(), lm_head=lm,
                   layers=layers, intermediate_padded=ip or cfg.intermediate_size)

    @classmethod
    def random(cls, cfg: ModelConfig, seed: int = 0, device="cuda", dtype=torch.bfloat16,
               std: float = 0.02) -> "PreparedWeights":
        """Random-init directly in the kernel layout (no HF copy kept; for large benchmarks)."""
        g = torch.Generator(device=str(device) if str(device).startswith("cuda") else "cpu")
        g.manual_seed(seed)

        def rnd(*shape):
            t = torch.empty(*shape, dtype=torch.float32, device=device)
            t.normal_(0.0, std, generator=g)
            return t.to(dtype)

        h, d = cfg.hidden_size, cfg.head_dim
        ip = -(-cfg.intermediate_size // 128) * 128
        layers = []
        for _ in range(cfg.num_layers):
            gate = rnd(cfg.intermediate_size, h)
            up = rnd(cfg.intermediate_size, h)
            layers.append(LayerWeights(
                in_norm=torch.ones(h, dtype=dtype, device=device),
                wqkv=rnd(cfg.qkv_size, h),
                bqkv=rnd(cfg.qkv_size) if cfg.attention_bias else None,
                wo=rnd(h, cfg.num_heads * d),
                post_norm=torch.ones(h, dtype=dtype, device=device),
                wgu=interleave_gate_up(gate, up),
                wd=pad_down_proj(rnd(h, cfg.intermediate_size))))
            del gate, up
        embed = rnd(cfg.vocab_size, h)
        lm = embed if cfg.tie_word_embeddings else rnd(cfg.vocab_size, h)
        return cls(cfg=cfg, embed=embed, final_norm=torch.ones(h, dtype=dtype, device=device),
                   lm_head=lm, layers=layers, intermediate_padded=ip)


def model_dir_or_random(cfg: ModelConfig, model_dir: Optional[str], seed: int, device,
                        dtype=torch.bfloat16) -> ModelWeights:
    if model_dir and os.path.isdir(model_dir):
        return ModelWeights.from_dir(model_dir, device=device, dtype=dtype, cfg=cfg)
    return ModelWeights.random_init(cfg, seed=seed, device=device, dtype=dtype)
