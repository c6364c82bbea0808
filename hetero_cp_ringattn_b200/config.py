"""Model config (HF `config.json`), ring/domain config JSON and environment knobs.

Parity:
  * `ModelConfig` mirrors rust/src/model/config.rs:27-120 (field names, HF aliases, defaults:
    rope_theta 1e4, rms_norm_eps 1e-6, hidden_act "silu", eos single-or-list, sliding window
    and partial_rotary_factor parsed but unused).
  * `RingAttnConfig` / `DomainConfig` mirror the JSON schema of config/minimal_2domain_ring.json
    and include/hcp_ringattn/core/ringattn_protocol.h:45-60; validation follows
    rust/src/smoke/reference_algo.rs:92-116 (chunks sum to the global length, positive sizes).
  * `EnvConfig` reads the HCP_* variables of the reference (ring.rs:71-75,160-166,
    coordinator.rs:2735, cache.rs:421-440, protocol.rs:348-353); transport-specific knobs
    become HCP_P2P_* (spin budget for device-side peer waits).
"""

from __future__ import annotations

import dataclasses
import json
import os
from pathlib import Path
from typing import Any, Optional, Sequence

from .errors import InvalidChunkSum, InvalidDomain, RingError


@dataclasses.dataclass
class ModelConfig:
    hidden_size: int
    num_layers: int
    num_heads: int
    intermediate_size: int
    vocab_size: int
    num_kv_heads: Optional[int] = None
    head_dim_override: Optional[int] = None
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = False
    torch_dtype: Optional[str] = None
    hidden_act: str = "silu"
    max_position_embeddings: Optional[int] = None
    attention_bias: bool = False          # Qwen2 has q/k/v bias
    bos_token_id: Optional[int] = None
    eos_token_id: Optional[list] = None
    architectures: Optional[list] = None
    sliding_window: Optional[int] = None  # parsed, unused (as in the reference)
    use_sliding_window: Optional[bool] = None
    partial_rotary_factor: float = 1.0    # parsed, unused
    rope_scaling: Optional[dict] = None   # HF rope_scaling: linear / llama3 / yarn frequencies
    mlp_bias: bool = False                # HF Llama option; biases on the MLP are not supported
    name: str = "custom"

    # ------------------------------------------------------------------ derived
    @property
    def kv_heads(self) -> int:
        return self.num_kv_heads if self.num_kv_heads else self.num_heads

    @property
    def head_dim(self) -> int:
        if self.head_dim_override:
            return self.head_dim_override
        return self.hidden_size // self.num_heads

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def is_qwen2(self) -> bool:
        arch = self.architectures or []
        return self.attention_bias or any("Qwen2" in a for a in arch)

    def kv_bytes_per_token_per_layer(self, elem_bytes: int = 2) -> int:
        return 2 * self.kv_heads * self.head_dim * elem_bytes

    def num_params(self) -> int:
        h, i, v = self.hidden_size, self.intermediate_size, self.vocab_size
        per_layer = h * self.qkv_size + self.q_size * h + 3 * h * i + 2 * h
        if self.attention_bias:
            per_layer += self.qkv_size
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_layers * per_layer + emb + h

    def validate(self) -> None:
        if self.num_heads % self.kv_heads:
            raise RingError(f"num_heads {self.num_heads} not divisible by kv heads {self.kv_heads}")
        if self.head_dim % 2:
            raise RingError("head_dim must be even for rotate-half RoPE")
        if self.hidden_act not in ("silu", "swish"):
            raise RingError(f"unsupported hidden_act {self.hidden_act}")
        if self.mlp_bias:
            raise RingError("mlp_bias=true (biases on the MLP projections) is not supported")
        if self.rope_scaling:
            kind = self.rope_scaling.get("rope_type", self.rope_scaling.get("type", "default"))
            if kind not in ("default", "linear", "llama3", "yarn"):
                raise RingError(f"unsupported rope_scaling type {kind!r} (default, linear, llama3, "
                                "yarn)")

    # ------------------------------------------------------------------ io
    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        def pick(*names, default=None):
            for n in names:
                if n in d and d[n] is not None:
                    return d[n]
            return default

        eos = d.get("eos_token_id")
        if eos is not None and not isinstance(eos, list):
            eos = [eos]
        arch = d.get("architectures")
        bias = bool(d.get("attention_bias", False)) or any("Qwen2" in a for a in (arch or []))
        cfg = cls(
            hidden_size=int(d["hidden_size"]),
            num_layers=int(pick("num_layers", "num_hidden_layers")),
            num_heads=int(pick("num_heads", "num_attention_heads")),
            intermediate_size=int(d["intermediate_size"]),
            vocab_size=int(d["vocab_size"]),
            num_kv_heads=pick("num_kv_heads", "num_key_value_heads"),
            head_dim_override=d.get("head_dim"),
            rope_theta=float(d.get("rope_theta", 10000.0)),
            rms_norm_eps=float(d.get("rms_norm_eps", 1e-6)),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            torch_dtype=d.get("torch_dtype"),
            hidden_act=d.get("hidden_act", "silu"),
            max_position_embeddings=d.get("max_position_embeddings"),
            attention_bias=bias,
            bos_token_id=d.get("bos_token_id"),
            eos_token_id=eos,
            architectures=arch,
            sliding_window=d.get("sliding_window"),
            use_sliding_window=d.get("use_sliding_window"),
            partial_rotary_factor=float(d.get("partial_rotary_factor", 1.0)),
            rope_scaling=dict(d["rope_scaling"]) if d.get("rope_scaling") else None,
            mlp_bias=bool(d.get("mlp_bias", False)),
            name=d.get("_name_or_path", d.get("name", "custom")),
        )
        if cfg.num_kv_heads is not None:
            cfg.num_kv_heads = int(cfg.num_kv_heads)
        if cfg.use_sliding_window and cfg.sliding_window and cfg.max_position_embeddings and \
                cfg.sliding_window < cfg.max_position_embeddings:
            import logging
            logging.getLogger("hcp.config").warning(
                "use_sliding_window is set (window %d): this engine attends over the full "
                "context, so positions beyond the window differ from a sliding-window model",
                cfg.sliding_window)
        cfg.validate()
        return cfg

    @classmethod
    def from_file(cls, path: str | Path) -> "ModelConfig":
        with open(path) as f:
            return cls.from_dict(json.load(f))

    def to_hf_dict(self) -> dict:
        arch = self.architectures or (["Qwen2ForCausalLM"] if self.attention_bias else ["LlamaForCausalLM"])
        d = {
            "architectures": arch,
            "model_type": "qwen2" if self.attention_bias else "llama",
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_layers,
            "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.kv_heads,
            "intermediate_size": self.intermediate_size,
            "vocab_size": self.vocab_size,
            "rope_theta": self.rope_theta,
            "rms_norm_eps": self.rms_norm_eps,
            "tie_word_embeddings": self.tie_word_embeddings,
            "torch_dtype": self.torch_dtype or "bfloat16",
            "hidden_act": self.hidden_act,
            "max_position_embeddings": self.max_position_embeddings,
            "attention_bias": self.attention_bias,
            "bos_token_id": self.bos_token_id,
            "eos_token_id": self.eos_token_id,
        }
        if self.head_dim_override:
            d["head_dim"] = self.head_dim_override
        if self.rope_scaling:
            d["rope_scaling"] = dict(self.rope_scaling)
        return d


def _preset(**kw) -> ModelConfig:
    cfg = ModelConfig(**kw)
    cfg.validate()
    return cfg


# RoPE frequency scaling of the Llama 3.1 / 3.2 releases (their config.json `rope_scaling`)
LLAMA3_ROPE_SCALING = {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                       "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}

# Shapes named by the benchmark configs (random-init weights of these architectures).
PRESETS = {
    "llama-3.2-1b": dict(name="llama-3.2-1b", hidden_size=2048, num_layers=16, num_heads=32,
                         num_kv_heads=8, intermediate_size=8192, vocab_size=128256,
                         rope_theta=500000.0, rms_norm_eps=1e-5, tie_word_embeddings=True,
                         max_position_embeddings=131072, torch_dtype="bfloat16",
                         rope_scaling=dict(LLAMA3_ROPE_SCALING),
                         architectures=["LlamaForCausalLM"], eos_token_id=[128001]),
    "qwen2.5-3b": dict(name="qwen2.5-3b", hidden_size=2048, num_layers=36, num_heads=16,
                       num_kv_heads=2, intermediate_size=11008, vocab_size=151936,
                       rope_theta=1000000.0, rms_norm_eps=1e-6, tie_word_embeddings=True,
                       attention_bias=True, max_position_embeddings=131072,
                       torch_dtype="bfloat16", architectures=["Qwen2ForCausalLM"],
                       eos_token_id=[151643]),
    "llama-3-8b": dict(name="llama-3-8b", hidden_size=4096, num_layers=32, num_heads=32,
                       num_kv_heads=8, intermediate_size=14336, vocab_size=128256,
                       rope_theta=500000.0, rms_norm_eps=1e-5, tie_word_embeddings=False,
                       # the 128k-prompt benchmark decodes 256 tokens past position 131072
                       max_position_embeddings=262144, torch_dtype="bfloat16",
                       architectures=["LlamaForCausalLM"], eos_token_id=[128001]),
    # Further shapes of the model families the reference runs (its validation and serving runs
    # use Qwen2-0.5B and Qwen2.5-7B): GQA groups of 7 and 3 query heads per KV head.
    "qwen2-0.5b": dict(name="qwen2-0.5b", hidden_size=896, num_layers=24, num_heads=14,
                       num_kv_heads=2, intermediate_size=4864, vocab_size=151936,
                       rope_theta=1000000.0, rms_norm_eps=1e-6, tie_word_embeddings=True,
                       attention_bias=True, max_position_embeddings=131072,
                       torch_dtype="bfloat16", architectures=["Qwen2ForCausalLM"],
                       eos_token_id=[151643]),
    "qwen2.5-7b": dict(name="qwen2.5-7b", hidden_size=3584, num_layers=28, num_heads=28,
                       num_kv_heads=4, intermediate_size=18944, vocab_size=152064,
                       rope_theta=1000000.0, rms_norm_eps=1e-6, tie_word_embeddings=False,
                       attention_bias=True, max_position_embeddings=131072,
                       torch_dtype="bfloat16", architectures=["Qwen2ForCausalLM"],
                       eos_token_id=[151643]),
    "llama-3.2-3b": dict(name="llama-3.2-3b", hidden_size=3072, num_layers=28, num_heads=24,
                         num_kv_heads=8, intermediate_size=8192, vocab_size=128256,
                         rope_theta=500000.0, rms_norm_eps=1e-5, tie_word_embeddings=True,
                         max_position_embeddings=131072, torch_dtype="bfloat16",
                         rope_scaling=dict(LLAMA3_ROPE_SCALING),
                         architectures=["LlamaForCausalLM"], eos_token_id=[128001]),
    # Tiny shapes used by tests (the reference's synthetic model is hidden 32, 2 layers, GQA 4/1,
    # vocab 100: rust/src/model/model.rs:676-740).
    "tiny": dict(name="tiny", hidden_size=32, num_layers=2, num_heads=4, num_kv_heads=1,
                 intermediate_size=64, vocab_size=100, rope_theta=10000.0, rms_norm_eps=1e-6,
                 max_position_embeddings=4096, torch_dtype="float32"),
    "tiny-gpu": dict(name="tiny-gpu", hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=2,
                     intermediate_size=1024, vocab_size=1024, rope_theta=10000.0,
                     rms_norm_eps=1e-6, max_position_embeddings=65536, torch_dtype="bfloat16"),
    "tiny-qwen-gpu": dict(name="tiny-qwen-gpu", hidden_size=512, num_layers=2, num_heads=4,
                          num_kv_heads=2, intermediate_size=1024, vocab_size=1024,
                          rope_theta=1000000.0, rms_norm_eps=1e-6, attention_bias=True,
                          max_position_embeddings=65536, torch_dtype="bfloat16"),
}


def preset(name: str) -> ModelConfig:
    if name not in PRESETS:
        raise RingError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return _preset(**PRESETS[name])


# --------------------------------------------------------------------------- ring/domain config
@dataclasses.dataclass
class DomainConfig:
    domain_id: str
    seq_chunk_len: int
    block_size: int
    host: str = "127.0.0.1"
    port: int = 0
    device: str = "cuda"


@dataclasses.dataclass
class RingAttnConfig:
    global_seq_len: int
    num_heads: int
    head_dim: int
    domains: list
    dtype: str = "float32"
    num_kv_heads: Optional[int] = None

    def validate(self) -> None:
        for d in self.domains:
            if not d.domain_id or d.seq_chunk_len <= 0 or d.block_size <= 0:
                raise InvalidDomain(d.domain_id)
        total = sum(d.seq_chunk_len for d in self.domains)
        if total != self.global_seq_len:
            raise InvalidChunkSum(total, self.global_seq_len)
        if self.num_heads <= 0 or self.head_dim <= 0:
            raise RingError("num_heads and head_dim must be positive")

    @property
    def chunks(self) -> list:
        return [d.seq_chunk_len for d in self.domains]

    @property
    def block_sizes(self) -> list:
        return [d.block_size for d in self.domains]

    @classmethod
    def from_dict(cls, d: dict) -> "RingAttnConfig":
        doms = [DomainConfig(domain_id=str(x["domain_id"]), seq_chunk_len=int(x["seq_chunk_len"]),
                             block_size=int(x["block_size"]), host=x.get("host", "127.0.0.1"),
                             port=int(x.get("port", 0)), device=x.get("device", "cuda"))
                for x in d["domains"]]
        cfg = cls(global_seq_len=int(d["global_seq_len"]), num_heads=int(d["num_heads"]),
                  head_dim=int(d["head_dim"]), domains=doms, dtype=d.get("dtype", "float32"),
                  num_kv_heads=d.get("num_kv_heads"))
        cfg.validate()
        return cfg

    @classmethod
    def from_file(cls, path: str | Path) -> "RingAttnConfig":
        with open(path) as f:
            return cls.from_dict(json.load(f))

    def to_dict(self) -> dict:
        return {
            "global_seq_len": self.global_seq_len, "num_heads": self.num_heads,
            "head_dim": self.head_dim, "dtype": self.dtype,
            **({"num_kv_heads": self.num_kv_heads} if self.num_kv_heads else {}),
            "domains": [dataclasses.asdict(x) for x in self.domains],
        }


# --------------------------------------------------------------------------- environment
def _env_bool(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    if v is None:
        return default
    return v.strip().lower() not in ("0", "false", "no", "off", "")


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    try:
        return int(v) if v is not None and v.strip() else default
    except ValueError:
        return default


def _env_choice(name: str, default: str, choices) -> str:
    v = os.environ.get(name)
    if v is None or not v.strip():
        return default
    v = v.strip().lower()
    if v not in choices:
        raise ValueError(f"{name}={v!r}: expected one of {', '.join(choices)}")
    return v


@dataclasses.dataclass
class EnvConfig:
    perf_log: Optional[str] = None          # HCP_PERF_LOG: JSONL perf events
    micro_kv_block_size: int = 0            # HCP_MICRO_KV_BLOCK_SIZE: host-path ring fold block
                                            # (0 -> 128, the CUDA kernels' fixed KV tile)
    disable_overlap: Optional[bool] = None  # HCP_DISABLE_OVERLAP=1: serial ring (push every
                                            # rank's KV, wait for all, then attend); =0: the
                                            # overlapped in-kernel ring; unset: chosen per world
                                            # size by the engine
    decode_ring: bool = True                # HCP_RING_DECODE_RING=0: legacy KV re-send decode
                                            # (host path; CUDA ranks warn and keep the exchange)
    decode_sd: bool = True                  # HCP_RING_DECODE_SD: capacity-scheduled KV growth;
                                            # 0 -> Q-ring placement, position % N
    kv_block_table: bool = True             # HCP_KV_CACHE_BLOCK_TABLE (paged arena is always used)
    kv_block_size: int = 256                # HCP_KV_CACHE_BLOCK_SIZE: tokens per KV page
                                            # (engine default; CUDA needs a multiple of 128)
    control_timeout_s: int = 600            # HCP_QUIC_TIMEOUT_SECS: process-group timeout of serve
    p2p_spin_budget_ms: int = 5000          # HCP_P2P_SPIN_BUDGET_MS: device-side peer-wait limit
    device: Optional[str] = None            # HCP_TORCH_DEVICE / HCP_TCH_DEVICE
    nvtx: bool = False                      # HCP_NVTX: NVTX ranges per prefill layer / decode step
    decode_combine: str = "launch"          # HCP_DECODE_COMBINE: where several ranks' decode
                                            # (O, LSE) partials are waited for and combined:
                                            # "launch" (a combine kernel of its own), "gemv" (the
                                            # output projection's prologue), "attn" (the attention
                                            # kernel's last CTA per (row, KV head); also
                                            # HCP_DECODE_KERNEL_COMBINE=1). Measured on 2 B200s:
                                            # launch 1.156, gemv 1.231, attn 1.285 ms per token
    fused_qkv: Optional[bool] = None        # HCP_FUSED_QKV: the projection GEMM's epilogue does
                                            # RoPE + the K/V writes (default on; 0: GEMM + a
                                            # separate RoPE / K/V kernel)
    decode_prefetch: int = 0                # HCP_DECODE_PREFETCH: decode kernels pull later
                                            # kernels' weights into L2 while they run (1: bulk
                                            # prefetches of every GEMV's weights, 2: the same
                                            # with per-line prefetches, 3: per-line, only the
                                            # output and QKV projections' weights). Measured on
                                            # B200 (Llama-3.2-1B, 32k, ms per token): off 1.09,
                                            # 1: 1.19-1.20, 2: 1.20-1.22, 3: within the noise
    decode_splits: int = 0                  # HCP_DECODE_SPLITS: at most this many KV splits per
                                            # (row, KV head) in decode attention (0: one wave)
    decode_chain: bool = False              # HCP_DECODE_CHAIN=1: the decode GEMVs between two
                                            # attentions (output projection, gate/up, down, next
                                            # QKV or LM head) as one cooperative chain kernel
                                            # with grid barriers instead of four launches.
                                            # Measured on B200 (Llama-3.2-1B, 32k, ms per token):
                                            # batch 1 1.18-1.27 against 1.09-1.12 for the four
                                            # launches, batch 4 2.50-2.61 against 1.96-2.09
    split_lm_head: bool = True              # HCP_SPLIT_LM_HEAD=0: every rank runs the whole LM
                                            # head in greedy decode steps (default: each rank
                                            # takes 1/N of the vocabulary and the ranks exchange
                                            # their packed argmax over NVLink)

    @classmethod
    def from_env(cls) -> "EnvConfig":
        return cls(
            perf_log=os.environ.get("HCP_PERF_LOG") or None,
            micro_kv_block_size=_env_int("HCP_MICRO_KV_BLOCK_SIZE", 0),
            disable_overlap=(_env_bool("HCP_DISABLE_OVERLAP", False)
                             if os.environ.get("HCP_DISABLE_OVERLAP") else None),
            decode_ring=_env_bool("HCP_RING_DECODE_RING", True),
            decode_sd=_env_bool("HCP_RING_DECODE_SD", True),
            kv_block_table=_env_bool("HCP_KV_CACHE_BLOCK_TABLE", True),
            kv_block_size=_env_int("HCP_KV_CACHE_BLOCK_SIZE", 256),
            control_timeout_s=_env_int("HCP_QUIC_TIMEOUT_SECS", 600),
            p2p_spin_budget_ms=_env_int("HCP_P2P_SPIN_BUDGET_MS", 5000),
            device=os.environ.get("HCP_TORCH_DEVICE") or os.environ.get("HCP_TCH_DEVICE") or None,
            nvtx=_env_bool("HCP_NVTX", False),
            decode_combine=("attn" if _env_bool("HCP_DECODE_KERNEL_COMBINE", False)
                            else _env_choice("HCP_DECODE_COMBINE", "launch", ("launch", "gemv", "attn"))),
            fused_qkv=(_env_bool("HCP_FUSED_QKV", True) if os.environ.get("HCP_FUSED_QKV") else None),
            split_lm_head=_env_bool("HCP_SPLIT_LM_HEAD", True),
            decode_chain=_env_bool("HCP_DECODE_CHAIN", False),
            decode_prefetch=_env_int("HCP_DECODE_PREFETCH", 0),
            decode_splits=_env_int("HCP_DECODE_SPLITS", 0),
        )


def parse_ratio(spec: str | Sequence[int]) -> list:
    """Parse an integer ratio override such as "5:5:1" into [5, 5, 1]."""
    if not isinstance(spec, str):
        return [int(x) for x in spec]
    parts = [p for p in spec.replace(",", ":").split(":") if p.strip()]
    vals = [int(p) for p in parts]
    if not vals or any(v < 0 for v in vals) or sum(vals) == 0:
        raise RingError(f"invalid ratio {spec!r}")
    return vals


def as_jsonable(obj: Any) -> Any:
    if dataclasses.is_dataclass(obj):
        return dataclasses.asdict(obj)
    return obj
