"""Debug exports for parity work against other implementations (HF transformers, the reference).

`hcp infer --export-hidden-states DIR`: after the prefill of the prompt, the per-layer K/V as
cached (prefill_{k,v}_layer_{i}.bin, [1, Hkv, L, D], K after RoPE), then the first decode step's
hidden state after every layer (layer_{i}.bin, [1, 1, hidden]), its final-norm output
(final_norm.bin) and its logits (logits.bin in the logits-export layout with one row).
Parity: rust/src/infer.rs:234-373 and rust/src/model/model.rs:420-470.

`hcp infer --prefill-debug DIR [--qk-inject DIR]`: the layer-0 intermediates of the prefill
(embedding_output, layer_0_input_norm, {q,k,v}_proj_layer_0 before RoPE, layer_0_post_attn,
layer_0_post_mlp) and every layer's K/V; with --qk-inject the q/k projections of layer 0 are read
from q_proj_layer_0.bin / k_proj_layer_0.bin instead of computed. Parity:
rust/src/infer.rs:402-485, rust/src/model/model.rs:491-640, ring.rs:1440-1480 and 1620-1660.

Tensor files: [ndims u64 LE][dims u64 LE x ndims][float32 LE data], row-major (the same layout as
the reference's write_tensor_as_binary, so its comparison scripts read either side). The values
come from the framework's float32 model oracle (models/reference_model.py) on the same weights.
"""

from __future__ import annotations

import os
import struct
from typing import Dict, Optional

import numpy as np
import torch

from .models import reference_model
from .models.weights import ModelWeights


def write_tensor_bin(t: torch.Tensor, path: str) -> None:
    a = t.detach().float().contiguous().cpu().numpy()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", a.ndim))
        for d in a.shape:
            f.write(struct.pack("<Q", int(d)))
        f.write(a.astype("<f4").tobytes())


def read_tensor_bin(path: str) -> torch.Tensor:
    with open(path, "rb") as f:
        (nd,) = struct.unpack("<Q", f.read(8))
        shape = struct.unpack("<" + "Q" * nd, f.read(8 * nd))
        data = np.frombuffer(f.read(), dtype="<f4")
    return torch.from_numpy(data.copy()).view(*shape)


def _batched(name: str, t: torch.Tensor) -> torch.Tensor:
    # the reference's tensors carry a batch dimension
    return t if name.startswith("prefill_") else t.unsqueeze(0)


def export_hidden_states(w: ModelWeights, prompt_ids: torch.Tensor, export_dir: str) -> int:
    """Writes the files listed in the module docstring; returns the first generated token."""
    os.makedirs(export_dir, exist_ok=True)
    ids = prompt_ids.long()

    def tap_kv(name, t):
        if name.startswith("prefill_"):
            write_tensor_bin(t, os.path.join(export_dir, name + ".bin"))

    logits = reference_model.forward(w, ids, last_only=True, tap=tap_kv)[0]
    first = int(torch.argmax(logits))
    # decode step 1 = the last position of the prompt + first token
    ids1 = torch.cat([ids, torch.tensor([first], device=ids.device)])

    def tap_hidden(name, t):
        if name.startswith("layer_") and name[6:].isdigit():
            write_tensor_bin(t[-1:].unsqueeze(0), os.path.join(export_dir, name + ".bin"))
        elif name == "final_norm":
            write_tensor_bin(t[-1:].unsqueeze(0), os.path.join(export_dir, "final_norm.bin"))

    dec_logits = reference_model.forward(w, ids1, last_only=True, tap=tap_hidden)[0]
    vocab = dec_logits.numel()
    with open(os.path.join(export_dir, "logits.bin"), "wb") as f:
        f.write(struct.pack("<QQ", vocab, 1))
        f.write(dec_logits.float().cpu().numpy().astype("<f4").tobytes())
    return first


def prefill_debug_layer0(w: ModelWeights, prompt_ids: torch.Tensor, export_dir: str,
                         qk_inject_dir: Optional[str] = None) -> None:
    os.makedirs(export_dir, exist_ok=True)
    inject: Dict[str, torch.Tensor] = {}
    if qk_inject_dir:
        for name in ("q_proj_layer_0", "k_proj_layer_0"):
            t = read_tensor_bin(os.path.join(qk_inject_dir, name + ".bin"))
            inject[name] = t.reshape(t.shape[-2], t.shape[-1]) if t.dim() == 3 else t
    keep = {"embedding_output", "layer_0_input_norm", "q_proj_layer_0", "k_proj_layer_0",
            "v_proj_layer_0", "layer_0_post_attn"}

    def tap(name, t):
        if name in keep or name.startswith("prefill_"):
            write_tensor_bin(_batched(name, t), os.path.join(export_dir, name + ".bin"))
        elif name == "layer_0":
            write_tensor_bin(t.unsqueeze(0), os.path.join(export_dir, "layer_0_post_mlp.bin"))

    reference_model.forward(w, prompt_ids.long(), last_only=True, tap=tap, inject=inject)
