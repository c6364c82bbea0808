"""Python front-ends of the sm_100a kernels.

CUDA tensors always go to the native kernels (the extension must be present: see `_ext.native`);
CPU tensors use the plain PyTorch oracles in `reference.py`, which is what the CPU-rank tests run.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import reference as ref
from ._ext import native
from ..utils import launches

EPI = {"store": 0, "bias": 1, "residual": 2, "swiglu": 3}
GEMV = {"f32": 0, "residual": 1, "swiglu": 2, "argmax": 3}
SWIGLU_BLOCK = 128  # gate/up rows are interleaved in blocks of 128


# --------------------------------------------------------------------------- weight layouts
def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    """[I, K] gate and up -> [2 * I_pad, K] with rows [g0..g127, u0..u127, g128.., u128.., ...].

    I is zero-padded to a multiple of `block` (silu(0) * 0 = 0, and the down projection gets
    matching zero columns via `pad_down_proj`)."""
    i, k = gate.shape
    ip = -(-i // block) * block
    if ip != i:
        gate = torch.cat([gate, gate.new_zeros(ip - i, k)])
        up = torch.cat([up, up.new_zeros(ip - i, k)])
    g = gate.view(ip // block, block, k)
    u = up.view(ip // block, block, k)
    return torch.stack([g, u], dim=1).reshape(2 * ip, k).contiguous()


def pad_down_proj(down: torch.Tensor, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    n, i = down.shape
    ip = -(-i // block) * block
    if ip == i:
        return down.contiguous()
    return torch.cat([down, down.new_zeros(n, ip - i)], dim=1).contiguous()


def swiglu_from_interleaved(y: torch.Tensor, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    """CPU helper: split an interleaved gate||up projection and apply SwiGLU."""
    t, n2 = y.shape
    v = y.view(t, n2 // (2 * block), 2, block)
    return ref.swiglu(v[:, :, 0].reshape(t, -1), v[:, :, 1].reshape(t, -1))


# --------------------------------------------------------------------------- GEMM
def gemm(a: torch.Tensor, w: torch.Tensor, epi: str = "store", bias: Optional[torch.Tensor] = None,
         residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
         status: Optional[torch.Tensor] = None, variant: int = 0, group: int = -1) -> torch.Tensor:
    """out = a @ w.T with a fused epilogue (`store`, `bias`, `residual`, `swiglu`). `variant`: 0
    the default kernel, 1 one CTA per 128x256 tile, 2 CTA pairs on 256x256 tiles. `group`: tile
    order in bands of that many m-blocks (0: n fastest; -1: chosen by the weight's size)."""
    m, n = a.shape[0], w.shape[0]
    n_out = n // 2 if epi == "swiglu" else n
    if not a.is_cuda:
        y = a.float() @ w.float().t()
        if epi == "bias":
            y = y + bias.float()
        if epi == "residual":
            y = y.to(a.dtype).float() + residual.float()
        if epi == "swiglu":
            return swiglu_from_interleaved(y.to(a.dtype))
        y = y.to(a.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = residual if (epi == "residual" and residual is not None) else torch.empty(
            m, n_out, dtype=a.dtype, device=a.device)
    native().gemm(a, w, out, EPI[epi], bias, residual, status, variant, group)
    launches.count()
    return out


# --------------------------------------------------------------------------- attention
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, L: int,
              causal: bool = True, scale: Optional[float] = None,
              want_lse: bool = True, status: Optional[torch.Tensor] = None, variant: int = 0,
              order: int = -1):
    """Flash attention of q [T,H,D] over position-ordered k/v [Hkv, Lcap, D] (rows 0..L-1).
    `variant` picks the head_dim-64 kernel (0: the default; 1: one softmax stream per q tile;
    2: two streams; 3: pipelined, P in its own TMEM columns). `order` picks the CTA order (-1:
    the kernel's choice: pair major for grids of at most 8 waves; 0: KV-head major; 1: heaviest
    q-tile pairs of all heads first).

    Returns (o [T,H,D], lse [H,T] natural log or None)."""
    t, h, d = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if not q.is_cuda:
        kk = k[:, :L].transpose(0, 1)
        vv = v[:, :L].transpose(0, 1)
        o, lse = ref.full_attention(q.float(), kk.float(), vv.float(), q_pos.long(),
                                    torch.arange(L), causal=causal, scale=scale)
        return o.to(q.dtype), (lse if want_lse else None)
    o = torch.empty_like(q)
    lse = torch.empty(h, t, dtype=torch.float32, device=q.device) if want_lse else None
    native().attn_fwd(q, k, v, o, lse, q_pos, L, k.stride(0), scale, causal, status, variant,
                      order)
    launches.count()
    return o, lse


# --------------------------------------------------------------------------- norm / embedding
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None):
    if not x.is_cuda:
        y = ref.rmsnorm(x, w, eps)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty_like(x)
    native().rmsnorm(x, w, out, eps)
    launches.count()
    return out


def embedding(ids: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
              status: Optional[torch.Tensor] = None):
    if not w.is_cuda:
        return w[ids.long()]
    if out is None:
        out = torch.empty(ids.numel(), w.shape[1], dtype=w.dtype, device=w.device)
    native().embedding(ids, w, out, status)
    launches.count()
    return out


# --------------------------------------------------------------------------- GEMV (decode)
def gemv(x: torch.Tensor, w: torch.Tensor, epi: str, bias=None, y_f32=None, y_bf16=None,
         argmax=None, norm_w=None, eps: float = 1e-6, index_base: int = 0, prefetch=(),
         tc: int = -1, bulk: int = -1, status=None):
    """Decode GEMV y = f(x) @ w.T with a fused epilogue; `norm_w` applies RMSNorm to x first.
    With the "argmax" epilogue `index_base` is added to every row index of the packed maximum
    (w is then the vocabulary slice starting at that row). `prefetch`: up to two contiguous weight
    tensors of later kernels that the launch pulls into L2 while it runs. `tc`: the tensor-core
    kernel (-1: by batch size, 0: never, 1: whenever the shape allows). `bulk`: the streaming kernel
    that brings the weights in with bulk copies, where the tensor-core one is not used (-1: by
    HCP_GEMV_BULK, on unless it is 0; 0: never; 1: whenever the shape allows). `status`: an int32
    status word for its bounded pipeline waits."""
    if not x.is_cuda:
        if norm_w is not None:
            x = ref.rmsnorm(x, norm_w, eps)
        y = x.float() @ w.float().t()
        if epi == "f32":
            if bias is not None:
                y = y + bias.float()
            y_f32.copy_(y)
            return y_f32
        if epi == "residual":
            y_bf16.copy_((y.to(x.dtype).float() + y_bf16.float()).to(x.dtype))
            return y_bf16
        if epi == "swiglu":
            y_bf16.copy_(swiglu_from_interleaved(y.to(x.dtype)))
            return y_bf16
        if epi == "argmax":
            if y_f32 is not None:
                y_f32.copy_(y)
            return y.argmax(-1) + index_base
    native().gemv(x, w, GEMV[epi], bias, y_f32, y_bf16, argmax, norm_w, eps, index_base,
                  list(prefetch), tc, bulk, status)
    launches.count()
    return y_bf16 if y_bf16 is not None else y_f32
