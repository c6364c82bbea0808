"""Plain PyTorch oracles (fp32/fp64) for every hot op.

These are the numerics references that the sm_100a kernels are tested against, and the CPU
implementation used by CPU-rank (gloo) tests. None of them is on the GPU hot path.

Parity:
  * `full_attention` / `ring_attention_model` / `online_update_block` extend the reference's f64
    oracle (rust/src/smoke/reference_algo.rs:134-291, python/ringattn_kernel_stub.py:34-210) with
    causal masking on global positions, GQA and a log-sum-exp output. The ring model visits KV
    sources in (target + step) % N order and splits each source into blocks, as the reference does.
  * The fully-masked-row convention follows rust/src/model/attention/ring.rs:963-971: running max
    starts at -1e4 (scaled-score domain) so all-masked rows yield O = 0 and a finite LSE.
  * `rmsnorm`, `rope`, `swiglu` follow rust/src/model/layers/{norm,rotary,mlp}.rs (rotate-half
    RoPE at absolute positions, x * rsqrt(mean(x^2) + eps) * w).
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

NEG_INIT = -1e4  # initial running max of the reference's online softmax (ring.rs:963-971)


# --------------------------------------------------------------------------- attention
def _expand_kv(k: torch.Tensor, num_heads: int) -> torch.Tensor:
    hkv = k.shape[1]
    if hkv == num_heads:
        return k
    return k.repeat_interleave(num_heads // hkv, dim=1)


def full_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   q_pos: Optional[torch.Tensor] = None, k_pos: Optional[torch.Tensor] = None,
                   causal: bool = True, scale: Optional[float] = None,
                   q_chunk: Optional[int] = None):
    """Dense softmax attention.  q [Tq,H,D], k/v [Tk,Hkv,D] -> (o [Tq,H,D], lse [H,Tq]).

    lse is the natural-log log-sum-exp of the scaled scores over the unmasked keys; rows with no
    unmasked key get o = 0 and lse = -inf. With `q_chunk`, the queries are processed that many at
    a time (the score matrix of a chunk is [H, q_chunk, Tk]), for long contexts; each row's
    result is the same as without chunking."""
    tq, h, d = q.shape
    if q_chunk is not None and tq > q_chunk:
        if causal and q_pos is None:
            q_pos = torch.arange(tq, device=q.device)
        outs, lses = [], []
        for c0 in range(0, tq, q_chunk):
            qp = q_pos[c0:c0 + q_chunk] if q_pos is not None else None
            o, l = full_attention(q[c0:c0 + q_chunk], k, v, qp, k_pos, causal, scale)
            outs.append(o)
            lses.append(l)
        return torch.cat(outs), torch.cat(lses, dim=1)
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    kk = _expand_kv(k, h)
    vv = _expand_kv(v, h)
    s = torch.einsum("qhd,khd->hqk", q, kk) * scale
    if causal:
        if q_pos is None:
            q_pos = torch.arange(tq, device=q.device)
        if k_pos is None:
            k_pos = torch.arange(k.shape[0], device=q.device)
        mask = k_pos.view(1, 1, -1) > q_pos.view(1, -1, 1)
        s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)                      # [H, Tq]
    p = torch.exp(s - lse.unsqueeze(-1))
    p = torch.nan_to_num(p, nan=0.0)
    o = torch.einsum("hqk,khd->qhd", p, vv)
    return o, lse


def online_update_block(m: torch.Tensor, l: torch.Tensor, acc: torch.Tensor, q: torch.Tensor,
                        k: torch.Tensor, v: torch.Tensor, q_pos, k_pos, causal: bool,
                        scale: float):
    """One online-softmax step of a q chunk over one KV block (state m, l: [H,Tq]; acc [Tq,H,D]).

    Fully-future blocks (min k_pos > max q_pos) are skipped, as in ring.rs:220-273."""
    h = q.shape[1]
    if causal and k_pos.numel() and q_pos.numel() and int(k_pos.min()) > int(q_pos.max()):
        return m, l, acc
    kk = _expand_kv(k, h)
    vv = _expand_kv(v, h)
    s = torch.einsum("qhd,khd->hqk", q, kk) * scale
    if causal:
        mask = k_pos.view(1, 1, -1) > q_pos.view(1, -1, 1)
        s = s.masked_fill(mask, float("-inf"))
    m_blk = s.amax(dim=-1)
    m_new = torch.maximum(m, m_blk)
    alpha = torch.exp(m - m_new)
    p = torch.exp(s - m_new.unsqueeze(-1))
    l_new = l * alpha + p.sum(-1)
    acc_new = acc * alpha.transpose(0, 1).unsqueeze(-1) + torch.einsum("hqk,khd->qhd", p, vv)
    return m_new, l_new, acc_new


def finalize_state(m, l, acc):
    """(m, l, acc) -> (o, lse). All-masked rows (l == 0) give o = 0 and lse = -inf."""
    safe = torch.where(l > 0, l, torch.ones_like(l))
    o = acc / safe.transpose(0, 1).unsqueeze(-1)
    lse = torch.where(l > 0, m + torch.log(safe), torch.full_like(l, float("-inf")))
    return o, lse


def ring_attention_model(q_chunks: Sequence[torch.Tensor], k_chunks: Sequence[torch.Tensor],
                         v_chunks: Sequence[torch.Tensor], pos_chunks: Sequence[torch.Tensor],
                         block_sizes: Sequence[int], causal: bool = True,
                         scale: Optional[float] = None):
    """Per-domain ring attention with online softmax over uneven blocks.

    Domain `t` folds source `(t + step) % N` for step = 0..N-1, each source cut into blocks of
    block_sizes[source] tokens. Returns a list of (o, lse) per domain."""
    n = len(q_chunks)
    d = q_chunks[0].shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    out = []
    for t in range(n):
        q = q_chunks[t]
        tq, h, _ = q.shape
        m = torch.full((h, tq), NEG_INIT, dtype=q.dtype, device=q.device)
        l = torch.zeros((h, tq), dtype=q.dtype, device=q.device)
        acc = torch.zeros_like(q)
        for step in range(n):
            s = (t + step) % n
            k, v, kp = k_chunks[s], v_chunks[s], pos_chunks[s]
            bs = max(1, int(block_sizes[s]))
            for b0 in range(0, k.shape[0], bs):
                b1 = min(b0 + bs, k.shape[0])
                m, l, acc = online_update_block(m, l, acc, q, k[b0:b1], v[b0:b1], pos_chunks[t],
                                                kp[b0:b1], causal, scale)
        out.append(finalize_state(m, l, acc))
    return out


def merge_partials(os: Sequence[torch.Tensor], lses: Sequence[torch.Tensor]):
    """Exact log-sum-exp merge of partial attentions (o_i [T,H,D], lse_i [H,T]) in list order."""
    lse_stack = torch.stack(list(lses))                     # [N,H,T]
    m = lse_stack.amax(0)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(lse_stack - m_safe)                       # [N,H,T]
    tot = w.sum(0)
    o = torch.zeros_like(os[0])
    for i, oi in enumerate(os):
        o = o + oi * w[i].transpose(0, 1).unsqueeze(-1)
    safe = torch.where(tot > 0, tot, torch.ones_like(tot))
    o = o / safe.transpose(0, 1).unsqueeze(-1)
    lse = torch.where(tot > 0, m_safe + torch.log(safe), torch.full_like(tot, float("-inf")))
    return o, lse


# --------------------------------------------------------------------------- layer ops
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype)


def rope_inv_freq(head_dim: int, theta: float, scaling: Optional[dict] = None, device=None):
    """RoPE inverse frequencies (float64, [D/2]) and the cos/sin amplitude.

    Without `scaling`: theta ** (-2i / D). With an HF `rope_scaling` dict:
      * linear: every frequency divided by `factor` (positions interpolated);
      * llama3 (the Llama 3.1 release's frequency-dependent rule): wavelengths shorter than
        original_max_position_embeddings / high_freq_factor keep their frequency, wavelengths
        longer than original_max_position_embeddings / low_freq_factor are divided by `factor`,
        and the band between is interpolated linearly in original_max / wavelength;
      * yarn (Peng et al. 2023, "YaRN: Efficient Context Window Extension of Large Language
        Models"): dimensions that rotate fewer than beta_slow times over the original context are
        interpolated (divided by `factor`), those rotating more than beta_fast times are kept, a
        linear ramp in between; cos and sin are scaled by attention_factor (default
        0.1 ln(factor) + 1).
    """
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64, device=device) /
                           head_dim))
    amp = 1.0
    if not scaling:
        return inv, amp
    kind = scaling.get("rope_type", scaling.get("type", "default"))
    factor = float(scaling.get("factor", 1.0))
    if kind == "default":
        return inv, amp
    if kind == "linear":
        return inv / factor, amp
    orig = float(scaling.get("original_max_position_embeddings", 8192))
    if kind == "llama3":
        lo, hi = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
        wavelen = 2 * math.pi / inv
        smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        mixed = (1.0 - smooth) * inv / factor + smooth * inv
        out = torch.where(wavelen > orig / lo, inv / factor, mixed)
        return torch.where(wavelen < orig / hi, inv, out), amp
    if kind == "yarn":
        beta_fast = float(scaling.get("beta_fast", 32.0))
        beta_slow = float(scaling.get("beta_slow", 1.0))

        def dim_of(rotations: float) -> float:   # dimension index rotating `rotations` times
            return head_dim * math.log(orig / (rotations * 2 * math.pi)) / (2 * math.log(theta))

        low = max(math.floor(dim_of(beta_fast)), 0)
        high = min(math.ceil(dim_of(beta_slow)), head_dim - 1)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(head_dim // 2, dtype=torch.float64, device=device) - low) /
                 (high - low)).clamp(0.0, 1.0)
        keep = 1.0 - ramp                                  # 1: extrapolate (keep the frequency)
        out = inv / factor * (1.0 - keep) + inv * keep
        amp = float(scaling.get("attention_factor") or (0.1 * math.log(factor) + 1.0))
        return out, amp
    raise ValueError(f"unsupported rope_scaling type {kind!r}")


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float, dtype=torch.float32,
                 scaling: Optional[dict] = None):
    inv, amp = rope_inv_freq(head_dim, theta, scaling, positions.device)
    f = positions.to(torch.float64).unsqueeze(-1) * inv.unsqueeze(0)   # [T, D/2]
    return (f.cos() * amp).to(dtype), (f.sin() * amp).to(dtype)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float,
               scaling: Optional[dict] = None) -> torch.Tensor:
    """Rotate-half RoPE. x [T, heads, D] at absolute positions [T]."""
    d = x.shape[-1]
    cos, sin = rope_cos_sin(positions, d, theta, scaling=scaling)
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    out = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)
    return out.to(x.dtype)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    g = gate.float()
    return (g * torch.sigmoid(g) * up.float()).to(gate.dtype)


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y.to(x.dtype)
