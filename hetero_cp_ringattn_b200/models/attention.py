"""Attention backends: the interface between a decoder layer and the attention of one prefill or
continuation layer.

A backend takes the layer's normalised input rows of this rank, projects them to Q / K / V,
rotates Q and K at the rows' global positions, stores this rank's K / V rows in the request's
KV cache and returns the attention of its query rows over every rank's rows of the request
(causal on global positions), before the output projection. The engine owns everything else of
the layer (norms, output projection, MLP, residuals) and picks the backend at construction;
`LlamaCPEngine(..., attention_backend=...)` plugs in another one.

Parity: the reference's `AttentionBackend` trait (rust/src/model/attention/backend.rs:20-55:
`forward`, `set_distributed`, `set_strategy`) with its two implementations, the local GQA
backend (backend.rs:57-80) and the ring backend (rust/src/model/attention/ring.rs). Here:

* `CudaRingBackend`: the tcgen05 attention kernel with the NVLink KV ring of the domain runtime
  (one rank: plain local attention; several: the overlapped ring, whose attention kernel pushes
  the rank's rows to the peers and waits per KV tile, or the serial ring, push -> wait -> attend).
* `HostRingBackend`: float32 host ranks over gloo, the ring fold of the reference's CPU path
  (all-gather of K / V / positions, sources folded in ring order in micro blocks).
"""

from __future__ import annotations

import abc
import dataclasses
from typing import Any, Dict, Optional

import numpy as np
import torch

from ..ops import kernels as K
from ..ops import reference as ref
from ..parallel.strategy import RingStrategy
from ..utils import launches


@dataclasses.dataclass
class LayerCall:
    """One backend call: the request, the layer and this rank's rows of it.

    `pos` holds the rows' global positions ([T], on the engine's device). `L` is the request's
    context length once this call's rows are stored. A continuation segment (`existing` set)
    also attends to the `slot_base` rows already stored for the layer, whose positions
    `existing` lists. The CUDA backend writes into the `q_buf` / `o_buf` scratch, advances the
    runtime's layer-step `epoch` (the same on every rank), and follows the overlapped ring plan
    in `ring`. With `ev` (5 CUDA events), ev[2] is recorded between the projection + push and
    the attention."""
    st: Any
    layer: int
    pos: torch.Tensor
    L: int
    q_buf: Optional[torch.Tensor] = None
    o_buf: Optional[torch.Tensor] = None
    epoch: int = 0
    slot_base: int = 0
    existing: Optional[torch.Tensor] = None
    ring: Dict[str, torch.Tensor] = dataclasses.field(default_factory=dict)
    ev: Optional[list] = None


class AttentionBackend(abc.ABC):
    """Per-rank attention of prefill and continuation layers (see the module docstring)."""

    name = "abstract"

    def __init__(self, eng) -> None:
        self.eng = eng
        self.rank, self.world, self.group = eng.rank, eng.world, eng.group
        self.strategy = RingStrategy.VANILLA

    def set_distributed(self, rank: int, world: int, group=None) -> None:
        """Bind the rank, the number of ranks and the host process group (backend.rs:38-43)."""
        self.rank, self.world, self.group = int(rank), int(world), group

    def set_strategy(self, strategy) -> None:
        """Default layout of prompts whose prefill names none (backend.rs:45-50)."""
        self.strategy = RingStrategy.parse(strategy)

    @property
    def mode(self) -> str:
        """What runs: "local" on one rank, else the ring variant."""
        return "local" if self.world == 1 else "ring"

    @abc.abstractmethod
    def forward(self, xn: torch.Tensor, lw, call: LayerCall) -> torch.Tensor:
        """Q/K/V projection of `xn` [T, hidden] with the layer weights `lw`, RoPE, this rank's K/V
        rows into the KV cache, attention over every rank's rows. Returns o [T, H * D]."""


class CudaRingBackend(AttentionBackend):
    """The tcgen05 attention kernel over the domain runtime's KV staging ring."""

    name = "cuda_ring"

    @property
    def mode(self) -> str:
        e = self.eng
        if self.world == 1:
            return "local"
        return "overlap_in_kernel" if e.overlap else "serial"

    def forward(self, xn: torch.Tensor, lw, call: LayerCall) -> torch.Tensor:
        e = self.eng
        rt = e.rt
        T = int(call.pos.numel())
        tail = (call.pos, e.cos, e.sin, call.layer, call.st.kv.pt_device, call.slot_base, call.L,
                e.scale, True, call.q_buf, call.o_buf, None, call.epoch)
        if call.existing is not None:
            # continuation segment: the serial ring re-pushes the layer's stored rows as well
            tail = tail + (call.existing,)
            if T and e.fused_qkv_serial:
                rt.push_layer_fused(xn, lw.wqkv, lw.bqkv, *tail)
                rt.attend_layer(xn, *tail)
            else:
                qkv = (K.gemm(xn, lw.wqkv, "bias" if lw.bqkv is not None else "store", bias=lw.bqkv)
                       if T else torch.empty(0, e.cfg.qkv_size, dtype=torch.bfloat16, device=e.device))
                rt.push_layer(qkv, *tail)
                rt.attend_layer(qkv, *tail)
            return call.o_buf.view(T, e.H * e.D)
        ring = call.ring
        fused = e.fused_qkv if (self.world == 1 or ring) else e.fused_qkv_serial
        if fused:
            # one kernel: QKV GEMM whose epilogue rotates, writes Q and writes K/V (into every
            # rank's staging buffer in the serial ring, into this rank's own otherwise)
            rt.push_layer_fused(xn, lw.wqkv, lw.bqkv, *tail, **ring)
        else:
            qkv = K.gemm(xn, lw.wqkv, "bias" if lw.bqkv is not None else "store", bias=lw.bqkv)
            rt.push_layer(qkv, *tail, **ring)
            del qkv
        if call.ev is not None:
            call.ev[2].record()
        # overlapped ring: this one kernel also pushes the rank's rows to the peers
        rt.attend_layer(xn, *tail, **ring)
        if self.world == 1 or ring:
            launches.count(2)
        else:   # + wait for the released parity (after the first two steps), wait, signal
            launches.count(5 - (1 if call.epoch <= 2 else 0))
        return call.o_buf.view(T, e.H * e.D)


class HostRingBackend(AttentionBackend):
    """float32 host ranks: K / V rows all-gathered over the gloo group and folded in ring order
    (own rows first, then the predecessor's, ...) in micro blocks of HCP_MICRO_KV_BLOCK_SIZE
    rows with the online softmax and the fully-future block skip (ring.rs:861-1399)."""

    name = "host_ring"

    def _gather_rows(self, t: torch.Tensor):
        return self.eng._gather_rows(t)

    def _project(self, h: torch.Tensor, lw, pos: torch.Tensor):
        e, cfg = self.eng, self.eng.cfg
        T = h.shape[0]
        H, Hkv, D = e.H, e.Hkv, e.D
        qkv = ref.linear(h, lw.wqkv, lw.bqkv)
        q = ref.apply_rope(qkv[:, : H * D].view(T, H, D), pos, cfg.rope_theta, cfg.rope_scaling)
        k = ref.apply_rope(qkv[:, H * D:(H + Hkv) * D].view(T, Hkv, D), pos, cfg.rope_theta,
                           cfg.rope_scaling)
        v = qkv[:, (H + Hkv) * D:].reshape(T, Hkv, D)
        return q, k, v

    def _fold(self, q, q_pos, ks, vs, ps) -> torch.Tensor:
        e = self.eng
        Tq = q.shape[0]
        m = torch.full((e.H, Tq), ref.NEG_INIT, dtype=q.dtype)
        l = torch.zeros(e.H, Tq, dtype=q.dtype)
        acc = torch.zeros_like(q)
        for step in range(self.world):
            src = (self.rank - step) % self.world
            k, v, kp = ks[src], vs[src], ps[src]
            for b0 in range(0, k.shape[0], e.micro_kv):
                b1 = min(b0 + e.micro_kv, k.shape[0])
                m, l, acc = ref.online_update_block(m, l, acc, q, k[b0:b1].to(q.dtype),
                                                    v[b0:b1].to(q.dtype), q_pos, kp[b0:b1],
                                                    True, e.scale)
        return ref.finalize_state(m, l, acc)[0]

    def forward(self, xn: torch.Tensor, lw, call: LayerCall) -> torch.Tensor:
        e = self.eng
        st, pos = call.st, call.pos
        T = int(pos.numel())
        if call.existing is None:
            # prefill: this rank's rows become the layer's KV, then the ring fold
            q, k, v = self._project(xn, lw, pos)
            st.host_kv.append([k.clone(), v.clone(), pos.clone(), torch.ones(T, dtype=torch.bool)])
            o = self._fold(q, pos, self._gather_rows(k), self._gather_rows(v),
                           self._gather_rows(pos))
            return o.reshape(T, e.H * e.D)
        # continuation: the segment's rows join the stored ones; every rank takes part in the
        # gathers, ranks without rows in the segment return an empty output
        kv = st.host_kv[call.layer]
        q = None
        if T:
            q, k, v = self._project(xn, lw, pos)
            kv[0] = torch.cat([kv[0], k])
            kv[1] = torch.cat([kv[1], v])
            kv[2] = torch.cat([kv[2], pos])
            kv[3] = torch.cat([kv[3], torch.ones(T, dtype=torch.bool)])
        sh = kv[3]
        ks, vs, ps = (self._gather_rows(kv[0][sh]), self._gather_rows(kv[1][sh]),
                      self._gather_rows(kv[2][sh]))
        if not T:
            return torch.zeros(0, e.H * e.D)
        kk = torch.zeros(call.L, e.Hkv, e.D, dtype=torch.float32)
        vv = torch.zeros_like(kk)
        for a, b, p in zip(ks, vs, ps):
            kk[p] = a.float()
            vv[p] = b.float()
        # replicated legacy-decode rows (identical on every rank): once, from here
        kk[kv[2][~sh]] = kv[0][~sh].float()
        vv[kv[2][~sh]] = kv[1][~sh].float()
        o, _ = ref.full_attention(q, kk, vv, pos, torch.arange(call.L), causal=True)
        return o.reshape(T, e.H * e.D)


def default_backend(eng) -> AttentionBackend:
    """The CUDA ring on GPU engines, the host ring on CPU engines."""
    return CudaRingBackend(eng) if eng.cuda else HostRingBackend(eng)


def positions_tensor(positions: np.ndarray, device) -> torch.Tensor:
    """Global positions as the backend's `pos`: int32 on CUDA (the kernels' type), int64 on the
    host (the reference ops' index type)."""
    if device.type == "cuda":
        return torch.from_numpy(positions.astype(np.int32)).to(device, non_blocking=True)
    return torch.from_numpy(positions.astype(np.int64))
