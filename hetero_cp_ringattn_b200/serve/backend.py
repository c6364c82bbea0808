"""What a worker rank needs from its compute backend, and the CP engine as that backend.

Parity: the reference's worker backend trait (rust/src/worker_sdk/backend.rs:30-218: prefill,
decode / decode_batch, stationary continuation / decode, sync_global_seq_len, release_request,
capacity_mb, num_layers, device) implemented by its libtorch backend (worker_sdk/tch_backend.rs).
Here `LlamaCPEngine` is the one production backend (`EngineBackend`); the worker's command loop
talks only to this interface, so tests and tools can drive the control plane with other
implementations.
"""

from __future__ import annotations

import abc
from typing import List, Optional, Sequence, Tuple

import torch


class WorkerBackend(abc.ABC):
    """Per-rank compute backend. Every method is called SPMD: all ranks receive the same calls
    in the same order. Logits, when returned, stay wherever the backend keeps them."""

    @abc.abstractmethod
    def prefill(self, request_id: int, prompt: torch.Tensor, chunks: Sequence[int],
                strategy: str, decode_horizon: int, capacity_tickets: Optional[Sequence[int]],
                keep_kv: bool, want_logits: bool = True) -> Tuple[int, Optional[torch.Tensor]]:
        """Prefill the whole prompt (every rank its chunk); the first token and, if wanted, its
        logits."""

    @abc.abstractmethod
    def decode_batch(self, request_ids: Sequence[int], tokens: Sequence[int],
                     want_logits: bool = True) -> Tuple[List[int], Optional[torch.Tensor]]:
        """One greedy decode step for each request; the next tokens and, if wanted, their
        logits (greedy-only batches pass False, which lets the ranks split the LM head)."""

    @abc.abstractmethod
    def continuation(self, request_id: int, tokens: torch.Tensor, position_ids: Sequence[int],
                     capacity_tickets: Sequence[int], decode_horizon: int,
                     want_logits: bool = True) -> Tuple[int, Optional[torch.Tensor]]:
        """Append a segment to a kept request; the next token and, if wanted, its logits."""

    @abc.abstractmethod
    def release(self, request_id: int) -> bool:
        """Free the request's KV; False if it holds none."""

    @abc.abstractmethod
    def context_len(self, request_id: int) -> Optional[int]:
        """Tokens with KV for the request (None if unknown)."""

    @abc.abstractmethod
    def decode_offset(self, request_id: int) -> Optional[int]:
        """Decode steps taken by the request (None if unknown)."""

    @property
    @abc.abstractmethod
    def world(self) -> int:
        """Number of ranks."""

    @property
    @abc.abstractmethod
    def rank(self) -> int:
        """This rank."""

    @abc.abstractmethod
    def capacity_mb(self) -> int:
        """Free memory this rank offers for KV (the handshake value)."""

    @abc.abstractmethod
    def num_layers(self) -> int:
        """Decoder layers of the model."""

    @abc.abstractmethod
    def device(self) -> str:
        """The device the backend computes on."""


class EngineBackend(WorkerBackend):
    """`LlamaCPEngine` as a worker backend."""

    def __init__(self, engine):
        self.engine = engine

    def prefill(self, request_id, prompt, chunks, strategy, decode_horizon, capacity_tickets,
                keep_kv, want_logits=True):
        tok, logits = self.engine.prefill(request_id, prompt, chunks, strategy,
                                          decode_horizon=decode_horizon, tickets=capacity_tickets,
                                          return_logits=want_logits, keep_kv=keep_kv)
        return int(tok), logits

    def decode_batch(self, request_ids, tokens, want_logits=True):
        e = self.engine
        toks = torch.tensor([int(t) for t in tokens], dtype=torch.int64, device=e.device)
        out = e.decode_step([int(r) for r in request_ids], toks, logits=bool(want_logits))
        logits = e.last_logits(len(request_ids)) if want_logits else None
        return [int(v) for v in out.view(-1).tolist()], logits

    def continuation(self, request_id, tokens, position_ids, capacity_tickets, decode_horizon,
                     want_logits=True):
        tok, logits = self.engine.append(request_id, tokens, position_ids, capacity_tickets,
                                         return_logits=want_logits,
                                         extra_horizon=max(1, int(decode_horizon)))
        return int(tok), logits

    def release(self, request_id):
        return self.engine.release(request_id)

    def context_len(self, request_id):
        st = self.engine.reqs.get(request_id)
        return None if st is None else st.context_len

    def decode_offset(self, request_id):
        st = self.engine.reqs.get(request_id)
        return None if st is None else st.decode_offset

    @property
    def world(self):
        return self.engine.world

    @property
    def rank(self):
        return self.engine.rank

    def capacity_mb(self):
        from ..parallel.capacity import query_device_capacity_mb
        return query_device_capacity_mb(str(self.engine.device))

    def num_layers(self):
        return self.engine.L

    def device(self):
        return str(self.engine.device)
