"""Worker side of the control plane: execute coordinator commands on this rank's engine.

Parity: rust/src/worker_sdk/runtime.rs:136-379 (command loop mapping `WorkerCommand`s to backend
calls; a closed control stream ends the worker; stationary failures become `Error` responses) and
the backend trait rust/src/worker_sdk/backend.rs:30-218 (prefill, decode, decode_batch, stationary
continuation / decode, sync_global_seq_len, release_request, capacity_mb, num_layers, device).
One process per GPU under torchrun; rank 0 also hosts the coordinator and calls `execute` itself.
"""

from __future__ import annotations

import logging
import traceback
from typing import Optional

import torch

from . import protocol as P
from .backend import EngineBackend, WorkerBackend

log = logging.getLogger("hcp.worker")


class Worker:
    """Executes control commands on a `WorkerBackend` (an `LlamaCPEngine` is wrapped in
    `EngineBackend`). A failing command becomes an `Error` response; the worker keeps serving."""

    def __init__(self, backend, control: P.ControlPlane):
        self.backend = backend if isinstance(backend, WorkerBackend) else EngineBackend(backend)
        self.control = control
        self.last_logits: Optional[torch.Tensor] = None

    @property
    def engine(self):
        """The wrapped engine (for callers that need engine-level state)."""
        return getattr(self.backend, "engine", None)

    # ------------------------------------------------------------------ backend-trait surface
    def capacity_mb(self) -> int:
        return self.backend.capacity_mb()

    def num_layers(self) -> int:
        return self.backend.num_layers()

    def device(self) -> str:
        return self.backend.device()

    def handshake(self) -> bytes:
        return P.pack_handshake(self.backend.rank, self.capacity_mb())

    # ------------------------------------------------------------------ execution
    def execute(self, cmd):
        rid = getattr(cmd, "request_id", -1)
        b = self.backend
        try:
            if isinstance(cmd, P.Prefill):
                prompt = torch.as_tensor(cmd.prompt, dtype=torch.int64)  # no copy from the frame
                tok, self.last_logits = b.prefill(cmd.request_id, prompt, cmd.chunks, cmd.strategy,
                                                  cmd.decode_horizon, cmd.capacity_tickets,
                                                  cmd.keep_kv, cmd.want_logits)
                return P.PrefillDone(cmd.request_id, tok, len(cmd.prompt))
            if isinstance(cmd, (P.Decode, P.DecodeBatch)):
                pairs = [(cmd.request_id, cmd.token)] if isinstance(cmd, P.Decode) else \
                    [tuple(x) for x in cmd.request_tokens]
                rids = [int(r) for r, _ in pairs]
                vals, self.last_logits = b.decode_batch(rids, [int(t) for _, t in pairs],
                                                        want_logits=getattr(cmd, "want_logits", True))
                if isinstance(cmd, P.Decode):
                    return P.DecodeDone(cmd.request_id, vals[0])
                return P.DecodeBatchDone([[r, v] for r, v in zip(rids, vals)])
            if isinstance(cmd, P.StationaryDecode):
                P.validate_stationary_decode(b.world, cmd.capacity_tickets, cmd.starter_domain,
                                             cmd.token_offset, cmd.decode_horizon)
                off = b.decode_offset(cmd.request_id)
                if off is None:
                    raise P.ProtocolError(f"unknown request {cmd.request_id}")
                if off != cmd.token_offset:
                    raise P.ProtocolError(f"request {cmd.request_id}: token_offset {cmd.token_offset} "
                                          f"!= engine offset {off}")
                vals, self.last_logits = b.decode_batch([cmd.request_id], [cmd.token])
                return P.DecodeDone(cmd.request_id, vals[0])
            if isinstance(cmd, P.StationaryContinuation):
                P.validate_stationary_continuation(b.world, cmd.tokens, cmd.position_ids,
                                                   cmd.capacity_tickets, cmd.starter_domain)
                tok, self.last_logits = b.continuation(
                    cmd.request_id, torch.as_tensor(cmd.tokens, dtype=torch.int64),
                    cmd.position_ids, cmd.capacity_tickets, cmd.decode_horizon, cmd.want_logits)
                return P.StationaryContinuationDone(cmd.request_id, tok)
            if isinstance(cmd, P.SyncGlobalSeqLen):
                n = b.context_len(cmd.request_id)
                if n is not None and n != cmd.len:
                    raise P.ProtocolError(f"request {cmd.request_id}: global length {n} "
                                          f"!= coordinator's {cmd.len}")
                return P.Ack(cmd.request_id)
            if isinstance(cmd, P.ReleaseRequest):
                b.release(cmd.request_id)
                return P.Ack(cmd.request_id)
            if isinstance(cmd, P.Shutdown):
                return P.Ack()
            raise P.ProtocolError(f"unsupported command {type(cmd).__name__}")
        except Exception as ex:  # the failing request is reported, the worker keeps serving
            log.warning("rank %d: %s failed: %s", b.rank, type(cmd).__name__, ex)
            log.debug(traceback.format_exc())
            return P.Error(rid, f"{type(ex).__name__}: {ex}")

    def loop(self) -> None:
        """Non-coordinator ranks: receive, execute, respond, until Shutdown."""
        while True:
            cmd = self.control.broadcast(None)
            resp = self.execute(cmd)
            if isinstance(cmd, P.Shutdown):
                break
            self.control.gather(resp)
