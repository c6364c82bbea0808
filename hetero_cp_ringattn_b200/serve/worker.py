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

log = logging.getLogger("hcp.worker")


class Worker:
    def __init__(self, engine, control: P.ControlPlane):
        self.engine = engine
        self.control = control
        self.last_logits: Optional[torch.Tensor] = None

    # ------------------------------------------------------------------ backend-trait surface
    def capacity_mb(self) -> int:
        from ..parallel.capacity import query_device_capacity_mb
        return query_device_capacity_mb(str(self.engine.device))

    def num_layers(self) -> int:
        return self.engine.L

    def device(self) -> str:
        return str(self.engine.device)

    def handshake(self) -> bytes:
        return P.pack_handshake(self.engine.rank, self.capacity_mb())

    # ------------------------------------------------------------------ execution
    def execute(self, cmd):
        rid = getattr(cmd, "request_id", -1)
        e = self.engine
        try:
            if isinstance(cmd, P.Prefill):
                prompt = torch.as_tensor(cmd.prompt, dtype=torch.int64)  # no copy from the frame
                tok, logits = e.prefill(cmd.request_id, prompt, cmd.chunks, cmd.strategy,
                                        decode_horizon=cmd.decode_horizon,
                                        tickets=cmd.capacity_tickets, return_logits=True,
                                        keep_kv=cmd.keep_kv)
                self.last_logits = logits
                return P.PrefillDone(cmd.request_id, int(tok), len(cmd.prompt))
            if isinstance(cmd, (P.Decode, P.DecodeBatch)):
                pairs = [(cmd.request_id, cmd.token)] if isinstance(cmd, P.Decode) else \
                    [tuple(x) for x in cmd.request_tokens]
                rids = [int(r) for r, _ in pairs]
                toks = torch.tensor([int(t) for _, t in pairs], dtype=torch.int64, device=e.device)
                out = e.decode_step(rids, toks)
                self.last_logits = e.last_logits(len(rids))
                vals = [int(v) for v in out.view(-1).tolist()]
                if isinstance(cmd, P.Decode):
                    return P.DecodeDone(cmd.request_id, vals[0])
                return P.DecodeBatchDone([[r, v] for r, v in zip(rids, vals)])
            if isinstance(cmd, P.StationaryDecode):
                P.validate_stationary_decode(e.world, cmd.capacity_tickets, cmd.starter_domain,
                                             cmd.token_offset, cmd.decode_horizon)
                st = e.reqs.get(cmd.request_id)
                if st is None:
                    raise P.ProtocolError(f"unknown request {cmd.request_id}")
                if st.decode_offset != cmd.token_offset:
                    raise P.ProtocolError(f"request {cmd.request_id}: token_offset {cmd.token_offset} "
                                          f"!= engine offset {st.decode_offset}")
                toks = torch.tensor([cmd.token], dtype=torch.int64, device=e.device)
                out = e.decode_step([cmd.request_id], toks)
                self.last_logits = e.last_logits(1)
                return P.DecodeDone(cmd.request_id, int(out.view(-1)[0]))
            if isinstance(cmd, P.StationaryContinuation):
                P.validate_stationary_continuation(e.world, cmd.tokens, cmd.position_ids,
                                                   cmd.capacity_tickets, cmd.starter_domain)
                tok, logits = e.append(cmd.request_id, torch.as_tensor(cmd.tokens, dtype=torch.int64),
                                       cmd.position_ids, cmd.capacity_tickets, return_logits=True,
                                       extra_horizon=max(1, int(cmd.decode_horizon)))
                self.last_logits = logits
                return P.StationaryContinuationDone(cmd.request_id, int(tok))
            if isinstance(cmd, P.SyncGlobalSeqLen):
                st = e.reqs.get(cmd.request_id)
                if st is not None and st.context_len != cmd.len:
                    raise P.ProtocolError(f"request {cmd.request_id}: global length {st.context_len} "
                                          f"!= coordinator's {cmd.len}")
                return P.Ack(cmd.request_id)
            if isinstance(cmd, P.ReleaseRequest):
                e.release(cmd.request_id)
                return P.Ack(cmd.request_id)
            if isinstance(cmd, P.Shutdown):
                return P.Ack()
            raise P.ProtocolError(f"unsupported command {type(cmd).__name__}")
        except Exception as ex:  # the failing request is reported, the worker keeps serving
            log.warning("rank %d: %s failed: %s", e.rank, type(cmd).__name__, ex)
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
