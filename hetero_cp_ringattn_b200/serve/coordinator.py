"""Coordinator: request admission, chunking, KV byte ledger, sessions, iterative decode batching.

Parity: rust/src/distributed/coordinator.rs:
  * chunk selection (:900-960): explicit `--chunk-sizes`, `--capacity-aware` (handshake capacities
    minus `--activation-reserve-mb`, default 1536), else equal splits; plus ratio overrides;
  * ring strategy (:57-74, :962);
  * KV byte admission with a per-domain ledger and rollback on failure (:784-871, :1678);
  * sessions: `keep_kv` keeps a finished request's KV, `append` continues it (:1246-1407,
    :1746-1822), with `--session-continuation-tokens` of headroom (:1719-1730);
  * iterative scheduling (:2563-2916): pending -> prefill -> active, one decode step per iteration
    for every active request (batched), streaming deltas, stop on EOS / max_tokens;
  * trace JSONL (:621-782): enqueue / prefill-accepted / first-token / completed timestamps,
    reserved / released KV bytes.
It runs inside rank 0's process; every engine step is issued to all ranks over the control plane.
"""

from __future__ import annotations

import dataclasses
import itertools
import json
import logging
import threading
import time
from typing import Dict, List, Optional, Sequence

from ..errors import AdmissionError, CapacityError, Overloaded, ProtocolError, RingError
from ..models.sampling import sample_token
from ..parallel.capacity import (DEFAULT_ACTIVATION_RESERVE_MB, KvLedger, UNKNOWN_CAPACITY,
                                 chunk_sizes, continuation_split)
from . import protocol as P
from .logits_dump import export_logits_dump
from .scheduler import ActiveRequest, BatchScheduler, Job

log = logging.getLogger("hcp.coordinator")


@dataclasses.dataclass
class CoordinatorArgs:
    strategy: str = "vanilla"
    chunk_sizes: Optional[List[int]] = None
    capacity_aware: bool = False
    ratio: Optional[List[int]] = None
    max_batch_size: int = 4
    activation_reserve_mb: int = DEFAULT_ACTIVATION_RESERVE_MB
    session_continuation_tokens: int = 64
    trace_jsonl: Optional[str] = None
    eos_ids: Optional[List[int]] = None
    export_logits_dir: Optional[str] = None  # per-request logits dumps (coordinator.rs:1170)
    max_queue: int = 0                       # >0: submissions beyond this many queued get 503
    kv_page_tokens: int = 1                  # ledger rounds each rank's rows up to whole pages
    session_ttl_s: float = 0.0               # >0: sessions idle this long release their KV
    decode_batch_limit: int = 8              # rows per engine decode step; more active requests
                                             # decode in several steps per iteration
    prefill_chunk_tokens: int = 0            # >0: prompts longer than this prefill in pieces,
                                             # with decode steps of the active requests between


class TraceSink:
    def __init__(self, path: Optional[str]):
        self.path = path
        self.lock = threading.Lock()

    def emit(self, kind: str, **kw) -> None:
        if not self.path:
            return
        with self.lock, open(self.path, "a") as f:
            f.write(json.dumps({"ts": time.time(), "event": kind, **kw}) + "\n")


@dataclasses.dataclass
class ChunkedPrefill:
    """A prompt being prefilled piece by piece: `done` tokens have KV on the ranks."""
    job: Job
    chunks: List[int]        # per-rank token shares used for tickets and the KV ledger
    done: int
    horizon: int


@dataclasses.dataclass
class Session:
    request_id: int
    context_len: int
    chunks: List[int]
    last_token: int
    last_used: float = dataclasses.field(default_factory=time.time)


class Metrics:
    """Request counters (the JSON `/metrics` fields) plus generated tokens and latency
    histograms for the Prometheus text endpoint."""

    BUCKETS = (0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0, 60.0)

    def __init__(self):
        self.total = 0
        self.completed = 0
        self.failed = 0
        self.aborted = 0                 # ended early because the client went away
        self.tokens = 0
        self.lock = threading.Lock()
        self.hist = {"ttft_seconds": [0] * (len(self.BUCKETS) + 1) + [0.0],
                     "request_latency_seconds": [0] * (len(self.BUCKETS) + 1) + [0.0]}

    def bump(self, field: str, n: int = 1) -> None:
        with self.lock:
            setattr(self, field, getattr(self, field) + n)

    def observe(self, name: str, value: float) -> None:
        """Histogram sample: per-bucket counts (non-cumulative), the overflow count, the sum."""
        with self.lock:
            h = self.hist[name]
            i = next((k for k, le in enumerate(self.BUCKETS) if value <= le), len(self.BUCKETS))
            h[i] += 1
            h[-1] += value

    def prometheus(self, queued: int, active: int) -> str:
        """Prometheus text exposition format (version 0.0.4)."""
        with self.lock:
            out = []
            for name, help_, kind, v in (
                    ("hcp_requests_total", "requests submitted", "counter", self.total),
                    ("hcp_requests_completed_total", "requests finished", "counter", self.completed),
                    ("hcp_requests_failed_total", "requests failed", "counter", self.failed),
                    ("hcp_requests_aborted_total", "requests ended by a client disconnect",
                     "counter", self.aborted),
                    ("hcp_generated_tokens_total", "tokens generated", "counter", self.tokens),
                    ("hcp_requests_queued", "requests waiting for admission", "gauge", queued),
                    ("hcp_requests_active", "requests decoding", "gauge", active)):
                out += [f"# HELP {name} {help_}", f"# TYPE {name} {kind}", f"{name} {v}"]
            for name, h in self.hist.items():
                full = f"hcp_{name}"
                out += [f"# HELP {full} {name.replace('_', ' ')}", f"# TYPE {full} histogram"]
                acc = 0
                for le, c in zip(self.BUCKETS, h):
                    acc += c
                    out.append(f'{full}_bucket{{le="{le}"}} {acc}')
                acc += h[len(self.BUCKETS)]
                out += [f'{full}_bucket{{le="+Inf"}} {acc}', f"{full}_sum {h[-1]}",
                        f"{full}_count {acc}"]
            return "\n".join(out) + "\n"


class Coordinator:
    def __init__(self, worker, control: P.ControlPlane, tokenizer, cfg, args: CoordinatorArgs,
                 capacities_mb: Optional[Sequence[int]] = None,
                 kv_budget_bytes: Optional[Sequence[int]] = None):
        self.worker = worker
        self.control = control
        self.tok = tokenizer
        self.cfg = cfg
        self.args = args
        self.world = control.world
        self.sched = BatchScheduler(args.max_batch_size)
        self.trace = TraceSink(args.trace_jsonl)
        self.metrics = Metrics()
        self.sessions: Dict[str, Session] = {}
        self._busy: set = set()   # session ids with a keep_kv / append request in flight
        self._prefilling: List[ChunkedPrefill] = []
        self.control_failed: Optional[str] = None   # set when the control group broke
        self._ids = itertools.count(1)
        caps = list(capacities_mb) if capacities_mb else [UNKNOWN_CAPACITY] * self.world
        self.capacities_mb = caps
        budgets = []
        for c in caps:
            if c == UNKNOWN_CAPACITY:
                budgets.append(1 << 62)
            else:
                budgets.append(max(0, int(c) - args.activation_reserve_mb) * 1024 * 1024)
        if kv_budget_bytes:
            # the ranks' preallocated KV arenas bound what can be admitted, whatever the free
            # device memory says
            budgets = [min(b, int(k)) for b, k in zip(budgets, kv_budget_bytes)]
        self.ledger = KvLedger(budgets)
        self.bytes_per_token_layer = cfg.kv_bytes_per_token_per_layer(2)
        self._stop = threading.Event()
        self.lock = threading.Lock()   # serialises engine steps issued by API threads

    # ------------------------------------------------------------------ submission
    def next_request_id(self) -> int:
        return next(self._ids)

    def submit(self, job: Job) -> None:
        self.metrics.bump("total")
        if self.args.max_queue and self.sched.queued >= self.args.max_queue:
            self.metrics.bump("failed")
            raise Overloaded(f"{self.sched.queued} requests queued (limit {self.args.max_queue}); "
                             "retry later")
        if job.append or job.keep_kv:
            if not job.session_id:
                raise ProtocolError(("append" if job.append else "keep_kv") + "=true requires session_id")
        if job.append and job.session_id not in self.sessions:
            raise ProtocolError(f"unknown or expired session {job.session_id!r}")
        if job.keep_kv and not job.append and job.session_id in self.sessions:
            raise ProtocolError(f"session_id {job.session_id!r} already has resident KV")
        self.trace.emit("enqueue", request=job.request_id, prompt_tokens=len(job.prompt_ids))
        self.sched.enqueue(job)

    # ------------------------------------------------------------------ engine commands
    def run_command(self, cmd):
        """Broadcast `cmd`, execute it here, gather every rank's response. A failure of the
        control group itself (a rank died, the group timed out) leaves the job unusable: it is
        recorded in `control_failed`, which /health reports, and re-raised."""
        with self.lock:
            try:
                self.control.broadcast(cmd)
                resp = self.worker.execute(cmd)
                all_resp = self.control.gather(resp)
            except (RuntimeError, OSError) as e:
                self.control_failed = f"{type(e).__name__}: {e}"
                self.trace.emit("control_failed", error=self.control_failed)
                raise
        errs = [r for r in (all_resp or [resp]) if isinstance(r, P.Error)]
        if errs:
            msg = "; ".join(f"rank error: {e.message}" for e in errs)
            if all(e.message.startswith("CapacityError:") for e in errs):
                raise CapacityError(msg)   # a rank's KV arena is full: wait or reject (400)
            raise ProtocolError(msg)
        return resp

    def shutdown(self) -> bool:
        """Stop the loop and tell the worker ranks to exit. Returns False when the ranks were
        already gone (an interrupt that reached every rank makes the broadcast fail; that is not
        an error here)."""
        self._stop.set()
        with self.lock:
            try:
                self.control.broadcast(P.Shutdown())
            except (RuntimeError, OSError) as e:
                self.trace.emit("shutdown_broadcast_failed", error=str(e))
                return False
        return True

    # ------------------------------------------------------------------ admission
    def _chunks(self, n: int) -> List[int]:
        return chunk_sizes(n, self.world, explicit=self.args.chunk_sizes,
                           capacities_mb=self.capacities_mb, capacity_aware=self.args.capacity_aware,
                           ratio=self.args.ratio, activation_reserve_mb=self.args.activation_reserve_mb)

    def _tickets(self, chunks: Sequence[int]) -> List[int]:
        if self.args.ratio:
            return list(self.args.ratio)
        return [max(1, c) for c in chunks]

    def _wants_logits(self, job: Job) -> bool:
        """Full logits travel to the ranks only when something reads them: sampling or dumps."""
        return job.temperature > 0 or bool(self.args.export_logits_dir)

    def _pages(self, rows: int) -> int:
        """Rows rounded up to whole KV pages (the arena hands out pages, not rows)."""
        p = max(1, int(self.args.kv_page_tokens))
        return -(-int(rows) // p) * p

    def _reserve(self, rid: int, chunks: Sequence[int], horizon: int) -> List[int]:
        tickets = self._tickets(chunks)
        tot = sum(tickets)
        per = []
        for c, t in zip(chunks, tickets):
            growth = -(-horizon * t // tot) + 1
            per.append(self._pages(c + growth) * self.cfg.num_layers * self.bytes_per_token_layer)
        self.ledger.try_reserve(rid, per)
        self.trace.emit("kv_reserved", request=rid, bytes=per)
        return per

    def _prefill(self, job: Job) -> None:
        rid = job.request_id
        if job.append:
            return self._append(job)
        horizon = max(1, job.max_tokens) + (self.args.session_continuation_tokens if job.keep_kv else 0)
        if job.keep_kv and (job.session_id in self.sessions or job.session_id in self._busy):
            raise AdmissionError(f"session_id {job.session_id!r} already has resident KV")
        try:
            chunks = self._chunks(len(job.prompt_ids))
        except RingError as e:
            raise AdmissionError(str(e)) from e
        self._reserve(rid, chunks, horizon)  # CapacityError: requeued while others hold KV
        if job.keep_kv:   # own the session only once admitted (a requeued job owns nothing)
            self._busy.add(job.session_id)
            job.holds_session = True
        piece = int(self.args.prefill_chunk_tokens)
        if piece > 0 and len(job.prompt_ids) > max(piece, self.world) and not self.args.chunk_sizes:
            return self._start_chunked(job, chunks, horizon, max(piece, self.world))
        try:
            resp = self.run_command(P.Prefill(rid, list(job.prompt_ids), chunks, self.args.strategy,
                                              horizon, self._tickets(chunks), job.keep_kv,
                                              self._wants_logits(job)))
        except Exception:
            self.ledger.release(rid)
            raise
        self.trace.emit("prefill_accepted", request=rid, chunks=chunks,
                        hops_per_prefill=self.cfg.num_layers * max(0, self.world - 1))
        if self.args.export_logits_dir and self.worker.last_logits is not None:
            export_logits_dump(self._dump_dir(rid), {"prefill_last_logits": self.worker.last_logits}, {
                "mode": "service", "device": "distributed-workers", "request_id": rid,
                "session_id": job.session_id, "keep_kv": job.keep_kv, "domains": self.world,
                "layers": self.cfg.num_layers, "prompt_tokens": len(job.prompt_ids),
                "prefill_argmax": int(resp.token)})
        req = ActiveRequest(job=job, chunks=chunks, next_position=len(job.prompt_ids))
        self._emit_token(req, resp.token)

    # ------------------------------------------------------------------ chunked prefill
    def _start_chunked(self, job: Job, chunks: List[int], horizon: int, first: int) -> None:
        """Prefill the first `first` tokens with the ring layout; the rest follows one piece per
        iteration as continuation segments (the engine's append path), so decode steps of the
        active requests run between the pieces. The request holds a batch slot meanwhile."""
        rid = job.request_id
        pchunks = chunk_sizes(first, self.world, capacities_mb=self.capacities_mb,
                              capacity_aware=self.args.capacity_aware, ratio=self.args.ratio,
                              activation_reserve_mb=self.args.activation_reserve_mb)
        try:
            self.run_command(P.Prefill(rid, list(job.prompt_ids[:first]), pchunks,
                                       self.args.strategy, horizon, self._tickets(chunks),
                                       job.keep_kv, False))
        except Exception:
            self.ledger.release(rid)
            raise
        self.sched.occupy(rid)
        self._prefilling.append(ChunkedPrefill(job, list(chunks), first, horizon))
        self.trace.emit("prefill_chunk", request=rid, done=first, total=len(job.prompt_ids))

    def _advance_chunked(self, pf: ChunkedPrefill) -> None:
        job, rid = pf.job, pf.job.request_id
        if job.cancelled:
            self._prefilling.remove(pf)
            self._abort_started(job)
            return
        n = len(job.prompt_ids)
        end = min(n, pf.done + max(int(self.args.prefill_chunk_tokens), 1))
        try:
            resp = self.run_command(P.StationaryContinuation(
                rid, list(job.prompt_ids[pf.done:end]), list(range(pf.done, end)),
                self._tickets(pf.chunks), 0, pf.horizon, self._wants_logits(job) and end == n))
        except Exception as e:
            self._prefilling.remove(pf)
            self._fail(job, e)
            return
        pf.done = end
        self.trace.emit("prefill_chunk", request=rid, done=end, total=n)
        if end == n:
            self._prefilling.remove(pf)
            self.trace.emit("prefill_accepted", request=rid, chunks=pf.chunks,
                            hops_per_prefill=self.cfg.num_layers * max(0, self.world - 1))
            self._emit_token(ActiveRequest(job=job, chunks=pf.chunks, next_position=n), resp.token)

    def _abort_started(self, job: Job) -> None:
        """A request that holds KV but produced no token yet, whose client went away."""
        self.sched.complete(job.request_id)
        if job.holds_session:
            self._busy.discard(job.session_id)
            job.holds_session = False
        self.run_command(P.ReleaseRequest(job.request_id))
        self.ledger.release(job.request_id)
        self.metrics.bump("aborted")
        self.trace.emit("aborted", request=job.request_id, completion_tokens=0)
        if job.done:
            job.done({"request_id": job.request_id, "tokens": [],
                      "prompt_tokens": len(job.prompt_ids), "finish_reason": "abort"})

    def _append(self, job: Job) -> None:
        sess = self.sessions.get(job.session_id)
        if sess is None:
            raise AdmissionError(f"unknown or expired session {job.session_id!r}")
        if job.session_id in self._busy:
            raise AdmissionError(f"session {job.session_id!r} already has a request in flight")
        rid = sess.request_id
        # the session's last generated token was never fed back, so it has no KV yet: it leads
        # the continuation segment (the context is exactly the text the client has seen)
        seg = [sess.last_token] + list(job.prompt_ids)
        n = len(seg)
        positions = list(range(sess.context_len, sess.context_len + n))
        tickets = self._tickets(sess.chunks)
        # KV bytes of the segment and its decode growth join the session's ledger entry
        tot = sum(tickets)
        per = [self._pages(c + -(-max(1, job.max_tokens) * t // tot) + 1) * self.cfg.num_layers *
               self.bytes_per_token_layer for c, t in zip(continuation_split(n, tickets), tickets)]
        self.ledger.try_reserve(rid, per)   # CapacityError: requeued while others hold KV
        self.trace.emit("kv_reserved", request=rid, bytes=per)
        self._busy.add(job.session_id)      # own the session only once admitted
        job.holds_session = True
        horizon = max(1, job.max_tokens) + (self.args.session_continuation_tokens if job.keep_kv else 0)
        resp = self.run_command(P.StationaryContinuation(rid, seg, positions, tickets, 0, horizon,
                                                         self._wants_logits(job)))
        if self.args.export_logits_dir and self.worker.last_logits is not None:
            export_logits_dump(self._dump_dir(rid), {"continuation_last_logits": self.worker.last_logits}, {
                "mode": "service", "device": "distributed-workers", "request_id": rid,
                "append_request_id": job.request_id, "session_id": job.session_id,
                "domains": self.world, "layers": self.cfg.num_layers, "tickets": tickets,
                "capacity_tickets": tickets, "starter_domain": 0,
                "continuation_offsets_by_domain": self._offsets_by_domain(n, tickets),
                "continuation_base_position": sess.context_len, "continuation_tokens": n,
                "continuation_argmax": int(resp.token)})
        job.request_id = rid
        req = ActiveRequest(job=job, chunks=sess.chunks, next_position=sess.context_len + n)
        self._emit_token(req, resp.token)

    def _dump_dir(self, request_id: int) -> str:
        import os
        return os.path.join(self.args.export_logits_dir, f"request_{request_id}")

    def _snapshot_logits(self):
        lg = self.worker.last_logits
        return None if lg is None else lg.detach().float().reshape(-1).cpu().clone()

    def _offsets_by_domain(self, n: int, tickets: Sequence[int]) -> List[List[int]]:
        """Segment offsets stored by each rank (the engine's contiguous continuation split)."""
        out, o = [], 0
        for c in continuation_split(n, tickets):
            out.append(list(range(o, o + c)))
            o += c
        return out

    def continuation_e2e(self, request_id: int, prompt_ids: Sequence[int], segment: Sequence[int],
                         max_tokens: int, tickets: Optional[Sequence[int]] = None) -> dict:
        """The reference's experimental continuation run (coordinator.rs:1973-2245, CLI
        `--continuation-segment`): prefill the prompt (vanilla layout, `--chunk-sizes` or an even
        split), decode its first token, prefill `segment` as a continuation right after it,
        then greedy-decode `max_tokens - 2` more. Logits of the prefill, of the decode step and
        of the continuation go to `export_logits_dir` when it is set."""
        if max_tokens < 2:
            raise AdmissionError("continuation E2E needs --max-tokens >= 2")
        if not segment:
            raise AdmissionError("continuation E2E needs a non-empty segment")
        if self.args.strategy != "vanilla":
            raise AdmissionError("--continuation-segment requires the vanilla ring strategy")
        L, n, N = len(prompt_ids), len(segment), self.world
        if self.args.chunk_sizes:
            chunks = list(self.args.chunk_sizes)
            if len(chunks) != N or sum(chunks) != L:
                raise AdmissionError(f"--chunk-sizes {chunks} must match domains {N} and prompt "
                                     f"length {L}")
        else:
            c = max(1, -(-L // N))
            chunks = [max(0, min(L, (i + 1) * c) - min(L, i * c)) for i in range(N)]
            chunks[-1] = L - sum(chunks[:-1])
        if 0 in chunks:
            raise AdmissionError("continuation E2E requires a non-zero chunk per domain")
        if not tickets:
            known = [int(c) for c in self.capacities_mb if c != UNKNOWN_CAPACITY]
            tickets = [max(1, int(c)) for c in self.capacities_mb] if len(known) == N else [1] * N
        if len(tickets) != N:
            raise AdmissionError(f"{len(tickets)} capacity tickets for {N} domains")
        tickets = [int(t) for t in tickets]
        rid = int(request_id)
        horizon = max_tokens + self.args.session_continuation_tokens
        resp = self.run_command(P.Prefill(rid, list(prompt_ids), chunks, "vanilla", horizon,
                                          tickets, True))
        prefill_logits = self._snapshot_logits()
        decode_token = int(resp.token)
        generated = [decode_token]
        try:
            d = self.run_command(P.Decode(rid, decode_token))
            decode_logits = self._snapshot_logits()  # the decode graph reuses its buffer
            decode_argmax = int(d.token)
            positions = list(range(L + 1, L + 1 + n))
            c = self.run_command(P.StationaryContinuation(rid, list(segment), positions, tickets, 0,
                                                          max_tokens))
            cont_logits = self._snapshot_logits()
            nxt = int(c.token)
            generated.append(nxt)
            for _ in range(max_tokens - 2):
                nxt = int(self.run_command(P.Decode(rid, nxt)).token)
                generated.append(nxt)
        finally:
            self.run_command(P.ReleaseRequest(rid))
        meta = {"mode": "production-nvlink", "device": "distributed-workers", "request_id": rid,
                "domains": N, "layers": self.cfg.num_layers, "tickets": tickets,
                "capacity_tickets": tickets, "prefix_splits": chunks, "starter_domain": 0,
                "continuation_offsets_by_domain": self._offsets_by_domain(n, tickets),
                "decode_token": decode_token, "prefill_argmax": decode_token,
                "decode_argmax": decode_argmax, "continuation_argmax": generated[1],
                "generated_ids": generated}
        if self.args.export_logits_dir:
            arts = {k: v for k, v in (("prefill_last_logits", prefill_logits),
                                      ("decode_logits", decode_logits),
                                      ("continuation_last_logits", cont_logits)) if v is not None}
            export_logits_dump(self.args.export_logits_dir, arts, meta)
        return meta

    def _eos(self, job: Job) -> set:
        """Tokens that end a request: its stop ids, else the model's EOS ids; none with
        ignore_eos."""
        if job.ignore_eos:
            return set()
        return set(job.stop_ids or self.args.eos_ids or [])

    def _finish_reason(self, req: ActiveRequest, tok: int) -> Optional[str]:
        """"stop" on an EOS / stop id or once the generated text contains a stop string (checked
        on a tail window of tokens that covers the longest one), "length" at max_tokens."""
        job = req.job
        if tok in self._eos(job):
            return "stop"
        if job.stop_strings and self.tok is not None:
            window = max(len(x) for x in job.stop_strings) + 8
            tail = self.tok.decode(req.generated[-window:])
            if any(x and x in tail for x in job.stop_strings):
                return "stop"
        if len(req.generated) >= job.max_tokens:
            return "length"
        return None

    def _emit_token(self, req: ActiveRequest, argmax_token: int) -> None:
        job = req.job
        tok = argmax_token
        if job.temperature > 0 and self.worker.last_logits is not None:
            logits = self.worker.last_logits
            tok = sample_token(logits[0] if logits.dim() > 1 else logits, job.temperature, job.top_p)
        req.generated.append(tok)
        req.next_token = tok
        if req.first_token_at is None:
            req.first_token_at = time.time()
            self.metrics.observe("ttft_seconds", req.first_token_at - job.enqueued_at)
            self.trace.emit("first_token", request=job.request_id,
                            ttft_s=req.first_token_at - job.enqueued_at)
        req.finish_reason = self._finish_reason(req, tok)
        if job.on_token:
            job.on_token(tok, req.finish_reason)
        if req.finish_reason:
            self._finish(req)
        elif job.request_id not in self.sched.active:
            self.sched.activate(req)

    def _finish(self, req: ActiveRequest) -> None:
        """Session rules (coordinator.rs:1743-1810, 2770-2830): a keep_kv request registers or
        advances its session and keeps the KV; an append without keep_kv ends the session it
        rode on; any other request releases its KV."""
        job = req.job
        self.sched.complete(job.request_id)
        if job.holds_session:
            self._busy.discard(job.session_id)
            job.holds_session = False
        if job.keep_kv:
            ctx = req.next_position + len(req.generated) - 1
            self.sessions[job.session_id] = Session(job.request_id, ctx, req.chunks, req.next_token)
            # the last generated token has no KV yet: the next append starts with it
        else:
            if job.append:
                self.sessions.pop(job.session_id, None)
            self.run_command(P.ReleaseRequest(job.request_id))
            released = self.ledger.release(job.request_id)
            self.trace.emit("kv_released", request=job.request_id, bytes=released)
        self.metrics.bump("completed")
        if req.finish_reason == "abort":
            self.metrics.bump("aborted")
        self.metrics.bump("tokens", len(req.generated))
        self.metrics.observe("request_latency_seconds", time.time() - job.enqueued_at)
        self.trace.emit("completed", request=job.request_id, completion_tokens=len(req.generated),
                        finish_reason=req.finish_reason,
                        decode_hops=self.cfg.num_layers * max(0, self.world - 1) * max(0, len(req.generated) - 1))
        if job.done:
            job.done({"request_id": job.request_id, "tokens": list(req.generated),
                      "prompt_tokens": len(job.prompt_ids), "finish_reason": req.finish_reason})

    def _fail(self, job: Job, err: Exception) -> None:
        """A failed request leaves no half-live KV: its rows on the workers and its ledger bytes
        are released, and a failed append drops the session it rode on
        (coordinator.rs:2636-2652). A request rejected before it owned its session (unknown or
        busy session, a keep_kv id that already holds KV) touches no session."""
        self.metrics.bump("failed")
        self.sched.complete(job.request_id)
        rid = job.request_id
        if job.holds_session:
            self._busy.discard(job.session_id)
            job.holds_session = False
            if job.append:
                sess = self.sessions.pop(job.session_id, None)
                rid = sess.request_id if sess is not None else rid
        try:
            self.run_command(P.ReleaseRequest(rid))
        except (ProtocolError, RuntimeError, OSError) as e:  # a rank is gone: nothing to free
            self.trace.emit("release_failed", request=rid, error=str(e))
        self.ledger.release(rid)
        self.trace.emit("failed", request=job.request_id, error=str(err))
        if job.done:
            job.done({"request_id": job.request_id, "error": str(err),
                      "status": 400 if isinstance(err, (AdmissionError, CapacityError)) else 500})

    # ------------------------------------------------------------------ iteration
    def _expire_sessions(self) -> None:
        """Release sessions idle longer than session_ttl_s (their KV would otherwise stay
        resident until an append without keep_kv ends them)."""
        now = time.time()
        for sid, sess in list(self.sessions.items()):
            if sid in self._busy or now - sess.last_used <= self.args.session_ttl_s:
                continue
            del self.sessions[sid]
            try:
                self.run_command(P.ReleaseRequest(sess.request_id))
            except (ProtocolError, RuntimeError, OSError) as e:
                self.trace.emit("release_failed", request=sess.request_id, error=str(e))
            self.ledger.release(sess.request_id)
            self.trace.emit("session_expired", session=sid, request=sess.request_id)

    def iteration(self) -> bool:
        did = False
        if self.args.session_ttl_s > 0 and self.sessions:
            self._expire_sessions()
        while self.sched.has_capacity():
            job = self.sched.pop_pending()
            if job is None:
                break
            did = True
            if job.cancelled:   # the client left while the request was queued
                self.metrics.bump("aborted")
                self.trace.emit("aborted", request=job.request_id, completion_tokens=0)
                if job.done:
                    job.done({"request_id": job.request_id, "tokens": [],
                              "prompt_tokens": len(job.prompt_ids), "finish_reason": "abort"})
                continue
            try:
                self._prefill(job)
            except CapacityError as e:
                if self.sched.active:
                    self.sched.requeue_front(job)   # wait for KV to be released
                    break
                self._fail(job, e)
            except Exception as e:
                self._fail(job, e)
        for pf in list(self._prefilling):
            did = True
            self._advance_chunked(pf)
        active = self.sched.active_list()
        for a in [a for a in active if a.job.cancelled]:
            # the client went away: finish now (KV released, or kept for a keep_kv session)
            a.finish_reason = "abort"
            self._finish(a)
            did = True
        active = [a for a in active if not a.job.cancelled]
        step = max(1, int(self.args.decode_batch_limit))
        for b0 in range(0, len(active), step):
            did = True
            self._decode_rows(active[b0:b0 + step])
        return did

    def _decode_rows(self, active: List[ActiveRequest]) -> None:
        """One engine decode step for up to `decode_batch_limit` active requests."""
        if active:
            pairs = [[a.job.request_id, a.next_token] for a in active]
            try:
                # greedy-only batches ask for no logits, so the ranks may split the LM head
                want = any(a.job.temperature > 0 for a in active)
                resp = self.run_command(P.DecodeBatch(pairs, want))
            except Exception as e:
                for a in active:
                    self._fail(a.job, e)
                return
            logits = self.worker.last_logits
            for i, (a, (_, tok)) in enumerate(zip(active, resp.request_tokens)):
                if a.job.temperature > 0 and logits is not None:
                    tok = sample_token(logits[i], a.job.temperature, a.job.top_p)
                a.generated.append(tok)
                a.next_token = tok
                a.finish_reason = self._finish_reason(a, tok)
                if a.job.on_token:
                    a.job.on_token(tok, a.finish_reason)
                if a.finish_reason:
                    self._finish(a)

    def run_forever(self) -> None:
        while not self._stop.is_set():
            if not self.iteration():
                self.sched.wait_for_work(0.02)

    # ------------------------------------------------------------------ convenience (CLI batch)
    def generate(self, prompt_ids: Sequence[int], max_tokens: int = 20, temperature: float = 0.0,
                 top_p: float = 1.0, session_id=None, keep_kv=False, append=False) -> dict:
        out = {}
        job = Job(request_id=self.next_request_id(), prompt_ids=list(prompt_ids),
                  max_tokens=max_tokens, temperature=temperature, top_p=top_p,
                  session_id=session_id, keep_kv=keep_kv, append=append,
                  done=lambda r: out.update(r))
        self.submit(job)
        while not out:
            self.iteration()
        return out
