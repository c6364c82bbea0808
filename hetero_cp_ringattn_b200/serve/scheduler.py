"""Iterative batch scheduler: FIFO pending queue, active map, bounded decode batch.

Parity: rust/src/distributed/scheduler.rs:18-160 (`ActiveRequest`, `BatchScheduler` with
`enqueue`, admission up to `max_batch_size` (default 4), removal on completion) and the
coordinator's iteration order (coordinator.rs:2563-2916: pending -> prefill (serial) -> active;
each iteration runs one decode step for the active requests). The queue and the active set
live in the native host library.
"""

from __future__ import annotations

import dataclasses
import time
from typing import Callable, Dict, List, Optional

from ..host import lib


@dataclasses.dataclass
class Job:
    request_id: int
    prompt_ids: List[int]
    max_tokens: int = 20
    temperature: float = 0.0
    top_p: float = 1.0
    session_id: Optional[str] = None
    keep_kv: bool = False
    append: bool = False
    stop_ids: Optional[List[int]] = None
    stop_strings: Optional[List[str]] = None   # text stop sequences (excluded from the output)
    ignore_eos: bool = False      # generate exactly max_tokens (benchmarks)
    on_token: Optional[Callable[[int, Optional[str]], None]] = None   # (token, finish_reason)
    done: Optional[Callable[[dict], None]] = None
    enqueued_at: float = dataclasses.field(default_factory=time.time)
    holds_session: bool = False   # set by the coordinator while this job owns its session
    cancelled: bool = False       # set by the API when the client went away: stop generating


@dataclasses.dataclass
class ActiveRequest:
    job: Job
    chunks: List[int]
    generated: List[int] = dataclasses.field(default_factory=list)
    next_token: int = 0
    next_position: int = 0
    first_token_at: Optional[float] = None
    finish_reason: Optional[str] = None


class BatchScheduler:
    """Admission order and the active set are kept by the native scheduler core
    (`csrc/host/scheduler.cpp`, thread safe); this wrapper holds the request objects by id."""

    def __init__(self, max_batch_size: int = 4):
        self._core = lib().BatchSchedulerCore(int(max_batch_size))
        self.max_batch_size = int(max_batch_size)
        self._pending: Dict[int, Job] = {}
        self.active: Dict[int, ActiveRequest] = {}

    def enqueue(self, job: Job) -> None:
        self._pending[job.request_id] = job
        self._core.enqueue(job.request_id)

    def has_capacity(self) -> bool:
        return self._core.has_capacity()

    def pop_pending(self) -> Optional[Job]:
        rid = self._core.pop_pending()
        return None if rid is None else self._pending.pop(rid)

    def requeue_front(self, job: Job) -> None:
        self._pending[job.request_id] = job
        self._core.requeue_front(job.request_id)

    def activate(self, req: ActiveRequest) -> None:
        self.active[req.job.request_id] = req
        self._core.activate(req.job.request_id)

    def occupy(self, request_id: int) -> None:
        """Take a batch slot for a request that is not decoding yet (a chunked prefill)."""
        self._core.activate(request_id)

    def complete(self, request_id: int) -> Optional[ActiveRequest]:
        self._core.complete(request_id)
        return self.active.pop(request_id, None)

    def active_list(self) -> List[ActiveRequest]:
        return [self.active[i] for i in self._core.active() if i in self.active]

    def wait_for_work(self, timeout: float = 0.05) -> None:
        self._core.wait_for_work(float(timeout))

    @property
    def queued(self) -> int:
        return self._core.queued
