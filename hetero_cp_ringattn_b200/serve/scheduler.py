"""Iterative batch scheduler: FIFO pending queue, active map, bounded decode batch.

Parity: rust/src/distributed/scheduler.rs:18-160 (`ActiveRequest`, `BatchScheduler` with
`enqueue`, admission up to `max_batch_size` (default 4), removal on completion) and the
coordinator's iteration order (coordinator.rs:2563-2916: pending -> prefill (serial) -> active;
each iteration runs one decode step for the active requests).
"""

from __future__ import annotations

import collections
import dataclasses
import threading
import time
from typing import Any, Callable, Deque, Dict, List, Optional


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
    on_token: Optional[Callable[[int, Optional[str]], None]] = None   # (token, finish_reason)
    done: Optional[Callable[[dict], None]] = None
    enqueued_at: float = dataclasses.field(default_factory=time.time)


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
    def __init__(self, max_batch_size: int = 4):
        if max_batch_size < 1:
            raise ValueError("max_batch_size must be >= 1")
        self.max_batch_size = max_batch_size
        self.pending: Deque[Job] = collections.deque()
        self.active: Dict[int, ActiveRequest] = {}
        self.lock = threading.Lock()
        self.cv = threading.Condition(self.lock)

    def enqueue(self, job: Job) -> None:
        with self.cv:
            self.pending.append(job)
            self.cv.notify_all()

    def has_capacity(self) -> bool:
        return len(self.active) < self.max_batch_size

    def pop_pending(self) -> Optional[Job]:
        with self.lock:
            if self.pending and self.has_capacity():
                return self.pending.popleft()
            return None

    def requeue_front(self, job: Job) -> None:
        with self.lock:
            self.pending.appendleft(job)

    def activate(self, req: ActiveRequest) -> None:
        with self.lock:
            self.active[req.job.request_id] = req

    def complete(self, request_id: int) -> Optional[ActiveRequest]:
        with self.lock:
            return self.active.pop(request_id, None)

    def active_list(self) -> List[ActiveRequest]:
        with self.lock:
            return list(self.active.values())

    def wait_for_work(self, timeout: float = 0.05) -> None:
        with self.cv:
            if not self.pending and not self.active:
                self.cv.wait(timeout)

    @property
    def queued(self) -> int:
        return len(self.pending)
