"""Counts launches of this package's own kernels (eager calls and CUDA-graph replays).

Every front-end that launches a native kernel calls `count(n)`; a captured decode graph records how
many launches it contains and adds that number on every replay.
"""

from __future__ import annotations

_count = 0
_capturing = 0
_captured = 0


def count(n: int = 1) -> None:
    global _count, _captured
    if _capturing:
        _captured += n
    else:
        _count += n


def total() -> int:
    return _count


def reset() -> None:
    global _count
    _count = 0


class capture:
    """Context manager used while a CUDA graph is captured: launches are recorded, not counted."""

    def __enter__(self):
        global _capturing, _captured
        _capturing += 1
        _captured = 0
        return self

    def __exit__(self, *exc):
        global _capturing
        _capturing -= 1
        self.launches = _captured
        return False
