"""Token -> rank layouts for context parallelism: vanilla, striped and zigzag.

Parity: rust/src/model/attention/strategy.rs:16-146 (`RingSchedulingStrategy`,
`build_assignment`, `build_domain_positions`, `build_inverse_perm`). The three layouts are kept
exactly as the reference defines them because the coordinator, the workers' RoPE positions and
the attention kernels' causal skip all derive from the same assignment:

  * vanilla: contiguous chunks in rank order;
  * striped: weighted round-robin - one slot per rank with remaining quota, repeated;
  * zigzag:  rank i owns a prefix segment of ceil(c_i/2) tokens (prefixes in rank order) and a
             suffix segment of floor(c_i/2) tokens (suffixes in reverse rank order).

Every layout preserves exact attention; the kernels only ever see per-token global positions.
"""

from __future__ import annotations

import enum
from typing import Sequence

import numpy as np


class RingStrategy(enum.Enum):
    VANILLA = "vanilla"
    STRIPED = "striped"
    ZIGZAG = "zigzag"

    @classmethod
    def parse(cls, s: "str | RingStrategy") -> "RingStrategy":
        if isinstance(s, RingStrategy):
            return s
        try:
            return cls(s.lower())
        except ValueError:
            raise ValueError(f"unknown ring strategy {s!r} (vanilla|striped|zigzag)") from None

    @classmethod
    def all(cls) -> list:
        return [cls.VANILLA, cls.STRIPED, cls.ZIGZAG]


def build_assignment(chunks: Sequence[int], strategy: "RingStrategy | str") -> np.ndarray:
    """Return `a` with a[p] = rank owning global position p; rank i owns chunks[i] positions."""
    strategy = RingStrategy.parse(strategy)
    chunks = [int(c) for c in chunks]
    seq_len = sum(chunks)
    n = len(chunks)
    if strategy is RingStrategy.VANILLA:
        return np.repeat(np.arange(n, dtype=np.int64), chunks)
    if strategy is RingStrategy.STRIPED:
        remaining = list(chunks)
        sched = []
        while any(c > 0 for c in remaining):
            for d in range(n):
                if remaining[d] > 0:
                    sched.append(d)
                    remaining[d] -= 1
        sched = np.asarray(sched, dtype=np.int64)
        if seq_len == 0:
            return sched
        return sched[np.arange(seq_len) % len(sched)]
    # zigzag
    prefix = [c - c // 2 for c in chunks]
    suffix = [c // 2 for c in chunks]
    out = np.empty(seq_len, dtype=np.int64)
    pos = 0
    for d in range(n):
        out[pos:pos + prefix[d]] = d
        pos += prefix[d]
    for d in reversed(range(n)):
        out[pos:pos + suffix[d]] = d
        pos += suffix[d]
    return out


def build_domain_positions(assignment: np.ndarray, num_domains: int | None = None) -> list:
    """Ordered global positions owned by each rank (local storage order)."""
    assignment = np.asarray(assignment)
    n = int(assignment.max()) + 1 if num_domains is None and assignment.size else (num_domains or 0)
    return [np.nonzero(assignment == d)[0].astype(np.int64) for d in range(n)]


def build_inverse_perm(assignment: np.ndarray) -> np.ndarray:
    """inverse[p] = index of global position p inside concat(rank0 tokens, rank1 tokens, ...)."""
    positions = build_domain_positions(assignment)
    inverse = np.empty(len(assignment), dtype=np.int64)
    off = 0
    for pos in positions:
        inverse[pos] = np.arange(off, off + len(pos), dtype=np.int64)
        off += len(pos)
    return inverse


def layout_positions(chunks: Sequence[int], strategy: "RingStrategy | str") -> list:
    """Convenience: per-rank global position arrays for a chunk split and strategy."""
    return build_domain_positions(build_assignment(chunks, strategy), num_domains=len(chunks))


def causal_work(positions: Sequence[np.ndarray]) -> list:
    """Causal attention work per rank (number of (q, k) pairs with k <= q), for load reports."""
    return [int(np.sum(np.asarray(p, dtype=np.int64) + 1)) for p in positions]
