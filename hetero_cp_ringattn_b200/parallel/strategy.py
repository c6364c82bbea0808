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
The layouts are computed by the native host library (`csrc/host/layout.cpp`).
"""

from __future__ import annotations

import enum
from typing import Sequence

import numpy as np

from ..host import lib


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
    return lib().build_assignment([int(c) for c in chunks], strategy.value)


def build_domain_positions(assignment: np.ndarray, num_domains: int | None = None) -> list:
    """Ordered global positions owned by each rank (local storage order)."""
    return list(lib().build_domain_positions(np.asarray(assignment, dtype=np.int64),
                                             -1 if num_domains is None else int(num_domains)))


def build_inverse_perm(assignment: np.ndarray) -> np.ndarray:
    """inverse[p] = index of global position p inside concat(rank0 tokens, rank1 tokens, ...)."""
    return lib().build_inverse_perm(np.asarray(assignment, dtype=np.int64))


def layout_positions(chunks: Sequence[int], strategy: "RingStrategy | str") -> list:
    """Convenience: per-rank global position arrays for a chunk split and strategy."""
    return build_domain_positions(build_assignment(chunks, strategy), num_domains=len(chunks))


def causal_work(positions: Sequence[np.ndarray]) -> list:
    """Causal attention work per rank (number of (q, k) pairs with k <= q), for load reports."""
    return [int(np.sum(np.asarray(p, dtype=np.int64) + 1)) for p in positions]
