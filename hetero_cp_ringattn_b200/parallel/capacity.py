"""Capacity-weighted chunking and KV byte admission.

The arithmetic runs in the native host library (`csrc/host/capacity.cpp`); this module binds it.

Parity:
  * `allocate_by_capacity` is the largest-remainder method of rust/src/capacity.rs:67-150
    (floor of the proportional share, at least one token per rank, excess trimmed from the largest
    chunk, remainder handed out by descending fractional part). Kept step-for-step because chunk
    boundaries must agree with the reference for the same capacities.
  * `admit_reserved_kv_bytes` mirrors capacity.rs:227-297: 2 * Hkv * D * elem bytes per token per
    layer against per-rank byte budgets; `capacity_mb_to_bytes` rejects the unknown-capacity
    sentinel (capacity.rs:200-225).
  * `query_device_capacity_mb` replaces the nvidia-smi/rocm-smi subprocess probes
    (capacity.rs:42-65) with `torch.cuda.mem_get_info`; CPU keeps the "available RAM / 4" rule.
  * `chunk_sizes` is the coordinator's three-tier chooser (coordinator.rs:900-960): explicit
    sizes, capacity-aware (capacities minus the activation reserve), else equal ceil(L/N) splits,
    plus an integer ratio override ("5:5:1").
"""

from __future__ import annotations

import dataclasses
import os
from typing import List, Optional, Sequence

from ..host import lib

UNKNOWN_CAPACITY = (1 << 64) - 1
DEFAULT_ACTIVATION_RESERVE_MB = 1536


def allocate_by_capacity(prompt_len: int, capacities: Sequence[int]) -> list:
    return list(lib().allocate_by_capacity(int(prompt_len), [int(c) for c in capacities]))


def equal_chunks(prompt_len: int, n: int) -> list:
    """Equal split with ceil(L/N) leading chunks (the coordinator's default tier)."""
    return list(lib().equal_chunks(int(prompt_len), int(n)))


def chunks_from_ratio(prompt_len: int, ratio: Sequence[int]) -> list:
    """Integer ratio override, e.g. 5:5:1 -> capacity tickets [5, 5, 1]."""
    return allocate_by_capacity(prompt_len, ratio)


def chunk_sizes(prompt_len: int, num_domains: int, *, explicit: Optional[Sequence[int]] = None,
                capacities_mb: Optional[Sequence[int]] = None, capacity_aware: bool = False,
                ratio: Optional[Sequence[int]] = None,
                activation_reserve_mb: int = DEFAULT_ACTIVATION_RESERVE_MB) -> list:
    return list(lib().chunk_sizes(int(prompt_len), int(num_domains),
                                  [int(x) for x in (explicit or [])],
                                  [int(c) for c in (capacities_mb or [])], bool(capacity_aware),
                                  [int(r) for r in (ratio or [])], int(activation_reserve_mb)))


def continuation_split(segment_len: int, tickets: Sequence[int]) -> List[int]:
    """Tokens of a continuation segment per rank, in rank order (the segment is cut into
    contiguous pieces, so each rank's new rows stay position-ordered). Long segments follow the
    capacity tickets (largest remainder); a segment shorter than the number of ranks gives one
    token each to the ranks with the most tickets (ties: lower rank)."""
    return list(lib().continuation_split(int(segment_len), [int(t) for t in tickets]))


# --------------------------------------------------------------------------- admission
@dataclasses.dataclass
class KvByteAdmission:
    bytes_per_token_per_layer: int
    required_bytes_per_domain: list


def capacity_mb_to_bytes(capacity_mb_by_domain: Sequence[int]) -> list:
    return list(lib().capacity_mb_to_bytes([int(c) for c in capacity_mb_by_domain]))


def admit_reserved_kv_bytes(layer_capacities_by_domain: Sequence[Sequence[int]],
                            budget_bytes_by_domain: Sequence[int], num_kv_heads: int,
                            head_dim: int, element_size_bytes: int) -> KvByteAdmission:
    bpt, req = lib().admit_reserved_kv_bytes(
        [[int(c) for c in caps] for caps in layer_capacities_by_domain],
        [int(b) for b in budget_bytes_by_domain], int(num_kv_heads), int(head_dim),
        int(element_size_bytes))
    return KvByteAdmission(int(bpt), list(req))


class KvLedger:
    """Per-domain KV byte ledger with reserve/release (coordinator.rs:784-871), kept natively.

    `try_reserve` is all-or-nothing; `ReservationGuard` rolls back if the prefill fails."""

    def __init__(self, budgets_bytes: Sequence[int]):
        self._l = lib().KvLedger([int(b) for b in budgets_bytes])

    def try_reserve(self, request_id: int, bytes_per_domain: Sequence[int]) -> None:
        self._l.try_reserve(int(request_id), [int(b) for b in bytes_per_domain])

    def release(self, request_id: int) -> list:
        return list(self._l.release(int(request_id)))

    def free_bytes(self) -> list:
        return list(self._l.free_bytes())

    def holds(self, request_id: int) -> bool:
        return self._l.holds(int(request_id))

    @property
    def budgets(self) -> list:
        return list(self._l.budgets)

    @property
    def used(self) -> list:
        return list(self._l.used)


class ReservationGuard:
    def __init__(self, ledger: KvLedger, request_id: int, bytes_per_domain: Sequence[int]):
        self.ledger = ledger
        self.request_id = request_id
        ledger.try_reserve(request_id, bytes_per_domain)
        self.committed = False

    def commit(self) -> None:
        self.committed = True

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        if exc_type is not None or not self.committed:
            self.ledger.release(self.request_id)
        return False


# --------------------------------------------------------------------------- device probes
def query_device_capacity_mb(device: str = "cuda") -> int:
    if device.startswith("cuda"):
        try:
            import torch
            if torch.cuda.is_available():
                idx = torch.device(device).index
                free, _ = torch.cuda.mem_get_info(idx if idx is not None else torch.cuda.current_device())
                return int(free // (1024 * 1024))
        except (RuntimeError, ValueError) as e:  # no usable device: capacity unknown
            import logging
            logging.getLogger("hcp.capacity").warning("capacity probe of %s failed: %s", device, e)
        return UNKNOWN_CAPACITY
    return _available_ram_mb() // 4


def _available_ram_mb() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) // 1024
    except OSError:
        pass
    try:
        return (os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_AVPHYS_PAGES")) // (1024 * 1024)
    except (ValueError, OSError):
        return 0
