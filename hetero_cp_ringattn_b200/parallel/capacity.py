"""Capacity-weighted chunking and KV byte admission.

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

from ..errors import CapacityError, RingError

UNKNOWN_CAPACITY = (1 << 64) - 1
DEFAULT_ACTIVATION_RESERVE_MB = 1536


def allocate_by_capacity(prompt_len: int, capacities: Sequence[int]) -> list:
    n = len(capacities)
    if n == 0:
        raise RingError("capacities must not be empty")
    if prompt_len < n:
        raise RingError(f"prompt_len ({prompt_len}) must be >= num_domains ({n}) to give each "
                        "domain at least 1 token")
    caps = [int(c) for c in capacities]
    total = sum(caps)
    if total == 0:
        base, rem = divmod(prompt_len, n)
        return [base + (1 if i < rem else 0) for i in range(n)]
    chunks = [(prompt_len * c) // total for c in caps]
    consumed = 0
    for i, c in enumerate(chunks):
        if c == 0:
            chunks[i] = 1
        consumed += chunks[i]
    if consumed > prompt_len:
        excess = consumed - prompt_len
        while excess > 0:
            # max_by_key picks the last maximal element in Rust's iterator semantics
            mx = max(chunks)
            idx = max(i for i, v in enumerate(chunks) if v == mx)
            if chunks[idx] > 1:
                chunks[idx] -= 1
                excess -= 1
            else:
                break
    remainder = prompt_len - sum(chunks)
    if remainder > 0:
        fr = [(i, prompt_len * c / total - chunks[i]) for i, c in enumerate(caps)]
        fr.sort(key=lambda t: -t[1])  # stable: ties keep index order
        for i, _ in fr[:remainder]:
            chunks[i] += 1
    assert sum(chunks) == prompt_len
    return chunks


def equal_chunks(prompt_len: int, n: int) -> list:
    """Equal split with ceil(L/N) leading chunks (the coordinator's default tier)."""
    if n <= 0:
        raise RingError("need at least one domain")
    if prompt_len < n:
        raise RingError(f"prompt_len ({prompt_len}) must be >= num_domains ({n})")
    size = -(-prompt_len // n)
    out = []
    left = prompt_len
    for i in range(n):
        c = min(size, left - (n - i - 1))
        out.append(c)
        left -= c
    return out


def chunks_from_ratio(prompt_len: int, ratio: Sequence[int]) -> list:
    """Integer ratio override, e.g. 5:5:1 -> capacity tickets [5, 5, 1]."""
    return allocate_by_capacity(prompt_len, list(ratio))


def chunk_sizes(prompt_len: int, num_domains: int, *, explicit: Optional[Sequence[int]] = None,
                capacities_mb: Optional[Sequence[int]] = None, capacity_aware: bool = False,
                ratio: Optional[Sequence[int]] = None,
                activation_reserve_mb: int = DEFAULT_ACTIVATION_RESERVE_MB) -> list:
    if explicit:
        ex = [int(x) for x in explicit]
        if len(ex) != num_domains:
            raise RingError(f"--chunk-sizes has {len(ex)} entries for {num_domains} domains")
        if sum(ex) != prompt_len:
            raise RingError(f"--chunk-sizes sum {sum(ex)} != prompt length {prompt_len}")
        if any(x < 1 for x in ex):
            raise RingError("every domain needs at least one token")
        return ex
    if ratio:
        if len(ratio) != num_domains:
            raise RingError(f"ratio has {len(ratio)} entries for {num_domains} domains")
        return chunks_from_ratio(prompt_len, ratio)
    if capacity_aware and capacities_mb:
        caps = [0 if c == UNKNOWN_CAPACITY else max(0, int(c) - activation_reserve_mb)
                for c in capacities_mb]
        return allocate_by_capacity(prompt_len, caps)
    return equal_chunks(prompt_len, num_domains)


def round_chunks_to_tile(chunks: Sequence[int], tile: int) -> list:
    """Move boundaries to multiples of `tile` (the last rank keeps the tail), keeping >= 1 token.

    Used for kernel-friendly splits; the sum is preserved."""
    total = sum(chunks)
    n = len(chunks)
    bounds = [0]
    acc = 0
    for c in chunks[:-1]:
        acc += c
        b = int(round(acc / tile)) * tile
        b = max(b, bounds[-1] + 1)
        bounds.append(min(b, total - (n - len(bounds))))
    bounds.append(total)
    return [bounds[i + 1] - bounds[i] for i in range(n)]


# --------------------------------------------------------------------------- admission
@dataclasses.dataclass
class KvByteAdmission:
    bytes_per_token_per_layer: int
    required_bytes_per_domain: list


def capacity_mb_to_bytes(capacity_mb_by_domain: Sequence[int]) -> list:
    out = []
    for d, mb in enumerate(capacity_mb_by_domain):
        if mb == UNKNOWN_CAPACITY:
            raise CapacityError(f"KV byte admission domain {d} reported unknown capacity")
        if mb * 1024 * 1024 >= (1 << 64):
            raise CapacityError(f"KV byte admission domain {d} capacity {mb} MB cannot be "
                                "represented in bytes")
        out.append(int(mb) * 1024 * 1024)
    return out


def admit_reserved_kv_bytes(layer_capacities_by_domain: Sequence[Sequence[int]],
                            budget_bytes_by_domain: Sequence[int], num_kv_heads: int,
                            head_dim: int, element_size_bytes: int) -> KvByteAdmission:
    domains = len(layer_capacities_by_domain)
    if domains == 0:
        raise CapacityError("KV byte admission requires at least one domain")
    if len(budget_bytes_by_domain) != domains:
        raise CapacityError(f"KV byte admission has {domains} domains but "
                            f"{len(budget_bytes_by_domain)} byte budgets")
    layers = len(layer_capacities_by_domain[0])
    if layers == 0:
        raise CapacityError("KV byte admission requires at least one layer")
    for d, caps in enumerate(layer_capacities_by_domain):
        if len(caps) != layers:
            raise CapacityError(f"KV byte admission domain {d} has {len(caps)} layers, "
                                f"expected {layers}")
    if num_kv_heads == 0 or head_dim == 0 or element_size_bytes == 0:
        raise CapacityError("KV byte admission requires non-zero KV heads, head dimension, and "
                            "element bytes")
    bpt = 2 * num_kv_heads * head_dim * element_size_bytes
    req = []
    for d, caps in enumerate(layer_capacities_by_domain):
        need = sum(int(c) for c in caps) * bpt
        if need >= (1 << 64):
            raise CapacityError("KV byte admission arithmetic overflow")
        if need > budget_bytes_by_domain[d]:
            raise CapacityError(f"KV byte admission domain {d} requires {need} bytes, budget is "
                                f"{budget_bytes_by_domain[d]} bytes")
        req.append(need)
    return KvByteAdmission(bpt, req)


class KvLedger:
    """Per-domain KV byte ledger with reserve/release (coordinator.rs:784-871).

    `try_reserve` is all-or-nothing; `ReservationGuard` rolls back if the prefill fails."""

    def __init__(self, budgets_bytes: Sequence[int]):
        self.budgets = [int(b) for b in budgets_bytes]
        self.used = [0] * len(self.budgets)
        self.by_request: dict = {}

    def try_reserve(self, request_id: int, bytes_per_domain: Sequence[int]) -> None:
        if len(bytes_per_domain) != len(self.budgets):
            raise CapacityError("reservation domain count mismatch")
        for d, b in enumerate(bytes_per_domain):
            if self.used[d] + b > self.budgets[d]:
                raise CapacityError(f"KV reservation for request {request_id} exceeds domain {d} "
                                    f"budget: used {self.used[d]} + {b} > {self.budgets[d]}")
        prev = self.by_request.get(request_id, [0] * len(self.budgets))
        for d, b in enumerate(bytes_per_domain):
            self.used[d] += b
            prev[d] += b
        self.by_request[request_id] = prev

    def release(self, request_id: int) -> list:
        held = self.by_request.pop(request_id, None)
        if held is None:
            return [0] * len(self.budgets)
        for d, b in enumerate(held):
            self.used[d] -= b
        return held

    def free_bytes(self) -> list:
        return [b - u for b, u in zip(self.budgets, self.used)]


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


def continuation_split(segment_len: int, tickets: Sequence[int]) -> List[int]:
    """Tokens of a continuation segment per rank, in rank order (the segment is cut into
    contiguous pieces, so each rank's new rows stay position-ordered). Long segments follow the
    capacity tickets (largest remainder); a segment shorter than the number of ranks gives one
    token each to the ranks with the most tickets (ties: lower rank)."""
    n = len(tickets)
    if segment_len >= n:
        return allocate_by_capacity(segment_len, list(tickets))
    order = sorted(range(n), key=lambda r: (-int(tickets[r]), r))
    out = [0] * n
    for r in order[:segment_len]:
        out[r] = 1
    return out
