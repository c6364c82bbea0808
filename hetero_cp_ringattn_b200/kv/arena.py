"""Host-side bookkeeping of the paged, position-tagged KV arena.

Parity: the reference's KV caches (rust/src/model/cache.rs:12-440: contiguous `cat` cache,
16-token block table, `update_sharded(keep)` for decode growth) and the reserved positioned shard
(rust/src/model/self_driving.rs:146-331: pre-allocated [1, Hkv, cap, D] slab with explicit
positions and capacity errors). Here the device memory is one arena per rank
([layers][pages][2][Hkv][page][D], owned by the native runtime); this module hands out pages,
tracks per-request / per-layer slot counts and the global position of every slot, and raises a
capacity error instead of growing with a copy.
"""

from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional

import numpy as np

from ..errors import CapacityError
from ..host import lib


def staging_bytes(stage_cap: int, kv_heads: int, head_dim: int) -> int:
    """Bytes of one rank's prefill KV staging buffers: two parities (layer steps alternate) of
    position-ordered bf16 K and V for every position up to `stage_cap` (the engine's
    `max_context`), [2][2][Hkv][stage_cap][D]. This is per rank whatever the number of ranks, so
    it bounds the longest context a rank can prefill: a Llama-3-8B shape (8 KV heads, head_dim
    128) at 512k positions needs 4.3 GB on every rank."""
    return 2 * 2 * int(kv_heads) * int(stage_cap) * int(head_dim) * 2


def max_staged_context(budget_bytes: int, kv_heads: int, head_dim: int) -> int:
    """Longest context whose staging buffers fit in `budget_bytes` on a rank."""
    return int(budget_bytes) // staging_bytes(1, kv_heads, head_dim)


class PageAllocator:
    """Page ids of this rank's arena, handed out and taken back by the native allocator
    (`csrc/host/pages.cpp`)."""

    def __init__(self, num_pages: int, page_size: int):
        self._a = lib().PageAllocator(int(num_pages), int(page_size))
        self.num_pages = int(num_pages)
        self.page_size = int(page_size)

    @property
    def free_pages(self) -> int:
        return self._a.free_pages

    def alloc(self, n: int, req_id: int) -> List[int]:
        return list(self._a.alloc(int(n), int(req_id)))

    def free(self, pages: List[int]) -> None:
        self._a.free([int(p) for p in pages])

    def owner_of(self, page: int) -> Optional[int]:
        o = self._a.owner_of(int(page))
        return None if o < 0 else o


@dataclasses.dataclass
class RequestKv:
    """One request's shard on this rank."""

    req_id: int
    pages: List[int]
    page_size: int
    num_layers: int
    n_prefill: int                       # slots 0..n_prefill-1 hold this rank's prompt tokens
    layer_counts: np.ndarray             # [layers] rows stored per layer (prefill + decode growth)
    slot_pos: np.ndarray                 # [layers, capacity] global position per slot (-1 empty)
    pt_device: Optional[object] = None   # int32 device tensor of the page ids

    @property
    def capacity(self) -> int:
        return len(self.pages) * self.page_size

    def check_room(self, layer: int, extra: int = 1) -> None:
        if self.layer_counts[layer] + extra > self.capacity:
            raise CapacityError(f"request {self.req_id} layer {layer}: reserved KV slab full "
                                f"({self.layer_counts[layer]} + {extra} > {self.capacity})")


class KvArenaManager:
    def __init__(self, num_pages: int, page_size: int, num_layers: int):
        self.alloc = PageAllocator(num_pages, page_size)
        self.page_size = page_size
        self.num_layers = num_layers
        self.requests: Dict[int, RequestKv] = {}

    def pages_for(self, slots: int) -> int:
        return max(1, -(-int(slots) // self.page_size))

    def reserve(self, req_id: int, n_prefill: int, capacity_slots: int,
                positions: Optional[np.ndarray] = None) -> RequestKv:
        if req_id in self.requests:
            raise CapacityError(f"request {req_id} already holds KV on this rank")
        cap = max(int(capacity_slots), int(n_prefill), 1)
        pages = self.alloc.alloc(self.pages_for(cap), req_id)
        rk = RequestKv(req_id=req_id, pages=pages, page_size=self.page_size,
                       num_layers=self.num_layers, n_prefill=int(n_prefill),
                       layer_counts=np.full(self.num_layers, int(n_prefill), dtype=np.int64),
                       slot_pos=np.full((self.num_layers, len(pages) * self.page_size), -1,
                                        dtype=np.int64))
        if positions is not None and n_prefill:
            rk.slot_pos[:, :n_prefill] = np.asarray(positions, dtype=np.int64)[None, :]
        self.requests[req_id] = rk
        return rk

    def extend(self, req_id: int, extra_slots: int) -> RequestKv:
        """Grow a request's reservation (session append) by whole pages."""
        rk = self.requests[req_id]
        need = int(rk.layer_counts.max()) + int(extra_slots)
        if need > rk.capacity:
            more = self.pages_for(need) - len(rk.pages)
            rk.pages += self.alloc.alloc(more, req_id)
            sp = np.full((rk.num_layers, len(rk.pages) * self.page_size), -1, dtype=np.int64)
            sp[:, :rk.slot_pos.shape[1]] = rk.slot_pos
            rk.slot_pos = sp
            rk.pt_device = None
        return rk

    def release(self, req_id: int) -> bool:
        rk = self.requests.pop(req_id, None)
        if rk is None:
            return False
        self.alloc.free(rk.pages)
        return True

    def get(self, req_id: int) -> RequestKv:
        if req_id not in self.requests:
            raise CapacityError(f"request {req_id} has no KV on this rank (released or unknown)")
        return self.requests[req_id]
