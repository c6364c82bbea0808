"""Capacity-weighted placement of decode-time KV growth.

Parity: `FrozenKvAssigneeSchedule` and `stationary_layer_starters` of
rust/src/model/self_driving.rs:12-144. The schedule decides which rank stores the K/V of each
(decode token, layer) unit: per-rank quotas by largest remainder over the capacity tickets, then a
smooth weighted round-robin sequence, read with a per-request phase (request_id mod total). The
algorithm is reproduced step for step because coordinator and workers must derive the same owner
for every unit without talking to each other.

On B200 the reference's serial hop-by-hop packet walk is replaced by parallel per-rank partial
attention plus an (O, LSE) combine, so "starter"/"finisher" no longer route compute; the starter
sequence is still derived (and validated) for protocol parity.
"""

from __future__ import annotations

from typing import Optional, Sequence

from ..errors import RingError


class FrozenKvAssigneeSchedule:
    def __init__(self, capacity_tickets: Sequence[int], request_id: int, total_kv_units: int):
        if len(capacity_tickets) == 0:
            raise RingError("KV assignee schedule requires at least one worker")
        if total_kv_units == 0:
            raise RingError("KV assignee schedule requires at least one KV unit")
        cap_sum = sum(int(t) for t in capacity_tickets)
        if cap_sum == 0:
            raise RingError("KV assignee schedule requires non-zero capacity")
        total = int(total_kv_units)
        counts = []
        remainders = []
        for d, t in enumerate(capacity_tickets):
            num = total * int(t)
            counts.append(num // cap_sum)
            remainders.append((d, num % cap_sum))
        remainders.sort(key=lambda x: (-x[1], x[0]))
        remaining = total - sum(counts)
        for d, _ in remainders[:remaining]:
            counts[d] += 1
        scores = [0] * len(counts)
        seq = []
        for _ in range(total):
            for i, c in enumerate(counts):
                scores[i] += c
            # max score, ties broken toward the lowest rank index
            best = max(range(len(scores)), key=lambda i: (scores[i], -i))
            scores[best] -= total
            seq.append(best)
        self.sequence = seq
        self.counts = counts
        self.phase = int(request_id) % total

    def total_units(self) -> int:
        return len(self.sequence)

    def assignee_for(self, token_offset: int, layer_idx: int, num_layers: int) -> Optional[int]:
        if num_layers == 0 or layer_idx >= num_layers or layer_idx < 0 or token_offset < 0:
            return None
        ordinal = token_offset * num_layers + layer_idx
        if ordinal >= len(self.sequence):
            return None
        return self.sequence[(self.phase + ordinal) % len(self.sequence)]

    def per_rank_units(self, num_ranks: int, token_offsets: range, num_layers: int) -> list:
        out = [0] * num_ranks
        for t in token_offsets:
            for layer in range(num_layers):
                a = self.assignee_for(t, layer, num_layers)
                if a is not None:
                    out[a] += 1
        return out


def stationary_layer_starters(initial_starter: int, layers: int, domains: int) -> list:
    if domains == 0:
        raise RingError("stationary ring requires at least one domain")
    if initial_starter >= domains or initial_starter < 0:
        raise RingError(f"stationary ring starter {initial_starter} out of {domains} domains")
    out = []
    s = initial_starter
    for _ in range(layers):
        out.append(s)
        s = (s + domains - 1) % domains
    return out


def layer_finisher(starter: int, domains: int) -> int:
    """The rank that completes a layer started at `starter` (N-1 hops later)."""
    return (starter + domains - 1) % domains
