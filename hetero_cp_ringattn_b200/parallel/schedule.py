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

The schedule is computed by the native host library (`csrc/host/schedule.cpp`).
"""

from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

from ..host import lib


class FrozenKvAssigneeSchedule:
    def __init__(self, capacity_tickets: Sequence[int], request_id: int, total_kv_units: int):
        self._s = lib().FrozenKvAssigneeSchedule([int(t) for t in capacity_tickets],
                                                 int(request_id), int(total_kv_units))

    @property
    def sequence(self) -> list:
        return list(self._s.sequence)

    @property
    def counts(self) -> list:
        return list(self._s.counts)

    @property
    def phase(self) -> int:
        return int(self._s.phase)

    def total_units(self) -> int:
        return int(self._s.total_units())

    def assignee_for(self, token_offset: int, layer_idx: int, num_layers: int) -> Optional[int]:
        return self._s.assignee_for(int(token_offset), int(layer_idx), int(num_layers))

    def per_rank_units(self, num_ranks: int, token_offsets: range, num_layers: int) -> list:
        if token_offsets.step != 1:
            return [sum(1 for t in token_offsets for l in range(num_layers)
                        if self.assignee_for(t, l, num_layers) == r) for r in range(num_ranks)]
        return list(self._s.per_rank_units(int(num_ranks), token_offsets.start, token_offsets.stop,
                                           int(num_layers)))


def assignee_table(capacity_tickets: Sequence[int], request_id: int, horizon: int,
                   num_layers: int) -> np.ndarray:
    """[horizon, layers] rank that stores each decoded (token, layer) KV row: the frozen schedule
    over horizon * layers units read from the request's phase."""
    return lib().assignee_table([int(t) for t in capacity_tickets], int(request_id), int(horizon),
                                int(num_layers))


def stationary_layer_starters(initial_starter: int, layers: int, domains: int) -> list:
    return list(lib().stationary_layer_starters(int(initial_starter), int(layers), int(domains)))


def layer_finisher(starter: int, domains: int) -> int:
    """The rank that completes a layer started at `starter` (N-1 hops later)."""
    return (starter + domains - 1) % domains
