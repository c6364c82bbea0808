"""Layouts, capacity chunking, KV admission and the frozen KV assignee schedule.

Golden vectors are the reference's own unit-test expectations:
  rust/src/model/attention/strategy.rs:154-202, rust/src/capacity.rs:445-668,
  rust/src/model/self_driving.rs:1066-1105, 1856-1940.
"""

import numpy as np
import pytest

from hetero_cp_ringattn_b200.errors import CapacityError, RingError
from hetero_cp_ringattn_b200.parallel import capacity as C
from hetero_cp_ringattn_b200.parallel.schedule import (FrozenKvAssigneeSchedule,
                                                       stationary_layer_starters)
from hetero_cp_ringattn_b200.parallel.strategy import (RingStrategy, build_assignment,
                                                       build_domain_positions, build_inverse_perm,
                                                       causal_work, layout_positions)


def test_layouts_match_reference_vectors():
    assert build_assignment([3, 1], "vanilla").tolist() == [0, 0, 0, 1]
    assert build_assignment([3, 1], "striped").tolist() == [0, 1, 0, 0]
    z = build_assignment([3, 1], "zigzag")
    assert z.tolist() == [0, 0, 1, 0]
    pos = build_domain_positions(z)
    assert pos[0].tolist() == [0, 1, 3] and pos[1].tolist() == [2]
    z2 = build_assignment([4, 4], RingStrategy.ZIGZAG)
    assert z2.tolist() == [0, 0, 1, 1, 1, 1, 0, 0]
    pos2 = build_domain_positions(z2)
    assert pos2[0].tolist() == [0, 1, 6, 7] and pos2[1].tolist() == [2, 3, 4, 5]
    assert build_inverse_perm(build_assignment([3, 1], "striped")).tolist() == [0, 3, 1, 2]
    with pytest.raises(ValueError):
        RingStrategy.parse("ring")


@pytest.mark.parametrize("strategy", ["vanilla", "striped", "zigzag"])
@pytest.mark.parametrize("chunks", [[5, 5, 1], [5, 5, 5, 5, 2, 2, 1, 1], [8192, 8192], [7]])
def test_layouts_partition_positions(strategy, chunks):
    pos = layout_positions(chunks, strategy)
    assert [len(p) for p in pos] == chunks
    allp = np.concatenate(pos)
    assert sorted(allp.tolist()) == list(range(sum(chunks)))


def test_zigzag_balances_causal_work():
    chunks = [4096] * 8
    van = causal_work(layout_positions(chunks, "vanilla"))
    zig = causal_work(layout_positions(chunks, "zigzag"))
    assert max(zig) / min(zig) < 1.01
    assert max(van) / min(van) > 10


def test_allocate_by_capacity_matches_reference():
    assert C.allocate_by_capacity(10, [4096, 4096]) == [5, 5]
    assert C.allocate_by_capacity(9, [8192, 4096]) == [6, 3]
    c = C.allocate_by_capacity(10, [12288, 4096])
    assert sum(c) == 10 and c[0] >= c[1]
    assert C.allocate_by_capacity(14, [4096, 2048, 1024]) == [8, 4, 2]
    c = C.allocate_by_capacity(10, [4096, 2048, 1024])
    assert sum(c) == 10 and c[0] >= c[1] >= c[2]
    assert C.allocate_by_capacity(5, [0, 4096]) == [1, 4]
    assert C.allocate_by_capacity(3, [100, 100, 100]) == [1, 1, 1]
    c = C.allocate_by_capacity(20, [100000, 1000])
    assert sum(c) == 20 and c[0] > c[1] >= 1
    assert C.allocate_by_capacity(8, [0, 0, 0]) == [3, 3, 2]
    assert C.allocate_by_capacity(11, [8192, 12288]) == [4, 7]
    assert C.allocate_by_capacity(11, [8192, 12288, 6144]) == [3, 5, 3]
    assert C.allocate_by_capacity(16, [8192, 20480, 16384]) == [3, 7, 6]
    with pytest.raises(RingError):
        C.allocate_by_capacity(2, [1, 1, 1])
    with pytest.raises(RingError):
        C.allocate_by_capacity(2, [])


def test_chunk_sizes_tiers_and_ratios():
    assert C.chunk_sizes(65536, 3, ratio=[5, 5, 1]) == C.allocate_by_capacity(65536, [5, 5, 1])
    c8 = C.chunk_sizes(65536, 8, ratio=[5, 5, 5, 5, 2, 2, 1, 1])
    assert sum(c8) == 65536 and c8[0] == c8[3] and c8[4] == c8[5] and c8[6] == c8[7]
    assert C.chunk_sizes(10, 2, explicit=[7, 3]) == [7, 3]
    with pytest.raises(RingError):
        C.chunk_sizes(10, 2, explicit=[7, 4])
    assert C.chunk_sizes(10, 3) == [4, 4, 2]
    assert C.chunk_sizes(12, 2, capacities_mb=[1536 + 100, 1536 + 300], capacity_aware=True) == [3, 9]
    assert C.equal_chunks(32768, 8) == [4096] * 8


def test_kv_admission_and_ledger():
    adm = C.admit_reserved_kv_bytes([[10, 10], [5, 5]], [1 << 20, 1 << 20], 2, 64, 2)
    assert adm.bytes_per_token_per_layer == 2 * 2 * 64 * 2
    assert adm.required_bytes_per_domain == [20 * 512, 10 * 512]
    with pytest.raises(CapacityError):
        C.admit_reserved_kv_bytes([[1]], [1], 0, 64, 2)
    with pytest.raises(CapacityError):
        C.admit_reserved_kv_bytes([[10]], [100], 2, 64, 2)
    with pytest.raises(CapacityError):
        C.capacity_mb_to_bytes([C.UNKNOWN_CAPACITY])
    assert C.capacity_mb_to_bytes([1, 4096]) == [1 << 20, 4096 << 20]
    led = C.KvLedger([100, 100])
    led.try_reserve(1, [60, 10])
    with pytest.raises(CapacityError):
        led.try_reserve(2, [50, 10])
    assert led.free_bytes() == [40, 90]
    # a failed prefill rolls its reservation back
    with pytest.raises(RuntimeError):
        with C.ReservationGuard(led, 3, [30, 30]):
            raise RuntimeError("prefill failed")
    assert led.free_bytes() == [40, 90]
    with C.ReservationGuard(led, 4, [30, 30]) as g:
        g.commit()
    assert led.free_bytes() == [10, 60]
    assert led.release(1) == [60, 10]


def test_frozen_schedule_matches_reference():
    s = FrozenKvAssigneeSchedule([1, 3], 75, 4)
    assert s.counts == [1, 3]
    assert sorted(s.assignee_for(o, 0, 1) for o in range(4)) == sorted(s.sequence)
    assert FrozenKvAssigneeSchedule([1, 2, 3], 75, 4).counts == [1, 1, 2]
    assert FrozenKvAssigneeSchedule([1, 2, 3], 75, 24).counts == [4, 8, 12]
    first = FrozenKvAssigneeSchedule([1, 3, 2], 41, 24)
    assert first.counts == [4, 12, 8] and first.total_units() == 24
    obs = [0, 0, 0]
    for t in range(8):
        for layer in range(3):
            obs[first.assignee_for(t, layer, 3)] += 1
    assert obs == first.counts
    other = FrozenKvAssigneeSchedule([1, 3, 2], 42, 24)
    assert other.phase != first.phase and other.counts == first.counts
    assert first.assignee_for(0, 3, 3) is None and first.assignee_for(8, 0, 3) is None
    for bad in [([], 41, 24), ([0, 0, 0], 41, 24), ([1, 3, 2], 41, 0)]:
        with pytest.raises(RingError):
            FrozenKvAssigneeSchedule(*bad)
    z = FrozenKvAssigneeSchedule([1, 0, 3], 7, 16)
    assert z.counts == [4, 0, 12] and 1 not in z.sequence
    for tickets, total, expected in [([7], 5, [5]), ([1, 1], 6, [3, 3]), ([1, 1, 1, 1], 8, [2, 2, 2, 2])]:
        assert FrozenKvAssigneeSchedule(tickets, 3, total).counts == expected


@pytest.mark.parametrize("tickets,total", [([7], 5), ([1, 1], 6), ([1, 1, 1], 7), ([1, 3, 2], 24),
                                           ([1, 0, 3], 16), ([2, 5, 1, 4], 19)])
def test_frozen_schedule_prefix_bounded_by_reservation(tickets, total):
    for rid in range(total):
        s = FrozenKvAssigneeSchedule(tickets, rid, total)
        used = [0] * len(tickets)
        for o in range(total):
            a = s.assignee_for(o, 0, 1)
            used[a] += 1
            assert all(u <= r for u, r in zip(used, s.counts))
        assert used == s.counts and s.assignee_for(total, 0, 1) is None


def test_layer_starters():
    assert stationary_layer_starters(1, 4, 2) == [1, 0, 1, 0]
    assert stationary_layer_starters(2, 7, 3) == [2, 1, 0, 2, 1, 0, 2]
    with pytest.raises(RingError):
        stationary_layer_starters(2, 1, 2)
    with pytest.raises(RingError):
        stationary_layer_starters(0, 1, 0)


@pytest.mark.parametrize("strategy", ["vanilla", "striped", "zigzag"])
@pytest.mark.parametrize("chunks", [[4096] * 8, [5000, 5000, 1000], [700, 1], [3000, 3000, 3000, 3000, 1200, 1200, 600, 600]])
def test_ring_plan_covers_every_row_once(strategy, chunks):
    """The overlapped ring's host plan: tile_src names exactly the ranks with rows in each KV tile
    and each rank's push ranges cover its rows once (last tile first)."""
    import numpy as np
    from hetero_cp_ringattn_b200.models.llama import ring_plan
    from hetero_cp_ringattn_b200.parallel.strategy import layout_positions
    L = sum(chunks)
    positions = layout_positions(chunks, strategy)
    owner = np.empty(L, dtype=np.int64)
    for r, p in enumerate(positions):
        owner[np.asarray(p)] = r
    for r, p in enumerate(positions):
        p = np.asarray(p, dtype=np.int64)
        src, push = ring_plan(positions, r, L)
        src = src.view(np.uint64)
        for t in range(len(src)):
            want = set(owner[t * 128:(t + 1) * 128].tolist())
            got = {s for s in range(len(chunks)) if (int(src[t]) >> s) & 1}
            assert got == want
        covered = np.zeros(len(p), dtype=np.int64)
        assert list(push[:, 0]) == sorted(push[:, 0], reverse=True)
        for tile, lo, hi in push:
            assert np.all(p[lo:hi] // 128 == tile)
            covered[lo:hi] += 1
        assert np.all(covered == 1)
