"""KV arena bookkeeping and token sampling on CPU.

Parity: the reference's cache tests (rust/src/model/cache.rs:447-625: block table capacity,
sharded growth) and reserved-slab capacity errors (self_driving.rs:146-331), and its sampling
rules (rust/src/model/sampling.rs:8-119: greedy at temperature 0, top-p keeps the most likely
token).
"""

import numpy as np
import pytest
import torch

from hetero_cp_ringattn_b200.errors import CapacityError
from hetero_cp_ringattn_b200.kv.arena import KvArenaManager, PageAllocator
from hetero_cp_ringattn_b200.models.sampling import sample_token


def test_page_allocator_exhaustion_and_reuse():
    a = PageAllocator(4, 128)
    p = a.alloc(3, req_id=1)
    assert len(set(p)) == 3 and a.free_pages == 1
    assert all(a.owner_of(x) == 1 for x in p) and a.owner_of(3) is None
    with pytest.raises(CapacityError):
        a.alloc(2, req_id=2)
    a.free(p[:2])
    q = a.alloc(3, req_id=2)
    assert set(p[:2]) <= set(q) and a.free_pages == 0


def test_arena_reserve_extend_release():
    m = KvArenaManager(num_pages=8, page_size=128, num_layers=3)
    pos = np.arange(10, 110)
    rk = m.reserve(7, n_prefill=100, capacity_slots=200, positions=pos)
    assert len(rk.pages) == 2 and rk.capacity == 256
    assert (rk.layer_counts == 100).all()
    assert (rk.slot_pos[:, :100] == pos[None]).all() and (rk.slot_pos[:, 100:] == -1).all()
    with pytest.raises(CapacityError):
        m.reserve(7, 1, 1)
    # growth on one layer only (a sharded decode row), then a session extension
    rk.slot_pos[1, 100] = 500
    rk.layer_counts[1] += 1
    m.extend(7, 300)
    assert len(rk.pages) == 4 and rk.slot_pos.shape == (3, 512)
    assert rk.slot_pos[1, 100] == 500 and (rk.slot_pos[:, :100] == pos[None]).all()
    assert m.alloc.free_pages == 4
    assert m.release(7) and not m.release(7)
    assert m.alloc.free_pages == 8
    with pytest.raises(CapacityError):
        m.get(7)


def test_reserved_slab_full_raises():
    m = KvArenaManager(num_pages=2, page_size=128, num_layers=2)
    rk = m.reserve(1, n_prefill=127, capacity_slots=128)
    rk.check_room(0)                 # one slot left
    rk.layer_counts[0] += 1
    with pytest.raises(CapacityError):
        rk.check_room(0)
    rk.check_room(1)


def test_decode_past_horizon_raises():
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    cfg = preset("tiny")
    w = ModelWeights.random_init(cfg, seed=0, dtype=torch.float32, std=0.2)
    eng = LlamaCPEngine(cfg, PreparedWeights.from_weights(w, dtype=torch.float32),
                        device=torch.device("cpu"), max_context=128)
    tok, _ = eng.prefill(1, torch.arange(9), [9], decode_horizon=2)
    tok = eng.decode_step([1], tok)
    tok = eng.decode_step([1], tok)
    with pytest.raises(CapacityError):
        eng.decode_step([1], tok)


def test_greedy_and_degenerate_top_p_pick_argmax():
    logits = torch.tensor([0.1, 3.0, -1.0, 2.9])
    assert sample_token(logits) == 1
    g = torch.Generator().manual_seed(0)
    assert all(sample_token(logits, 1.0, 1e-6, generator=g) == 1 for _ in range(50))


def test_temperature_sampling_follows_softmax():
    logits = torch.tensor([0.0, 1.0, 2.0, -0.5])
    g = torch.Generator().manual_seed(1)
    n = 20000
    counts = np.bincount([sample_token(logits, 1.0, generator=g) for _ in range(n)], minlength=4)
    p = torch.softmax(logits, -1).numpy()
    assert np.abs(counts / n - p).max() < 0.015


def test_top_p_samples_only_the_nucleus():
    # probabilities ~ [0.64, 0.24, 0.09, 0.03]: top_p 0.8 keeps the first two
    logits = torch.log(torch.tensor([0.64, 0.24, 0.09, 0.03]))
    g = torch.Generator().manual_seed(2)
    draws = [sample_token(logits, 1.0, 0.8, generator=g) for _ in range(4000)]
    assert set(draws) == {0, 1}
    frac0 = draws.count(0) / len(draws)
    assert abs(frac0 - 0.64 / 0.88) < 0.03


def _old_meta_advance(eng, rids):
    """The per-layer loop form of the decode bookkeeping (the oracle for the vectorised one)."""
    B = len(rids)
    pos = np.zeros(B, dtype=np.int32)
    owner = np.zeros((B, eng.L), dtype=np.int32)
    slot = np.zeros((B, eng.L), dtype=np.int32)
    ntok = np.zeros((eng.L, B), dtype=np.int32)
    for b, rid in enumerate(rids):
        st = eng.reqs[rid]
        pos[b] = st.context_len
        own = (st.assignee[st.decode_offset] == eng.rank)
        for li in np.nonzero(own)[0]:
            st.kv.check_room(int(li))
        owner[b], slot[b], ntok[:, b] = own, st.kv.layer_counts, st.kv.layer_counts + own
    for b, rid in enumerate(rids):
        st = eng.reqs[rid]
        for li in np.nonzero(owner[b])[0]:
            st.kv.slot_pos[li, st.kv.layer_counts[li]] = pos[b]
        st.kv.layer_counts += owner[b]
        st.decode_offset += 1
        st.context_len += 1
    return pos, owner, slot, ntok


def test_vectorised_decode_bookkeeping_matches_the_loop_form():
    """Decode metadata and KV slot bookkeeping (owner, slot, token counts, slot positions,
    the reserved-slab capacity error) on the CUDA path's data, vectorised vs per-layer loops."""
    from hetero_cp_ringattn_b200.config import preset
    from hetero_cp_ringattn_b200.models.llama import LlamaCPEngine, RequestState
    from hetero_cp_ringattn_b200.models.weights import ModelWeights, PreparedWeights
    from hetero_cp_ringattn_b200.parallel.strategy import RingStrategy
    cfg = preset("tiny")
    cfg.num_layers = 6
    w = PreparedWeights.from_weights(ModelWeights.random_init(cfg, seed=0, dtype=torch.float32),
                                     dtype=torch.float32)
    engines = []
    for _ in range(2):
        e = LlamaCPEngine(cfg, w, device=torch.device("cpu"), max_context=1024, kv_pages=64,
                          page_size=16)
        e.rank, e.world = 1, 3          # owners vary per (token, layer)
        for b, rid in enumerate((5, 6, 7)):
            st = RequestState(req_id=rid, prompt_len=100, chunks=[100], strategy=RingStrategy.VANILLA,
                              positions=np.arange(100), owner_of_last=0, horizon=400,
                              assignee=e._schedule(rid, [2, 1, 1], 400, 0, 100), context_len=100)
            st.kv = e.kv.reserve(rid, 30 + b, 30 + b + 5 + 3 * b, np.arange(30 + b))
            e.reqs[rid] = st
        e.cuda = True                   # the CUDA branch of the bookkeeping is pure host code
        engines.append(e)
    new, old = engines
    rids = [5, 6, 7]
    for step in range(400):
        try:
            ref = _old_meta_advance(old, rids)
        except CapacityError as e_old:
            with pytest.raises(CapacityError) as e_new:
                new._decode_meta(rids)
            assert str(e_new.value) == str(e_old)
            break
        got = new._decode_meta(rids)
        new._advance(rids, got[1], got[0])
        for a, b in zip(got, ref):
            assert np.array_equal(a, b), step
        for rid in rids:
            assert np.array_equal(new.reqs[rid].kv.layer_counts, old.reqs[rid].kv.layer_counts)
            assert np.array_equal(new.reqs[rid].kv.slot_pos, old.reqs[rid].kv.slot_pos)
    else:
        raise AssertionError("the reserved slabs never filled up")


def test_staging_memory_ceiling():
    """The prefill staging buffers are O(L) per rank whatever the number of ranks: two parities of
    position-ordered bf16 K and V. 512k positions of the Llama-3-8B shape need 4.3 GB per rank;
    the ceiling for a budget inverts the formula."""
    from hetero_cp_ringattn_b200.kv.arena import max_staged_context, staging_bytes
    assert staging_bytes(524288, 8, 128) == 2 * 2 * 8 * 524288 * 128 * 2
    assert abs(staging_bytes(524288, 8, 128) / 1e9 - 4.29) < 0.01
    assert staging_bytes(32768, 8, 64) == 134217728          # Llama-3.2-1B shape at 32k: 128 MiB
    ctx = max_staged_context(16 << 30, 8, 128)
    assert staging_bytes(ctx, 8, 128) <= 16 << 30 < staging_bytes(ctx + 1, 8, 128)
