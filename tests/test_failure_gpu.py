"""Failure detection on the GPU without a GPU fault: a bounded device wait on a flag that nothing
sets runs out after its budget, records a peer-timeout status and returns; the context stays
usable and the next launch works."""

import time

import pytest
import torch

from hetero_cp_ringattn_b200.ops._ext import native

pytestmark = pytest.mark.gpu


def test_device_wait_times_out_into_status(dev):
    rt = native().Runtime(0, 1, dev.index or 0, 1, 2, 256, 2, 64, 8, 1024, 1, 200)
    t0 = time.time()
    rt.wait_flags(0, 2, 7, 100)          # kv_ready[0..1] >= 7 never happens
    torch.cuda.synchronize(dev)
    waited = time.time() - t0
    with pytest.raises(RuntimeError, match="code=17"):
        rt.check()                        # kPeerTimeout, then the status word is cleared
    assert waited < 5.0
    # the context is still usable: a satisfied wait passes and the status stays clean
    rt.flags()[0:2] = 7
    rt.wait_flags(0, 2, 7, 100)
    torch.cuda.synchronize(dev)
    rt.check()
    x = torch.ones(1024, device=dev)
    assert float(x.sum()) == 1024.0
    rt.shutdown()


def test_overlapped_ring_missing_peer_times_out_into_status(dev):
    """The overlapped ring's per-tile wait on a peer that never publishes its tiles runs out after
    the runtime's budget (100 ms here), reports a peer timeout at the producer's wait site and the
    kernel returns; the runtime stays usable."""
    import math
    from hetero_cp_ringattn_b200.models.llama import ring_plan
    from hetero_cp_ringattn_b200.ops import reference as ref
    from hetero_cp_ringattn_b200.parallel.strategy import layout_positions
    H, HKV, D, PAGE = 8, 2, 64, 256
    rts = [native().Runtime(r, 2, dev.index or 0, 1, 8, PAGE, HKV, D, H, 1024, 1, 100) for r in range(2)]
    for rt in rts:
        rt.open_peers_local(rts)
    chunks = [256, 256]
    L = sum(chunks)
    positions = layout_positions(chunks, "zigzag")
    src, push = ring_plan(positions, 0, L)
    plan = dict(tile_src=torch.from_numpy(src).to(dev), push_tiles=torch.from_numpy(push).to(dev))
    p = torch.as_tensor(positions[0], device=dev).int()
    cos, sin = ref.rope_cos_sin(torch.arange(2048, device=dev), D, 10000.0)
    qkv = torch.randn(len(p), (H + 2 * HKV) * D, device=dev).bfloat16()
    q_out = torch.empty(len(p), H, D, device=dev, dtype=torch.bfloat16)
    o_out = torch.empty_like(q_out)
    args = (qkv, p, cos.contiguous(), sin.contiguous(), 0, torch.arange(0, 2, dtype=torch.int32, device=dev),
            0, L, 1.0 / math.sqrt(D), True, q_out, o_out, None, 1)
    t0 = time.time()
    rts[0].push_layer(*args, **plan)
    rts[0].attend_layer(*args, **plan)     # rank 1 never pushes or publishes its tiles
    torch.cuda.synchronize(dev)
    assert time.time() - t0 < 5.0
    with pytest.raises(RuntimeError, match="code=17.*site 210"):
        rts[0].check()
    x = torch.ones(1024, device=dev)
    assert float(x.sum()) == 1024.0
    for rt in rts:
        rt.shutdown()


def test_argmax_exchange_missing_peer_times_out_into_status(dev):
    """The vocabulary-split LM head's argmax exchange waits (bounded, 100 ms here) for a peer
    that never stores its maximum: it reports a peer timeout at its wait site, returns with this
    rank's own maximum as the token, and the runtime stays usable."""
    rts = [native().Runtime(r, 2, dev.index or 0, 1, 2, 256, 2, 64, 8, 1024, 1, 100) for r in range(2)]
    for rt in rts:
        rt.open_peers_local(rts)
    packed = ((0x3F800000 | 0x80000000) << 32) | (0xFFFFFFFF - 42)   # value 1.0 at id 42
    local = torch.tensor([packed - (1 << 64)], dtype=torch.int64, device=dev)
    step = torch.tensor([3], dtype=torch.int64, device=dev)
    tok = torch.full((1,), -1, dtype=torch.int64, device=dev)
    t0 = time.time()
    rts[0].argmax_exchange(local, step, None, tok)    # rank 1 never runs its exchange
    torch.cuda.synchronize(dev)
    assert time.time() - t0 < 5.0
    with pytest.raises(RuntimeError, match="code=17.*site 306"):
        rts[0].check()
    assert int(tok[0]) == 42
    x = torch.ones(1024, device=dev)
    assert float(x.sum()) == 1024.0
    for rt in rts:
        rt.shutdown()


def test_output_projection_combine_missing_peer_times_out_into_status(dev):
    """The combine prologue of the decode output projection waits (bounded, 100 ms here) for a
    peer whose partial never arrives: it reports a peer timeout at its wait site and returns;
    the runtime stays usable."""
    H, D = 8, 64
    rts = [native().Runtime(r, 2, dev.index or 0, 1, 2, 256, 2, D, H, 1024, 1, 100) for r in range(2)]
    for rt in rts:
        rt.open_peers_local(rts)
    x = torch.zeros(1, H * D, device=dev, dtype=torch.bfloat16)
    W = torch.zeros(128, H * D, device=dev, dtype=torch.bfloat16)
    y = torch.zeros(1, 128, device=dev, dtype=torch.bfloat16)
    step = torch.zeros(1, dtype=torch.int64, device=dev)
    t0 = time.time()
    rts[0].o_proj_combine(x, W, y, step, 1, 3)          # no rank ever releases epoch 3
    torch.cuda.synchronize(dev)
    assert time.time() - t0 < 5.0
    with pytest.raises(RuntimeError, match="code=17.*site 402"):
        rts[0].check()
    x1 = torch.ones(1024, device=dev)
    assert float(x1.sum()) == 1024.0
    for rt in rts:
        rt.shutdown()
