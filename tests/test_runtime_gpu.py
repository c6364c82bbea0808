"""Domain runtime on the GPU: KV push + ring attention and the decode (O, LSE) exchange, for one
rank and for ranks emulated inside one process on one GPU (push phase for every rank before any
attend phase, so no launch ever waits on a later launch)."""

import math

import pytest
import torch

from hetero_cp_ringattn_b200.ops import reference as ref
from hetero_cp_ringattn_b200.ops._ext import native
from hetero_cp_ringattn_b200.parallel.strategy import layout_positions

pytestmark = pytest.mark.gpu

H, HKV, D, PAGE = 8, 2, 64, 256


def make_rt(rank, world, cap=2048, pages=16, layers=2):
    return native().Runtime(rank, world, 0, layers, pages, PAGE, HKV, D, H, cap, 8, 2000)


def tables(dev, max_pos=4096):
    cos, sin = ref.rope_cos_sin(torch.arange(max_pos, device=dev), D, 10000.0)
    return cos.contiguous(), sin.contiguous()


def reference_layer(qkv_all, pos_all, theta=10000.0):
    q = qkv_all[:, : H * D].view(-1, H, D)
    k = qkv_all[:, H * D:(H + HKV) * D].view(-1, HKV, D)
    v = qkv_all[:, (H + HKV) * D:].view(-1, HKV, D)
    q = ref.apply_rope(q.float(), pos_all, theta)
    k = ref.apply_rope(k.float(), pos_all, theta)
    o, lse = ref.full_attention(q, k, v.float(), pos_all, pos_all, causal=True)
    return q, k, v, o, lse


def run_ranks(dev, chunks, strategy, layer=0, epoch=1, rts=None):
    L = sum(chunks)
    n = len(chunks)
    torch.manual_seed(7)
    qkv_all = (torch.randn(L, (H + 2 * HKV) * D, device=dev) * 0.5).bfloat16()
    pos_all = torch.arange(L, device=dev)
    cos, sin = tables(dev)
    positions = [torch.as_tensor(p, device=dev) for p in layout_positions(chunks, strategy)]
    if rts is None:
        rts = [make_rt(r, n) for r in range(n)]
        if n > 1:
            for rt in rts:
                rt.open_peers_local(rts)
    outs = []
    args = []
    for r in range(n):
        p = positions[r]
        qkv = qkv_all[p].contiguous()
        pt = torch.arange(r * 4, r * 4 + 4, dtype=torch.int32, device=dev)  # 4 pages
        q_out = torch.empty(len(p), H, D, device=dev, dtype=torch.bfloat16)
        o_out = torch.empty_like(q_out)
        lse = torch.empty(H, len(p), device=dev, dtype=torch.float32)
        a = (qkv, p.int().contiguous(), cos, sin, layer, pt, 0, L, 1.0 / math.sqrt(D), True,
             q_out, o_out, lse, epoch)
        args.append(a)
        outs.append((o_out, lse))
    for r in range(n):
        rts[r].push_layer(*args[r])
    for r in range(n):
        rts[r].attend_layer(*args[r])
    torch.cuda.synchronize()
    for rt in rts:
        rt.check()
    _, k_ref, v_ref, o_ref, lse_ref = reference_layer(qkv_all, pos_all)
    for r in range(n):
        p = positions[r]
        o, lse = outs[r]
        assert (o.float() - o_ref[p]).abs().max() < 2e-2, f"rank {r}"
        assert (lse - lse_ref[:, p]).abs().max() < 2e-2
        # the local arena holds this rank's K/V rows in local order
        arena = rts[r].arena()
        pages = torch.arange(r * 4, r * 4 + 4, device=dev)
        kk = arena[layer, pages, 0].permute(1, 0, 2, 3).reshape(HKV, -1, D)[:, : len(p)]
        assert (kk.float().transpose(0, 1) - k_ref[p]).abs().max() < 2e-2
    return rts, qkv_all, positions


def test_single_rank_layer(dev):
    run_ranks(dev, [700], "vanilla")


@pytest.mark.parametrize("strategy", ["vanilla", "zigzag", "striped"])
def test_emulated_two_ranks(dev, strategy):
    run_ranks(dev, [400, 300], strategy)


def test_emulated_uneven_three_ranks_two_layers(dev):
    rts, _, _ = run_ranks(dev, [500, 500, 100], "vanilla", layer=0, epoch=1)
    run_ranks(dev, [500, 500, 100], "zigzag", layer=1, epoch=2, rts=rts)
    run_ranks(dev, [500, 500, 100], "vanilla", layer=0, epoch=3, rts=rts)


@pytest.mark.parametrize("world,b", [(1, 1), (2, 1), (3, 4)])
def test_decode_exchange(dev, world, b):
    torch.manual_seed(9)
    counts = [300, 257, 129][:world]
    rts = [make_rt(r, world) for r in range(world)]
    if world > 1:
        for rt in rts:
            rt.open_peers_local(rts)
    q = torch.randn(b, H, D, device=dev, dtype=torch.bfloat16)
    ks, vs = [], []
    pts = []
    for r in range(world):
        arena = rts[r].arena()
        n = counts[r]
        k = torch.randn(n, HKV, D, device=dev, dtype=torch.bfloat16)
        v = torch.randn(n, HKV, D, device=dev, dtype=torch.bfloat16)
        pages = [3, 1]  # non-contiguous page ids
        for i in range(n):
            pg, row = pages[i // PAGE], i % PAGE
            arena[1, pg, 0, :, row] = k[i]
            arena[1, pg, 1, :, row] = v[i]
        ks.append(k)
        vs.append(v)
        pts.append(torch.tensor([pages] * b, dtype=torch.int32, device=dev))
    splits = 4
    outs = []
    bufs = []
    for r in range(world):
        part_o = torch.empty(b * H * splits * D, device=dev)
        part_l = torch.empty(b * H * splits, device=dev)
        cnt = torch.zeros(b * HKV + 1, dtype=torch.int32, device=dev)
        ntok = torch.full((b,), counts[r], dtype=torch.int32, device=dev)
        bufs.append((part_o, part_l, cnt, ntok))
        rts[r].decode_attn(q, 1, pts[r], ntok, 1.0 / math.sqrt(D), splits, part_o, part_l, cnt, None, 1, 5)
    for r in range(world):
        out = torch.empty(b, H * D, device=dev, dtype=torch.bfloat16)
        rts[r].decode_combine(out, b, H, None, 1, 5)
        outs.append(out)
    torch.cuda.synchronize()
    for rt in rts:
        rt.check()
    k_all = torch.cat(ks)
    v_all = torch.cat(vs)
    L = k_all.shape[0]
    for bb in range(b):
        ro, _ = ref.full_attention(q[bb:bb + 1].float(), k_all.float(), v_all.float(), causal=False)
        for r in range(world):
            assert (outs[r][bb].view(H, D).float() - ro[0]).abs().max() < 2e-2
    for r in range(1, world):
        assert torch.equal(outs[r], outs[0]), "ranks must produce bit-identical combined outputs"


@pytest.mark.parametrize("world,b", [(2, 1), (3, 4), (4, 2)])
def test_decode_in_kernel_combine(dev, world, b):
    """The multi-rank decode attention with the exchange and the rank-order combine inside the
    kernel (the last CTA of each (row, KV head) publishes its partial, waits for the other ranks'
    and combines), with ranks emulated on one GPU: ranks 1.. first store their partials with the
    plain kernel and publish their group flags, so every wait is satisfied when it is launched.
    All ranks' outputs are bit-identical and match float32 attention over every rank's KV."""
    torch.manual_seed(19)
    counts = [300, 257, 129, 64][:world]
    rts = [make_rt(r, world) for r in range(world)]
    for rt in rts:
        rt.open_peers_local(rts)
    q = torch.randn(b, H, D, device=dev, dtype=torch.bfloat16)
    ks, vs, pts = [], [], []
    for r in range(world):
        arena = rts[r].arena()
        k = torch.randn(counts[r], HKV, D, device=dev, dtype=torch.bfloat16)
        v = torch.randn(counts[r], HKV, D, device=dev, dtype=torch.bfloat16)
        for i in range(counts[r]):
            arena[0, [2, 5][i // PAGE], 0, :, i % PAGE] = k[i]
            arena[0, [2, 5][i // PAGE], 1, :, i % PAGE] = v[i]
        ks.append(k)
        vs.append(v)
        pts.append(torch.tensor([[2, 5]] * b, dtype=torch.int32, device=dev))
    splits, epoch = 4, 9

    def attn(r, combine_out=None):
        part_o = torch.empty(b * H * splits * D, device=dev)
        part_l = torch.empty(b * H * splits, device=dev)
        cnt = torch.zeros(b * HKV + 1, dtype=torch.int32, device=dev)
        ntok = torch.full((b,), counts[r], dtype=torch.int32, device=dev)
        rts[r].decode_attn(q, 0, pts[r], ntok, 1.0 / math.sqrt(D), splits, part_o, part_l, cnt,
                           None, 1, epoch, None, combine_out)
        torch.cuda.synchronize()   # the scratch tensors live until the launch is done

    for r in range(1, world):
        attn(r)
        rts[r].publish_decode_groups(b, epoch)
    outs = [torch.full((b, H * D), float("nan"), device=dev, dtype=torch.bfloat16) for _ in range(world)]
    for r in range(world):
        attn(r, outs[r])
    for rt in rts:
        rt.check()
    k_all, v_all = torch.cat(ks), torch.cat(vs)
    for bb in range(b):
        ro, _ = ref.full_attention(q[bb:bb + 1].float(), k_all.float(), v_all.float(), causal=False)
        assert (outs[0][bb].view(H, D).float() - ro[0]).abs().max() < 2e-2
    for r in range(1, world):
        assert torch.equal(outs[r], outs[0]), "ranks must produce bit-identical combined outputs"


@pytest.mark.parametrize("d,chunks,strategy", [(64, [700], "vanilla"), (128, [333, 400], "zigzag"),
                                               (64, [300, 200, 257], "striped")])
def test_fused_projection_push(dev, d, chunks, strategy):
    """QKV GEMM whose epilogue adds the bias, rotates, writes Q and pushes K/V to every rank's
    staging buffer and arena (no projection output in memory), then ring attention; against an
    fp32 reference of projection + RoPE + causal attention."""
    torch.manual_seed(11)
    hid, n, L = 320, len(chunks), sum(chunks)
    nq = (H + 2 * HKV) * d
    rts = [native().Runtime(r, n, 0, 1, 16, PAGE, HKV, d, H, 2048, 8, 2000) for r in range(n)]
    if n > 1:
        for rt in rts:
            rt.open_peers_local(rts)
    x_all = (torch.randn(L, hid, device=dev) * 0.5).bfloat16()
    w = (torch.randn(nq, hid, device=dev) / math.sqrt(hid)).bfloat16()
    bias = (torch.randn(nq, device=dev) * 0.1).bfloat16()
    qkv_all = x_all.float() @ w.float().t() + bias.float()
    pos_all = torch.arange(L, device=dev)
    cos, sin = ref.rope_cos_sin(torch.arange(4096, device=dev), d, 10000.0)
    cos, sin = cos.contiguous(), sin.contiguous()
    positions = [torch.as_tensor(p, device=dev) for p in layout_positions(chunks, strategy)]
    runs = []
    for r in range(n):
        p = positions[r]
        x = x_all[p].contiguous()
        pt = torch.arange(r * 4, r * 4 + 4, dtype=torch.int32, device=dev)
        q_out = torch.empty(len(p), H, d, device=dev, dtype=torch.bfloat16)
        o_out = torch.empty_like(q_out)
        lse = torch.empty(H, len(p), device=dev, dtype=torch.float32)
        tail = (p.int().contiguous(), cos, sin, 0, pt, 0, L, 1.0 / math.sqrt(d), True,
                q_out, o_out, lse, 1)
        runs.append((x, tail, q_out, o_out, lse))
    for r in range(n):
        rts[r].push_layer_fused(runs[r][0], w, bias, *runs[r][1])
    for r in range(n):
        rts[r].attend_layer(runs[r][0], *runs[r][1])
    torch.cuda.synchronize()
    for rt in rts:
        rt.check()
    q = ref.apply_rope(qkv_all[:, : H * d].view(-1, H, d), pos_all, 10000.0)
    k = ref.apply_rope(qkv_all[:, H * d:(H + HKV) * d].view(-1, HKV, d), pos_all, 10000.0)
    v = qkv_all[:, (H + HKV) * d:].view(-1, HKV, d)
    o_ref, lse_ref = ref.full_attention(q, k, v, pos_all, pos_all, causal=True)
    for r in range(n):
        p = positions[r]
        _, _, q_out, o_out, lse = runs[r]
        assert (q_out.float() - q[p]).abs().max() < 3e-2, f"rank {r} q"
        assert (o_out.float() - o_ref[p]).abs().max() < 3e-2, f"rank {r} o"
        assert (lse - lse_ref[:, p]).abs().max() < 3e-2
        arena = rts[r].arena()
        pages = torch.arange(r * 4, r * 4 + 4, device=dev)
        kk = arena[0, pages, 0].permute(1, 0, 2, 3).reshape(HKV, -1, d)[:, : len(p)]
        vv = arena[0, pages, 1].permute(1, 0, 2, 3).reshape(HKV, -1, d)[:, : len(p)]
        assert (kk.float().transpose(0, 1) - k[p]).abs().max() < 3e-2
        assert (vv.float().transpose(0, 1) - v[p]).abs().max() < 3e-2
    for rt in rts:
        rt.shutdown()


@pytest.mark.parametrize("b,d,tc", [(1, 64, 0), (4, 128, 0), (4, 64, 1), (8, 128, 1)])
def test_qkv_gemv_rope_matches_two_kernel_path(dev, b, d, tc):
    """Decode QKV GEMV with the RoPE + KV-append epilogue against GEMV (fp32 out) + qkv_decode."""
    from hetero_cp_ringattn_b200.ops import kernels as K
    torch.manual_seed(13)
    hid, layers = 512, 2
    nq = (H + 2 * HKV) * d
    rt = native().Runtime(0, 1, 0, layers, 8, PAGE, HKV, d, H, 1024, 8, 2000)
    x = torch.randn(b, hid, device=dev).bfloat16()
    w = (torch.randn(nq, hid, device=dev) / math.sqrt(hid)).bfloat16()
    bias = (torch.randn(nq, device=dev) * 0.1).bfloat16()
    nw = (torch.rand(hid, device=dev) + 0.5).bfloat16()
    cos, sin = ref.rope_cos_sin(torch.arange(2048, device=dev), d, 10000.0)
    cos, sin = cos.contiguous(), sin.contiguous()
    pos = torch.tensor([5, 700, 1000, 33, 2, 1500, 64, 999][:b], dtype=torch.int32, device=dev)
    pt = torch.tensor([[1, 2, 3]] * b, dtype=torch.int32, device=dev)
    owner = torch.tensor([[1, 1], [0, 1], [1, 0], [1, 1], [0, 0], [1, 1], [1, 0], [0, 1]][:b],
                         dtype=torch.int32, device=dev)
    slot = torch.tensor([[3, 3], [300, 301], [600, 7], [17, 18], [5, 6], [400, 401], [700, 9],
                         [10, 767]][:b], dtype=torch.int32, device=dev)
    layer = 1
    qa = torch.empty(b, H, d, device=dev, dtype=torch.bfloat16)
    rt.arena().zero_()
    rt.qkv_gemv_rope(x, w, bias, nw, 1e-5, pos, cos, sin, layer, pt, owner, slot, qa, tc=tc)
    torch.cuda.synchronize()
    arena_a = rt.arena().clone()
    rt.arena().zero_()
    qkv = torch.empty(b, nq, device=dev, dtype=torch.float32)
    K.gemv(x, w, "f32", bias=bias, y_f32=qkv, norm_w=nw, eps=1e-5)
    qb = torch.empty_like(qa)
    rt.qkv_decode(qkv, pos, cos, sin, layer, pt, owner, slot, qb)
    torch.cuda.synchronize()
    rt.check()
    assert (qa.float() - qb.float()).abs().max() < 2e-2
    assert (arena_a.float() - rt.arena().float()).abs().max() < 2e-2
    assert arena_a.abs().sum() > 0
    rt.shutdown()


@pytest.mark.parametrize("h,hkv,d,n", [(16, 2, 128, 5000), (4, 4, 64, 70), (8, 1, 64, 1),
                                       (14, 2, 64, 333), (24, 8, 128, 1000), (40, 8, 128, 300),
                                       (12, 2, 128, 700), (32, 2, 64, 900), (128, 8, 128, 600),
                                       (9, 1, 64, 200), (24, 2, 128, 450)])
def test_decode_attention_group_shapes(dev, h, hkv, d, n):
    """Tensor-core split-KV decode attention for 8-head GQA groups at head_dim 128 (Qwen2.5-3B),
    no GQA, MQA with a single cached token, the groups of 7 (Qwen2-0.5B), 3 (Llama-3.2-3B),
    5 (Qwen2.5-14B) and 6 (Qwen2.5-1.5B) query heads per KV head, and groups of 9 to 16 heads,
    which use the MMA tile's second row group (16: Llama-3.1-405B's 128 / 8), against an fp32
    reference."""
    torch.manual_seed(14)
    pages_n = -(-n // PAGE) + 1
    rt = native().Runtime(0, 1, 0, 1, pages_n + 1, PAGE, hkv, d, h, 1024, 8, 2000)
    arena = rt.arena()
    arena.zero_()
    k = torch.randn(n, hkv, d, device=dev, dtype=torch.bfloat16)
    v = torch.randn(n, hkv, d, device=dev, dtype=torch.bfloat16)
    page_ids = list(range(pages_n, 0, -1))  # reversed page order
    for i in range(n):
        arena[0, page_ids[i // PAGE], 0, :, i % PAGE] = k[i]
        arena[0, page_ids[i // PAGE], 1, :, i % PAGE] = v[i]
    pt = torch.tensor([page_ids], dtype=torch.int32, device=dev)
    q = torch.randn(1, h, d, device=dev, dtype=torch.bfloat16)
    ntok = torch.tensor([n], dtype=torch.int32, device=dev)
    splits = 7
    part_o = torch.empty(h * splits * d, device=dev)
    part_l = torch.empty(h * splits, device=dev)
    cnt = torch.zeros(hkv + 1, dtype=torch.int32, device=dev)
    out = torch.empty(1, h * d, device=dev, dtype=torch.bfloat16)
    rt.decode_attn(q, 0, pt, ntok, 1.0 / math.sqrt(d), splits, part_o, part_l, cnt, None, 1, 5, out)
    torch.cuda.synchronize()
    rt.check()
    ro, _ = ref.full_attention(q[0][None].float(), k.float(), v.float(), torch.tensor([n - 1], device=dev),
                               torch.arange(n, device=dev), causal=True)
    assert (out.view(h, d).float() - ro[0]).abs().max() < 2e-2
    rt.shutdown()


def _plan(positions, rank, L, dev):
    from hetero_cp_ringattn_b200.models.llama import ring_plan
    src, push = ring_plan([p.cpu().numpy() for p in positions], rank, L)
    return dict(tile_src=torch.from_numpy(src).to(dev), push_tiles=torch.from_numpy(push).to(dev))


def run_overlap_ranks(dev, chunks, strategy, epoch, rts=None, layer=0):
    """The overlapped ring (the attention kernel pushes this rank's rows to the peers and waits
    per KV tile) with ranks emulated on one GPU. No launch may wait on a later one, so ranks
    1..n-1 first store their rows everywhere with the serial push and mark their tiles present;
    rank 0 then runs the overlapped path (local projection, attention that pushes its rows to the
    others and waits per tile); then ranks 1..n-1 run the overlapped attention, whose waits rank
    0's finished kernel satisfied. Rank 0's rows reach the other ranks only through its kernel."""
    L = sum(chunks)
    n = len(chunks)
    torch.manual_seed(100 + epoch)
    qkv_all = (torch.randn(L, (H + 2 * HKV) * D, device=dev) * 0.5).bfloat16()
    pos_all = torch.arange(L, device=dev)
    cos, sin = tables(dev)
    positions = [torch.as_tensor(p, device=dev) for p in layout_positions(chunks, strategy)]
    if rts is None:
        rts = [make_rt(r, n) for r in range(n)]
        for rt in rts:
            rt.open_peers_local(rts)
    args, plans, outs = [], [], []
    for r in range(n):
        p = positions[r]
        qkv = qkv_all[p].contiguous()
        pt = torch.arange(r * 4, r * 4 + 4, dtype=torch.int32, device=dev)
        q_out = torch.empty(len(p), H, D, device=dev, dtype=torch.bfloat16)
        o_out = torch.empty_like(q_out)
        lse = torch.empty(H, len(p), device=dev, dtype=torch.float32)
        args.append((qkv, p.int().contiguous(), cos, sin, layer, pt, 0, L, 1.0 / math.sqrt(D),
                     True, q_out, o_out, lse, epoch))
        plans.append(_plan(positions, r, L, dev))
        outs.append((o_out, lse))
    for r in range(1, n):
        rts[r].push_layer(*args[r])                              # serial push to every rank
        rts[r].publish_tiles(plans[r]["push_tiles"], epoch)
    rts[0].push_layer(*args[0], **plans[0])                      # local rows only
    rts[0].attend_layer(*args[0], **plans[0])                    # pushes rank 0's rows, waits
    for r in range(1, n):
        rts[r].attend_layer(*args[r], **plans[r])
    torch.cuda.synchronize()
    for rt in rts:
        rt.check()
    _, _, _, o_ref, lse_ref = reference_layer(qkv_all, pos_all)
    # one rank over the whole sequence: every row folds its KV tiles in the same order, so the
    # ranks' rows are the same bits as the single rank's
    one = make_rt(0, 1)
    o_one = torch.empty(L, H, D, device=dev, dtype=torch.bfloat16)
    a1 = (qkv_all, pos_all.int(), cos, sin, 0, torch.arange(0, 8, dtype=torch.int32, device=dev), 0,
          L, 1.0 / math.sqrt(D), True, torch.empty_like(o_one), o_one, None, 1)
    one.push_layer(*a1)
    one.attend_layer(*a1)
    torch.cuda.synchronize()
    one.check()
    one.shutdown()
    for r in range(n):
        p = positions[r]
        o, lse = outs[r]
        assert (o.float() - o_ref[p]).abs().max() < 2e-2, f"rank {r}"
        assert (lse - lse_ref[:, p]).abs().max() < 2e-2, f"rank {r}"
        assert torch.equal(o, o_one[p]), f"rank {r}: not bit-identical to one rank"
    return rts


@pytest.mark.parametrize("strategy", ["vanilla", "zigzag", "striped"])
def test_overlapped_ring_emulated_two_ranks(dev, strategy):
    run_overlap_ranks(dev, [640, 300], strategy, epoch=1)


def test_overlapped_ring_uneven_three_ranks_several_steps(dev):
    """5:5:1-like uneven chunks, several layer steps on the same runtimes (both staging parities,
    the consumed handshake of step epoch - 2, counters reset by the last CTA)."""
    rts = run_overlap_ranks(dev, [500, 500, 100], "vanilla", epoch=1)
    for epoch, strategy in [(2, "zigzag"), (3, "vanilla"), (4, "striped"), (5, "zigzag")]:
        run_overlap_ranks(dev, [500, 500, 100], strategy, epoch=epoch, rts=rts, layer=epoch % 2)


@pytest.mark.parametrize("world,b", [(2, 1), (3, 4), (8, 8)])
def test_split_lm_head_argmax_exchange(dev, world, b):
    """Greedy decode with the LM head split over the vocabulary: each emulated rank runs the
    argmax GEMV over its own vocabulary rows (global row ids through `index_base`) and the
    exchange kernel keeps the largest packed maximum over the ranks. Every rank's tokens equal
    the whole head's argmax, including an exact tie across slices, which goes to the smaller id.
    Ranks 1.. publish by storing into every rank's slots before rank 0's launch, so no wait
    depends on a later launch."""
    from hetero_cp_ringattn_b200.ops import kernels as K
    torch.manual_seed(23)
    V, KD, EPOCH = 1000, 256, 7                       # epoch 7: parity 1
    x = torch.randn(b, KD, device=dev, dtype=torch.bfloat16)
    W = (torch.randn(V, KD, device=dev) * 0.05).bfloat16()
    part = -(-V // (world * 8)) * 8
    lo = [min(V, r * part) for r in range(world)]
    hi = [min(V, lo_r + part) for lo_r in lo]
    tie = lo[-1] + 3                                  # a row of the last rank's slice
    W[5] = W[tie] = (torch.sign(x[0].float()) * 0.25).bfloat16()
    rts = [make_rt(r, world) for r in range(world)]
    for rt in rts:
        rt.open_peers_local(rts)
    step = torch.tensor([EPOCH], dtype=torch.int64, device=dev)
    am = []
    for r in range(world):
        a = torch.zeros(b, dtype=torch.int64, device=dev)
        K.gemv(x, W[lo[r]:hi[r]], "argmax", argmax=a, index_base=lo[r])
        am.append(a)
    for r in range(1, world):
        for d in range(world):
            sl = rts[d].argmax_slots()
            sl[1, r, :b, 0] = am[r]
            sl[1, r, :b, 1] = EPOCH
    toks = []
    for r in range(world):
        t32 = torch.full((b,), -1, dtype=torch.int32, device=dev)
        t64 = torch.full((b,), -1, dtype=torch.int64, device=dev)
        rts[r].argmax_exchange(am[r], step, t32, t64)
        torch.cuda.synchronize()
        toks.append((t32, t64))
    for rt in rts:
        rt.check()
    full = torch.zeros(b, dtype=torch.int64, device=dev)
    K.gemv(x, W, "argmax", argmax=full)
    want = torch.zeros(b, dtype=torch.int64, device=dev)
    native().argmax_finalize(full, None, want)
    assert int(want[0]) == 5
    logits = x.float() @ W.float().t()
    assert bool((logits.gather(1, want.view(-1, 1)).view(-1) >= logits.max(1).values - 1e-2).all())
    for t32, t64 in toks:
        assert torch.equal(t64, want) and torch.equal(t32.long(), want)
    for d in range(world):      # rank 0's kernel stored its maxima into every rank's slots
        sl = rts[d].argmax_slots()
        assert torch.equal(sl[1, 0, :b, 0], am[0]) and bool((sl[1, 0, :b, 1] == EPOCH).all())
    for rt in rts:
        rt.shutdown()


@pytest.mark.parametrize("world,b", [(2, 1), (3, 4), (4, 8)])
def test_output_projection_with_combine_prologue(dev, world, b):
    """The decode step's output projection with the cross-rank combine in its prologue (the
    default on several ranks): after every emulated rank's split-KV attention has stored its
    (O, LSE) partial into every rank's slots and released its ready flag, each rank's
    `o_proj_combine` equals the combine launch followed by the plain residual GEMV, bit for
    bit, and the combined attention matches float32 attention over every rank's KV."""
    from hetero_cp_ringattn_b200.ops import kernels as K
    torch.manual_seed(29)
    counts = [300, 257, 129, 64][:world]
    rts = [make_rt(r, world) for r in range(world)]
    for rt in rts:
        rt.open_peers_local(rts)
    q = torch.randn(b, H, D, device=dev, dtype=torch.bfloat16)
    ks, vs, pts = [], [], []
    for r in range(world):
        arena = rts[r].arena()
        k = torch.randn(counts[r], HKV, D, device=dev, dtype=torch.bfloat16)
        v = torch.randn(counts[r], HKV, D, device=dev, dtype=torch.bfloat16)
        for i in range(counts[r]):
            arena[0, [4, 2][i // PAGE], 0, :, i % PAGE] = k[i]
            arena[0, [4, 2][i // PAGE], 1, :, i % PAGE] = v[i]
        ks.append(k)
        vs.append(v)
        pts.append(torch.tensor([[4, 2]] * b, dtype=torch.int32, device=dev))
    splits, epoch = 4, 11
    keep = []
    for r in range(world):
        part_o = torch.empty(b * H * splits * D, device=dev)
        part_l = torch.empty(b * H * splits, device=dev)
        cnt = torch.zeros(b * HKV + 1, dtype=torch.int32, device=dev)
        ntok = torch.full((b,), counts[r], dtype=torch.int32, device=dev)
        keep.append((part_o, part_l, cnt, ntok))
        rts[r].decode_attn(q, 0, pts[r], ntok, 1.0 / math.sqrt(D), splits, part_o, part_l, cnt,
                           None, 1, epoch)
    torch.cuda.synchronize()
    W = (torch.randn(384, H * D, device=dev) * 0.05).bfloat16()
    y0 = torch.randn(b, 384, device=dev).bfloat16()
    step = torch.zeros(1, dtype=torch.int64, device=dev)     # epoch = 0 * 1 + epoch
    k_all, v_all = torch.cat(ks).float(), torch.cat(vs).float()
    for r in range(world):
        o = torch.empty(b, H * D, device=dev, dtype=torch.bfloat16)
        rts[r].decode_combine(o, b, H, None, 1, epoch)
        want = y0.clone()
        K.gemv(o, W, "residual", y_bf16=want)
        got = y0.clone()
        rts[r].o_proj_combine(torch.empty_like(o), W, got, step, 1, epoch)
        torch.cuda.synchronize()
        rts[r].check()
        assert torch.equal(got, want), f"rank {r}: max diff {(got.float() - want.float()).abs().max()}"
        for bb in range(b):
            ro, _ = ref.full_attention(q[bb:bb + 1].float(), k_all, v_all, causal=False)
            assert (o[bb].view(H, D).float() - ro[0]).abs().max() < 2e-2
    for rt in rts:
        rt.shutdown()


def test_context_longer_than_staging_is_rejected_before_any_kernel(dev):
    """The staging buffers bound the context a rank can prefill (two parities of position-ordered
    K/V up to the runtime's staging capacity): a layer step over a longer context is rejected by
    the runtime's host check with a clear error, nothing is launched, and the runtime stays
    usable for a context that fits."""
    cap = 512
    rt = native().Runtime(0, 1, 0, 1, 8, PAGE, HKV, D, H, cap, 8, 2000)
    cos, sin = tables(dev)
    T = 640
    qkv = torch.zeros(T, (H + 2 * HKV) * D, device=dev, dtype=torch.bfloat16)
    pos = torch.arange(T, device=dev, dtype=torch.int32)
    pt = torch.arange(0, 4, dtype=torch.int32, device=dev)
    q_out = torch.empty(T, H, D, device=dev, dtype=torch.bfloat16)
    o_out = torch.empty_like(q_out)
    with pytest.raises(RuntimeError, match="staging capacity"):
        rt.push_layer(qkv, pos, cos, sin, 0, pt, 0, T, 1.0 / math.sqrt(D), True, q_out, o_out, None, 1)
    torch.cuda.synchronize()
    rt.check()
    run_ranks(dev, [cap], "vanilla", rts=[rt])
    rt.shutdown()
