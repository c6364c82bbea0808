"""Numerics of the sm_100a kernels against plain PyTorch fp32 references (GPU only)."""

import math

import pytest
import torch

from hetero_cp_ringattn_b200.ops import kernels as K
from hetero_cp_ringattn_b200.ops import reference as ref
from hetero_cp_ringattn_b200.ops._ext import native

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a = a.float()
    b = b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


def status_tensor(dev):
    return torch.zeros(8, dtype=torch.int32, device=dev)


def assert_status_clean(st):
    torch.cuda.synchronize()
    assert int(st[0]) == 0, f"device status {st.tolist()}"


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 512, 256), (1000, 768, 1000), (4096, 3072, 2048),
                                   (260, 384, 128)])
def test_gemm_store(dev, m, n, k, variant):
    """Both GEMM kernels (one CTA per 128x256 tile; CTA pairs on 256x256 tiles with
    cta_group::2) against float32, including row and column tails (M = 260: the second CTA of
    the last pair holds 4 rows; N = 384: the last tile's second half of B is out of range)."""
    torch.manual_seed(0)
    a = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
    w = torch.randn(n, k, device=dev, dtype=torch.bfloat16) / math.sqrt(k)
    st = status_tensor(dev)
    y = K.gemm(a, w, "store", status=st, variant=variant)
    assert_status_clean(st)
    r = a.float() @ w.float().t()
    assert rel_err(y, r) < 1e-2


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("m,n", [(1000, 768), (4096, 3072)])
def test_gemm_tile_orders_bit_identical(dev, variant, m, n):
    """Banded tile orders (3 or 16 m-blocks per band, m fastest inside a band; a short last
    band when the blocks do not divide) only change which CTA computes a tile when: the output is
    the same bits as n-fastest order, and matches float32."""
    torch.manual_seed(4)
    k = 256
    a = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
    w = torch.randn(n, k, device=dev, dtype=torch.bfloat16) / math.sqrt(k)
    st = status_tensor(dev)
    outs = [K.gemm(a, w, "store", status=st, variant=variant, group=g) for g in (0, 3, 16)]
    assert_status_clean(st)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert rel_err(outs[0], a.float() @ w.float().t()) < 1e-2


@pytest.mark.parametrize("variant", [1, 2])
def test_gemm_bias_residual(dev, variant):
    torch.manual_seed(1)
    m, n, k = 513, 1280, 512
    a = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
    w = torch.randn(n, k, device=dev, dtype=torch.bfloat16) / math.sqrt(k)
    b = torch.randn(n, device=dev, dtype=torch.bfloat16)
    st = status_tensor(dev)
    y = K.gemm(a, w, "bias", bias=b, status=st, variant=variant)
    r = a.float() @ w.float().t() + b.float()
    assert rel_err(y, r) < 1e-2
    res = torch.randn(m, n, device=dev, dtype=torch.bfloat16)
    expect = (a.float() @ w.float().t()).bfloat16().float() + res.float()
    y2 = K.gemm(a, w, "residual", residual=res, status=st, variant=variant)  # in place on res
    assert_status_clean(st)
    assert y2.data_ptr() == res.data_ptr()
    assert rel_err(y2, expect) < 1e-2


@pytest.mark.parametrize("variant", [1, 2])
def test_gemm_swiglu(dev, variant):
    torch.manual_seed(2)
    m, i, k = 700, 512, 384
    a = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
    g = torch.randn(i, k, device=dev, dtype=torch.bfloat16) / math.sqrt(k)
    u = torch.randn(i, k, device=dev, dtype=torch.bfloat16) / math.sqrt(k)
    wgu = K.interleave_gate_up(g, u)
    st = status_tensor(dev)
    y = K.gemm(a, wgu, "swiglu", status=st, variant=variant)
    assert_status_clean(st)
    gg = (a.float() @ g.float().t()).bfloat16().float()
    uu = (a.float() @ u.float().t()).bfloat16().float()
    r = torch.nn.functional.silu(gg) * uu
    assert y.shape == (m, i)
    assert rel_err(y, r) < 2e-2


def _stage(k_tok, v_tok, cap):
    """[L, Hkv, D] tokens in position order -> staging [Hkv, cap, D] K and V."""
    L, hkv, d = k_tok.shape
    ks = torch.zeros(hkv, cap, d, dtype=k_tok.dtype, device=k_tok.device)
    vs = torch.zeros_like(ks)
    ks[:, :L] = k_tok.transpose(0, 1)
    vs[:, :L] = v_tok.transpose(0, 1)
    return ks, vs


@pytest.mark.parametrize("d,variant", [(64, 0), (64, 1), (64, 3), (128, 0)])
@pytest.mark.parametrize("layout", ["prefix", "suffix", "striped", "noncausal"])
def test_attention(dev, d, variant, layout):
    torch.manual_seed(3)
    L, h, hkv = 700, 8, 2
    q_all = torch.randn(L, h, d, device=dev, dtype=torch.bfloat16)
    k_all = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    v_all = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    if layout == "prefix":
        pos = torch.arange(0, 300, device=dev)
    elif layout == "suffix":
        pos = torch.arange(300, L, device=dev)
    elif layout == "striped":
        pos = torch.arange(1, L, 3, device=dev)
    else:
        pos = torch.arange(100, 400, device=dev)
    causal = layout != "noncausal"
    q = q_all[pos].contiguous()
    ks, vs = _stage(k_all, v_all, cap=1024)
    st = status_tensor(dev)
    o, lse = K.attention(q, ks, vs, pos.int(), L, causal=causal, status=st, variant=variant)
    assert_status_clean(st)
    ro, rl = ref.full_attention(q.float(), k_all.float(), v_all.float(), pos, torch.arange(L, device=dev),
                                causal=causal)
    assert (o.float() - ro).abs().max() < 2e-2
    assert (lse - rl).abs().max() < 2e-2


@pytest.mark.parametrize("variant", [0, 3])
def test_attention_long_gqa(dev, variant):
    torch.manual_seed(4)
    L, h, hkv, d = 4096, 32, 8, 64
    q = torch.randn(L, h, d, device=dev, dtype=torch.bfloat16)
    k = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    v = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    pos = torch.arange(L, device=dev)
    ks, vs = _stage(k, v, cap=L)
    st = status_tensor(dev)
    o, lse = K.attention(q, ks, vs, pos.int(), L, causal=True, status=st, variant=variant)
    assert_status_clean(st)
    ro, rl = ref.full_attention(q.float(), k.float(), v.float(), pos, pos, causal=True)
    assert (o.float() - ro).abs().max() < 2e-2
    assert (lse - rl).abs().max() < 2e-2


def test_rmsnorm_embedding(dev):
    torch.manual_seed(5)
    x = torch.randn(1000, 2048, device=dev, dtype=torch.bfloat16)
    w = torch.rand(2048, device=dev, dtype=torch.bfloat16) + 0.5
    y = K.rmsnorm(x, w, 1e-5)
    r = ref.rmsnorm(x.float(), w.float(), 1e-5)
    assert rel_err(y, r) < 1e-2
    emb = torch.randn(500, 256, device=dev, dtype=torch.bfloat16)
    ids = torch.randint(0, 500, (77,), device=dev, dtype=torch.int32)
    e = K.embedding(ids, emb)
    assert torch.equal(e, emb[ids.long()])


# the three decode GEMV kernels: CUDA-core register loads, bulk-copy streaming, tensor cores
GEMV_KERNELS = {"cuda": dict(tc=0, bulk=0), "bulk": dict(tc=0, bulk=1), "tc": dict(tc=1, bulk=0)}


@pytest.mark.parametrize("kern", list(GEMV_KERNELS))
@pytest.mark.parametrize("b", [1, 2, 4, 8])
def test_gemv(dev, b, kern):
    """Decode GEMV epilogues (f32 + bias, residual, SwiGLU, argmax with logits) on each GEMV
    kernel against float32 (the streaming kernel takes batches up to 4, 8 runs on CUDA cores)."""
    tc = GEMV_KERNELS[kern]
    torch.manual_seed(6)
    kdim, n = 2048, 3072
    x = torch.randn(b, kdim, device=dev, dtype=torch.bfloat16)
    w = torch.randn(n, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    bias = torch.randn(n, device=dev, dtype=torch.bfloat16)
    y = torch.empty(b, n, device=dev, dtype=torch.float32)
    K.gemv(x, w, "f32", bias=bias, y_f32=y, **tc)
    r = x.float() @ w.float().t() + bias.float()
    assert rel_err(y, r) < 1e-3
    res = torch.randn(b, n, device=dev, dtype=torch.bfloat16)
    expect = (x.float() @ w.float().t()).bfloat16().float() + res.float()
    K.gemv(x, w, "residual", y_bf16=res, **tc)
    assert rel_err(res, expect) < 1e-2
    g = torch.randn(1024, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    u = torch.randn(1024, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    out = torch.empty(b, 1024, device=dev, dtype=torch.bfloat16)
    K.gemv(x, K.interleave_gate_up(g, u), "swiglu", y_bf16=out, **tc)
    gg = (x.float() @ g.float().t()).bfloat16().float()
    uu = (x.float() @ u.float().t()).bfloat16().float()
    assert rel_err(out, torch.nn.functional.silu(gg) * uu) < 2e-2
    vocab = 50000
    wl = torch.randn(vocab, kdim, device=dev, dtype=torch.bfloat16)
    am = torch.zeros(b, dtype=torch.int64, device=dev)
    logits = torch.empty(b, vocab, device=dev, dtype=torch.float32)
    K.gemv(x, wl, "argmax", y_f32=logits, argmax=am, **tc)
    tok = torch.empty(b, dtype=torch.int64, device=dev)
    native().argmax_finalize(am, None, tok)
    rl = x.float() @ wl.float().t()
    assert torch.equal(tok, logits.argmax(-1))
    assert rel_err(logits, rl) < 1e-3


@pytest.mark.parametrize("kern", list(GEMV_KERNELS))
@pytest.mark.parametrize("b", [1, 4, 8])
def test_gemv_fused_rmsnorm(dev, b, kern):
    tc = GEMV_KERNELS[kern]
    torch.manual_seed(7)
    kdim, n = 2048, 1024
    x = torch.randn(b, kdim, device=dev, dtype=torch.bfloat16) * 3
    nw = (torch.rand(kdim, device=dev) + 0.5).bfloat16()
    w = torch.randn(n, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    y = torch.empty(b, n, device=dev, dtype=torch.float32)
    K.gemv(x, w, "f32", y_f32=y, norm_w=nw, eps=1e-5, **tc)
    xn = K.rmsnorm(x, nw, 1e-5)
    r = xn.float() @ w.float().t()
    assert rel_err(y, r) < 1e-3
    g = torch.randn(512, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    u = torch.randn(512, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    out = torch.empty(b, 512, device=dev, dtype=torch.bfloat16)
    K.gemv(x, K.interleave_gate_up(g, u), "swiglu", y_bf16=out, norm_w=nw, eps=1e-5, **tc)
    gg = (xn.float() @ g.float().t()).bfloat16().float()
    uu = (xn.float() @ u.float().t()).bfloat16().float()
    assert rel_err(out, torch.nn.functional.silu(gg) * uu) < 2e-2


@pytest.mark.parametrize("kdim,n", [(8192, 2048), (11008, 1001), (1000, 37), (896, 4864), (576, 1600)])
def test_gemv_k_chunks_and_row_tails(dev, kdim, n):
    """K that spans several per-lane chunks or ends mid-chunk, row counts that leave a partial
    row group, and (tensor-core kernel, B = 4 and 8) K ranges that give the 8 warps 1 or 2
    64-element chunks each, against an fp32 reference; shapes the tensor-core kernel does not
    take (rows not a multiple of 16, K not a multiple of 64) run on the CUDA-core kernel."""
    torch.manual_seed(8)
    for b, kw in ((1, GEMV_KERNELS["tc"]), (4, GEMV_KERNELS["tc"]), (8, GEMV_KERNELS["tc"]),
                  (1, GEMV_KERNELS["bulk"]), (2, GEMV_KERNELS["bulk"])):
        x = torch.randn(b, kdim, device=dev, dtype=torch.bfloat16)
        w = torch.randn(n, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
        y = torch.empty(b, n, device=dev, dtype=torch.float32)
        K.gemv(x, w, "f32", y_f32=y, **kw)
        assert rel_err(y, x.float() @ w.float().t()) < 1e-3
        am = torch.zeros(b, dtype=torch.int64, device=dev)
        logits = torch.empty(b, n, device=dev, dtype=torch.float32)
        K.gemv(x, w, "argmax", y_f32=logits, argmax=am, **kw)
        tok = torch.empty(b, dtype=torch.int64, device=dev)
        native().argmax_finalize(am, None, tok)
        assert torch.equal(tok, logits.argmax(-1))


@pytest.mark.parametrize("kdim", [2048, 4096, 896])
@pytest.mark.parametrize("b", [1, 2, 4])
def test_gemv_bulk_bit_identical_to_cuda_core(dev, b, kdim):
    """The streaming kernel keeps the CUDA-core kernel's per-lane summation order: every epilogue
    (f32 + bias, fused RMSNorm, residual, SwiGLU, argmax with logits) gives the same bits, for
    32 KB stages (K = 2048), 64 KB stages (K = 4096; its SwiGLU rows exceed a stage and run on
    the CUDA-core kernel) and a K that is not a multiple of 256 (896)."""
    torch.manual_seed(14)
    n = 1536
    x = torch.randn(b, kdim, device=dev, dtype=torch.bfloat16)
    w = torch.randn(n, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    bias = torch.randn(n, device=dev, dtype=torch.bfloat16)
    nw = (torch.rand(kdim, device=dev) + 0.5).bfloat16()
    res0 = torch.randn(b, n, device=dev, dtype=torch.bfloat16)
    st = status_tensor(dev)
    out = {}
    for kern in ("cuda", "bulk"):
        kw = dict(GEMV_KERNELS[kern], status=st)
        y = torch.empty(b, n, device=dev, dtype=torch.float32)
        K.gemv(x, w, "f32", bias=bias, y_f32=y, **kw)
        yn = torch.empty(b, n, device=dev, dtype=torch.float32)
        K.gemv(x, w, "f32", y_f32=yn, norm_w=nw, eps=1e-5, **kw)
        res = res0.clone()
        K.gemv(x, w, "residual", y_bf16=res, **kw)
        sw = torch.empty(b, n // 2, device=dev, dtype=torch.bfloat16)
        K.gemv(x, w, "swiglu", y_bf16=sw, **kw)
        am = torch.zeros(b, dtype=torch.int64, device=dev)
        logits = torch.empty(b, n, device=dev, dtype=torch.float32)
        K.gemv(x, w, "argmax", y_f32=logits, argmax=am, index_base=7, **kw)
        out[kern] = (y, yn, res, sw, am, logits)
    assert_status_clean(st)
    for u, v in zip(out["cuda"], out["bulk"]):
        assert torch.equal(u, v)


@pytest.mark.parametrize("b", [1, 2, 4])
def test_gemv_chain_matches_separate_launches(dev, b):
    """One cooperative chain launch (output projection + residual, RMSNorm + gate/up + SwiGLU,
    down projection + residual, RMSNorm + LM head + argmax with logits; each phase reads what
    the previous one wrote) gives the same bits as the four GEMVs launched one by one, on two
    launches in a row that share one counter pair (each launch leaves it zeroed)."""
    torch.manual_seed(15)
    hid, inter, vocab = 2048, 8192, 32000
    o = torch.randn(b, hid, device=dev, dtype=torch.bfloat16)
    wo = torch.randn(hid, hid, device=dev, dtype=torch.bfloat16) / math.sqrt(hid)
    wgu = torch.randn(2 * inter, hid, device=dev, dtype=torch.bfloat16) / math.sqrt(hid)
    wd = torch.randn(hid, inter, device=dev, dtype=torch.bfloat16) / math.sqrt(inter)
    wl = torch.randn(vocab, hid, device=dev, dtype=torch.bfloat16) / math.sqrt(hid)
    n1 = (torch.rand(hid, device=dev) + 0.5).bfloat16()
    n2 = (torch.rand(hid, device=dev) + 0.5).bfloat16()
    x0 = torch.randn(b, hid, device=dev, dtype=torch.bfloat16)
    ctr = torch.zeros(2, dtype=torch.int32, device=dev)

    def run(chain):
        x = x0.clone()
        g = torch.empty(b, inter, device=dev, dtype=torch.bfloat16)
        am = torch.zeros(b, dtype=torch.int64, device=dev)
        logits = torch.empty(b, vocab, device=dev, dtype=torch.float32)
        st = status_tensor(dev)
        if chain:
            native().gemv_chain_begin()
        K.gemv(o, wo, "residual", y_bf16=x)
        K.gemv(x, wgu, "swiglu", y_bf16=g, norm_w=n1, eps=1e-5)
        K.gemv(g, wd, "residual", y_bf16=x)
        K.gemv(x, wl, "argmax", y_f32=logits, argmax=am, norm_w=n2, eps=1e-5)
        if chain:
            assert native().gemv_chain_end(ctr, st)
        torch.cuda.synchronize()
        assert_status_clean(st)
        return x, g, am, logits

    want = run(False)
    for _ in range(2):
        got = run(True)
        for u, v in zip(want, got):
            assert torch.equal(u, v)
        assert int(ctr.abs().sum()) == 0


def test_gemv_chain_falls_back_to_separate_launches(dev):
    """A recorded sequence that is not the chain's phase order (two GEMVs), or the chain's order
    at a batch of 8 rows, runs as separate launches: gemv_chain_end returns False and the results
    are those of direct launches."""
    torch.manual_seed(16)
    hid, inter = 2048, 4096
    wo = torch.randn(hid, hid, device=dev, dtype=torch.bfloat16) / math.sqrt(hid)
    wgu = torch.randn(2 * inter, hid, device=dev, dtype=torch.bfloat16) / math.sqrt(hid)
    wd = torch.randn(hid, inter, device=dev, dtype=torch.bfloat16) / math.sqrt(inter)
    wl = torch.randn(1024, hid, device=dev, dtype=torch.bfloat16) / math.sqrt(hid)
    nw = (torch.rand(hid, device=dev) + 0.5).bfloat16()
    ctr = torch.zeros(2, dtype=torch.int32, device=dev)
    for b, full in ((2, False), (8, True)):
        o = torch.randn(b, hid, device=dev, dtype=torch.bfloat16)
        x0 = torch.randn(b, hid, device=dev, dtype=torch.bfloat16)

        def run(record):
            x = x0.clone()
            g = torch.zeros(b, inter, device=dev, dtype=torch.bfloat16)
            am = torch.zeros(b, dtype=torch.int64, device=dev)
            if record:
                native().gemv_chain_begin()
            K.gemv(o, wo, "residual", y_bf16=x)
            K.gemv(x, wgu, "swiglu", y_bf16=g, norm_w=nw, eps=1e-5)
            if full:
                K.gemv(g, wd, "residual", y_bf16=x)
                K.gemv(x, wl, "argmax", argmax=am, norm_w=nw, eps=1e-5)
            if record:
                assert native().gemv_chain_end(ctr) is False
            torch.cuda.synchronize()
            return x, g, am

        for u, v in zip(run(False), run(True)):
            assert torch.equal(u, v)
    assert int(ctr.abs().sum()) == 0


@pytest.mark.parametrize("kern", list(GEMV_KERNELS))
def test_gemv_batch_larger_than_staging(dev, kern):
    """B x K too large for one shared-memory x stage (8 rows x 14336, the Llama-3-8B down
    projection at batch 8): the batch is run in halves; same result as per-row GEMVs."""
    tc = GEMV_KERNELS[kern]
    torch.manual_seed(9)
    b, kdim, n = 8, 14336, 256
    x = torch.randn(b, kdim, device=dev, dtype=torch.bfloat16)
    w = torch.randn(n, kdim, device=dev, dtype=torch.bfloat16) / math.sqrt(kdim)
    res = torch.randn(b, n, device=dev, dtype=torch.bfloat16)
    expect = (x.float() @ w.float().t()).bfloat16().float() + res.float()
    K.gemv(x, w, "residual", y_bf16=res, **tc)
    assert rel_err(res, expect) < 1e-2


@pytest.mark.parametrize("L,T,h,hkv,d", [(1, 1, 4, 1, 64), (129, 1, 4, 1, 128), (300, 300, 16, 2, 128),
                                         (257, 2, 8, 8, 64), (1000, 130, 16, 2, 64),
                                         (500, 200, 14, 2, 64), (300, 300, 24, 8, 128)])
def test_attention_edge_shapes(dev, L, T, h, hkv, d):
    """A single key, a single query, MQA (one KV head), 8-head GQA groups, no GQA, a query block
    one row past a tile, groups of 7 and 3 query heads: the queries are the last T positions of
    an L-token context."""
    torch.manual_seed(12)
    q_all = torch.randn(L, h, d, device=dev, dtype=torch.bfloat16)
    k_all = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    v_all = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    pos = torch.arange(L - T, L, device=dev)
    ks, vs = _stage(k_all, v_all, cap=max(128, L))
    st = status_tensor(dev)
    o, lse = K.attention(q_all[pos].contiguous(), ks, vs, pos.int(), L, causal=True, status=st)
    assert_status_clean(st)
    ro, rl = ref.full_attention(q_all[pos].float(), k_all.float(), v_all.float(), pos,
                                torch.arange(L, device=dev), causal=True)
    assert (o.float() - ro).abs().max() < 2e-2
    assert (lse - rl).abs().max() < 2e-2


@pytest.mark.parametrize("d", [64, 128])
def test_attention_cta_orders_bit_identical(dev, d):
    """The two CTA orders (KV-head major; heaviest q-tile pairs of all heads first) only change
    which CTA runs when: every row's output and LSE are the same bits, here on one context-
    parallel rank's zigzag rows (the case the pair-major order is for)."""
    from hetero_cp_ringattn_b200.parallel.capacity import equal_chunks
    from hetero_cp_ringattn_b200.parallel.strategy import layout_positions
    torch.manual_seed(6)
    L, h, hkv = 4096, 8, 2
    pos = torch.as_tensor(layout_positions(equal_chunks(L, 4), "zigzag")[1], device=dev)
    k_all = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    v_all = torch.randn(L, hkv, d, device=dev, dtype=torch.bfloat16)
    q = torch.randn(len(pos), h, d, device=dev, dtype=torch.bfloat16)
    ks, vs = _stage(k_all, v_all, cap=L)
    outs = []
    for order in (0, 1):
        st = status_tensor(dev)
        outs.append(K.attention(q, ks, vs, pos.int(), L, causal=True, status=st, order=order))
        assert_status_clean(st)
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    ro, _ = ref.full_attention(q.float(), k_all.float(), v_all.float(), pos, torch.arange(L, device=dev),
                               causal=True)
    assert (outs[1][0].float() - ro).abs().max() < 2e-2
