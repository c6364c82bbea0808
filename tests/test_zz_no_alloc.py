"""The allocation-free decode-attention entry point, called through its exported C symbol.

For callers that cannot allocate device memory (they only hand over inputs and outputs), the
library offers `hcp_decode_attention_noalloc`, whose split-KV scratch and status word live in a
static device array inside the library. This test loads the extension as a plain shared library
with ctypes, calls that symbol twice in a row per shape, and checks each result against both the
regular entry point (the domain runtime's decode attention + combine, which takes its scratch as
arguments) and a float32 PyTorch reference of the same attention. It covers head_dim 64 and 128
and GQA groups of 1, 4 and 8 query heads per KV head, the device status query, the bound on a
row's KV length and the argument checks.

The file is named so that pytest collects it last; it passes both alone in a fresh process and
after the rest of the suite.
"""

import ctypes
import math

import pytest
import torch

from hetero_cp_ringattn_b200.ops import _ext

pytestmark = pytest.mark.gpu

PAGE = 256
K_OUT_OF_BOUNDS = 18      # StatusCode::kOutOfBounds
SITE_KV_LENGTH = 304      # decode_attn_kernel: n_tokens[b] outside [0, pt_stride * page]


def _lib():
    lib = ctypes.CDLL(_ext.so_path())
    fn = lib.hcp_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p]
    err = lib.hcp_decode_attention_noalloc_error
    err.restype = ctypes.c_char_p
    nbytes = lib.hcp_decode_attention_noalloc_scratch_bytes
    nbytes.restype = ctypes.c_ulonglong
    nbytes.argtypes = [ctypes.c_int] * 5
    status = lib.hcp_decode_attention_noalloc_status
    status.restype = ctypes.c_int
    status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    return fn, err, nbytes, status


def _status(status_fn, stream):
    words = (ctypes.c_int * 4)()
    assert status_fn(words, ctypes.c_void_p(stream.cuda_stream)) == 0
    return list(words)


def _reference(q, arena, layer, page_tables, n_tokens, scale, hkv):
    """float32 attention of each row's query heads over its first n_tokens keys / values."""
    B, H, D = q.shape
    G = H // hkv
    out = torch.empty(B, H, D, device=q.device)
    for b in range(B):
        n = int(n_tokens[b])
        s = torch.arange(n, device=q.device)
        pages = page_tables[b].long()[s // PAGE]
        k = arena[layer, pages, 0, :, s % PAGE].float()      # [n, Hkv, D]
        v = arena[layer, pages, 1, :, s % PAGE].float()
        for h in range(H):
            sc = (k[:, h // G] @ q[b, h].float()) * scale
            out[b, h] = torch.softmax(sc, 0) @ v[:, h // G]
    return out.view(B, H * D)


@pytest.mark.parametrize("d,heads,hkv", [(64, 8, 2), (128, 4, 4), (128, 16, 2), (64, 8, 1), (64, 24, 2)])
def test_noalloc_decode_matches_runtime_entry_point_and_fp32(dev, d, heads, hkv):
    fn, err, nbytes, status = _lib()
    native = _ext.native()
    layers, pages = 2, 8
    rt = native.Runtime(0, 1, dev.index or 0, layers, pages, PAGE, hkv, d, heads, 1024, 4, 2000)
    arena = rt.arena()
    g = torch.Generator(device=dev).manual_seed(21 + d + heads)
    arena.copy_(torch.randn(arena.shape, device=dev, generator=g).to(torch.bfloat16))
    B, splits = 3, 8
    page_tables = torch.tensor([[5, 2, 7], [1, 3, 0], [6, 4, 2]], dtype=torch.int32, device=dev)
    n_tokens = torch.tensor([700, 257, 31], dtype=torch.int32, device=dev)
    scale = 1.0 / math.sqrt(d)
    stream = torch.cuda.current_stream(dev)
    _status(status, stream)   # start from a clean status word
    for call, layer in enumerate([1, 0]):
        q = torch.randn(B, heads, d, device=dev, generator=g).to(torch.bfloat16)
        # regular entry point: scratch passed in by the caller
        part_o = torch.empty(B * heads * splits * d, device=dev)
        part_l = torch.empty(B * heads * splits, device=dev)
        cnt = torch.zeros(B * hkv + 1, dtype=torch.int32, device=dev)
        want = torch.empty(B, heads * d, device=dev, dtype=torch.bfloat16)
        rt.decode_attn(q, layer, page_tables, n_tokens, scale, splits, part_o, part_l, cnt,
                       None, 1, 2 * call + 1)
        rt.decode_combine(want, B, heads, None, 1, 2 * call + 1)
        # allocation-free entry point through the C ABI
        got = torch.empty(B, heads * d, device=dev, dtype=torch.bfloat16)
        rc = fn(q.data_ptr(), arena.data_ptr(), layers, pages, PAGE, hkv, d, layer,
                page_tables.data_ptr(), page_tables.stride(0), n_tokens.data_ptr(), B, heads,
                scale, splits, got.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, err().decode()
        assert _status(status, stream) == [0, 0, 0, 0]
        ref = _reference(q, arena, layer, page_tables, n_tokens, scale, hkv)
        assert torch.isfinite(got.float()).all()
        assert (got.float() - want.float()).abs().max() < 2e-2, f"call {call}: vs runtime"
        assert (got.float() - ref).abs().max() < 2e-2, f"call {call}: vs fp32 reference"
    rt.check()
    rt.shutdown()


def test_noalloc_decode_bounds_and_rejections(dev):
    fn, err, nbytes, status = _lib()
    native = _ext.native()
    d, heads, hkv, layers, pages = 64, 8, 2, 1, 8
    rt = native.Runtime(0, 1, dev.index or 0, layers, pages, PAGE, hkv, d, heads, 1024, 4, 2000)
    arena = rt.arena()
    g = torch.Generator(device=dev).manual_seed(5)
    arena.copy_(torch.randn(arena.shape, device=dev, generator=g).to(torch.bfloat16))
    stream = torch.cuda.current_stream(dev)
    scale = 1.0 / math.sqrt(d)
    B, splits = 2, 4
    q = torch.randn(B, heads, d, device=dev, generator=g).to(torch.bfloat16)
    page_tables = torch.tensor([[3, 1], [0, 6]], dtype=torch.int32, device=dev)
    got = torch.empty(B, heads * d, device=dev, dtype=torch.bfloat16)
    _status(status, stream)
    # row 1 claims more keys than its page-table row holds: clamped to 2 pages, and reported
    n_tokens = torch.tensor([300, 2 * PAGE + 40], dtype=torch.int32, device=dev)
    rc = fn(q.data_ptr(), arena.data_ptr(), layers, pages, PAGE, hkv, d, 0, page_tables.data_ptr(),
            page_tables.stride(0), n_tokens.data_ptr(), B, heads, scale, splits, got.data_ptr(),
            ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, err().decode()
    words = _status(status, stream)
    assert words[0] == K_OUT_OF_BOUNDS and words[1] == SITE_KV_LENGTH and words[3] == 1, words
    assert _status(status, stream) == [0, 0, 0, 0]          # reading the status resets it
    clamped = torch.tensor([300, 2 * PAGE], dtype=torch.int32, device=dev)
    ref = _reference(q, arena, 0, page_tables, clamped, scale, hkv)
    assert (got.float() - ref).abs().max() < 2e-2
    # argument checks: a page-table stride below 1, non-positive sizes, too much scratch
    rc = fn(q.data_ptr(), arena.data_ptr(), layers, pages, PAGE, hkv, d, 0, page_tables.data_ptr(),
            0, n_tokens.data_ptr(), B, heads, scale, splits, got.data_ptr(),
            ctypes.c_void_p(stream.cuda_stream))
    assert rc < 0 and b"stride" in err()
    assert nbytes(-1, heads, hkv, d, splits) == 2 ** 64 - 1
    assert nbytes(B, heads, hkv, d, 4096) > (4 << 20)
    rc = fn(q.data_ptr(), arena.data_ptr(), layers, pages, PAGE, hkv, d, 0, page_tables.data_ptr(),
            page_tables.stride(0), n_tokens.data_ptr(), B, heads, scale, 4096, got.data_ptr(),
            ctypes.c_void_p(stream.cuda_stream))
    assert rc < 0 and b"static maximum" in err()
    rt.check()
    rt.shutdown()
