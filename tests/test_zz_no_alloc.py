"""The allocation-free decode-attention entry point, called through its exported C symbol.

For callers that cannot allocate device memory (they only hand over inputs and outputs), the
library offers `hcp_decode_attention_noalloc`, whose split-KV scratch lives in a static device
array inside the library. This test loads the extension as a plain shared library with ctypes,
calls that symbol twice in a row, and checks each result against the regular entry point (the
domain runtime's decode attention + combine, which takes its scratch as arguments).

The file is named so that pytest collects it last; it passes both alone in a fresh process and
after the rest of the suite.
"""

import ctypes
import math

import pytest
import torch

from hetero_cp_ringattn_b200.ops import _ext

pytestmark = pytest.mark.gpu

H, HKV, D, PAGE = 8, 2, 64, 256


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
    return fn, err, nbytes


def test_noalloc_decode_matches_runtime_entry_point(dev):
    fn, err, nbytes = _lib()
    native = _ext.native()
    layers, pages = 2, 8
    rt = native.Runtime(0, 1, dev.index or 0, layers, pages, PAGE, HKV, D, H, 1024, 4, 2000)
    arena = rt.arena()
    g = torch.Generator(device=dev).manual_seed(21)
    arena.copy_(torch.randn(arena.shape, device=dev, generator=g).to(torch.bfloat16))
    B, splits = 3, 8
    page_tables = torch.tensor([[5, 2, 7], [1, 3, 0], [6, 4, 2]], dtype=torch.int32, device=dev)
    n_tokens = torch.tensor([700, 257, 31], dtype=torch.int32, device=dev)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream(dev)
    for call, layer in enumerate([1, 0]):
        q = torch.randn(B, H, D, device=dev, generator=g).to(torch.bfloat16)
        # regular entry point: scratch passed in by the caller
        part_o = torch.empty(B * H * splits * D, device=dev)
        part_l = torch.empty(B * H * splits, device=dev)
        cnt = torch.zeros(B * HKV + 1, dtype=torch.int32, device=dev)
        want = torch.empty(B, H * D, device=dev, dtype=torch.bfloat16)
        rt.decode_attn(q, layer, page_tables, n_tokens, scale, splits, part_o, part_l, cnt,
                       None, 1, 2 * call + 1)
        rt.decode_combine(want, B, H, None, 1, 2 * call + 1)
        # allocation-free entry point through the C ABI
        got = torch.empty(B, H * D, device=dev, dtype=torch.bfloat16)
        rc = fn(q.data_ptr(), arena.data_ptr(), layers, pages, PAGE, HKV, D, layer,
                page_tables.data_ptr(), page_tables.stride(0), n_tokens.data_ptr(), B, H, scale,
                splits, got.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, err().decode()
        torch.cuda.synchronize(dev)
        assert torch.isfinite(got.float()).all()
        assert (got.float() - want.float()).abs().max() < 2e-2, f"call {call}"
    rt.check()
    # a problem larger than the static scratch is rejected with a clear message
    too_many_splits = 4096
    assert nbytes(B, H, HKV, D, too_many_splits) > (4 << 20)
    rc = fn(q.data_ptr(), arena.data_ptr(), layers, pages, PAGE, HKV, D, 0, page_tables.data_ptr(),
            page_tables.stride(0), n_tokens.data_ptr(), B, H, scale, too_many_splits,
            got.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
    assert rc < 0 and b"static maximum" in err()
    rt.shutdown()
