"""The native extension's host-side checks, on a machine without a GPU.

Parity: the reference's no-op domain runtime validates its configuration before doing anything
(src/ringattn_runtime.cc:10-70: domain id, positive chunk and block sizes, a complete global
config). Here `DomainRuntime::Init` rejects a bad arena geometry or rank layout with an
`InvalidArgument` status before the first CUDA call, and a machine without a usable device gets a
CUDA status back, not a crash. Skipped when the extension is not built.
"""

import pytest
import torch

from hetero_cp_ringattn_b200.ops import _ext

pytestmark = pytest.mark.skipif(not _ext.available(), reason="extension not built")

# rank, world, device, layers, pages, page, hkv, d, num_heads, stage_cap, max_batch, budget_ms
GOOD = dict(rank=0, world=2, device=0, layers=2, pages=4, page=128, hkv=8, d=64, num_heads=32,
            stage_cap=1024, max_batch=1, budget_ms=1000)


def _runtime(**kw):
    a = dict(GOOD, **kw)
    return _ext.native().Runtime(a["rank"], a["world"], a["device"], a["layers"], a["pages"],
                                 a["page"], a["hkv"], a["d"], a["num_heads"], a["stage_cap"],
                                 a["max_batch"], a["budget_ms"])


@pytest.mark.parametrize("kw,msg", [
    ({"world": 0}, "world out of range"),
    ({"world": 100}, "world out of range"),
    ({"rank": 2}, "rank out of range"),
    ({"rank": -1}, "rank out of range"),
    ({"d": 96}, "head_dim must be 64 or 128"),
    ({"page": 100}, "page size must be a multiple of 128"),
    ({"page": 0}, "page size must be a multiple of 128"),
    ({"layers": 0}, "arena geometry must be positive"),
    ({"pages": 0}, "arena geometry must be positive"),
    ({"num_heads": 30}, "num_heads % hkv"),
])
def test_runtime_rejects_bad_config_before_touching_the_device(kw, msg):
    with pytest.raises(RuntimeError, match="code=1: " + msg):
        _runtime(**kw)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_runtime_without_a_device_returns_a_cuda_status():
    with pytest.raises(RuntimeError, match="cudaSetDevice"):
        _runtime()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the host-tensor path")
def test_kernel_entry_points_refuse_host_tensors():
    m = _ext.native()
    x = torch.zeros(128, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        m.rmsnorm(x, torch.ones(64, dtype=torch.bfloat16), torch.empty_like(x), 1e-5)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        m.gemv(x, torch.zeros(256, 64, dtype=torch.bfloat16), 0)
