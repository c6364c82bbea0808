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
