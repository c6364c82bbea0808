"""Native coordinator smoke (no Python in the loop): build the C++ program against the runtime and
kernels with nvcc for sm_100a, run it (config checks everywhere; one emulated 3-domain ring layer
on a GPU)."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "hetero_cp_ringattn_b200", "csrc")
OUT = os.path.join(ROOT, "build", "native")


def build_smoke() -> str:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    os.makedirs(OUT, exist_ok=True)
    exe = os.path.join(OUT, "hcp_runtime_smoke")
    srcs = ["tests/runtime_smoke.cu", "core/runtime.cu", "kernels/attn_fwd_sm100.cu",
            "kernels/elementwise.cu", "kernels/gemm_sm100.cu", "kernels/decode.cu"]
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-lineinfo",
           "-I" + os.path.join(CSRC, "include"), "-I" + CSRC, "-o", exe] + \
        [os.path.join(CSRC, s) for s in srcs] + ["-lcudart"]
    subprocess.run(cmd, check=True, capture_output=True, text=True, timeout=600)
    return exe


@pytest.fixture(scope="module")
def smoke_exe():
    if not (shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc")):
        pytest.skip("nvcc not available")
    return build_smoke()


def test_native_smoke_builds_and_checks_config(smoke_exe):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([smoke_exe], capture_output=True, text=True, timeout=120, env=env)
    assert r.returncode == 0, r.stderr
    assert "config ok" in r.stdout


@pytest.mark.gpu
def test_native_smoke_runs_ring_layer_on_gpu(smoke_exe):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    r = subprocess.run([smoke_exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "[smoke] ok" in r.stdout
