"""The debug build's extra device-side index checks (`HCP_DEBUG_BOUNDS=1`): the kernels that read
page ids from page tables compile with the checks enabled (nvcc for sm_100a, compile only, no GPU
needed). In default builds the checks are compiled out."""

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

import pytest

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    "hetero_cp_ringattn_b200", "csrc")


@pytest.mark.skipif(not (shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc")),
                    reason="nvcc not available")
def test_kernels_compile_with_debug_bounds_checks(tmp_path):
    import torch.utils.cpp_extension as ce
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    inc = ["-I" + os.path.join(CSRC, "include"), "-I" + CSRC] + ["-I" + p for p in ce.include_paths()]

    def build(src):
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-DHCP_DEBUG_BOUNDS=1", "-O3",
               "-std=c++17", "--use_fast_math", "--expt-relaxed-constexpr", *inc, "-c",
               os.path.join(CSRC, "kernels", src), "-o", str(tmp_path / (src + ".o"))]
        return subprocess.run(cmd, capture_output=True, text=True, timeout=1500)

    with ThreadPoolExecutor(2) as ex:
        results = list(ex.map(build, ["decode.cu", "elementwise.cu"]))
    for r in results:
        assert r.returncode == 0, r.stderr[-3000:]
