"""The host runtime library's own C++ test (`csrc/tests/host_test.cpp`), built with g++ and run
on the CPU: reference golden vectors for layouts, capacity allocation, admission and the KV-growth
schedule, the page allocator, the batch scheduler core under concurrent producers, and the control
protocol's binary frames (round trips, every truncation, versions, lying counts), and the f64
ring-attention oracle against full attention on the reference's cases plus causal GQA layouts."""

import os
import shutil
import subprocess

import pytest

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    "hetero_cp_ringattn_b200", "csrc")
SOURCES = ["tests/host_test.cpp"] + [f"host/{f}" for f in ("layout.cpp", "capacity.cpp",
                                                         "schedule.cpp", "pages.cpp",
                                                         "scheduler.cpp", "protocol.cpp",
                                                         "ref_attention.cpp")]


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_host_library_native_tests(tmp_path):
    exe = str(tmp_path / "host_test")
    cc = subprocess.run(["g++", "-O2", "-std=c++17", "-Wall", "-Wextra", "-Wshadow", "-Werror",
                         "-pthread", "-o", exe] +
                        [os.path.join(CSRC, s) for s in SOURCES], capture_output=True, text=True,
                        timeout=300)
    assert cc.returncode == 0, cc.stderr[-4000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and "host_test ok" in run.stdout, run.stdout + run.stderr
