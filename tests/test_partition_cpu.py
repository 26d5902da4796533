"""The launch partitions (alveare_b200/csrc/stream.cuh: FastDiv, Partition)
are host-built 32-bit arithmetic; tests/partition_check.cu compares them
with plain 64-bit division over the kernels' shapes and several grids.
Compiled as host code with nvcc (no GPU needed)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "alveare_b200", "csrc")


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="nvcc not available")
def test_partition_arithmetic_matches_64bit(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "partition_check"
    subprocess.run([nvcc, "-std=c++17", "-O2", "-Wno-deprecated-gpu-targets", "-I", CSRC, "-o", str(exe),
                    os.path.join(HERE, "partition_check.cu")], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "0 bad" in out.stdout
