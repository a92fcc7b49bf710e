"""The stream-K work decomposition of the CTA-pair kernels (PairWork in
csrc/gemm_common.cuh), checked on the host: tests/pairwork_check.cu is built
with nvcc against the kernels' own header and run (see its header for the
invariants)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


@pytest.mark.skipif(not os.path.exists(NVCC), reason="nvcc not available")
def test_pair_work_decomposition_covers_every_k_block_once(tmp_path):
    exe = tmp_path / "pairwork_check"
    subprocess.run([NVCC, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", os.path.join(ROOT, "lightx2v-rs_b200", "csrc"),
                    os.path.join(ROOT, "tests", "pairwork_check.cu"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout[-2000:]
    assert " 0 failing" in out.stdout
