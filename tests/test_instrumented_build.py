"""The diagnostic builds of libq2b (per-role cycle counters of the pair GEMM
and of the RHT/EDEN kernel) still compile: nvcc cross-compiles sm_100a without
a GPU, so the flags cannot rot unnoticed between the runs that use them."""
import os
import shutil
import subprocess

import pytest

from cloverlm_b200 import build as b


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="nvcc not available")
def test_stats_build_compiles(tmp_path):
    out = tmp_path / "libq2b_stats.o"
    cmd = [b._nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17", "-c",
           "-DQ2B_GEMM2_STATS", "-DQ2B_RHT_STATS", "-o", str(out), os.path.join(b.SRC_DIR, "libq2b.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-4000:]
    assert out.stat().st_size > 0
