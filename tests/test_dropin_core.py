"""The unchanged magnetron core driving this backend through MAG_ENABLE_CUDA.

oracle/_ref/libmagnetron_cudacore.so is the reference's magnetron.c and
magnetron_cpu.c compiled from their own sources with -DMAG_ENABLE_CUDA and
linked against libmagnetron_cuda.so (oracle/Makefile, target cudacore).  It
exists where the reference sources were available at build time.
"""
import json
import os
import subprocess
import sys

import pytest

from oracle import CUDACORE_SO

HERE = os.path.dirname(os.path.abspath(__file__))
needs_core = pytest.mark.skipif(not os.path.exists(CUDACORE_SO), reason="reference core not built here")


def run(mode):
    out = subprocess.run([sys.executable, os.path.join(HERE, "dropin_driver.py"), mode], capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


@needs_core
def test_core_falls_back_to_cpu_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    res = run("fallback")
    assert res["device_type"] == 0  # mag_compute_device_init retries with the CPU (magnetron/magnetron.c:895-899)


@needs_core
@pytest.mark.gpu
def test_core_runs_ops_on_cuda():
    res = run("ops")
    assert res["device_type"] == 1 and "B200" in res["device_name"], res
    assert res["matmul_exact"] and res["sigmoid_inplace_exact"] and res["h2_aliases_h4"], res
    assert res["sum_rel_err"] <= 1e-6 and res["scalar_accessor"], res
    assert res["tanh_dv_max_rel"] <= 1e-6, res
    assert res["launches"] >= 5, res
