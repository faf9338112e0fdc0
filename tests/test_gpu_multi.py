"""Sharded element ranges on two GPUs (skipped with fewer): each rank adds its
contiguous range of x + y and the ranges are all-gathered over NCCL, bit-exact
against the host sum; each rank reduces its range to a record, the records are
all-gathered in rank order and combined into the full SUM/MEAN/MIN/MAX on every
rank, equal on all ranks and within the reduction tolerance of the oracle.
No rank fails on purpose here (failure paths are covered with gloo ranks)."""
import os
import socket
import subprocess
import sys
import textwrap

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

pytestmark = pytest.mark.gpu

WORKER = textwrap.dedent("""
    import datetime, os, sys
    rank, world = int(sys.argv[1]), int(sys.argv[2])
    os.environ["MAG_CUDA_DEVICE"] = str(rank)
    import numpy as np, torch, torch.distributed as dist
    sys.path[:0] = [{pkg!r}, {orc!r}, {tests!r}]
    import dp, mag_b200 as MB
    from oracle import Oracle, pad6
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    o = Oracle()
    n = (1 << 22) + 6
    x = o.stream(0x5EED0E00).normal(n, 0.0, 1.0)
    y = o.stream(0x5EED0E01).normal(n, 0.0, 1.0)
    start, cnt = dp.shard_rows(n, world, rank)
    dev = MB.Device()
    assert dev.ordinal == rank
    xs, ys = dev.tensor((cnt,)), dev.tensor((cnt,))
    xs.write(x[start:start + cnt])
    ys.write(y[start:start + cnt])
    r = dev.op("ADD", xs, ys)
    dev.sync()

    class _A:
        def __init__(self, ptr, k):
            self.__cuda_array_interface__ = {{"shape": (k,), "typestr": "<f4", "data": (ptr, False),
                                              "version": 3, "stream": None}}

    local = torch.as_tensor(_A(r.data_ptr, cnt), device=f"cuda:{{rank}}")
    full = dp.gather_rows(local, n, 1, world, rank).cpu().numpy()
    assert np.array_equal(full.view(np.uint32), (x + y).view(np.uint32)), "gathered ADD differs"
    s6 = pad6((n,))
    res = dev.tensor((4,))
    for i, op in enumerate(["SUM", "MEAN", "MIN", "MAX"]):
        dp.reduce_full(dev, op, xs, res.data_ptr + 4 * i, world)
    got = res.read()
    everyone = [None] * world
    dist.all_gather_object(everyone, got.tobytes())
    assert all(e == everyone[0] for e in everyone), "ranks disagree"
    for i, op in enumerate(["SUM", "MEAN", "MIN", "MAX"]):
        want = o.reduce(op, x, s6)
        tol = 0.0 if op in ("MIN", "MAX") else 1e-6 * max(1.0, abs(want))
        assert abs(got[i] - want) <= tol, (op, got[i], want)
    dist.barrier(device_ids=[rank])
    dev.close()
    dist.destroy_process_group()
    print("OK", flush=True)
""")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_gpus_shard_elements_and_reduce():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    code = WORKER.format(pkg=os.path.join(ROOT, "magnetron-pre-oss-release-old_b200"),
                         orc=os.path.join(ROOT, "oracle"), tests=HERE, port=_port())
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-c", code, str(r), "2"], stdout=subprocess.PIPE,
                              stderr=subprocess.PIPE, text=True, env=env) for r in range(2)]
    outs = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, err = p.communicate()
        outs.append((p.returncode, out, err))
    for rc, out, err in outs:
        assert rc == 0 and "OK" in out, err[-3000:]
