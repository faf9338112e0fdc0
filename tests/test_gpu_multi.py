"""Sharded work on two GPUs (skipped with fewer).  Element ranges: each rank adds its
contiguous range of x + y and the ranges are all-gathered over NCCL, bit-exact
against the host sum; each rank reduces its range to a record, the records are
all-gathered in rank order and combined into the full SUM/MEAN/MIN/MAX on every
rank, equal on all ranks and within the reduction tolerance of the oracle.  The deep MLP: rows
sharded, logits gathered, bit-identical with one GPU's forward of every row.
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


MLP_WORKER = textwrap.dedent("""
    import datetime, os, sys
    rank, world = int(sys.argv[1]), int(sys.argv[2])
    os.environ["MAG_CUDA_DEVICE"] = str(rank)
    import numpy as np, torch, torch.distributed as dist
    sys.path[:0] = [{pkg!r}, {orc!r}, {tests!r}]
    import dp, mag_b200 as MB
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    total, d, hidden, d_out = 10240, 4096, 8, 1000
    dev = MB.Device()

    class _A:
        def __init__(self, ptr, k):
            self.__cuda_array_interface__ = {{"shape": (k,), "typestr": "<f4", "data": (ptr, False),
                                              "version": 3, "stream": None}}

    std = (2.0 / d) ** 0.5
    Ws = []
    for i in range(hidden):
        W = dev.tensor((d, d))
        dev.fill_random_normal(W, 0.0, std, MB.Pcg(0x5EED1005 + i))
        Ws.append(W)
    Wo = dev.tensor((d, d_out))
    dev.fill_random_normal(Wo, 0.0, std, MB.Pcg(0x5EED1105))
    xall = torch.randn(total * d, generator=torch.Generator().manual_seed(0x5EED1205)).numpy()

    def forward(rows, x):
        X = dev.tensor((rows, d))
        X.write(x)
        keep = [X]
        dev.eager = False
        try:
            h = X
            for W in Ws:
                B = dev.tensor((rows, d))
                keep.append(B)
                h = dev.op("GELU", dev.op("ADD", dev.op("MATMUL", h, W), B), inplace=True)
            Bo = dev.tensor((rows, d_out))
            keep.append(Bo)
            z = dev.op("ADD", dev.op("MATMUL", h, Wo), Bo)
        finally:
            dev.eager = True
        P = dev.tensor((rows * d_out,))
        dev.graph_exec(z, fused=True)
        MB.check(dev.L.mag_cuda_softmax_rows_f32(dev.p, P.data_ptr, z.data_ptr, rows, d_out), "softmax")
        MB.check(dev.L.mag_cuda_synchronize(dev.p), "sync")
        logits = torch.as_tensor(_A(z.data_ptr, rows * d_out), device=f"cuda:{{rank}}").clone()
        probs = torch.as_tensor(_A(P.data_ptr, rows * d_out), device=f"cuda:{{rank}}").clone()
        dev.graph_release(z)
        return logits, probs

    start, rows = dp.shard_rows(total, world, rank)
    assert rows % 4 == 0
    lz, lp = forward(rows, xall[start * d:(start + rows) * d])
    gz = dp.gather_rows(lz, total, d_out, world, rank).cpu().numpy()
    gp = dp.gather_rows(lp, total, d_out, world, rank).cpu().numpy()
    if rank == 0:
        fz, fp = forward(total, xall)
        fz, fp = fz.cpu().numpy(), fp.cpu().numpy()
        assert np.array_equal(gz.view(np.uint32), fz.view(np.uint32)), "gathered logits differ from one GPU's"
        assert np.array_equal(gp.view(np.uint32), fp.view(np.uint32)), "gathered probabilities differ"
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


def _run_two(worker):
    code = worker.format(pkg=os.path.join(ROOT, "magnetron-pre-oss-release-old_b200"),
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


def test_two_gpus_shard_elements_and_reduce():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_two(WORKER)


def test_two_gpus_deep_mlp_gathered_logits_equal_one_gpu():
    """The deep MLP (8 x 4096^2 + GELU, 4096 x 1000, row softmax; 10240 rows) with rows sharded
    over two GPUs and the logits and probabilities all-gathered over NCCL: bit-identical with
    the same forward of all rows on one GPU.  Each shard holds 5120 rows (a multiple of 4, and
    enough tiles on every layer that neither run splits K), so every output is computed the
    same way in both."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_two(MLP_WORKER)
