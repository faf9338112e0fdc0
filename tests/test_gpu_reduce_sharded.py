"""Sharded full reductions on one GPU: per-shard records combined in shard order.

One record over a whole tensor combines to exactly what the full reduction
(mag_blas_{sum,mean,min,max}_f32, magnetron/magnetron_cpu.c:1034-1152) gives on
the device.  Several shards combine to the oracle's value within the reduction
tolerance (MIN/MAX exactly); the combine is deterministic; bad arguments are
rejected before any launch.
"""
import ctypes as C

import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle, pad6
from gpu_util import device

pytestmark = pytest.mark.gpu

OPS = ["SUM", "MEAN", "MIN", "MAX"]


def _records(dev, n):
    import torch
    return torch.zeros(3 * n, dtype=torch.float64, device=f"cuda:{dev.ordinal}")


def _combine(dev, op, recs, n):
    r = dev.tensor((1,))
    dev.reduce_combine(op, r.data_ptr, recs.data_ptr(), n)
    return r.read()[0]


@pytest.mark.parametrize("shape", [(1,), (7, 3, 2), (4097, 5, 3), (1 << 22,), (8, 8, 8, 8, 8, 8)])
def test_one_record_equals_full_reduction(shape):
    dev, o = device(), oracle()
    x = o.stream(0x5EED7000 + len(shape)).uniform(int(np.prod(shape)), -1.0, 1.0)
    t = dev.tensor(shape)
    t.write(x)
    recs = _records(dev, 1)
    dev.reduce_partial(t, recs.data_ptr())
    for op in OPS:
        full = dev.op(op, t).read()[0]
        got = _combine(dev, op, recs, 1)
        assert np.float32(got).view(np.uint32) == np.float32(full).view(np.uint32), (op, got, full)
    assert MB.ReducePart.from_buffer_copy(recs.cpu().numpy().tobytes()).count == x.size


@pytest.mark.parametrize("nshards", [2, 3, 8])
def test_shards_combine_to_oracle(nshards):
    dev, o = device(), oracle()
    n = (1 << 20) + 37
    x = o.stream(0x5EED7100 + nshards).normal(n + (n & 1), 0.0, 1.0)[:n]
    recs = _records(dev, nshards)
    base = recs.data_ptr()
    keep = []
    bounds = np.linspace(0, n, nshards + 1).astype(np.int64)
    for i in range(nshards):
        part = x[bounds[i]:bounds[i + 1]]
        t = dev.tensor((part.size,))
        t.write(part)
        dev.reduce_partial(t, base + i * MB.REDUCE_PART_BYTES)
        keep.append(t)
    s6 = pad6((n,))
    for op in OPS:
        want = o.reduce(op, x, s6)
        got = _combine(dev, op, recs, nshards)
        if op in ("MIN", "MAX"):
            assert got == want, (op, got, want)
        else:
            assert abs(got - want) <= 1e-6 * max(1.0, abs(want)), (op, got, want)
        assert _combine(dev, op, recs, nshards) == got  # deterministic
    # records carry each shard's own count, so MEAN divides by the total
    rec = recs.cpu().numpy().reshape(nshards, 3)
    assert rec[:, 2].view(np.uint64).sum() == n


def test_record_fields():
    dev, o = device(), oracle()
    x = o.stream(0x5EED7200).uniform(5000, -3.0, 2.0)
    t = dev.tensor((50, 100))
    t.write(x)
    recs = _records(dev, 1)
    dev.reduce_partial(t, recs.data_ptr())
    raw = recs.cpu().numpy().tobytes()
    rec = MB.ReducePart.from_buffer_copy(raw)
    assert rec.count == 5000
    assert np.float32(rec.min) == x.min() and np.float32(rec.max) == x.max()
    assert abs(rec.sum - float(np.sum(x.astype(np.float64)))) <= 1e-9 * 5000


def test_rejections():
    dev = device()
    t = dev.tensor((16,))
    recs = _records(dev, 2)
    r = dev.tensor((1,))
    L = dev.L
    assert L.mag_cuda_reduce_combine_f32(dev.p, MB.OP["SUM"], r.data_ptr, recs.data_ptr(), 0) == MB.E_INVALID
    assert L.mag_cuda_reduce_combine_f32(dev.p, MB.OP["ADD"], r.data_ptr, recs.data_ptr(), 1) == MB.E_INVALID
    assert L.mag_cuda_reduce_combine_f32(dev.p, MB.OP["SUM"], r.data_ptr, recs.data_ptr() + 4, 1) == MB.E_INVALID
    d = (C.c_int64 * 6)(*[int(v) for v in t.t.shape])
    s = (C.c_int64 * 6)(*[int(v) for v in t.t.strides])
    assert L.mag_cuda_reduce_partial_f32(dev.p, recs.data_ptr() + 4, t.data_ptr, d, s) == MB.E_INVALID
    assert L.mag_cuda_reduce_partial_f32(dev.p, None, t.data_ptr, d, s) == MB.E_INVALID
    dev.sync()
