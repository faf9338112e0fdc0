"""Asynchronous host copies: ordering against the compute stream.

An upload queued after an op still lets that op read the old contents; every later
access reads the new ones.  A download sees the values before any later in-place write.
Graph replays wait for uploads of their inputs.
"""
import numpy as np
import pytest

import mag_b200 as MB
from gpu_util import device

pytestmark = pytest.mark.gpu


def _pinned(a):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).pin_memory()
    return t, t.data_ptr()


def test_upload_ordered_after_earlier_readers():
    dev = device()
    n = 1 << 22
    old = np.arange(n, dtype=np.float32)
    new = -np.arange(n, dtype=np.float32) - 1.0
    x = dev.tensor((n,))
    x.write(old)
    y = dev.op("NEG", x)  # queued before the upload: reads the old contents
    hold, p = _pinned(new)
    dev.upload_async(x, p, n * 4)
    z = dev.op("ABS", x)  # queued after: reads the new contents
    assert np.array_equal(y.read(), -old)
    assert np.array_equal(z.read(), np.abs(new))
    assert np.array_equal(x.read(), new)
    dev.copies_sync()


def test_download_sees_values_before_later_writes():
    import torch
    dev = device()
    n = 1 << 20
    v = np.linspace(-3, 3, n).astype(np.float32)
    x = dev.tensor((n,))
    x.write(v)
    r = dev.op("SQR", x)
    out = torch.empty(n, dtype=torch.float32).pin_memory()
    dev.download_async(r, out.data_ptr(), n * 4)
    dev.op("NEG", r, inplace=True)  # writes r after the download was queued
    dev.copies_sync()
    assert np.array_equal(out.numpy(), v * v)
    assert np.array_equal(r.read(), -(v * v))


def test_graph_replay_waits_for_input_upload():
    dev = device()
    rows, cols = 512, 256
    x = dev.tensor((rows, cols))
    dev.eager = False
    y = dev.op("ADDS", dev.op("SQR", x), xi=1.0)
    dev.eager = True
    rng = np.random.default_rng(3)
    try:
        for i in range(3):
            v = rng.standard_normal(rows * cols).astype(np.float32)
            hold, p = _pinned(v)
            dev.upload_async(x, p, v.nbytes)
            dev.graph_exec(y)
            assert np.array_equal(y.read(), v * v + np.float32(1.0)), i
    finally:
        dev.graph_release(y)


def test_partial_upload_zero_fills_and_rejections():
    dev = device()
    n = 4096
    x = dev.tensor((n,))
    v = np.full(100, 2.5, np.float32)
    hold, p = _pinned(v)
    dev.upload_async(x, p, v.nbytes)
    got = x.read()
    assert np.all(got[:100] == 2.5) and np.all(got[100:] == 0)
    pageable = np.ones(n, np.float32)
    assert dev.L.mag_cuda_tensor_upload_async(dev.p, x.ptr, pageable.ctypes.data, n * 4) == MB.E_INVALID
    big, pb = _pinned(np.ones(n + 1, np.float32))
    assert dev.L.mag_cuda_tensor_upload_async(dev.p, x.ptr, pb, (n + 1) * 4) == MB.E_INVALID
