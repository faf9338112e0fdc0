"""The allocation-free skinny matmul entry point.

mag_cuda_matmul_skinny_f32_noalloc exists for callers that cannot allocate
device memory when they need the product (for example, a latency-critical
host path that must not enter the CUDA allocator, which can block or
synchronise, or code that runs under a memory budget fixed up front): its
split-K partial sums live in a fixed
array inside the library's device image instead of a buffer from cudaMalloc.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle
from gpu_util import device

pytestmark = pytest.mark.gpu


def _raw(dev, ptr, n):
    import torch

    class _A:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                             "version": 3, "stream": None}

    return torch.as_tensor(_A(), device=f"cuda:{dev.L.mag_cuda_device_ordinal(dev.p)}").cpu().numpy()


def _scratch_bytes(m, k, n, sms):
    """Partial-sum bytes of an m x k x n skinny product: K cut into slices so that about four
    CTAs per SM (256 threads, 4 columns each, 16 rows per CTA) stream Y, 16 <= slice <= 64 k
    (the sizing rule of skinny_slices, csrc/k_matmul_exact.cu), times m x n floats."""
    colblocks, rowblocks = -(-n // 1024), -(-m // 16)
    want = max(1, -(-4 * sms // (colblocks * rowblocks)))
    kc = min(64, max(16, -(-(-(-k // want)) // 16) * 16))
    return -(-k // kc) * m * n * 4


def _normwise_ok(got, x, y, m, k, n, tol=1e-5):
    x64 = x.reshape(m, k).astype(np.float64)
    y64 = y.reshape(k, n).astype(np.float64)
    err = np.abs(got.reshape(m, n).astype(np.float64) - x64 @ y64)
    return float((err / np.maximum(np.abs(x64) @ np.abs(y64), 1e-30)).max()) <= tol


@pytest.mark.parametrize("m", [1, 8])
def test_noalloc_matches_allocating_entry_point_twice(m):
    """M = 1 and M = 8 at K = N = 4096.  On a 148-SM B200 the M = 8 product needs exactly the
    whole array (128 slices x 8 x 4096 x 4 B = 16 MiB): it covers the boundary, where a call is
    still accepted."""
    dev = device()
    L = dev.L
    k = n = 4096
    assert L.mag_cuda_matmul_skinny_noalloc_limit() == 16 << 20
    import torch
    sms = torch.cuda.get_device_properties(dev.ordinal).multi_processor_count
    assert _scratch_bytes(m, k, n, sms) <= 16 << 20
    s = oracle().stream(0x5EED0A00 + m)
    x = s.normal(m * k, 0.0, k ** -0.5) if (m * k) % 2 == 0 else s.uniform(m * k, -1, 1)
    y = s.normal(k * n, 0.0, k ** -0.5)
    tx, ty = dev.tensor((m * k,)), dev.tensor((k * n,))
    tx.write(x)
    ty.write(y)
    ref_t, out_t = dev.tensor((m * n,)), dev.tensor((m * n,))
    MB.check(L.mag_cuda_matmul_f32(dev.p, ref_t.data_ptr, tx.data_ptr, ty.data_ptr, m, k, n), "allocating")
    dev.sync()
    ref = _raw(dev, ref_t.data_ptr, m * n)
    assert _normwise_ok(ref, x, y, m, k, n)
    for _ in range(2):  # the shared array keeps the previous call's partials; results must not depend on them
        MB.check(L.mag_cuda_matmul_skinny_f32_noalloc(dev.p, out_t.data_ptr, tx.data_ptr, ty.data_ptr, m, k, n),
                 "noalloc")
        assert L.mag_cuda_synchronize(dev.p) == 0
        got = _raw(dev, out_t.data_ptr, m * n)
        assert _normwise_ok(got, x, y, m, k, n)
        assert np.max(np.abs(got - ref)) <= 1e-5 * np.max(np.abs(ref))
    for t in (tx, ty, ref_t, out_t):
        t.free()


def test_noalloc_rejects_products_above_the_array():
    """Products whose partial sums exceed the array are refused before anything runs: 16 x 4096 x
    8192 (64 slices x 16 x 8192 x 4 B = 32 MiB) and, one row past the boundary above,
    9 x 4096 x 4096 (18 MiB on a 148-SM B200)."""
    dev = device()
    L = dev.L
    import torch
    sms = torch.cuda.get_device_properties(dev.ordinal).multi_processor_count
    m, k, n = 16, 4096, 8192
    assert _scratch_bytes(m, k, n, sms) > 16 << 20
    tx, ty, tr = dev.tensor((m * k,)), dev.tensor((k * n,)), dev.tensor((m * n,))
    rc = L.mag_cuda_matmul_skinny_f32_noalloc(dev.p, tr.data_ptr, tx.data_ptr, ty.data_ptr, m, k, n)
    assert rc == MB.E_SCRATCH_LIMIT
    if _scratch_bytes(9, 4096, 4096, sms) > 16 << 20:
        rc = L.mag_cuda_matmul_skinny_f32_noalloc(dev.p, tr.data_ptr, tx.data_ptr, ty.data_ptr, 9, 4096, 4096)
        assert rc == MB.E_SCRATCH_LIMIT
    assert L.mag_cuda_matmul_skinny_f32_noalloc(dev.p, tr.data_ptr, tx.data_ptr, ty.data_ptr, 17, k, n) == MB.E_INVALID
    assert L.mag_cuda_synchronize(dev.p) == 0
