"""Device fills against the oracle's restatement of the reference's host fills.

Uniform fills are bit-exact with the host PCG stream (magnetron/magnetron.c:779-790),
including where one fill leaves the stream and the next continues it.  Normal
fills (Box-Muller, magnetron/magnetron.c:1856-1876) differ from the host only by the
rounding of log/sin/cos: each value within 2^-21 of the pair's magnitude plus |mean|
(a few ulp), and the share of values not bit-identical is bounded.
"""
import ctypes as C

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
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                             "stream": None}

    dev.sync()
    return torch.as_tensor(_A(), device=f"cuda:{dev.L.mag_cuda_device_ordinal(dev.p)}").cpu().numpy()


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("n", [1, 3, 4, 5, 1000, 4099, (1 << 20) + 3, (1 << 26) + 5])
@pytest.mark.parametrize("lo,hi", [(0.0, 1.0), (-1.0, 1.0), (-0.0759, 0.0759)])
def test_uniform_bit_exact(n, lo, hi):
    dev, o = device(), oracle()
    seed = 0x5EED0000 + n
    g, ref = MB.Pcg(seed), o.stream(seed)
    assert (g.state.value, g.inc) == (ref.g.state, ref.g.inc)
    t = dev.tensor((n,))
    dev.fill_random_uniform(t, lo, hi, g)
    want = ref.uniform(n, lo, hi)
    assert np.array_equal(_bits(t.read()), _bits(want))
    assert g.state.value == ref.g.state  # the stream advanced by n, as on the host
    t.free()


def test_uniform_continues_stream_and_unaligned():
    """Three fills in a row, the middle one into a view starting 1 element into its
    buffer (no 16-byte alignment), equal one host fill of the total length."""
    dev, o = device(), oracle()
    g, ref = MB.Pcg(0x5EED0002), o.stream(0x5EED0002)
    want = ref.uniform(10 + 4097 + 33, -2.0, 3.0)
    base = dev.tensor((1 + 4097,))
    a, c = dev.tensor((10,)), dev.tensor((33,))
    dev.fill_random_uniform(a, -2.0, 3.0, g)
    ptr = base.data_ptr + 4
    MB.check(dev.L.mag_cuda_fill_uniform_pcg_f32(dev.p, ptr, 4097, -2.0, 3.0, C.byref(g.state), g.inc), "fill")
    dev.fill_random_uniform(c, -2.0, 3.0, g)
    got = np.concatenate([a.read(), _raw(dev, ptr, 4097), c.read()])
    assert np.array_equal(_bits(got), _bits(want))
    assert g.state.value == ref.g.state


def _normal_check(got, want, mean):
    mag = np.hypot((want[0::2] - mean).astype(np.float64), (want[1::2] - mean).astype(np.float64))
    bound = np.repeat(mag + abs(mean), 2) * 2.0 ** -21 + 1e-30
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= bound), f"max err/bound {np.max(err / bound):.3f}"
    return float(np.mean(_bits(got) != _bits(want)))


@pytest.mark.parametrize("n", [2, 6, 1000, 4098, (1 << 22) + 2])
@pytest.mark.parametrize("mean,std", [(0.0, 1.0), (0.0, 0.0221), (3.0, 0.5)])
def test_normal_within_rounding(n, mean, std):
    dev, o = device(), oracle()
    seed = 0x5EED1000 + n
    g, ref = MB.Pcg(seed), o.stream(seed)
    t = dev.tensor((n,))
    dev.fill_random_normal(t, mean, std, g)
    want = ref.normal(n, mean, std)
    diff = _normal_check(t.read(), want, mean)
    assert diff < 0.03, f"{diff:.4f} of values not bit-identical"  # 1.5% measured at 2^24
    assert g.state.value == ref.g.state
    t.free()


def test_normal_rejects_odd_count():
    dev = device()
    g = MB.Pcg(1)
    s0 = g.state.value
    t = dev.tensor((5,))
    rc = dev.L.mag_cuda_fill_normal_pcg_f32(dev.p, t.data_ptr, 5, 0.0, 1.0, C.byref(g.state), g.inc)
    assert rc == MB.E_INVALID and g.state.value == s0


@pytest.mark.parametrize("n", [1, 7, 4096, (1 << 20) + 1])
def test_fill_const(n):
    dev = device()
    t = dev.tensor((n + 1,))
    for x in (2.5, -0.0, float("inf")):
        dev.fill(t, 7.0)
        MB.check(dev.L.mag_cuda_fill_f32(dev.p, t.data_ptr + 4, n, x), "fill")
        got = t.read()
        assert got[0] == 7.0
        assert np.array_equal(_bits(got[1:]), _bits(np.full(n, x, np.float32)))


def test_fill_then_op_sees_values():
    """A filled buffer is marked written: the lazy zero of a fresh tensor must not
    overwrite it before an op reads it."""
    dev, o = device(), oracle()
    g, ref = MB.Pcg(9), o.stream(9)
    x = dev.tensor((256, 64))
    dev.fill_random_uniform(x, -1.0, 1.0, g)
    r = dev.op("ABS", x)
    assert np.array_equal(r.read(), np.abs(ref.uniform(256 * 64, -1.0, 1.0)))
