"""Helpers for the GPU parity tests (device fixture, comparisons)."""
import numpy as np

import mag_b200 as MB
from harness import ulp_diff, bits_equal, tanh_cr

_dev = None


def device() -> MB.Device:
    global _dev
    if _dev is None:
        _dev = MB.Device()
    return _dev


def run_op(dev, name, arrays, shapes, xi=None, inplace=False):
    ts = [dev.tensor(s) for s in shapes]
    for t, a in zip(ts, arrays):
        t.write(a)
    r = dev.op(name, *ts, xi=xi, inplace=inplace)
    out = r.read()
    return out, r, ts


def lane_mask(shape6):
    """True where the reference takes its vector-lane path (column < cols & ~3)."""
    cols = int(shape6[0])
    n = int(np.prod(shape6))
    c = np.arange(n) % cols
    return c < (cols & ~3)


def assert_unary_parity(op, x, got, ref, shape6):
    """Bit-exact on vector lanes; tails within 2 ulp of glibc; tanh/gelu by tolerance;
    tanh' within 8 ulp (it squares and inverts libm coshf, magnetron/magnetron_cpu.c:901-909)."""
    if op == "TANH":
        cr = tanh_cr(x)
        assert ulp_diff(got, cr).max() <= 2, op
        return
    if op == "GELU":
        x64 = x.astype(np.float64)
        a = 1.0 + 0.044715 * (x64 * x64)
        cr = 0.5 * (x64 * (1.0 + np.tanh(0.7978845608028654 * (x64 * a))))
        assert np.all(np.abs(got - cr) <= 1e-6 * np.maximum(1.0, np.abs(x64))), op
        return
    if op == "TANH_DV":
        # the reference squares and inverts glibc's coshf; the GPU rounds a double cosh once
        d = ulp_diff(got, ref)
        assert np.all((d <= 8) | (np.isnan(got) & np.isnan(ref))), (op, int(d.max()))
        return
    lanes = lane_mask(shape6)
    eq = bits_equal(got, ref)
    assert eq[lanes].all(), (op, np.where(~eq & lanes)[0][:5])
    tails = ~lanes
    if tails.any():
        d = ulp_diff(got[tails], ref[tails])
        nan = np.isnan(got[tails]) & np.isnan(ref[tails])
        assert np.all((d <= 2) | nan), (op, int(d.max()))
