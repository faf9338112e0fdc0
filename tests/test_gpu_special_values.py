"""Unary ops on special values: +-0, +-inf, NaN, subnormals, the largest finite values, and
arguments past exp's overflow, on vector lanes and scalar tails.

The oracle agrees with the reference library bit for bit on these inputs
(`test_oracle_matches_reference_on_special_values`, CPU).  The device must then match the
oracle as in the random sweeps: lanes bit-exact, tails within 2 ulp, TANH within 2 ulp of the
correctly rounded tanh, GELU within 1e-6 max(1, |x|) of its double-precision formula (or equal
to the oracle's f32 evaluation where that overflows, as the reference's does).  A NaN
result only has to be a NaN: the GPU returns the canonical NaN where x86 keeps the input's
payload, and the reference gives NaN payloads no meaning.
"""
import os

import numpy as np
import pytest

from harness import oracle, pad6, ulp_diff, tanh_cr
from gpu_util import device, run_op, lane_mask

SPECIALS = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 1.17e-38, 3.4e38, -3.4e38, 88.7, -88.7,
                     100.0, -100.0, 1e20, -1e20, 0.5, -0.5, 1.0, -1.0, 1e-30, -1e-30], np.float32)
OPS = ["ABS", "NEG", "LOG", "SQR", "SQRT", "SIN", "COS", "STEP", "SOFTMAX", "SOFTMAX_DV", "SIGMOID",
       "SIGMOID_DV", "HARD_SIGMOID", "SILU", "TANH", "TANH_DV", "RELU", "RELU_DV", "GELU"]
# 22 columns: lanes 0..19 and tails 20, 21 of every row; 4 columns: lanes only
SHAPES = [(22, 4), (4, 22)]


def same(a, b):
    """Equal bits, or both NaN."""
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))


def test_oracle_matches_reference_on_special_values():
    """CPU: the oracle's restatement against the reference library itself."""
    from oracle import RefLib, REF_SO
    if not os.path.exists(REF_SO):
        pytest.skip("reference library not built (make -C oracle ref)")
    o, R = oracle(), RefLib()
    try:
        for shape in SHAPES:
            x = np.resize(SPECIALS, int(np.prod(shape))).astype(np.float32)
            for op in OPS:
                if op in ("TANH", "GELU"):  # the reference's rcpps-based tanh is not restated
                    continue
                t = R.tensor_nd(shape)
                R.write(t, x)
                got = R.read(R.op(op, t))
                want = o.unary(op, x, pad6(shape))
                assert same(got, want).all(), (op, shape, x[~same(got, want)][:4])
    finally:
        R.close()


@pytest.mark.gpu
@pytest.mark.parametrize("op", OPS)
def test_device_on_special_values(op):
    dev, o = device(), oracle()
    for shape in SHAPES:
        s6 = pad6(shape)
        x = np.resize(SPECIALS, int(np.prod(shape))).astype(np.float32)
        got, _, _ = run_op(dev, op, [x], [shape])
        if op == "TANH":
            cr = tanh_cr(x)
            fin = np.isfinite(x)
            assert ulp_diff(got[fin], cr[fin]).max() <= 2, op
            assert same(got[~fin], np.tanh(x[~fin])).all(), op
            continue
        if op == "GELU":
            x64 = x.astype(np.float64)
            with np.errstate(all="ignore"):
                a = 1.0 + 0.044715 * (x64 * x64)
                cr = 0.5 * (x64 * (1.0 + np.tanh(0.7978845608028654 * (x64 * a))))
            # the reference evaluates 0.5f * (x * b) in f32, so x * b overflows to inf for |x| above
            # about 1.7e38 where the double formula stays finite: there (and for non-finite
            # results) the oracle's f32 evaluation is the comparison
            want = o.unary(op, x, s6)
            f32 = ~np.isfinite(cr) | ~np.isfinite(want) | (np.abs(x64) > 1e38)
            assert np.all(np.abs(got[~f32] - cr[~f32]) <= 1e-6 * np.maximum(1.0, np.abs(x64[~f32]))), op
            assert same(got[f32], want[f32]).all(), (op, x[f32], got[f32], want[f32])
            continue
        want = o.unary(op, x, s6)
        if op == "TANH_DV":  # the reference squares and inverts glibc's coshf (8 ulp, as in the sweep)
            d = ulp_diff(got, want)
            assert np.all((d <= 8) | same(got, want)), op
            continue
        lanes = lane_mask(s6)
        assert same(got, want)[lanes].all(), (op, shape, x[lanes & ~same(got, want)][:4])
        tails = ~lanes
        if tails.any():
            g, w = got[tails], want[tails]
            ok = same(g, w) | (np.isfinite(g) & np.isfinite(w) & (ulp_diff(g, w) <= 2))
            assert ok.all(), (op, shape, x[tails][~ok])


def _pairs():
    """Every ordered pair of special values, as two (n,) vectors."""
    a, b = np.meshgrid(SPECIALS, SPECIALS, indexing="ij")
    return a.reshape(-1).astype(np.float32), b.reshape(-1).astype(np.float32)


BINARY = ["ADD", "SUB", "MUL", "DIV"]


def test_oracle_binary_matches_reference_on_special_values():
    from oracle import RefLib, REF_SO
    if not os.path.exists(REF_SO):
        pytest.skip("reference library not built (make -C oracle ref)")
    o, R = oracle(), RefLib()
    x, y = _pairs()
    try:
        for op in BINARY:
            tx, ty = R.tensor_nd((x.size,)), R.tensor_nd((y.size,))
            R.write(tx, x)
            R.write(ty, y)
            got = R.read(R.op(op, tx, ty))
            want = o.binary(op, x, pad6((x.size,)), y, pad6((y.size,)))
            assert same(got, want).all(), (op, x[~same(got, want)][:4], y[~same(got, want)][:4])
    finally:
        R.close()


@pytest.mark.gpu
@pytest.mark.parametrize("op", BINARY)
def test_device_binary_on_special_values(op):
    dev, o = device(), oracle()
    x, y = _pairs()
    got, _, _ = run_op(dev, op, [x, y], [(x.size,), (y.size,)])
    want = o.binary(op, x, pad6((x.size,)), y, pad6((y.size,)))
    assert same(got, want).all(), (op, x[~same(got, want)][:4], y[~same(got, want)][:4])


@pytest.mark.gpu
@pytest.mark.parametrize("op", ["SUM", "MEAN", "MIN", "MAX"])
def test_device_reductions_on_special_values(op):
    """Full reductions over vectors holding infinities, NaN, signed zeros and subnormals: the
    reference's double sums and fminf/fmaxf (which skip NaN, from +-inf) give the same value.
    Values compare with ==: over zeros of both signs the reference's MIN/MAX keep whichever
    zero glibc's argument order leaves, which a reduction tree cannot reproduce; the mixed
    finite case is exact in double in any summation order."""
    dev, o = device(), oracle()
    cases = [SPECIALS, np.array([0.5, -0.25, 1.0, 88.5, -100.0, 0.0, -0.0, 3.0], np.float32),
             np.array([np.inf, 1.0, -2.0], np.float32), np.array([np.nan, np.nan], np.float32),
             np.array([np.nan, 1.0, np.nan], np.float32), np.array([-0.0, 0.0, -0.0], np.float32),
             np.array([1e-40, -3e-40, 2e-45] * 300, np.float32)]
    for v in cases:
        got, _, _ = run_op(dev, op, [v], [(v.size,)])
        want = np.float32(o.reduce(op, v, pad6((v.size,))))
        assert got[0] == want or (np.isnan(got[0]) and np.isnan(want)), (op, v[:6], got[0], want)


@pytest.mark.gpu
def test_exact_matmul_on_special_values():
    """The bit-exact MATMUL path (the reference's i-k-j loop, separately rounded multiply and add)
    propagates infinities and NaN exactly as the oracle's restatement of it."""
    import mag_b200 as MB
    dev, o = device(), oracle()
    m, k, n = 8, 11, 8
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, m * k).astype(np.float32)
    y = rng.uniform(-1, 1, k * n).astype(np.float32)
    x[[3, 17, 40, 41]] = [np.inf, -np.inf, np.nan, -0.0]
    y[[5, 22, 60]] = [0.0, np.inf, 1e-40]
    MB.check(dev.L.mag_cuda_set_matmul_mode(dev.p, 1), "exact")
    try:
        got, _, _ = run_op(dev, "MATMUL", [x, y], [(m, k), (k, n)])
    finally:
        dev.L.mag_cuda_set_matmul_mode(dev.p, 0)
    want = o.matmul(x, y, m, k, n)
    assert same(got, want).all(), np.where(~same(got, want))


@pytest.mark.gpu
def test_softmax_rows_with_masked_entries():
    """Rows with -inf entries (masked positions) give exact zeros there and a normal softmax over
    the rest; a row that is all -inf gives NaN, as exp(x - max) / sum does in the oracle.  The
    200003-wide rows take the L2-resident cluster (7 parts of 28572 columns), and row 3 there also
    has its second part fully masked (that CTA's statistics are skipped in the cluster combine)."""
    dev, o = device(), oracle()
    for cols in (10, 1024, 8193, 200003):
        rows = 4
        x = np.random.default_rng(cols).uniform(-5, 5, rows * cols).astype(np.float32)
        x[0:cols:3] = -np.inf               # row 0: every third entry masked
        x[cols:2 * cols] = -np.inf          # row 1: fully masked
        x[2 * cols + 1] = np.inf            # row 2: one +inf (max - max is NaN there)
        if cols > 65536:
            x[3 * cols + 28572:3 * cols + 57144] = -np.inf  # row 3: its second part masked
        tx, tr = dev.tensor((rows * cols,)), dev.tensor((rows * cols,))
        tx.write(x)
        import mag_b200 as MB
        MB.check(dev.L.mag_cuda_softmax_rows_f32(dev.p, tr.data_ptr, tx.data_ptr, rows, cols), "softmax")
        got = tr.read()
        want = o.softmax_rows(x, rows, cols)
        assert np.array_equal(np.isnan(got), np.isnan(want)), cols
        fin = ~np.isnan(want)
        assert np.all(got[fin][want[fin] == 0] == 0), cols
        nz = fin & (want != 0)
        assert np.all(np.abs(got[nz] - want[nz]) <= 1e-6 * np.abs(want[nz])), cols
