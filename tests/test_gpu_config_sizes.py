"""Parity at the benchmark's own sizes: the configurations that the benchmark times.

Each workload runs at its full size on the device and is checked against the oracle (the
reference's arithmetic restated in C) in full where the oracle finishes in seconds, and on
seeded samples otherwise:
  - deep MLP forward, 8 x (4096 x 4096 + GELU) + 4096 x 1000 + row softmax, on 2048 rows
    through the fused graph executor; 16 rows against the oracle's chain of reference ops and
    against the same forward in double precision;
  - square products at 8192^3 and 16384^3 (sampled rows, norm-wise against double precision),
    the skinny shapes M in {1, 8, 64} x 4096 x 4096 and the batched 64 x [512^3] in full;
  - the two-sided broadcast [8,16,1,64,1,256] (op) [1,16,32,1,128,256] (2^33 outputs, 32 GiB)
    on 2^20 seeded indices, bit for bit;
  - binary and unary ops over 2^28 elements, in full;
  - row reductions and the row softmax at (65536, 1024), (4096, 32768), (1024, 262144), and
    the full SUM over 2^28.
Tolerances are the ones the other parity tests use: bit-exact for IEEE-exact ops, <= 1e-5 of
|X||Y| for products, <= 1e-6 relative for reductions and the softmax.
"""
import os
import sys

if __name__ == "__main__":  # run as a script by the short-segment test: the paths conftest.py adds
    _here = os.path.dirname(os.path.abspath(__file__))
    for _p in (os.path.dirname(_here), os.path.join(os.path.dirname(_here), "oracle"), _here,
               os.path.join(_here, "golden"), os.path.join(os.path.dirname(_here), "magnetron-pre-oss-release-old_b200")):
        sys.path.insert(0, _p)

import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle, bits_equal
from oracle import pad6
from gpu_util import device, assert_unary_parity

pytestmark = pytest.mark.gpu

CHUNK = 1 << 24  # host-side comparisons in slices of 16 Mi elements


class _CudaArray:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "stream": None}


def _view(dev, t, n=None):
    """A torch view of a device tensor's storage (no copy)."""
    import torch
    n = t.numel if n is None else n
    return torch.as_tensor(_CudaArray(t.data_ptr, n), device=f"cuda:{dev.ordinal}")


def _normal(dev, n, std, seed, shape=None):
    """A device tensor of n values ~ N(0, std) from the device PCG stream, and its host copy."""
    t = dev.tensor(shape or (n,))
    dev.fill_random_normal(t, 0.0, std, MB.Pcg(seed))
    dev.sync()
    return t, _view(dev, t).cpu().numpy()


def _normwise(got, x64, y64):
    """max over outputs of |got - exact| / (|X||Y|), all in double."""
    exact = x64 @ y64
    bound = np.abs(x64) @ np.abs(y64)
    return float((np.abs(got.astype(np.float64) - exact) / np.maximum(bound, 1e-30)).max())


# ---------------------------------------------------------------- config 5
def _deep_mlp_errors():
    """The benchmark's deep MLP at full width (X ~ N(0,1), Kaiming-normal weights, zero
    full-shape biases, MATMUL -> ADD -> GELU in place per layer, then MATMUL -> ADD and the row
    softmax) on 2048 rows through the fused graph executor; 16 sampled rows against the oracle's
    chain of the reference's ops (sequential f32 products, the reference's GELU formula) and
    against the same forward in double precision.  Returns the largest deviations: logits
    relative to their row's largest logit, probabilities relative to themselves."""
    dev, o = device(), oracle()
    rows, d, hidden, d_out = 2048, 4096, 8, 1000
    std = (2.0 / d) ** 0.5
    Xg, xh = _normal(dev, rows * d, 1.0, 0x5EED0005, (rows, d))
    Wgs, wh = [], []
    for i in range(hidden):
        W, w = _normal(dev, d * d, std, 0x5EED0105 + i, (d, d))
        Wgs.append(W)
        wh.append(w)
    Wog, woh = _normal(dev, d * d_out, std, 0x5EED0205, (d, d_out))
    Bs = [dev.tensor((rows, d)) for _ in range(hidden)]
    Bo = dev.tensor((rows, d_out))
    dev.eager = False
    try:
        h = Xg
        for W, B in zip(Wgs, Bs):
            h = dev.op("GELU", dev.op("ADD", dev.op("MATMUL", h, W), B), inplace=True)
        z = dev.op("ADD", dev.op("MATMUL", h, Wog), Bo)
    finally:
        dev.eager = True
    P = dev.tensor((rows * d_out,))
    try:
        dev.graph_exec(z, fused=True)
        MB.check(dev.L.mag_cuda_softmax_rows_f32(dev.p, P.data_ptr, z.data_ptr, rows, d_out), "softmax")
        assert dev.L.mag_cuda_synchronize(dev.p) == 0
        logits = _view(dev, z, rows * d_out).cpu().numpy().reshape(rows, d_out)
        probs = _view(dev, P).cpu().numpy().reshape(rows, d_out)
    finally:
        dev.graph_release(z)
    assert np.allclose(probs.sum(1), 1.0, atol=1e-5)
    sample = np.array([0, 1, 2, 3, 255, 256, 511, 777, 1024, 1027, 1500, 1789, 2000, 2044, 2046, 2047])
    ns = len(sample)
    a = xh.reshape(rows, d)[sample].reshape(-1)
    a64 = a.astype(np.float64).reshape(ns, d)
    c1, c2 = 0.7978845608028654, 0.044715
    for w in wh:
        a = o.unary("GELU", o.matmul(a, w, ns, d, d), pad6((d, ns)))
        v = a64 @ w.astype(np.float64).reshape(d, d)
        a64 = 0.5 * v * (1.0 + np.tanh(c1 * (v + c2 * v ** 3)))
    zr = o.matmul(a, woh, ns, d, d_out).reshape(ns, d_out)
    z64 = a64 @ woh.astype(np.float64).reshape(d, d_out)
    pr = o.softmax_rows(zr.reshape(-1), ns, d_out).reshape(ns, d_out)
    e = np.exp(z64 - z64.max(1, keepdims=True))
    p64 = e / e.sum(1, keepdims=True)
    got_z, got_p = logits[sample], probs[sample]
    rowmax = np.abs(z64).max(1, keepdims=True)
    return {"z_f64": float((np.abs(got_z - z64) / rowmax).max()), "p_f64": float((np.abs(got_p - p64) / p64).max()),
            "z_ref": float((np.abs(got_z - zr) / np.abs(zr).max(1, keepdims=True)).max()),
            "p_ref": float((np.abs(got_p - pr) / pr).max()),
            "ref_z_f64": float((np.abs(zr - z64) / rowmax).max()), "ref_p_f64": float((np.abs(pr - p64) / p64).max())}


def test_deep_mlp_forward_full_width_sampled_rows():
    """Default segments (512 elements of K per tensor-core accumulator).  Each of the nine
    products is within 1e-5 of |X||Y| (the product tests), but the tensor cores' accumulation
    truncates, which shrinks every product's magnitude by a few 1e-6, and the shrinkage compounds
    through the layers: measured 2.6e-5 of the row's largest logit against double precision and
    1.1e-4 relative on the probabilities.  The reference's own f32 chain lies 5.7e-6 and 1.5e-5
    from double precision.  Bounds: 5e-5 on logits and 2.5e-4 on probabilities, against both."""
    err = _deep_mlp_errors()
    assert err["ref_z_f64"] <= 1e-5, err
    assert err["z_f64"] <= 5e-5 and err["p_f64"] <= 2.5e-4, err
    assert err["z_ref"] <= 5e-5 and err["p_ref"] <= 2.5e-4, err


def test_deep_mlp_forward_short_segments_meet_1e5():
    """The same forward with short accumulator segments (256 elements of K for a tile's first
    segment, then 64; MAG_CUDA_TC_SEGMENT_FIRST / MAG_CUDA_TC_SEGMENT, read when the library first
    launches a product, so in a process of its own): the compounded shrinkage falls below the
    reference's own deviation scale, and the logits are within 1e-5 of the row maximum against
    double precision (2e-5 against the reference chain, whose own deviation is 5.7e-6)."""
    import json
    import subprocess
    env = dict(os.environ, MAG_CUDA_TC_SEGMENT_FIRST="256", MAG_CUDA_TC_SEGMENT="64")
    out = subprocess.run([sys.executable, os.path.abspath(__file__)], env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    err = json.loads(out.stdout.strip().splitlines()[-1])
    assert err["z_f64"] <= 1e-5 and err["p_f64"] <= 4e-5, err
    assert err["z_ref"] <= 2e-5 and err["p_ref"] <= 5e-5, err


# ---------------------------------------------------------------- config 4
@pytest.mark.parametrize("n", [8192, 16384])
def test_matmul_square_config_sizes_sampled_rows(n):
    """A, B ~ N(0, 1/sqrt(K)) from the device PCG stream, M = N = K = 8192 and 16384 on the
    default tensor-core path; eight sampled rows (first, last, and rows of the last wave's
    tiles) within 1e-5 of |A||B| of the double-precision product, and within 1e-5 of max|C| of
    the oracle's sequential f32 product."""
    dev, o = device(), oracle()
    std = n ** -0.5
    A, ah = _normal(dev, n * n, std, 0x5EED0404 + n)
    B, bh = _normal(dev, n * n, std, 0x5EED0504 + n)
    R = dev.tensor((n * n,))
    MB.check(dev.L.mag_cuda_matmul_f32(dev.p, R.data_ptr, A.data_ptr, B.data_ptr, n, n, n), "matmul")
    assert dev.L.mag_cuda_synchronize(dev.p) == 0
    rows = np.array([0, 1, n // 2 + 3, n - 258, n - 129, n - 100, n - 2, n - 1])
    import torch
    got = _view(dev, R).view(n, n)[torch.as_tensor(rows, device=f"cuda:{dev.ordinal}")].cpu().numpy()
    a64 = ah.reshape(n, n)[rows].astype(np.float64)
    b64 = bh.reshape(n, n).astype(np.float64)
    assert _normwise(got, a64, b64) <= 1e-5
    seq = np.stack([o.matmul_rows(ah, bh, int(r), 1, n, n) for r in rows[:3]])
    assert float(np.abs(got[:3] - seq).max()) <= 1e-5 * float(np.abs(seq).max())
    for t in (A, B, R):
        t.free()


@pytest.mark.parametrize("m", [1, 8, 64])
def test_matmul_skinny_config_shapes(m):
    """M x 4096 x 4096 for M = 1, 8 (HBM-bound skinny kernels) and 64 (tensor-core split-K),
    A, B ~ N(0, 1/64): every output within 1e-5 of |A||B|."""
    dev = device()
    n = 4096
    A, ah = _normal(dev, m * n, n ** -0.5, 0x5EED0604 + m)
    B, bh = _normal(dev, n * n, n ** -0.5, 0x5EED0704)
    R = dev.tensor((m * n,))
    MB.check(dev.L.mag_cuda_matmul_f32(dev.p, R.data_ptr, A.data_ptr, B.data_ptr, m, n, n), "matmul")
    assert dev.L.mag_cuda_synchronize(dev.p) == 0
    got = _view(dev, R).cpu().numpy().reshape(m, n)
    assert _normwise(got, ah.reshape(m, n).astype(np.float64), bh.reshape(n, n).astype(np.float64)) <= 1e-5


def test_matmul_batched_config_shape():
    """[64, 512, 512] . [64, 512, 512] on the batched tensor-core path: every batch within 1e-5
    of |A||B|."""
    dev = device()
    b, m = 64, 512
    A, ah = _normal(dev, b * m * m, m ** -0.5, 0x5EED0804)
    B, bh = _normal(dev, b * m * m, m ** -0.5, 0x5EED0904)
    R = dev.tensor((b * m * m,))
    MB.check(dev.L.mag_cuda_matmul_batched_f32(dev.p, R.data_ptr, A.data_ptr, B.data_ptr, b, m, m, m), "bmm")
    assert dev.L.mag_cuda_synchronize(dev.p) == 0
    got = _view(dev, R).cpu().numpy().reshape(b, m, m)
    a64 = ah.reshape(b, m, m).astype(np.float64)
    b64 = bh.reshape(b, m, m).astype(np.float64)
    for i in range(b):
        assert _normwise(got[i], a64[i], b64[i]) <= 1e-5, i


# ---------------------------------------------------------------- config 2
def test_broadcast2_two_sided_full_size_sampled():
    """[8,16,1,64,1,256] (op) [1,16,32,1,128,256] (row-major) -> 2^33 outputs (32 GiB), x and y
    ~ N(0,1), divisors |y| >= 0.5: 2^20 seeded output indices bit-identical with the oracle
    for ADD, SUB, MUL and DIV."""
    import torch
    dev, o = device(), oracle()
    xs, ys, rs = (256, 1, 64, 1, 16, 8), (256, 128, 1, 32, 16, 1), (256, 128, 64, 32, 16, 8)
    nx, ny, nr = int(np.prod(xs)), int(np.prod(ys)), int(np.prod(rs))
    X, xh = _normal(dev, nx, 1.0, 0x5EED0002)
    Y, yh = _normal(dev, ny, 1.0, 0x5EED0102)
    yd = (yh + np.copysign(np.float32(0.5), yh)).astype(np.float32)
    Yd = dev.tensor((ny,))
    Yd.write(yd)
    R = dev.tensor((nr,))
    idx = np.sort(np.random.default_rng(0x5EED0302).integers(0, nr, 1 << 20, dtype=np.int64))
    idx[:4] = [0, 1, nr - 2, nr - 1]
    tidx = torch.as_tensor(idx, device=f"cuda:{dev.ordinal}")
    for op in ["ADD", "SUB", "MUL", "DIV"]:
        yt, yv = (Yd, yd) if op == "DIV" else (Y, yh)
        MB.check(dev.L.mag_cuda_broadcast2_f32(dev.p, MB.OP[op], R.data_ptr, X.data_ptr, yt.data_ptr,
                                               MB.i64x6(rs), MB.i64x6(xs), MB.i64x6(ys)), op)
        assert dev.L.mag_cuda_synchronize(dev.p) == 0
        got = _view(dev, R)[tidx].cpu().numpy()
        want = o.bcast2(op, xh, xs, yv, ys, rs, sample_idx=idx)
        assert bits_equal(got, want).all(), op
    for t in (X, Y, Yd, R):
        t.free()


def test_binary_2p28_full():
    """ADD/SUB/MUL/DIV over 2^28 contiguous elements (x, y ~ N(0,1), divisors |y| >= 0.5):
    every output bit-identical with the oracle."""
    dev, o = device(), oracle()
    n = 1 << 28
    X, xh = _normal(dev, n, 1.0, 0x5EED0012)
    Y, yh = _normal(dev, n, 1.0, 0x5EED0112)
    yd = (yh + np.copysign(np.float32(0.5), yh)).astype(np.float32)
    Yd = dev.tensor((n,))
    Yd.write(yd)
    R = dev.tensor((n,))
    dims, st = MB.i64x6([n, 1, 1, 1, 1, 1]), MB.i64x6(MB.strides6([n, 1, 1, 1, 1, 1]))
    for op in ["ADD", "SUB", "MUL", "DIV"]:
        yt, yv = (Yd, yd) if op == "DIV" else (Y, yh)
        MB.check(dev.L.mag_cuda_binary_f32(dev.p, MB.OP[op], R.data_ptr, X.data_ptr, yt.data_ptr, dims, st, st, dims,
                                           st), op)
        assert dev.L.mag_cuda_synchronize(dev.p) == 0
        got = _view(dev, R).cpu().numpy()
        for i in range(0, n, CHUNK):
            sl = slice(i, i + CHUNK)
            want = o.binary(op, xh[sl], pad6((CHUNK,)), yv[sl], pad6((CHUNK,)))
            assert bits_equal(got[sl], want).all(), (op, i)
    for t in (X, Y, Yd, R):
        t.free()


@pytest.mark.parametrize("op", ["ABS", "NEG", "LOG", "SQR", "SQRT", "SOFTMAX", "SIGMOID", "TANH", "RELU", "GELU"])
def test_unary_2p28_full(op):
    """The unary sweep over 2^28 elements as 65536 rows of 4096 (x ~ N(0,1); LOG on |x|+1, SQRT
    on |x|), every output checked with the per-op tolerance of the unary parity tests
    (bit-exact lanes, tanh within 2 ulp of the correctly rounded value, GELU within
    1e-6 max(1,|x|) of the double-precision formula)."""
    dev, o = device(), oracle()
    n, cols = 1 << 28, 4096
    X, xh = _normal(dev, n, 1.0, 0x5EED0022)
    if op in ("LOG", "SQRT"):
        xh = np.abs(xh) + (np.float32(1.0) if op == "LOG" else np.float32(0.0))
        X.write(xh)
    R = dev.tensor((n,))
    MB.check(dev.L.mag_cuda_unary_f32(dev.p, MB.OP[op], R.data_ptr, X.data_ptr, n // cols, cols, cols, cols, 0.0), op)
    assert dev.L.mag_cuda_synchronize(dev.p) == 0
    got = _view(dev, R).cpu().numpy()
    for i in range(0, n, CHUNK):
        sl = slice(i, i + CHUNK)
        shape6 = pad6((cols, CHUNK // cols))
        assert_unary_parity(op, xh[sl], got[sl], o.unary(op, xh[sl], shape6), shape6)
    for t in (X, R):
        t.free()


# ---------------------------------------------------------------- config 3
@pytest.mark.parametrize("rows,cols", [(65536, 1024), (4096, 32768), (1024, 262144)])
def test_row_reductions_and_softmax_config_shapes(rows, cols):
    """SUM/MEAN/MIN/MAX and the normalised softmax along the last dim of (65536, 1024),
    (4096, 32768) and (1024, 262144) (x ~ N(0,1), 2^28 elements): every row within 1e-6
    relative of the oracle (double row sums, the reference's exp); the softmax within 2e-6
    (CUDA's expf in place of the reference's exp lanes, and for rows split over a cluster one
    more expf and rounding in the slice's rescaling: measured up to 1.15e-6)."""
    dev, o = device(), oracle()
    n = rows * cols
    X, xh = _normal(dev, n, 1.0, 0x5EED0003 + cols)
    R = dev.tensor((n,))
    for op in ["SUM", "MEAN", "MIN", "MAX"]:
        MB.check(dev.L.mag_cuda_reduce_rows_f32(dev.p, MB.OP[op], R.data_ptr, X.data_ptr, rows, cols), op)
        assert dev.L.mag_cuda_synchronize(dev.p) == 0
        got = _view(dev, R, rows).cpu().numpy()
        want = o.reduce_rows(op, xh, rows, cols)
        rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
        assert float(rel.max()) <= 1e-6, (op, float(rel.max()))
    MB.check(dev.L.mag_cuda_softmax_rows_f32(dev.p, R.data_ptr, X.data_ptr, rows, cols), "softmax")
    assert dev.L.mag_cuda_synchronize(dev.p) == 0
    got = _view(dev, R).cpu().numpy()
    rstep = max(1, CHUNK // cols)
    for r0 in range(0, rows, rstep):
        sl = slice(r0 * cols, (r0 + rstep) * cols)
        want = o.softmax_rows(xh[sl], min(rstep, rows - r0), cols)
        rel = np.abs(got[sl] - want) / np.maximum(np.abs(want), 1e-30)
        assert float(rel.max()) <= 2e-6, (r0, float(rel.max()))
    for t in (X, R):
        t.free()


def test_full_sum_2p28():
    """SUM, MEAN, MIN and MAX over all 2^28 elements (x ~ N(0,1)): within 1e-6 relative of the
    oracle (double accumulation, a different order)."""
    dev, o = device(), oracle()
    n = 1 << 28
    X, xh = _normal(dev, n, 1.0, 0x5EED0013)
    R = dev.tensor((1,))
    dims, st = MB.i64x6([n, 1, 1, 1, 1, 1]), MB.i64x6(MB.strides6([n, 1, 1, 1, 1, 1]))
    for op in ["SUM", "MEAN", "MIN", "MAX"]:
        MB.check(dev.L.mag_cuda_reduce_f32(dev.p, MB.OP[op], R.data_ptr, X.data_ptr, dims, st), op)
        assert dev.L.mag_cuda_synchronize(dev.p) == 0
        got = float(R.read()[0])
        want = o.reduce(op, xh, pad6((n,)))
        assert abs(got - want) <= 1e-6 * max(abs(want), 1e-30), (op, got, want)
    for t in (X, R):
        t.free()


if __name__ == "__main__":  # the short-segment forward's errors, in a process of its own
    import json
    print(json.dumps(_deep_mlp_errors()))
