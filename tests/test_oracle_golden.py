"""The oracle (CPU restatement) against golden vectors made by the reference library.

Bit-exact for every op except TANH/GELU, whose reference lanes use x86 rcpps
(magnetron/magnetron_cpu.c:192-204): those are checked within the reference's
own test tolerance of 1e-3 (test/compute_cpu.cpp:151,165), scaled by |x| for
GELU, on finite values (the reference tanh is NaN below x = -44.4).
"""
import numpy as np
import pytest

import cases as CS
from harness import case_inputs, golden, oracle_output, bits_equal, oracle

G = golden()
CASES = CS.cases()


@pytest.mark.parametrize("c", CASES, ids=[CS.case_id(c) for c in CASES])
def test_oracle_matches_reference(c):
    cid = CS.case_id(c)
    x, y = case_inputs(c)
    # the PCG + Box-Muller restatement reproduces the reference's own fills
    assert bits_equal(x[:16], G[cid + "/x16"]).all()
    if y is not None:
        assert bits_equal(y[:16], G[cid + "/y16"]).all()
    got = oracle_output(c, x, y)
    ref = G[cid + "/out"]
    assert got.shape == ref.shape
    if c["op"] in CS.RCP_OPS:
        # tanh error is absolute; gelu scales it by 0.5*|x|
        fin = np.isfinite(ref)
        scale = np.maximum(1.0, np.abs(x)) if c["op"] == "GELU" else 1.0
        assert np.all((np.abs(got - ref) <= 1e-3 * scale)[fin])
    else:
        assert bits_equal(got, ref).all(), cid


def test_known_answer_matmul():
    """Known answers of the reference's tests (test/compute_cpu.cpp:380-452)."""
    o = oracle()
    A = np.array([1.6354027, -1.3607267, 1.8556793, 1.1689897], np.float32)
    B = np.array([-0.6105532, 0.10695228, -1.0069681, -0.40955952], np.float32)
    exp = np.array([0.3717081, 0.7322086, -2.3101263, -0.28030172], np.float32)
    np.testing.assert_allclose(o.matmul(A, B, 2, 2, 2), exp, rtol=4 * 2**-23)
    A = np.array([1, 2, 3, 4, 5, 6], np.float32)
    B = np.array([0.5, -1.0], np.float32)
    np.testing.assert_array_equal(o.matmul(A, B, 3, 2, 1), np.array([-1.5, -2.5, -3.5], np.float32))


def test_normal_generator_moments():
    """PRNG moment check in the style of test/tensor.cpp:455-563."""
    x = oracle().normal(1 << 20, 0.0, 1.0, 0x5EED0003)
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01
