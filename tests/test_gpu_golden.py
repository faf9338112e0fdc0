"""The CUDA backend against the golden vectors made by the reference library,
driven through the device vtable exactly as the magnetron core drives it."""
import numpy as np
import pytest

import cases as CS
from harness import case_inputs, golden, bits_equal
from oracle import pad6
from gpu_util import device, run_op, assert_unary_parity

G = golden()
CASES = CS.cases()


@pytest.mark.gpu
@pytest.mark.parametrize("c", CASES, ids=[CS.case_id(c) for c in CASES])
def test_cuda_matches_reference_golden(c):
    dev = device()
    x, y = case_inputs(c)
    ref = G[CS.case_id(c) + "/out"]
    if c["kind"] == "matmul":
        shapes = [tuple(c["x"]), tuple(c["y"])]
    else:
        shapes = [tuple(c["x"])] + ([tuple(c["y"])] if "y" in c else [])
    arrays = [x] + ([y] if y is not None else [])
    got, r, ts = run_op(dev, c["op"], arrays, shapes, xi=c.get("xi"))
    if c["kind"] in ("unary",):
        assert_unary_parity(c["op"], x, got, ref, pad6(c["x"]))
    else:
        assert bits_equal(got, ref).all(), CS.case_id(c)
    for t in ts + [r]:
        t.free()
