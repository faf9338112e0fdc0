"""Shared test helpers: regenerate golden-case inputs and compare floats."""
import os

import numpy as np

import cases as CS
from oracle import Oracle, pad6

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
_oracle = None


def oracle() -> Oracle:
    global _oracle
    if _oracle is None:
        _oracle = Oracle()
    return _oracle


def golden():
    return np.load(GOLDEN)


def case_inputs(c):
    """Inputs of a golden case, drawn from the oracle's restatement of the PCG stream."""
    o = oracle()
    s = o.stream(c["seed"])
    x = s.draw(int(np.prod(c["x"])), c["dist"][0])
    y = s.draw(int(np.prod(c["y"])), c["dist"][1]) if "y" in c else None
    return x, y


def oracle_output(c, x, y):
    o = oracle()
    k = c["kind"]
    if k in ("unary", "scalar"):
        return o.unary(c["op"], x, pad6(c["x"]), c.get("xi", 0.0))
    if k == "binary":
        return o.binary(c["op"], x, pad6(c["x"]), y, pad6(c["y"]))
    if k == "reduce":
        r = np.zeros(int(np.prod(pad6(c["x"])[1:])), np.float32)
        r[0] = o.reduce(c["op"], x, pad6(c["x"]))
        return r
    if k == "matmul":
        m, kk = c["x"]
        n = c["y"][1]
        return o.matmul(x, y, m, kk, n)
    raise ValueError(k)


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))


def ulp_diff(a, b):
    """Distance in units in the last place between float32 arrays (NaN==NaN -> 0)."""
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, np.int64(-2**31) - a, a)
    b = np.where(b < 0, np.int64(-2**31) - b, b)
    return np.abs(a - b)


def tanh_cr(x):
    return np.tanh(np.asarray(x, np.float64)).astype(np.float32)
