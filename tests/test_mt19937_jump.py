"""The jump arithmetic behind the device Mersenne-twister fills, checked on the host.

The reference's generator (magnetron/magnetron.c:751-777) as a word stream is an affine
recurrence over GF(2); the library finds its minimal polynomial (Berlekamp-Massey) and jumps
a 624-word window d words ahead as x^d mod that polynomial.  Here the library's host jump is
compared with the oracle's stream for many distances, including the substream lengths and the
doubling distances the device uses.
"""
import ctypes as C

import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle

U32P = C.POINTER(C.c_uint32)


def _jump(L, win, d):
    out = np.zeros(624, np.uint32)
    rc = L.mag_cuda_mt19937_jump(win.ctypes.data_as(U32P), d, out.ctypes.data_as(U32P))
    assert rc == 0
    return out


def test_minimal_polynomial_degree():
    """19937 for the linear part, plus the factor x + 1 of the affine constant (the all-ones
    window is the affine map's fixed point)."""
    assert MB.load_library().mag_cuda_mt19937_degree() == 19938


@pytest.mark.parametrize("seed", [5489, 0x5EED0001])
@pytest.mark.parametrize("d", [0, 1, 226, 227, 623, 624, 19937, 19938, 30011, 624 * 96 - 624, 624 * 96,
                               624 * 384 + 1, 250001])
def test_jump_matches_the_stream(seed, d):
    """A window one block into the stream (the first twisted block of a fresh seed), jumped by d,
    equals the stream's window d words later."""
    L = MB.load_library()
    w = oracle().mt_stream(seed).words(d + 624)
    assert np.array_equal(_jump(L, w[:624], d), w[d:d + 624])


def test_jump_composes_over_doubling_distances():
    """Window at 3 * 59904 reached by the device's path (59904 - 624 from the first twisted
    block, then 59904, then 2 * 59904) equals one jump and the stream itself."""
    L = MB.load_library()
    sub = 624 * 96
    mt = oracle().mt_stream(77)
    w = mt.words(3 * sub + 624)  # w[0:624] = the first twisted block = stream words 624..1247
    win0 = w[:624]
    w1 = _jump(L, win0, sub - 624)
    w2 = _jump(L, w1, sub)
    w3 = _jump(L, w1, 2 * sub)
    assert np.array_equal(w1, w[sub - 624:sub])
    assert np.array_equal(w2, w[2 * sub - 624:2 * sub])
    assert np.array_equal(w3, w[3 * sub - 624:3 * sub])
