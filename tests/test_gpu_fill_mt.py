"""Device fills from the reference's default Mersenne-twister stream against the oracle.

A reference context draws uniform values from its MT19937 state (magnetron/magnetron.c:751-777)
unless it was switched to PCG.  The device fill reproduces that stream by jump-ahead: uniform
values are bit-exact with the host fill, the state struct is left exactly as the host generator
leaves it (block, next, remaining), and fills continue one another.  Normal values are
Box-Muller pairs (magnetron/magnetron.c:1856-1876) within the rounding of log/sin/cos.
"""
import ctypes as C
import os

import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle
from gpu_util import device
from test_gpu_fill import _bits, _normal_check, _raw

pytestmark = pytest.mark.gpu


def _same_state(g: MB.Mt19937, ref) -> bool:
    a, b = g.st, ref.g
    return (a.remaining, a.next) == (b.remaining, b.next) and list(a.state) == list(b.state)


@pytest.mark.parametrize("n", [1, 3, 623, 624, 625, 1000, 4099, 2 * 59904 + 17, 3 * 59904 + 5, (1 << 22) + 3, (1 << 26) + 5,
                               (1 << 27) + 7])
@pytest.mark.parametrize("lo,hi", [(0.0, 1.0), (-0.0759, 0.0759)])
def test_uniform_bit_exact(n, lo, hi):
    """Sizes inside the first block, at block edges, across a few substreams (3 * 59904 + 5 ends
    five words into its last substream), and at each of the three substream lengths (2^22 + 3
    just past the first size threshold, 18 substreams; 2^26 + 5 and 2^27 + 7 in the longest, 71
    and 141 substreams, the latter from eight doubling launches)."""
    if n > (1 << 26) and lo != 0.0:
        pytest.skip("one range is enough at 2^27")
    dev, o = device(), oracle()
    seed = 0x5EED1000 + n
    g, ref = MB.Mt19937(seed), o.mt_stream(seed)
    assert _same_state(g, ref)
    t = dev.tensor((n,))
    dev.fill_random_uniform(t, lo, hi, g)
    want = ref.uniform(n, lo, hi)
    assert np.array_equal(_bits(t.read()), _bits(want))
    assert _same_state(g, ref)
    t.free()


def test_fills_continue_the_stream_mid_block_and_unaligned():
    """Fills of 10, 100, 4097 (into a view one float into its buffer), 1, 160, 624, 2 * 10^6 and
    33 values in a row equal one host fill of the total: each fill starts where the last one left
    the block.  The 160 use up the current block without a twist (next = 624, remaining = 1) and
    the 624 are exactly the next block."""
    dev, o = device(), oracle()
    g, ref = MB.Mt19937(0x5EED1001), o.mt_stream(0x5EED1001)
    sizes = [10, 100, 4097, 1, 160, 624, 2_000_000, 33]
    want = ref.uniform(sum(sizes), -2.0, 3.0)
    got = []
    for n in sizes:
        if n == 4097:
            base = dev.tensor((1 + n,))
            ptr = base.data_ptr + 4
            MB.check(dev.L.mag_cuda_fill_uniform_mt19937_f32(dev.p, ptr, n, -2.0, 3.0, C.byref(g.st)), "fill")
            got.append(_raw(dev, ptr, n))
        else:
            t = dev.tensor((n,))
            dev.fill_random_uniform(t, -2.0, 3.0, g)
            got.append(t.read())
    assert np.array_equal(_bits(np.concatenate(got)), _bits(want))
    assert _same_state(g, ref)


def test_deep_doubling_levels(monkeypatch):
    """The shortest substreams forced at 2^26 + 9 values: 1121 substreams, eleven doubling
    launches (jumps up to 2^10 L), bit-exact."""
    monkeypatch.setenv("MAG_CUDA_MT_SUBSTREAM_SET", "0")
    dev, o = device(), oracle()
    n = (1 << 26) + 9
    g, ref = MB.Mt19937(0x5EED1002), o.mt_stream(0x5EED1002)
    first = ref.uniform(300, 0.0, 1.0)  # start mid-block
    t0 = dev.tensor((300,))
    dev.fill_random_uniform(t0, 0.0, 1.0, g)
    t = dev.tensor((n,))
    dev.fill_random_uniform(t, 0.0, 1.0, g)
    want = ref.uniform(n, 0.0, 1.0)
    assert np.array_equal(_bits(t0.read()), _bits(first))
    assert np.array_equal(_bits(t.read()), _bits(want))
    assert _same_state(g, ref)


@pytest.mark.parametrize("n", [2, 6, 1000, 4098, (1 << 22) + 2])
@pytest.mark.parametrize("mean,std", [(0.0, 1.0), (3.0, 0.5)])
def test_normal_within_rounding(n, mean, std):
    dev, o = device(), oracle()
    seed = 0x5EED2000 + n
    g, ref = MB.Mt19937(seed), o.mt_stream(seed)
    t = dev.tensor((n,))
    dev.fill_random_normal(t, mean, std, g)
    want = ref.normal(n, mean, std)
    frac = _normal_check(t.read(), want, mean)
    assert frac < 0.05
    assert _same_state(g, ref)


def test_rejects_odd_normal_and_impossible_states():
    """An odd normal fill (the core asserts pairs) and states the host generator cannot be in
    (remaining 0, or next + remaining - 1 past the block) return MAG_CUDA_E_INVALID, launch
    nothing and leave the state alone."""
    dev = device()
    t = dev.tensor((8,))
    g = MB.Mt19937(5)
    before = MB.Mt19937(5)
    k0 = dev.L.mag_cuda_kernel_launches()
    assert dev.L.mag_cuda_fill_normal_mt19937_f32(dev.p, t.data_ptr, 7, 0.0, 1.0, C.byref(g.st)) == MB.E_INVALID
    for rem, nxt in [(0, 0), (625, 0), (300, 400)]:
        g.st.remaining, g.st.next = rem, nxt
        assert dev.L.mag_cuda_fill_uniform_mt19937_f32(dev.p, t.data_ptr, 8, 0.0, 1.0, C.byref(g.st)) == MB.E_INVALID
        assert (g.st.remaining, g.st.next) == (rem, nxt)
    assert dev.L.mag_cuda_kernel_launches() == k0
    assert list(g.st.state) == list(before.st.state)
