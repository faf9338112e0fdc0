"""The oracle's Mersenne-twister restatement against the reference's own fills.

tests/golden/mt19937.npz holds fills a reference context made with its default generator
(tests/golden/gen_mt.py): uniform fills bit for bit, normal fills within the rounding of
libm's logf/cosf/sinf (the oracle calls the same functions, so they match exactly here).
"""
import os

import numpy as np

from harness import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "mt19937.npz")

SEQUENCES = [
    (0x5EED0000, [("u", 1000, 0.0, 1.0), ("u", 1, -2.0, 3.0), ("n", 2000, 0.0, 1.0), ("u", 5000, -1.0, 1.0)]),
    (1, [("u", 624, 0.0, 1.0), ("u", 624, 0.0, 1.0), ("n", 1250, 2.0, 0.5)]),
    (0xDEADBEEFCAFE, [("n", 4096, 0.0, 0.01), ("u", 623, 5.0, 6.0), ("u", 3, 0.0, 1.0)]),
]


def test_oracle_mt19937_matches_the_reference_fills():
    g = np.load(GOLDEN)
    o = oracle()
    for si, (seed, fills) in enumerate(SEQUENCES):
        s = o.mt_stream(seed)
        for fi, (kind, n, a, b) in enumerate(fills):
            got = s.uniform(n, a, b) if kind == "u" else s.normal(n, a, b)
            want = g[f"s{si}/f{fi}"]
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (si, fi)


def test_oracle_mt19937_state_after_draws():
    """After n draws the state holds the block of the last word drawn, next = words drawn from
    it and remaining = 625 - next (magnetron/magnetron.c:751-777)."""
    o = oracle()
    for n in (1, 623, 624, 625, 1248, 1249, 5000):
        s = o.mt_stream(42)
        words = s.words(n + 1)
        s.uniform(n, 0.0, 1.0)
        t = (n - 1) % 624 + 1
        assert s.g.next == t and s.g.remaining == 625 - t
        assert s.g.state[t - 1] == words[n - 1]
        assert s.words(1)[0] == words[n]
