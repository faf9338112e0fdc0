"""Generate tests/golden/mt19937.npz from the reference library itself.

Run from the repository root after `make -C oracle all ref`:

    python tests/golden/gen_mt.py

A CPU context of the reference build (oracle/_ref/libmagnetron.so) is switched to its
Mersenne-twister generator with a seed (mag_ctx_set_prng_algorithm, the reference's default
algorithm) and fills tensors in sequence with mag_tensor_fill_random_uniform and
mag_tensor_fill_random_normal; each fill's output is stored.  The sizes cross the generator's
624-word blocks (so the later fills start in the middle of a block).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import RefLib  # noqa: E402

# (seed, [(kind, n, a, b), ...]) filled in order on one context
SEQUENCES = [
    (0x5EED0000, [("u", 1000, 0.0, 1.0), ("u", 1, -2.0, 3.0), ("n", 2000, 0.0, 1.0), ("u", 5000, -1.0, 1.0)]),
    (1, [("u", 624, 0.0, 1.0), ("u", 624, 0.0, 1.0), ("n", 1250, 2.0, 0.5)]),
    (0xDEADBEEFCAFE, [("n", 4096, 0.0, 0.01), ("u", 623, 5.0, 6.0), ("u", 3, 0.0, 1.0)]),
]


def main():
    R = RefLib()
    out = {}
    for si, (seed, fills) in enumerate(SEQUENCES):
        R.seed_mt(seed)
        for fi, (kind, n, a, b) in enumerate(fills):
            t = R.tensor_nd((n,))
            if kind == "u":
                R.L.mag_tensor_fill_random_uniform(t, a, b)
            else:
                R.L.mag_tensor_fill_random_normal(t, a, b)
            out[f"s{si}/f{fi}"] = R.read(t)
            R.free(t)
    R.close()
    np.savez_compressed(os.path.join(HERE, "mt19937.npz"), **out)
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main()
