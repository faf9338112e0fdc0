"""Generate tests/golden/golden.npz from the reference library itself.

Run from the repository root after `make -C oracle all ref`:

    python tests/golden/gen_golden.py

For every case in cases.py it creates a CPU context of the reference build
(oracle/_ref/libmagnetron.so), seeds its PCG generator, fills the inputs with
the reference's own fill_random_* calls, runs the op through
mag_tensor_operator and stores the output together with the first 16 values of
each input (which pin the oracle's restatement of the generator).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, HERE)

from oracle import RefLib, pad6  # noqa: E402
import cases as C  # noqa: E402


def fill(R, t, dist):
    kind, a, b = dist
    if kind == "u":
        R.L.mag_tensor_fill_random_uniform(t, a, b)
    else:
        R.L.mag_tensor_fill_random_normal(t, a, b)


def main():
    R = RefLib()
    out = {}
    for c in C.cases():
        cid = C.case_id(c)
        R.seed(c["seed"])
        if c["kind"] == "matmul":
            x = R.tensor_nd(c["x"])
            y = R.tensor_nd(c["y"])
        else:
            x = R.tensor(pad6(c["x"]))
            y = R.tensor(pad6(c["y"])) if "y" in c else None
        fill(R, x, c["dist"][0])
        if y is not None:
            fill(R, y, c["dist"][1])
        ins = [x] + ([y] if y is not None else [])
        r = R.op(c["op"], *ins, xi=c.get("xi"))
        out[cid + "/out"] = R.read(r)
        out[cid + "/x16"] = R.read(x)[:16]
        if y is not None:
            out[cid + "/y16"] = R.read(y)[:16]
        R.free(r, *ins)
    R.close()
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main()
