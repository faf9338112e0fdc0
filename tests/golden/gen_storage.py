"""Generate tests/golden/storage/*.magnetron with the reference library's own writer.

Run from the repository root after `make -C oracle all ref`:

    python tests/golden/gen_storage.py

Each file is one tensor saved by mag_tensor_save (magnetron/magnetron.c:2931-2950) from a
CPU context of the reference build (oracle/_ref/libmagnetron.so).  The tensor's values are
the reference's own fill_random_uniform draws from a PCG context seeded with `seed`, so the
tests regenerate them with the oracle's stream; storage.json lists name, shape and seed.
"""
import ctypes as C
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import RefLib  # noqa: E402

CASES = [
    {"file": "weight.magnetron", "shape": [4, 8], "name": "fc1.weight", "seed": 0x5EED5701},
    {"file": "bias.magnetron", "shape": [5], "name": "b", "seed": 0x5EED5702},
    {"file": "cube6d.magnetron", "shape": [1, 2, 3, 1, 2, 2], "name": "", "seed": 0x5EED5703},
    {"file": "longname.magnetron", "shape": [3, 3], "name": "n" * 70, "seed": 0x5EED5704},
    {"file": "rows.magnetron", "shape": [256, 33], "name": "rows", "seed": 0x5EED5705},
]


def main():
    R = RefLib()
    R.L.mag_tensor_set_name.argtypes = [C.c_void_p, C.c_char_p]
    R.L.mag_tensor_save.argtypes = [C.c_void_p, C.c_char_p]
    out_dir = os.path.join(HERE, "storage")
    os.makedirs(out_dir, exist_ok=True)
    for c in CASES:
        R.seed(c["seed"])
        t = R.tensor_nd(c["shape"])
        R.L.mag_tensor_set_name(t, c["name"].encode())
        R.L.mag_tensor_fill_random_uniform(t, -1.0, 1.0)
        R.L.mag_tensor_save(t, os.path.join(out_dir, c["file"]).encode())
        R.free(t)
    with open(os.path.join(out_dir, "storage.json"), "w") as f:
        json.dump({"lo": -1.0, "hi": 1.0, "cases": CASES}, f, indent=1)
    R.close()


if __name__ == "__main__":
    main()
