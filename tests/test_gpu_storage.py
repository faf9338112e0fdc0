"""Device save/load of .magnetron files against files the reference's own writer made
(tests/golden/storage) and through round trips at sizes spanning many 8 MiB chunks."""
import ctypes as C
import json
import os

import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle
from gpu_util import device

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "storage")
MANIFEST = json.load(open(os.path.join(GOLD, "storage.json")))
CASES = MANIFEST["cases"]


def _values(case):
    return oracle().stream(case["seed"]).uniform(int(np.prod(case["shape"])), MANIFEST["lo"], MANIFEST["hi"])


@pytest.mark.parametrize("case", CASES, ids=[c["file"] for c in CASES])
def test_device_save_matches_reference_file(case, tmp_path):
    dev = device()
    t = dev.tensor(tuple(case["shape"]))
    t.name = case["name"]
    t.write(_values(case))
    path = str(tmp_path / "t.magnetron")
    with open(path, "wb") as f:  # an older, longer file at the path is replaced, not patched
        f.write(b"\xff" * 100_000)
    dev.save(path, [t])
    assert open(path, "rb").read() == open(os.path.join(GOLD, case["file"]), "rb").read()


@pytest.mark.parametrize("case", CASES, ids=[c["file"] for c in CASES])
def test_device_load_reference_file(case):
    dev = device()
    (t,) = dev.load(os.path.join(GOLD, case["file"]))
    assert t.shape == tuple(case["shape"]) and t.name == case["name"][:63] and t.t.flags == MB.TFLAG_OWNER
    assert np.array_equal(t.read().view(np.uint32), _values(case).view(np.uint32))


def test_round_trip_many_chunks(tmp_path):
    """Three tensors, 64 MiB + 4 KB + 36 MB: chunk edges inside and between tensors."""
    dev = device()
    shapes = [(4096, 4096), (1000,), (8192, 1111)]
    ts, vals = [], []
    for i, s in enumerate(shapes):
        v = oracle().stream(77 + i).uniform(int(np.prod(s)), -3, 3)
        t = dev.tensor(s)
        t.name = f"t{i}"
        t.write(v)
        ts.append(t)
        vals.append(v)
    path = str(tmp_path / "many.magnetron")
    dev.save(path, ts)
    assert os.path.getsize(path) == 20 + 3 * 116 + sum(v.nbytes for v in vals)
    back = dev.load(path)
    for t, b, v, i in zip(ts, back, vals, range(3)):
        assert b.shape == t.shape and b.name == f"t{i}"
        assert np.array_equal(b.read(), v)
    ver, ents = MB.sto_parse(open(path, "rb").read(20 + 3 * 116), os.path.getsize(path))
    assert [e.dims for e in ents] == shapes


def test_save_never_written_tensor_is_zero(tmp_path):
    dev = device()
    t = dev.tensor((3, 1024))
    path = str(tmp_path / "z.magnetron")
    dev.save(path, [t])
    assert open(path, "rb").read()[136:] == b"\0" * (3 * 1024 * 4)


def test_save_waits_for_queued_ops_and_load_for_readers(tmp_path):
    dev, o = device(), oracle()
    x = dev.tensor((1 << 20,))
    v = o.stream(5).uniform(1 << 20, -1, 1)
    x.write(v)
    y = dev.op("NEG", x)  # eager: queued on the device stream
    path = str(tmp_path / "y.magnetron")
    dev.save(path, [y])
    assert np.array_equal(np.frombuffer(open(path, "rb").read()[136:], np.float32), -v)
    z = dev.op("ABS", x)  # reads x; the load below overwrites x
    other = dev.tensor((1 << 20,))
    other.write(np.full(1 << 20, 7.0, np.float32))
    dev.save(path, [other])
    MB.check(dev.L.mag_cuda_tensor_load(dev.p, path.encode(), (C.c_void_p * 1)(x.ptr), 1), "load")
    assert np.array_equal(z.read(), np.abs(v))
    assert np.array_equal(x.read(), np.full(1 << 20, 7.0, np.float32))


def test_load_rejects_shape_mismatch_and_bad_paths(tmp_path):
    dev = device()
    src = os.path.join(GOLD, CASES[0]["file"])
    wrong = dev.tensor((8, 4))
    assert dev.L.mag_cuda_tensor_load(dev.p, src.encode(), (C.c_void_p * 1)(wrong.ptr), 1) == MB.E_INVALID
    assert dev.L.mag_cuda_tensor_load(dev.p, b"/nonexistent/a.magnetron", (C.c_void_p * 1)(wrong.ptr), 1) == MB.E_IO
    assert dev.L.mag_cuda_tensor_save(dev.p, str(tmp_path / "a.bin").encode(), (C.c_void_p * 1)(wrong.ptr),
                                      1) == MB.E_INVALID
