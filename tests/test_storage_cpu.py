""".magnetron storage format on the CPU: the backend's header writer and parser against
files the reference's own mag_tensor_save wrote (tests/golden/storage, made by
tests/golden/gen_storage.py), and against the reference reader
(mag_sto_read_buffered, magnetron/magnetron.c:2884-2922) on malformed images.

No GPU: the parser and the header writer are host code of the backend library.
"""
import ctypes as C
import json
import os
import struct

import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "storage")
MANIFEST = json.load(open(os.path.join(GOLD, "storage.json")))
CASES = MANIFEST["cases"]


class HostTensor:
    """A mag_tensor_t with shape, name and flags but no storage (enough for the header writer)."""

    def __init__(self, shape, name, flags=MB.TFLAG_OWNER):
        self.t = t = MB.TensorT()
        s6 = MB.pad6(shape)
        t.rank = len(shape)
        for i in range(6):
            t.shape[i] = s6[i]
        t.numel = int(np.prod(s6))
        t.dtype = 0
        t.flags = flags
        t.storage.size = t.numel * 4
        raw = name.encode()[:63]
        C.memmove(C.addressof(t) + MB.TensorT.name.offset, raw, len(raw))

    @property
    def ptr(self):
        return C.addressof(self.t)


def _values(case):
    s = oracle().stream(case["seed"])
    return s.uniform(int(np.prod(case["shape"])), MANIFEST["lo"], MANIFEST["hi"])


def _gold(case) -> bytes:
    return open(os.path.join(GOLD, case["file"]), "rb").read()


@pytest.mark.parametrize("case", CASES, ids=[c["file"] for c in CASES])
def test_parse_reference_file(case):
    buf = _gold(case)
    ver, ents = MB.sto_parse(buf)
    assert ver == 1 and len(ents) == 1
    e = ents[0]
    assert e.name.decode() == case["name"][:63]
    assert e.dims == tuple(case["shape"]) and e.dtype == 0 and e.flags == MB.TFLAG_OWNER
    assert e.offset == 20 + 116 and e.bytes == 4 * int(np.prod(case["shape"])) == len(buf) - e.offset
    got = np.frombuffer(buf[e.offset:], np.float32)
    assert np.array_equal(got.view(np.uint32), _values(case).view(np.uint32))


@pytest.mark.parametrize("case", CASES, ids=[c["file"] for c in CASES])
def test_writer_matches_reference_bytes(case):
    t = HostTensor(case["shape"], case["name"])
    assert MB.sto_header([t]) + _values(case).tobytes() == _gold(case)


def _ref_reader():
    from oracle import RefLib, REF_SO
    if not os.path.exists(REF_SO):
        pytest.skip("reference library not built (make -C oracle ref)")
    R = RefLib()
    R.L.mag_sto_read_buffered.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_uint32),
                                          C.POINTER(C.c_uint32)]
    R.L.mag_sto_read_buffered.restype = C.POINTER(C.c_void_p)
    R.L.mag_tensor_get_name.argtypes = [C.c_void_p]
    R.L.mag_tensor_get_name.restype = C.c_char_p
    return R


def _mutations(base: bytes):
    """Malformed images the reference reader rejects in its header phase (returns NULL)."""
    b = bytearray(base)

    def put(off, fmt, v):
        m = bytearray(b)
        struct.pack_into(fmt, m, off, v)
        return bytes(m)

    aux = struct.unpack_from("<I", b, 84)[0]
    return {
        "bad magic": put(0, "<B", ord("M")),
        "version 0": put(8, "<I", 0),
        "version 2": put(8, "<I", 2),
        "no tensors": put(12, "<I", 0),
        "count beyond headers": put(12, "<I", 2),
        "flag bit 4": put(84, "<I", aux | (1 << 20)),
        "dtype 1": put(84, "<I", (aux & ~0xFF00) | (1 << 8)),
        "rank 0": put(84, "<I", aux & ~0xFF),
        "rank 7": put(84, "<I", (aux & ~0xFF) | 7),
        "zero dim": put(88 + 8, "<Q", 0),
        "dim above int64": put(88, "<Q", 1 << 63),
        "shape overflow": put(88 + 8 * 2, "<Q", 1 << 62),
        "too short": bytes(b[:137]),
    }


def test_malformed_rejected_like_reference():
    base = _gold(CASES[1])  # one 5-element tensor: a second header cannot fit
    muts = _mutations(base)
    for what, img in muts.items():
        with pytest.raises(MB.CudaError):
            MB.sto_parse(img)
    R = _ref_reader()
    for what, img in muts.items():
        n, ver = C.c_uint32(0), C.c_uint32(0)
        r = R.L.mag_sto_read_buffered(R.ctx, img, len(img), C.byref(n), C.byref(ver))
        assert not r, f"reference accepted '{what}'"
    n, ver = C.c_uint32(0), C.c_uint32(0)
    assert R.L.mag_sto_read_buffered(R.ctx, base, len(base), C.byref(n), C.byref(ver)) and n.value == 1
    R.close()


def test_truncated_data_rejected():
    """The reference aborts here (mag_assert2, magnetron/magnetron.c:2914); the backend returns an error."""
    base = _gold(CASES[4])
    with pytest.raises(MB.CudaError):
        MB.sto_parse(base[:-1])
    ver, ents = MB.sto_parse(base + b"\0" * 8)  # trailing bytes are not checked by the reader
    assert ents[0].bytes == len(base) - 136


def test_multi_tensor_file_read_by_reference():
    """mag_tensor_save writes one tensor; the format (and the exported reader) takes n.
    A three-tensor image from the backend's writer reads back in the reference."""
    shapes, names = [(3, 4), (7,), (2, 1, 3)], ["w", "bias.0", "z" * 63]
    hts = [HostTensor(s, n) for s, n in zip(shapes, names)]
    vals = [oracle().stream(900 + i).uniform(int(np.prod(s)), -1, 1) for i, s in enumerate(shapes)]
    img = MB.sto_header(hts) + b"".join(v.tobytes() for v in vals)
    ver, ents = MB.sto_parse(img)
    off = 20 + 3 * 116
    for e, s, v in zip(ents, shapes, vals):
        assert e.dims == s and e.offset == off
        off += v.nbytes
    R = _ref_reader()
    n, ver = C.c_uint32(0), C.c_uint32(0)
    ts = R.L.mag_sto_read_buffered(R.ctx, img, len(img), C.byref(n), C.byref(ver))
    assert ts and n.value == 3 and ver.value == 1
    for i in range(3):
        assert R.L.mag_tensor_get_name(ts[i]).decode() == names[i]
        assert np.array_equal(R.read(ts[i]), vals[i])
    R.close()


def test_paths_checked_before_any_device_work():
    L = MB.load_library()
    n, ver = C.c_uint32(0), C.c_uint32(0)
    assert L.mag_cuda_sto_read_directory(b"/nonexistent/x.bin", None, 0, C.byref(n), C.byref(ver)) == MB.E_INVALID
    assert L.mag_cuda_sto_read_directory(b".magnetron", None, 0, C.byref(n), C.byref(ver)) == MB.E_INVALID
    assert L.mag_cuda_sto_read_directory(b"/nonexistent/x.magnetron", None, 0, C.byref(n), C.byref(ver)) == MB.E_IO
    path = os.path.join(GOLD, CASES[1]["file"]).encode()
    ents = (MB.StoEntry * 1)()
    assert L.mag_cuda_sto_read_directory(path, ents, 1, C.byref(n), C.byref(ver)) == 0
    assert n.value == 1 and ents[0].dims == (5,) and ents[0].offset == 136
