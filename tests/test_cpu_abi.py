"""CPU-side checks of the C ABI: the library loads, exports every declared
entry point, its struct layout matches the core's, and it declines cleanly
(NULL device) where no GPU is present, which makes the core fall back to its
CPU device (magnetron/magnetron.c:895-899)."""
import ctypes as C
import os
import re

import pytest

import mag_b200 as MB

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def declared_symbols():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"MAG_CUDA_EXPORT[^;(]*?\b(mag_\w+)\s*\(", src)
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "mag_init_device_cuda" in names and "mag_destroy_device_cuda" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    L = C.CDLL(MB.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(L, name), name


def test_struct_layout_matches_core():
    assert C.sizeof(MB.TensorT) == 384
    assert MB.TensorT.storage.offset == 128 and MB.TensorT.op.offset == 196
    assert MB.TensorT.op_inputs.offset == 200 and MB.TensorT.op_params.offset == 216
    assert MB.ComputeDevice.eager_exec_fwd.offset == 144 and C.sizeof(MB.ComputeDevice) == 176


def test_op_numbering_matches_core():
    assert MB.OP["MATMUL"] == 38 and MB.OP["ADD"] == 30 and MB.OP["SOFTMAX"] == 17 and MB.OP["DIVS"] == 37


def test_f32_param_packing():
    # mag_op_param_float: raw f32 bits, tag 0 in bits 62..63 (magnetron/magnetron.c:1126-1130)
    assert MB.f32_param(1.0) == 0x3F800000


def test_init_without_gpu_returns_null():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = MB.load_library()
    assert not L.mag_init_device_cuda(None)


def test_pcg_seeding_matches_oracle():
    """The host-side stream handle starts where the reference context's PCG does."""
    from harness import oracle
    o = oracle()
    for seed in (1, 0x5EED0001, 2**63 + 5):
        g, ref = MB.Pcg(seed), o.stream(seed)
        assert (g.state.value, g.inc) == (ref.g.state, ref.g.inc)
