"""Drives the unchanged magnetron core (built with MAG_ENABLE_CUDA and linked
against this backend, oracle/_ref/libmagnetron_cudacore.so) through its public
C API, in a process of its own; prints one JSON line with the results.

Usage: python tests/dropin_driver.py {fallback|ops}
"""
import ctypes as C
import json
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, os.path.join(ROOT, "magnetron-pre-oss-release-old_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import mag_b200 as MB  # noqa: E402
from oracle import Oracle, CUDACORE_SO, OP, pad6  # noqa: E402


def bind(L):
    vp = C.c_void_p
    L.mag_ctx_create2.argtypes = [C.c_int]
    L.mag_ctx_create2.restype = vp
    L.mag_ctx_get_compute_device_type.argtypes = [vp]
    L.mag_ctx_get_compute_device_type.restype = C.c_int
    L.mag_ctx_get_compute_device_name.argtypes = [vp]
    L.mag_ctx_get_compute_device_name.restype = C.c_char_p
    L.mag_ctx_destroy.argtypes = [vp]
    L.mag_tensor_create_2d.argtypes = [vp, C.c_int, C.c_int64, C.c_int64]
    L.mag_tensor_create_2d.restype = vp
    L.mag_tensor_copy_buffer_from.argtypes = [vp, vp, C.c_size_t]
    L.mag_tensor_operator.argtypes = [vp, C.c_int, C.c_bool, C.POINTER(vp), C.c_uint32, vp]
    L.mag_tensor_operator.restype = vp
    L.mag_tensor_decref.argtypes = [vp]
    L.mag_tensor_get_scalar_virtual_index.argtypes = [vp, C.c_int64]
    L.mag_tensor_get_scalar_virtual_index.restype = C.c_float
    L.mag_tensor_numel.argtypes = [vp]
    L.mag_tensor_numel.restype = C.c_int64


def read(t):
    """storage.cpy_device_host through the tensor struct, as the core's accessors do."""
    tt = C.cast(t, C.POINTER(MB.TensorT)).contents
    out = np.empty(int(tt.numel), np.float32)
    tt.storage.cpy_device_host(C.byref(tt.storage), 0, out.ctypes.data, out.nbytes)
    return out


def main(mode):
    L = C.CDLL(CUDACORE_SO)
    bind(L)
    ctx = L.mag_ctx_create2(1)  # MAG_COMPUTE_DEVICE_TYPE_CUDA
    res = {"device_type": L.mag_ctx_get_compute_device_type(ctx),
           "device_name": L.mag_ctx_get_compute_device_name(ctx).decode()}
    if mode == "ops":
        o = Oracle()
        s = o.stream(0x5EED0077)
        M, K, N = 64, 96, 48
        x = s.uniform(M * K, -1, 1)
        w = s.uniform(K * N, -1, 1)
        b = s.uniform(M * N, -1, 1)
        tx = L.mag_tensor_create_2d(ctx, 0, M, K)
        tw = L.mag_tensor_create_2d(ctx, 0, K, N)
        tb = L.mag_tensor_create_2d(ctx, 0, M, N)
        for t, a in ((tx, x), (tw, w), (tb, b)):
            L.mag_tensor_copy_buffer_from(t, a.ctypes.data, a.nbytes)

        def op(name, *ins, inplace=False):
            arr = (C.c_void_p * len(ins))(*ins)
            r = L.mag_tensor_operator(ctx, OP[name], inplace, arr, len(ins), None)
            assert r, name
            return r

        h = op("MATMUL", tx, tw)
        h2 = op("ADD", h, tb)
        h3 = op("TANH_DV", h2)
        h4 = op("SIGMOID", h2, inplace=True)
        sm = op("SUM", h4)
        want_h = o.matmul(x, w, M, K, N)
        want_h2 = o.binary("ADD", want_h, pad6((M, N)), b, pad6((M, N)))
        want_h4 = o.unary("SIGMOID", want_h2, pad6((M, N)))
        res["matmul_exact"] = bool(np.array_equal(read(h).view(np.uint32), want_h.view(np.uint32)))
        res["sigmoid_inplace_exact"] = bool(np.array_equal(read(h4).view(np.uint32), want_h4.view(np.uint32)))
        res["h2_aliases_h4"] = bool(np.array_equal(read(h2).view(np.uint32), want_h4.view(np.uint32)))
        got_sum = float(read(sm)[0])
        res["sum_rel_err"] = abs(got_sum - o.reduce("SUM", want_h4, pad6((M, N)))) / max(1.0, abs(got_sum))
        res["scalar_accessor"] = float(L.mag_tensor_get_scalar_virtual_index(h4, 5)) == float(want_h4[5])
        d = o.unary("TANH_DV", want_h2, pad6((M, N)))
        g = read(h3)
        res["tanh_dv_max_rel"] = float(np.max(np.abs(g - d) / np.abs(d)))
        for t in (sm, h4, h3, h2, h, tb, tw, tx):
            L.mag_tensor_decref(t)
        res["launches"] = int(MB.load_library().mag_cuda_kernel_launches())
    L.mag_ctx_destroy(ctx)
    print(json.dumps(res))


if __name__ == "__main__":
    main(sys.argv[1])
