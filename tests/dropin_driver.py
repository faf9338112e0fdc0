"""Drives the unchanged magnetron core (built with MAG_ENABLE_CUDA and linked
against this backend, oracle/_ref/libmagnetron_cudacore.so) through its public
C API, in a process of its own; prints one JSON line with the results.

Usage: python tests/dropin_driver.py {fallback|ops|bench}

`bench` times, end to end through the core's eager C API (inputs in through
mag_tensor_copy_buffer_from, every op through mag_tensor_operator, results out
through the storage callback), the two-layer MLP forward at batch 256 and an
8192-row slice of the deep MLP (8 x [4096 x 4096 + bias + GELU], 4096 x 1000 +
bias, the row softmax through the backend's extension), in samples/s.
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


def bench(L, ctx, res):
    """End-to-end samples/s through the core's eager API (see the module docstring)."""
    import time
    import torch
    lib = MB.load_library()
    L.mag_tensor_create_1d.argtypes = [C.c_void_p, C.c_int, C.c_int64]
    L.mag_tensor_create_1d.restype = C.c_void_p
    g = torch.Generator().manual_seed(1234)

    def tensor(d1, d2, a=None):
        t = L.mag_tensor_create_2d(ctx, 0, d1, d2)
        if a is not None:
            a = np.ascontiguousarray(a, np.float32)
            L.mag_tensor_copy_buffer_from(t, a.ctypes.data, a.nbytes)
        return t

    def st(t):
        return C.cast(t, C.POINTER(MB.TensorT)).contents.storage

    def op(name, *ins, inplace=False):
        arr = (C.c_void_p * len(ins))(*ins)
        r = L.mag_tensor_operator(ctx, OP[name], inplace, arr, len(ins), None)
        assert r, name
        return r

    def timed(step, reps):
        for _ in range(3):
            step()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            step()
            ts.append(time.perf_counter() - t0)
        return float(np.median(ts))

    def forward(x_host, rows, layers, d_in, w_first, b_first, act, w_out, b_out, d_out, out_host):
        tx = tensor(rows, d_in, x_host)
        keep, h = [tx], tx
        for i, (w, b) in enumerate(layers):
            m = op("MATMUL", h, w)
            a = op("ADD", m, b)
            h = op(act, a, inplace=True)
            keep += [m, a, h]
        zm = op("MATMUL", h, w_out)
        z = op("ADD", zm, b_out)
        keep += [zm, z]
        p = tensor(rows, d_out)
        keep.append(p)
        dvc = st(z).host  # the backend device the core created for this context
        MB.check(lib.mag_cuda_softmax_rows_f32(dvc, int(st(p).base), int(st(z).base), rows, d_out), "softmax")
        sp = st(p)
        sp.cpy_device_host(C.byref(sp), 0, out_host.ctypes.data, out_host.nbytes)  # waits for the forward
        for t in reversed(keep):
            L.mag_tensor_decref(t)

    # two-layer MLP, batch 256: MATMUL -> ADD(1-D bias) -> SIGMOID -> MATMUL -> ADD, row softmax
    B, D, H, O = 256, 784, 256, 10
    lim1, lim2 = (6.0 / (D + H)) ** 0.5, (6.0 / (H + O)) ** 0.5
    x1 = torch.rand(B * D, generator=g).numpy()
    w1 = tensor(D, H, ((torch.rand(D * H, generator=g) * 2 - 1) * lim1).numpy())
    w2 = tensor(H, O, ((torch.rand(H * O, generator=g) * 2 - 1) * lim2).numpy())
    b1 = L.mag_tensor_create_1d(ctx, 0, H)
    b2 = tensor(B, O)
    o1 = np.empty(B * O, np.float32)
    t1 = timed(lambda: forward(x1, B, [(w1, b1)], D, None, None, "SIGMOID", w2, b2, O, o1), 50)
    res["mlp2_batch256_samples_per_s"] = B / t1
    res["mlp2_batch256_ms"] = t1 * 1e3
    for t in (b2, b1, w2, w1):
        L.mag_tensor_decref(t)

    # deep MLP slice: 8192 rows of 4096, 8 x [MATMUL -> ADD(zero bias) -> GELU], MATMUL -> ADD, softmax
    R, DH, DO = 8192, 4096, 1000
    std = (2.0 / DH) ** 0.5
    x5 = torch.randn(R * DH, generator=g).numpy()
    layers = [(tensor(DH, DH, (torch.randn(DH * DH, generator=g) * std).numpy()), tensor(R, DH)) for _ in range(8)]
    wo, bo = tensor(DH, DO, (torch.randn(DH * DO, generator=g) * std).numpy()), tensor(R, DO)
    o5 = np.empty(R * DO, np.float32)
    t5 = timed(lambda: forward(x5, R, layers, DH, None, None, "GELU", wo, bo, DO, o5), 5)
    res["deep_mlp_8192_samples_per_s"] = R / t5
    res["deep_mlp_8192_ms"] = t5 * 1e3
    res["deep_mlp_8192_tflops"] = 2.0 * R * (8 * DH * DH + DH * DO) / t5 / 1e12
    res["h2d_bytes_per_step"] = R * DH * 4
    res["d2h_bytes_per_step"] = R * DO * 4
    for w, b in layers:
        L.mag_tensor_decref(w)
        L.mag_tensor_decref(b)
    L.mag_tensor_decref(wo)
    L.mag_tensor_decref(bo)


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
    elif mode == "bench":
        bench(L, ctx, res)
    L.mag_ctx_destroy(ctx)
    print(json.dumps(res))


if __name__ == "__main__":
    main(sys.argv[1])
