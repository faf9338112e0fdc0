"""ctypes bindings for the parity checker.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py.  It never feeds the product path.

* ``Oracle`` wraps ``oracle/liboracle.so``, the C restatement of the reference
  kernels (mag_oracle.c).
* ``RefLib`` wraps ``oracle/_ref/libmagnetron.so``, the reference library built
  from its own sources (present only where the sources were available at build
  time); it drives the reference's public C API (magnetron/magnetron.h).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmagnetron.so")
CUDACORE_SO = os.path.join(HERE, "_ref", "libmagnetron_cudacore.so")

# op numbering of magnetron/magnetron.h:136-178
OPS = ["NOP", "CLONE", "VIEW", "TRANSPOSE", "PERMUTE", "MEAN", "MIN", "MAX", "SUM",
       "ABS", "NEG", "LOG", "SQR", "SQRT", "SIN", "COS", "STEP", "SOFTMAX", "SOFTMAX_DV",
       "SIGMOID", "SIGMOID_DV", "HARD_SIGMOID", "SILU", "SILU_DV", "TANH", "TANH_DV",
       "RELU", "RELU_DV", "GELU", "GELU_DV", "ADD", "SUB", "MUL", "DIV",
       "ADDS", "SUBS", "MULS", "DIVS", "MATMUL"]
OP = {n: i for i, n in enumerate(OPS)}

_f32p = C.POINTER(C.c_float)
_i64p = C.POINTER(C.c_int64)


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


def _ip(v) -> C.Array:
    return (C.c_int64 * 6)(*[int(t) for t in v])


def build():
    subprocess.check_call(["make", "-s", "-C", HERE, "all"])


class _Pcg(C.Structure):
    _fields_ = [("state", C.c_uint64), ("inc", C.c_uint64)]


class Stream:
    """One seeded PCG stream, drawn in order like a reference context's PRNG."""

    def __init__(self, oracle: "Oracle", seed: int):
        self.o = oracle
        self.g = _Pcg()
        oracle.L.orc_pcg_seed(C.byref(self.g), seed)

    def uniform(self, n: int, lo: float, hi: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.o.L.orc_fill_uniform(C.byref(self.g), _fp(out), n, lo, hi)
        return out

    def normal(self, n: int, mean: float, std: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.o.L.orc_fill_normal(C.byref(self.g), _fp(out), n, mean, std)
        return out

    def draw(self, n: int, dist):
        kind, a, b = dist
        return self.uniform(n, a, b) if kind == "u" else self.normal(n, a, b)


class MtState(C.Structure):
    """A reference context's Mersenne-twister state (magnetron/magnetron_internal.h:398-402)."""
    _fields_ = [("remaining", C.c_uint32), ("next", C.c_uint32), ("state", C.c_uint32 * 624)]


class MtStream:
    """One seeded Mersenne-twister stream, drawn in order like a default reference context."""

    def __init__(self, oracle: "Oracle", seed: int):
        self.o = oracle
        self.g = MtState()
        oracle.L.orc_mt_seed(C.byref(self.g), seed)

    def uniform(self, n: int, lo: float, hi: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.o.L.orc_fill_uniform_mt(C.byref(self.g), _fp(out), n, lo, hi)
        return out

    def normal(self, n: int, mean: float, std: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.o.L.orc_fill_normal_mt(C.byref(self.g), _fp(out), n, mean, std)
        return out

    def words(self, n: int) -> np.ndarray:
        """The next n untempered words, without drawing them."""
        out = np.empty(n, np.uint32)
        self.o.L.orc_mt_words(C.byref(self.g), out.ctypes.data_as(C.POINTER(C.c_uint32)), n)
        return out

    def copy_state(self) -> MtState:
        c = MtState()
        C.memmove(C.byref(c), C.byref(self.g), C.sizeof(MtState))
        return c


class Oracle:
    def stream(self, seed: int) -> Stream:
        return Stream(self, seed)

    def mt_stream(self, seed: int) -> MtStream:
        return MtStream(self, seed)

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        self.L = L
        L.orc_pcg_seed.argtypes = [C.POINTER(_Pcg), C.c_uint64]
        L.orc_fill_uniform.argtypes = [C.POINTER(_Pcg), _f32p, C.c_int64, C.c_float, C.c_float]
        L.orc_fill_normal.argtypes = [C.POINTER(_Pcg), _f32p, C.c_int64, C.c_float, C.c_float]
        L.orc_mt_seed.argtypes = [C.POINTER(MtState), C.c_uint64]
        L.orc_fill_uniform_mt.argtypes = [C.POINTER(MtState), _f32p, C.c_int64, C.c_float, C.c_float]
        L.orc_fill_normal_mt.argtypes = [C.POINTER(MtState), _f32p, C.c_int64, C.c_float, C.c_float]
        L.orc_mt_words.argtypes = [C.POINTER(MtState), C.POINTER(C.c_uint32), C.c_int64]
        L.orc_sse_expf.argtypes = [C.c_float]
        L.orc_sse_expf.restype = C.c_float
        L.orc_sse_logf.argtypes = [C.c_float]
        L.orc_sse_logf.restype = C.c_float
        L.orc_unary.argtypes = [C.c_int, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_float]
        L.orc_unary.restype = C.c_int
        L.orc_binary.argtypes = [C.c_int, _f32p, _f32p, _f32p, _i64p, _i64p, _i64p, _i64p, _i64p]
        L.orc_reduce.argtypes = [C.c_int, _f32p, _i64p, _i64p]
        L.orc_reduce.restype = C.c_float
        L.orc_matmul.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64]
        L.orc_matmul_rows.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64]
        L.orc_matmul_batched.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int64]
        L.orc_binary_bcast2.argtypes = [C.c_int, _f32p, _f32p, _f32p, _i64p, _i64p, _i64p, _i64p, C.c_int64]
        L.orc_reduce_rows.argtypes = [C.c_int, _f32p, _f32p, C.c_int64, C.c_int64]
        L.orc_softmax_rows.argtypes = [_f32p, _f32p, C.c_int64, C.c_int64]

    # ---- seeded inputs (the reference's PCG + Box-Muller) ----
    def uniform(self, n: int, lo: float, hi: float, seed: int) -> np.ndarray:
        g = _Pcg()
        self.L.orc_pcg_seed(C.byref(g), seed)
        out = np.empty(n, np.float32)
        self.L.orc_fill_uniform(C.byref(g), _fp(out), n, lo, hi)
        return out

    def normal(self, n: int, mean: float, std: float, seed: int) -> np.ndarray:
        g = _Pcg()
        self.L.orc_pcg_seed(C.byref(g), seed)
        out = np.empty(n, np.float32)
        self.L.orc_fill_normal(C.byref(g), _fp(out), n, mean, std)
        return out

    # ---- kernels ----
    def unary(self, op: str, x: np.ndarray, shape6, xi: float = 0.0) -> np.ndarray:
        """Contiguous unary/scalar op on a tensor of magnetron shape6 (dim 0 fastest)."""
        x = np.ascontiguousarray(x, np.float32)
        r = np.zeros_like(x)
        cols = int(shape6[0])
        rows = int(np.prod(shape6[1:]))
        rc = self.L.orc_unary(OP[op], _fp(r), _fp(x), rows, cols, cols, cols, xi)
        if rc != 0:
            raise RuntimeError(f"{op}: the reference panics (NYI)")
        return r

    def binary(self, op: str, x: np.ndarray, xshape6, y: np.ndarray, yshape6) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.ascontiguousarray(y, np.float32)
        r = np.zeros_like(x)
        xs, ys = strides6(xshape6), strides6(yshape6)
        self.L.orc_binary(OP[op], _fp(r), _fp(x), _fp(y), _ip(xshape6), _ip(xs), _ip(xs), _ip(yshape6), _ip(ys))
        return r

    def reduce(self, op: str, x: np.ndarray, shape6) -> float:
        x = np.ascontiguousarray(x, np.float32)
        return float(self.L.orc_reduce(OP[op], _fp(x), _ip(shape6), _ip(strides6(shape6))))

    def matmul(self, x: np.ndarray, y: np.ndarray, M: int, K: int, N: int) -> np.ndarray:
        r = np.zeros(M * N, np.float32)
        self.L.orc_matmul(_fp(r), _fp(np.ascontiguousarray(x, np.float32)), _fp(np.ascontiguousarray(y, np.float32)), M, K, N, N)
        return r

    def matmul_rows(self, x, y, row0: int, nrows: int, K: int, N: int) -> np.ndarray:
        r = np.empty(nrows * N, np.float32)
        self.L.orc_matmul_rows(_fp(r), _fp(np.ascontiguousarray(x, np.float32)), _fp(np.ascontiguousarray(y, np.float32)), row0, nrows, K, N)
        return r

    def matmul_batched(self, x, y, batch: int, M: int, K: int, N: int) -> np.ndarray:
        r = np.empty(batch * M * N, np.float32)
        self.L.orc_matmul_batched(_fp(r), _fp(np.ascontiguousarray(x, np.float32)), _fp(np.ascontiguousarray(y, np.float32)), batch, M, K, N)
        return r

    def bcast2(self, op: str, x, xshape6, y, yshape6, rshape6, sample_idx=None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.ascontiguousarray(y, np.float32)
        if sample_idx is None:
            n = int(np.prod(rshape6))
            r = np.empty(n, np.float32)
            self.L.orc_binary_bcast2(OP[op], _fp(r), _fp(x), _fp(y), _ip(rshape6), _ip(xshape6), _ip(yshape6), None, 0)
        else:
            idx = np.ascontiguousarray(sample_idx, np.int64)
            r = np.empty(idx.size, np.float32)
            self.L.orc_binary_bcast2(OP[op], _fp(r), _fp(x), _fp(y), _ip(rshape6), _ip(xshape6), _ip(yshape6),
                                     idx.ctypes.data_as(_i64p), idx.size)
        return r

    def reduce_rows(self, op: str, x, rows: int, cols: int) -> np.ndarray:
        r = np.empty(rows, np.float32)
        self.L.orc_reduce_rows(OP[op], _fp(r), _fp(np.ascontiguousarray(x, np.float32)), rows, cols)
        return r

    def softmax_rows(self, x, rows: int, cols: int) -> np.ndarray:
        r = np.empty(rows * cols, np.float32)
        self.L.orc_softmax_rows(_fp(r), _fp(np.ascontiguousarray(x, np.float32)), rows, cols)
        return r


def strides6(shape6):
    s = [1] * 6
    for i in range(1, 6):
        s[i] = s[i - 1] * int(shape6[i - 1])
    return s


def pad6(shape):
    shape = list(shape)
    return shape + [1] * (6 - len(shape))


class RefLib:
    """The reference library's public C API (magnetron/magnetron.h) on a CPU context."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        self.L = L
        vp = C.c_void_p
        L.mag_ctx_create2.argtypes = [C.c_int]
        L.mag_ctx_create2.restype = vp
        L.mag_ctx_destroy.argtypes = [vp]
        L.mag_ctx_set_prng_algorithm.argtypes = [vp, C.c_int, C.c_uint64]
        L.mag_tensor_create_6d.argtypes = [vp, C.c_int] + [C.c_int64] * 6
        L.mag_tensor_create_6d.restype = vp
        L.mag_tensor_create_2d.argtypes = [vp, C.c_int, C.c_int64, C.c_int64]
        L.mag_tensor_create_2d.restype = vp
        L.mag_tensor_create_1d.argtypes = [vp, C.c_int, C.c_int64]
        L.mag_tensor_create_1d.restype = vp
        L.mag_tensor_fill_random_uniform.argtypes = [vp, C.c_float, C.c_float]
        L.mag_tensor_fill_random_normal.argtypes = [vp, C.c_float, C.c_float]
        L.mag_tensor_fill.argtypes = [vp, C.c_float]
        L.mag_tensor_copy_buffer_from.argtypes = [vp, vp, C.c_size_t]
        L.mag_tensor_operator.argtypes = [vp, C.c_int, C.c_bool, C.POINTER(vp), C.c_uint32, vp]
        L.mag_tensor_operator.restype = vp
        L.mag_tensor_data_ptr.argtypes = [vp]
        L.mag_tensor_data_ptr.restype = vp
        L.mag_tensor_numel.argtypes = [vp]
        L.mag_tensor_numel.restype = C.c_int64
        L.mag_tensor_decref.argtypes = [vp]
        L.mag_tensor_decref.restype = C.c_bool
        L.mag_op_param_float.argtypes = [C.c_float]
        L.mag_op_param_float.restype = C.c_uint64
        self.ctx = L.mag_ctx_create2(0)
        self._live = []

    def seed(self, seed: int):
        self.L.mag_ctx_set_prng_algorithm(self.ctx, 1, seed)  # MAG_PRNG_PCG

    def seed_mt(self, seed: int):
        self.L.mag_ctx_set_prng_algorithm(self.ctx, 0, seed)  # MAG_PRNG_MERSENNE_TWISTER

    def tensor(self, shape6):
        return self.L.mag_tensor_create_6d(self.ctx, 0, *[int(s) for s in shape6])

    def tensor_nd(self, shape):
        if len(shape) == 1:
            return self.L.mag_tensor_create_1d(self.ctx, 0, int(shape[0]))
        if len(shape) == 2:
            return self.L.mag_tensor_create_2d(self.ctx, 0, int(shape[0]), int(shape[1]))
        return self.tensor(pad6(shape))

    def read(self, t) -> np.ndarray:
        n = self.L.mag_tensor_numel(t)
        p = C.cast(self.L.mag_tensor_data_ptr(t), _f32p)
        return np.ctypeslib.as_array(p, shape=(n,)).copy()

    def write(self, t, a: np.ndarray):
        a = np.ascontiguousarray(a, np.float32)
        self.L.mag_tensor_copy_buffer_from(t, a.ctypes.data, a.nbytes)

    def op(self, name: str, *inputs, xi=None, inplace=False):
        arr = (C.c_void_p * len(inputs))(*inputs)
        params = None
        if xi is not None:
            pa = (C.c_uint64 * 6)(self.L.mag_op_param_float(xi), 0, 0, 0, 0, 0)
            params = C.cast(C.pointer(pa), C.c_void_p)
            self._live.append(pa)
        r = self.L.mag_tensor_operator(self.ctx, OP[name], inplace, arr, len(inputs), params)
        if not r:
            raise ValueError(f"reference rejected {name}")
        return r

    def free(self, *ts):
        for t in ts:
            self.L.mag_tensor_decref(t)

    def close(self):
        if self.ctx:
            self.L.mag_ctx_destroy(self.ctx)
            self.ctx = None


# ---------------------------------------------------------------------------- images
# numpy float32 restatements (every op separately rounded, as the reference's x86 build
# computes them) of the reference's image pixel work.

def img_load(src: np.ndarray, w: int, h: int, c: int, rw: int = 0, rh: int = 0) -> np.ndarray:
    """mag_tensor_load_image's conversion and bilinear resize (magnetron/magnetron.c:3013-3087)."""
    f = np.float32
    ori = (src.reshape(h, w, c).astype(f) / f(255.0)).transpose(2, 0, 1)  # planar [c][h][w]
    if not (rw and rh):
        return np.ascontiguousarray(ori).reshape(-1)
    with np.errstate(divide="ignore", invalid="ignore"):
        ws = f(w - 1) / f(rw - 1)
        hs = f(h - 1) / f(rh - 1)
    part = np.empty((c, h, rw), f)
    for cc in range(rw):
        if cc == rw - 1 or w == 1:
            part[:, :, cc] = ori[:, :, w - 1]
        else:
            sx = f(cc) * ws
            ix = int(sx)
            dx = sx - f(ix)
            part[:, :, cc] = (f(1) - dx) * ori[:, :, ix] + dx * ori[:, :, ix + 1]
    dst = np.empty((c, rh, rw), f)
    for r in range(rh):
        with np.errstate(invalid="ignore"):
            sy = f(r) * hs
        iy = 0 if np.isnan(sy) else int(sy)
        dy = sy - f(iy)
        dst[:, r, :] = (f(1) - dy) * part[:, iy, :]
        if not (r == rh - 1 or h == 1):
            dst[:, r, :] = dst[:, r, :] + dy * part[:, iy + 1, :]
    return dst.reshape(-1)


def img_save(x: np.ndarray, w: int, h: int, c: int) -> np.ndarray:
    """mag_tensor_save_image's conversion (magnetron/magnetron.c:3089-3109): (uint8_t)(x * 255)
    as x86-64 compiles it, truncation to int32 (INT32_MIN when out of range or NaN), low byte."""
    v = (x.astype(np.float32) * np.float32(255.0)).reshape(c, h * w)
    ok = (v >= -2147483648.0) & (v < 2147483648.0)
    q = np.where(ok, np.trunc(np.where(ok, v, 0)), -2147483648.0).astype(np.int64)
    return (q & 0xFF).astype(np.uint8).T.reshape(-1)


def img_draw_box(img: np.ndarray, w: int, h: int, x1, y1, x2, y2, wi, rgb) -> np.ndarray:
    """mag_tensor_img_draw_box (magnetron/magnetron.c:2159-2214) on planar RGB."""
    out = img.astype(np.float32).copy()
    col = [np.float32((rgb >> s) & 0xFF) / np.float32(255.0) for s in (16, 8, 0)]
    plane = w * h

    def put(x, y):
        o = x + y * w
        for k in range(3):
            out[o + k * plane] = col[k]
    for i in range(max(1, wi)):
        xx1, yy1, xx2, yy2 = min(x1 + i, w - 1), min(y1 + i, h - 1), min(x2 - i, w - 1), min(y2 - i, h - 1)
        for j in range(xx1, xx2 + 1):
            put(j, yy1)
            put(j, yy2)
        for j in range(yy1, yy2 + 1):
            put(xx1, j)
            put(xx2, j)
    return out
