"""Python host mirror of the magnetron core's tensor/operator layer over the
B200 backend's C ABI.

The magnetron core hands its CUDA device a ``mag_tensor_t`` per result and
calls ``eager_exec_fwd`` on it (magnetron/magnetron.c:1747-1789); tensors get
their buffers from ``alloc_storage`` and move data with the storage callbacks
(magnetron/magnetron.c:1653-1656, :1820-1830).  This module creates the same
structs with ctypes, so Python code (tests, the benchmark, users without the C
core) can drive ``libmagnetron_cuda.so`` through exactly the interface the
core uses:

    dev = Device()                       # mag_init_device_cuda
    x = dev.tensor((4096, 65536)); x.write(host_array)
    r = dev.op("SIGMOID", x)             # result ctor + eager_exec_fwd
    r.read()                             # storage.cpy_device_host

Shapes use the core's convention: dim 0 is the fastest (contiguous) dim, so a
row-major (rows, cols) array is shape (cols, rows).  MATMUL is the exception:
it reads its buffers as row-major [shape0][shape1] (magnetron/magnetron_cpu.c:2151-2185).

There is no fallback: if the CUDA library is missing or no sm_100 GPU is
present, constructing a Device raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmagnetron_cuda.so")

OPS = ["NOP", "CLONE", "VIEW", "TRANSPOSE", "PERMUTE", "MEAN", "MIN", "MAX", "SUM",
       "ABS", "NEG", "LOG", "SQR", "SQRT", "SIN", "COS", "STEP", "SOFTMAX", "SOFTMAX_DV",
       "SIGMOID", "SIGMOID_DV", "HARD_SIGMOID", "SILU", "SILU_DV", "TANH", "TANH_DV",
       "RELU", "RELU_DV", "GELU", "GELU_DV", "ADD", "SUB", "MUL", "DIV",
       "ADDS", "SUBS", "MULS", "DIVS", "MATMUL"]
OP = {n: i for i, n in enumerate(OPS)}
UNARY = set(OPS[OP["ABS"]:OP["GELU_DV"] + 1])
SCALAR = {"ADDS", "SUBS", "MULS", "DIVS"}
BINARY = {"ADD", "SUB", "MUL", "DIV"}
REDUCE = {"MEAN", "MIN", "MAX", "SUM"}
# ops whose result may alias the first input (mag_op_def inplace column, magnetron/magnetron.h:136-178)
INPLACE_OK = UNARY | SCALAR | BINARY | {"MATMUL"}
TFLAG_OWNER, TFLAG_VIEW = 1, 2

E_INVALID, E_DEVICE_WAIT, E_UNSUPPORTED, E_SCRATCH_LIMIT, E_IO = 10001, 10002, 10003, 10004, 10005
TC_SPLIT_TF32, TC_SPLIT_F16 = 0, 1  # mag_cuda_set_tc_split


# ---------------------------------------------------------------- ABI structs
class StorageBuffer(C.Structure):
    pass


SET_FN = C.CFUNCTYPE(None, C.POINTER(StorageBuffer), C.c_size_t, C.c_uint8)
H2D_FN = C.CFUNCTYPE(None, C.POINTER(StorageBuffer), C.c_size_t, C.c_void_p, C.c_size_t)
D2H_FN = C.CFUNCTYPE(None, C.POINTER(StorageBuffer), C.c_size_t, C.c_void_p, C.c_size_t)
StorageBuffer._fields_ = [
    ("base", C.c_uint64), ("size", C.c_size_t), ("alignment", C.c_size_t), ("host", C.c_void_p),
    ("set", SET_FN), ("cpy_host_device", H2D_FN), ("cpy_device_host", D2H_FN),
]

EXEC_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)
ALLOC_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(StorageBuffer), C.c_size_t, C.c_size_t)
FREE_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(StorageBuffer))


class ComputeDevice(C.Structure):
    _fields_ = [
        ("name", C.c_char * 128), ("impl", C.c_void_p), ("is_async", C.c_bool), ("type", C.c_int32),
        ("eager_exec_fwd", EXEC_FN), ("eager_exec_bwd", EXEC_FN),
        ("alloc_storage", ALLOC_FN), ("free_storage", FREE_FN),
    ]


class TensorT(C.Structure):
    _fields_ = [
        ("rc_strong", C.c_uint32), ("rc_weak", C.c_uint32), ("ctx", C.c_void_p), ("rank", C.c_int64),
        ("shape", C.c_int64 * 6), ("strides", C.c_int64 * 6), ("dtype", C.c_int32),
        ("storage", StorageBuffer), ("numel", C.c_int64), ("flags", C.c_int32), ("op", C.c_int32),
        ("op_inputs", C.c_void_p * 2), ("op_params", C.c_uint64 * 6), ("view_uplink", C.c_void_p),
        ("view_offs", C.c_size_t), ("grad", C.c_void_p), ("pmon", C.c_uint64 * 3),
        ("name", C.c_char * 64), ("ud", C.c_void_p),
    ]


assert C.sizeof(StorageBuffer) == 56 and C.sizeof(ComputeDevice) == 176 and C.sizeof(TensorT) == 384

_lib = None


def load_library(path: str = LIB_PATH):
    """Loads libmagnetron_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `make -C {HERE}` (no CPU fallback exists)")
    L = C.CDLL(path)
    vp, i64, f32p = C.c_void_p, C.c_int64, C.POINTER(C.c_float)
    i64p = C.POINTER(C.c_int64)
    sig = {
        "mag_init_device_cuda": ([vp], vp),
        "mag_destroy_device_cuda": ([vp], None),
        "mag_cuda_device_ordinal": ([vp], C.c_int),
        "mag_cuda_set_matmul_mode": ([vp, C.c_int], C.c_int),
        "mag_cuda_set_tc_split": ([vp, C.c_int], C.c_int),
        "mag_cuda_stream": ([vp], vp),
        "mag_cuda_synchronize": ([vp], C.c_int),
        "mag_cuda_last_error": ([vp], C.c_int),
        "mag_cuda_memory_in_use": ([vp], C.c_size_t),
        "mag_cuda_graph_exec": ([vp, vp], C.c_int),
        "mag_cuda_graph_exec_fused": ([vp, vp], C.c_int),
        "mag_cuda_graph_release": ([vp, vp], C.c_int),
        "mag_cuda_exec_node": ([vp, vp], C.c_int),
        "mag_cuda_unary_f32": ([vp, C.c_int, vp, vp, i64, i64, i64, i64, C.c_float], C.c_int),
        "mag_cuda_binary_f32": ([vp, C.c_int, vp, vp, vp, i64p, i64p, i64p, i64p, i64p], C.c_int),
        "mag_cuda_reduce_f32": ([vp, C.c_int, vp, vp, i64p, i64p], C.c_int),
        "mag_cuda_matmul_f32": ([vp, vp, vp, vp, i64, i64, i64], C.c_int),
        "mag_cuda_broadcast2_f32": ([vp, C.c_int, vp, vp, vp, i64p, i64p, i64p], C.c_int),
        "mag_cuda_reduce_rows_f32": ([vp, C.c_int, vp, vp, i64, i64], C.c_int),
        "mag_cuda_reduce_partial_f32": ([vp, vp, vp, i64p, i64p], C.c_int),
        "mag_cuda_reduce_combine_f32": ([vp, C.c_int, vp, vp, C.c_int], C.c_int),
        "mag_cuda_softmax_rows_f32": ([vp, vp, vp, i64, i64], C.c_int),
        "mag_cuda_matmul_batched_f32": ([vp, vp, vp, vp, i64, i64, i64, i64], C.c_int),
        "mag_cuda_profile_start": ([vp], C.c_int),
        "mag_cuda_profile_stop": ([vp, C.c_char_p], C.c_int),
        "mag_cuda_profile_collect": ([vp], C.c_int),
        "mag_cuda_profile_stats": ([vp, C.c_int, C.POINTER(C.c_uint64), C.POINTER(C.c_double)], C.c_int),
        "mag_cuda_kernel_launches": ([], C.c_uint64),
        "mag_cuda_matmul_skinny_f32_noalloc": ([vp, vp, vp, vp, i64, i64, i64], C.c_int),
        "mag_cuda_matmul_skinny_noalloc_limit": ([], C.c_size_t),
        "mag_cuda_fill_uniform_pcg_f32": ([vp, vp, i64, C.c_float, C.c_float, C.POINTER(C.c_uint64), C.c_uint64],
                                          C.c_int),
        "mag_cuda_fill_normal_pcg_f32": ([vp, vp, i64, C.c_float, C.c_float, C.POINTER(C.c_uint64), C.c_uint64],
                                         C.c_int),
        "mag_cuda_fill_f32": ([vp, vp, i64, C.c_float], C.c_int),
        "mag_cuda_fill_uniform_mt19937_f32": ([vp, vp, i64, C.c_float, C.c_float, C.POINTER(MtState)], C.c_int),
        "mag_cuda_fill_normal_mt19937_f32": ([vp, vp, i64, C.c_float, C.c_float, C.POINTER(MtState)], C.c_int),
        "mag_cuda_mt19937_jump": ([C.POINTER(C.c_uint32), C.c_uint64, C.POINTER(C.c_uint32)], C.c_int),
        "mag_cuda_mt19937_degree": ([], C.c_int),
        "mag_cuda_tensor_upload_async": ([vp, vp, vp, C.c_size_t], C.c_int),
        "mag_cuda_tensor_download_async": ([vp, vp, vp, C.c_size_t], C.c_int),
        "mag_cuda_copies_synchronize": ([vp], C.c_int),
        "mag_cuda_sto_parse": ([vp, C.c_size_t, C.c_size_t, vp, C.c_uint32, C.POINTER(C.c_uint32),
                                C.POINTER(C.c_uint32)], C.c_int),
        "mag_cuda_sto_write_header": ([vp, C.c_uint32, vp, C.c_size_t, C.POINTER(C.c_size_t)], C.c_int),
        "mag_cuda_tensor_save": ([vp, C.c_char_p, vp, C.c_uint32], C.c_int),
        "mag_cuda_sto_read_directory": ([C.c_char_p, vp, C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)],
                                        C.c_int),
        "mag_cuda_tensor_load": ([vp, C.c_char_p, vp, C.c_uint32], C.c_int),
        "mag_cuda_img_from_u8": ([vp, vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32], C.c_int),
        "mag_cuda_img_to_u8": ([vp, vp, vp], C.c_int),
        "mag_cuda_img_draw_box": ([vp, vp] + [C.c_int32] * 5 + [C.c_uint32], C.c_int),
        "mag_cuda_img_draw_text": ([vp, vp, C.c_int32, C.c_int32, C.c_int32, C.c_uint32, C.c_char_p], C.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


class ReducePart(C.Structure):
    """mag_cuda_reduce_part: one shard's full-reduction record (24 bytes)."""
    _fields_ = [("sum", C.c_double), ("min", C.c_float), ("max", C.c_float), ("count", C.c_uint64)]


REDUCE_PART_BYTES = C.sizeof(ReducePart)


class StoEntry(C.Structure):
    """mag_cuda_sto_entry: one tensor of a .magnetron file's directory."""
    _fields_ = [("name", C.c_char * 64), ("flags", C.c_uint32), ("dtype", C.c_uint32), ("rank", C.c_int64),
                ("shape", C.c_int64 * 6), ("offset", C.c_uint64), ("bytes", C.c_uint64)]

    @property
    def dims(self):
        return tuple(int(self.shape[i]) for i in range(int(self.rank)))


def sto_parse(buf: bytes, total: int | None = None):
    """The reader's header checks over a .magnetron image (no GPU needed).
    Returns (version, entries) or raises CudaError with the library's code."""
    L = load_library()
    total = len(buf) if total is None else total
    n, ver = C.c_uint32(0), C.c_uint32(0)
    cap = 64
    ents = (StoEntry * cap)()
    check(L.mag_cuda_sto_parse(buf, len(buf), total, ents, cap, C.byref(n), C.byref(ver)), "sto_parse")
    return int(ver.value), list(ents[:min(cap, n.value)])


def sto_header(tensors) -> bytes:
    """Header bytes the writer emits for these tensors (no GPU needed)."""
    L = load_library()
    arr = (C.c_void_p * len(tensors))(*[t.ptr for t in tensors])
    size = C.c_size_t(0)
    check(L.mag_cuda_sto_write_header(arr, len(tensors), None, 0, C.byref(size)), "sto_write_header")
    out = C.create_string_buffer(size.value)
    check(L.mag_cuda_sto_write_header(arr, len(tensors), out, size.value, C.byref(size)), "sto_write_header")
    return out.raw[:size.value]


class Pcg:
    """A context's PCG stream: mag_prng_init, PCG branch (magnetron/magnetron.c:797-808).
    Fills draw from it in order and advance it, as the reference context's generator does."""

    def __init__(self, seed: int):
        seed &= (1 << 64) - 1
        if not seed:  # the reference derives a default seed from the context's address
            seed = 0x853C49E6748FEA9B ^ id(self)
        self.state = C.c_uint64(seed ^ 0x853C49E6748FEA9B)
        self.inc = 0xDA3E39CB94B95BDB


class MtState(C.Structure):
    """A context's Mersenne-twister state (magnetron/magnetron_internal.h:398-402)."""
    _fields_ = [("remaining", C.c_uint32), ("next", C.c_uint32), ("state", C.c_uint32 * 624)]


class Mt19937:
    """A context's Mersenne-twister stream, the reference's default generator: mag_prng_init,
    Mersenne-twister branch (magnetron/magnetron.c:797-805).  Fills draw from it in order and
    leave it as the reference context's generator would."""

    def __init__(self, seed: int):
        seed &= (1 << 64) - 1
        if not seed:  # the reference derives a default seed from the context's address
            seed = 0x853C49E6748FEA9B ^ id(self)
        self.st = MtState()
        w = seed & 0xFFFFFFFF
        self.st.state[0] = w
        for i in range(1, 624):
            w = ((w ^ (w >> 30)) * 1812433253 + i) & 0xFFFFFFFF
            self.st.state[i] = w
        self.st.next = 0
        self.st.remaining = 1


def i64x6(v) -> C.Array:
    return (C.c_int64 * 6)(*[int(t) for t in v])


def pad6(shape):
    shape = [int(s) for s in shape]
    return shape + [1] * (6 - len(shape))


def strides6(shape6):
    s = [1] * 6
    for i in range(1, 6):
        s[i] = s[i - 1] * int(shape6[i - 1])
    return s


def f32_param(x: float) -> int:
    return int(np.array([x], np.float32).view(np.uint32)[0])  # tag 0 = float (magnetron/magnetron.c:1126-1130)


class CudaError(RuntimeError):
    pass


def check(rc: int, what: str):
    if rc:
        raise CudaError(f"{what} failed with code {rc}")


# ------------------------------------------------------------------- tensors
class Tensor:
    """One ``mag_tensor_t`` owned by Python, with storage from the device."""

    def __init__(self, dev: "Device", shape, view_of: "Tensor | None" = None):
        self.dev = dev
        self.t = TensorT()
        self.inputs = []
        shape6 = pad6(shape)
        rank = len(shape)
        t = self.t
        t.rc_strong = 1
        t.rank = rank
        for i in range(6):
            t.shape[i] = shape6[i]
        for i, s in enumerate(strides6(shape6)):
            t.strides[i] = s
        t.dtype = 0
        t.numel = int(np.prod(shape6))
        t.op = 0
        self.base = view_of.base if view_of is not None and view_of.base is not None else view_of
        if view_of is not None:  # share the viewed tensor's storage (magnetron/magnetron.c:1654-1655)
            t.flags = TFLAG_VIEW
            t.storage = view_of.t.storage
            t.view_uplink = C.addressof(view_of.t)
            self.owner = False
        else:
            t.flags = TFLAG_OWNER
            dev.dev.alloc_storage(dev.p, C.byref(t.storage), t.numel * 4, 4)
            self.owner = True

    @property
    def ptr(self) -> int:
        return C.addressof(self.t)

    @property
    def data_ptr(self) -> int:
        return int(self.t.storage.base)

    @property
    def name(self) -> str:
        return self.t.name.decode()

    @name.setter
    def name(self, v: str):  # mag_tensor_set_name: strncpy into 64 bytes, NUL at [63] (magnetron/magnetron.c:1968-1971)
        raw = v.encode()[:63]
        C.memset(C.addressof(self.t) + TensorT.name.offset, 0, 64)
        C.memmove(C.addressof(self.t) + TensorT.name.offset, raw, len(raw))

    @property
    def shape(self):
        return tuple(int(self.t.shape[i]) for i in range(int(self.t.rank)))

    @property
    def numel(self) -> int:
        return int(self.t.numel)

    def write(self, a: np.ndarray, offset_elems: int = 0):
        a = np.ascontiguousarray(a, np.float32)
        st = self.t.storage
        st.cpy_host_device(C.byref(self.t.storage), offset_elems * 4, a.ctypes.data, a.nbytes)

    def read(self, n: int | None = None) -> np.ndarray:
        n = self.numel if n is None else n
        out = np.empty(n, np.float32)
        st = self.t.storage
        st.cpy_device_host(C.byref(self.t.storage), 0, out.ctypes.data, out.nbytes)
        return out

    def fill_zero(self):
        st = self.t.storage
        st.set(C.byref(self.t.storage), 0, 0)

    def free(self):
        if getattr(self, "owner", False) and self.t.storage.base:
            self.dev.dev.free_storage(self.dev.p, C.byref(self.t.storage))
        self.owner = False

    def __del__(self):
        try:
            if self.dev.alive:
                self.free()
        except Exception:
            pass


class Device:
    """The CUDA compute device, created through mag_init_device_cuda."""

    def __init__(self):
        L = load_library()
        p = L.mag_init_device_cuda(None)
        if not p:
            raise CudaError("mag_init_device_cuda returned NULL: no usable sm_100 GPU")
        self.L = L
        self.p = p
        self.dev = C.cast(p, C.POINTER(ComputeDevice)).contents
        self.alive = True
        self.eager = True

    @property
    def name(self) -> str:
        return self.dev.name.decode()

    @property
    def stream(self) -> int:
        return int(self.L.mag_cuda_stream(self.p) or 0)

    @property
    def ordinal(self) -> int:
        return int(self.L.mag_cuda_device_ordinal(self.p))

    def sync(self):
        check(self.L.mag_cuda_synchronize(self.p), "synchronize")

    def close(self):
        if self.alive:
            self.sync()
            self.alive = False
            self.L.mag_destroy_device_cuda(self.p)

    def tensor(self, shape) -> Tensor:
        return Tensor(self, shape)

    def from_numpy(self, a: np.ndarray, shape=None) -> Tensor:
        t = Tensor(self, shape if shape is not None else a.shape[::-1])
        t.write(a.reshape(-1))
        return t

    # ---- the core's result constructors + eager execution (magnetron/magnetron.c:1447-1588, :1762-1789)
    def op(self, name: str, *inputs: Tensor, xi: float | None = None, inplace: bool = False) -> Tensor:
        x = inputs[0]
        if inplace and name in INPLACE_OK:
            r = Tensor(self, x.shape, view_of=x)
        elif name in REDUCE:
            r = Tensor(self, [1] + list(pad6(x.shape)[1:]))
        elif name == "MATMUL":
            r = Tensor(self, (x.t.shape[0], inputs[1].t.shape[1]))
        elif name == "CLONE" or name in UNARY or name in SCALAR or name in BINARY:
            r = Tensor(self, x.shape)
        else:
            raise ValueError(name)
        if name in BINARY:
            y = inputs[1]
            if any(int(x.t.shape[i]) % int(y.t.shape[i]) for i in range(6)):
                raise ValueError(f"{name}: shapes are not broadcastable (magnetron/magnetron.c:1266-1300)")
        r.t.op = OP[name]
        for i, t in enumerate(inputs):
            r.t.op_inputs[i] = t.ptr
        r.inputs = list(inputs)
        if xi is not None:
            r.t.op_params[0] = f32_param(xi)
        if self.eager:
            self.exec(r)
        return r

    def exec(self, r: Tensor):
        self.dev.eager_exec_fwd(self.p, r.ptr)

    # ---- sharded full reductions (one record per shard, combined in shard order)
    def reduce_partial(self, x: Tensor, part_ptr: int):
        """Writes x's record (double sum, min, max, count) to device memory at part_ptr."""
        d = (C.c_int64 * 6)(*[int(v) for v in x.t.shape])
        s = (C.c_int64 * 6)(*[int(v) for v in x.t.strides])
        check(self.L.mag_cuda_reduce_partial_f32(self.p, part_ptr, x.data_ptr, d, s), "reduce_partial")

    def reduce_combine(self, name: str, r_ptr: int, parts_ptr: int, nparts: int):
        """r[0] = SUM/MEAN/MIN/MAX over nparts records at parts_ptr, in record order."""
        check(self.L.mag_cuda_reduce_combine_f32(self.p, OP[name], r_ptr, parts_ptr, nparts), "reduce_combine")

    # ---- .magnetron storage (mag_tensor_save / mag_tensor_load, magnetron/magnetron.c:2931-2977)
    def save(self, path: str, tensors):
        arr = (C.c_void_p * len(tensors))(*[t.ptr for t in tensors])
        check(self.L.mag_cuda_tensor_save(self.p, path.encode(), arr, len(tensors)), "tensor_save")

    def read_directory(self, path: str):
        n, ver = C.c_uint32(0), C.c_uint32(0)
        check(self.L.mag_cuda_sto_read_directory(path.encode(), None, 0, C.byref(n), C.byref(ver)), "read_directory")
        ents = (StoEntry * max(1, n.value))()
        check(self.L.mag_cuda_sto_read_directory(path.encode(), ents, n.value, C.byref(n), C.byref(ver)),
              "read_directory")
        return list(ents[:n.value])

    def load(self, path: str):
        """Every tensor of the file, as new device tensors named and flagged from the file."""
        ts = [self.tensor(e.dims) for e in self.read_directory(path)]
        arr = (C.c_void_p * len(ts))(*[t.ptr for t in ts])
        check(self.L.mag_cuda_tensor_load(self.p, path.encode(), arr, len(ts)), "tensor_load")
        return ts

    # ---- image tensors (c, h, w) (magnetron/magnetron.c:2159-2274, 3013-3109, pixel work on the device)
    def image_from_u8(self, src: np.ndarray, w: int, h: int, c: int, rw: int = 0, rh: int = 0) -> Tensor:
        src = np.ascontiguousarray(src, np.uint8)
        t = self.tensor((c, rh, rw) if rw and rh else (c, h, w))
        check(self.L.mag_cuda_img_from_u8(self.p, t.ptr, src.ctypes.data, w, h, c, rw, rh), "img_from_u8")
        return t

    def image_to_u8(self, t: Tensor) -> np.ndarray:
        out = np.empty(t.numel, np.uint8)
        check(self.L.mag_cuda_img_to_u8(self.p, t.ptr, out.ctypes.data), "img_to_u8")
        return out

    def draw_box(self, t: Tensor, x1: int, y1: int, x2: int, y2: int, wi: int, rgb: int):
        check(self.L.mag_cuda_img_draw_box(self.p, t.ptr, x1, y1, x2, y2, wi, rgb), "img_draw_box")

    def draw_text(self, t: Tensor, x: int, y: int, size: int, rgb: int, txt: str):
        check(self.L.mag_cuda_img_draw_text(self.p, t.ptr, x, y, size, rgb, txt.encode("latin-1")), "img_draw_text")

    # ---- asynchronous host copies (pinned host memory; ordered against the compute stream)
    def upload_async(self, t: Tensor, host_ptr: int, nbytes: int):
        check(self.L.mag_cuda_tensor_upload_async(self.p, t.ptr, host_ptr, nbytes), "tensor_upload_async")

    def download_async(self, t: Tensor, host_ptr: int, nbytes: int):
        check(self.L.mag_cuda_tensor_download_async(self.p, t.ptr, host_ptr, nbytes), "tensor_download_async")

    def copies_sync(self):
        check(self.L.mag_cuda_copies_synchronize(self.p), "copies_synchronize")

    # ---- seeded fills (mag_tensor_fill*, magnetron/magnetron.c:1826-1876, on the device)
    def fill(self, t: Tensor, x: float):
        check(self.L.mag_cuda_fill_f32(self.p, t.data_ptr, t.numel, x), "fill")

    def fill_random_uniform(self, t: Tensor, lo: float, hi: float, gen: "Pcg | Mt19937"):
        if isinstance(gen, Mt19937):
            rc = self.L.mag_cuda_fill_uniform_mt19937_f32(self.p, t.data_ptr, t.numel, lo, hi, C.byref(gen.st))
        else:
            rc = self.L.mag_cuda_fill_uniform_pcg_f32(self.p, t.data_ptr, t.numel, lo, hi, C.byref(gen.state), gen.inc)
        check(rc, "fill_random_uniform")

    def fill_random_normal(self, t: Tensor, mean: float, std: float, gen: "Pcg | Mt19937"):
        if isinstance(gen, Mt19937):
            rc = self.L.mag_cuda_fill_normal_mt19937_f32(self.p, t.data_ptr, t.numel, mean, std, C.byref(gen.st))
        else:
            rc = self.L.mag_cuda_fill_normal_pcg_f32(self.p, t.data_ptr, t.numel, mean, std, C.byref(gen.state),
                                                     gen.inc)
        check(rc, "fill_random_normal")

    def graph_exec(self, root: Tensor, fused: bool = False):
        fn = self.L.mag_cuda_graph_exec_fused if fused else self.L.mag_cuda_graph_exec
        check(fn(self.p, root.ptr), "graph_exec")

    def graph_release(self, root: Tensor):
        self.L.mag_cuda_graph_release(self.p, root.ptr)

    def launches(self) -> int:
        return int(self.L.mag_cuda_kernel_launches())

    # ---- per-op device timing
    def profile_start(self):
        check(self.L.mag_cuda_profile_start(self.p), "profile_start")

    def profile_collect(self):
        check(self.L.mag_cuda_profile_collect(self.p), "profile_collect")

    def profile_stats(self, op: str):
        n, us = C.c_uint64(0), C.c_double(0.0)
        check(self.L.mag_cuda_profile_stats(self.p, OP[op], C.byref(n), C.byref(us)), "profile_stats")
        return int(n.value), float(us.value)

    def profile_stop(self, csv_path: str | None = None):
        check(self.L.mag_cuda_profile_stop(self.p, csv_path.encode() if csv_path else None), "profile_stop")
