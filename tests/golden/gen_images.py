"""Generate tests/golden/images.npz from the reference library's own image code.

Run from the repository root after `make -C oracle all ref`:

    python tests/golden/gen_images.py

A CPU context of the reference build (oracle/_ref/libmagnetron.so) is created with image
callbacks of this script (mag_ctx_info_t, magnetron/magnetron.h:85-98): the loader hands the
reference seeded interleaved u8 pixels, so mag_tensor_load_image runs its own conversion and
bilinear resize on them; the saver captures the u8 pixels mag_tensor_save_image produces.
Box and text drawing run mag_tensor_img_draw_box / mag_tensor_img_draw_text on CPU tensors.
Inputs and outputs are stored together.
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import REF_SO  # noqa: E402

LOAD_FN = C.CFUNCTYPE(C.c_void_p, C.c_char_p, C.POINTER(C.c_uint32 * 3), C.c_int)
FREE_FN = C.CFUNCTYPE(None, C.c_void_p)
SAVE_FN = C.CFUNCTYPE(C.c_bool, C.c_char_p, C.POINTER(C.c_uint8), C.POINTER(C.c_uint32 * 3))


class CtxInfo(C.Structure):
    _fields_ = [("device", C.c_int), ("pool_chunk_size", C.c_size_t), ("pool_chunks_cap", C.c_size_t),
                ("prng_seed", C.c_uint64), ("warmup_chunks", C.c_bool), ("prng_algorithm", C.c_int),
                ("exec_mode", C.c_int), ("image_load_fn", LOAD_FN), ("image_load_free_fn", FREE_FN),
                ("image_save_fn", SAVE_FN), ("user_data", C.c_void_p)]


# (w, h, c, rw, rh): no resize when rw = rh = 0
LOADS = [(7, 5, 3, 0, 0), (64, 48, 4, 0, 0), (33, 17, 1, 50, 40), (64, 48, 3, 20, 13), (1, 9, 3, 5, 4),
         (9, 1, 3, 4, 5), (10, 10, 3, 1, 6), (320, 240, 3, 112, 112), (6, 4, 1, 3, 1)]
SAVES = [(7, 5, 3), (16, 9, 1), (8, 8, 4)]
# (w, h, x1, y1, x2, y2, wi, rgb, random background)
BOXES = [(50, 40, 5, 5, 30, 20, 2, 0xFF8000, False), (50, 40, 10, 8, 1000, 1000, 3, 0x00FF7F, False),
         (50, 40, 3, 4, 12, 40, 20, 0x123456, False), (64, 32, 1, 1, 63, 31, 4, 0xFFFFFF, True),
         (20, 20, 2, 3, 9, 9, 0, 0x808080, True)]
# (w, h, x, y, rgb, text)
TEXTS = [(120, 40, 3, 2, 0xFFFFFF, "Hello, B200!\nline 2\ttab"), (40, 20, 30, 10, 0xFF0000, "clipped text"),
         (8 * 48 + 4, 14 * 3 + 2, 0, 0, 0x00FF00, "".join(chr(c) for c in range(33, 81)) + "\n" +
          "".join(chr(c) for c in range(81, 127)) + "\n\x01\x7f\xe9 ~")]


def main():
    L = C.CDLL(REF_SO)
    vp = C.c_void_p
    L.mag_ctx_create.argtypes = [C.POINTER(CtxInfo)]
    L.mag_ctx_create.restype = vp
    L.mag_ctx_destroy.argtypes = [vp]
    L.mag_tensor_load_image.argtypes = [vp, C.c_char_p, C.c_int, C.c_uint32, C.c_uint32]
    L.mag_tensor_load_image.restype = vp
    L.mag_tensor_save_image.argtypes = [vp, C.c_char_p]
    L.mag_tensor_create_3d.argtypes = [vp, C.c_int, C.c_int64, C.c_int64, C.c_int64]
    L.mag_tensor_create_3d.restype = vp
    L.mag_tensor_img_draw_box.argtypes = [vp] + [C.c_int32] * 5 + [C.c_uint32]
    L.mag_tensor_img_draw_text.argtypes = [vp, C.c_int32, C.c_int32, C.c_int32, C.c_uint32, C.c_char_p]
    L.mag_tensor_data_ptr.argtypes = [vp]
    L.mag_tensor_data_ptr.restype = vp
    L.mag_tensor_numel.argtypes = [vp]
    L.mag_tensor_numel.restype = C.c_int64
    L.mag_tensor_copy_buffer_from.argtypes = [vp, vp, C.c_size_t]
    L.mag_tensor_decref.argtypes = [vp]

    pending = {}
    captured = {}

    @LOAD_FN
    def load(path, whc, channels):
        buf, (w, h, c) = pending["img"]
        whc.contents[0], whc.contents[1], whc.contents[2] = w, h, c
        return buf.ctypes.data

    @FREE_FN
    def free(p):
        pass

    @SAVE_FN
    def save(path, data, whc):
        w, h, c = whc.contents[0], whc.contents[1], whc.contents[2]
        captured["u8"] = np.ctypeslib.as_array(data, shape=(w * h * c,)).copy()
        return True

    info = CtxInfo()
    info.image_load_fn, info.image_load_free_fn, info.image_save_fn = load, free, save
    ctx = L.mag_ctx_create(C.byref(info))

    def read(t):
        n = L.mag_tensor_numel(t)
        return np.ctypeslib.as_array(C.cast(L.mag_tensor_data_ptr(t), C.POINTER(C.c_float)), shape=(n,)).copy()

    out = {}
    for i, (w, h, c, rw, rh) in enumerate(LOADS):
        src = np.random.default_rng(100 + i).integers(0, 256, w * h * c, dtype=np.uint8)
        pending["img"] = (src, (w, h, c))
        t = L.mag_tensor_load_image(ctx, b"synthetic", 0, rw, rh)
        out[f"load{i}_src"] = src
        out[f"load{i}_out"] = read(t)
        L.mag_tensor_decref(t)
    for i, (w, h, c) in enumerate(SAVES):
        x = np.random.default_rng(200 + i).uniform(-0.5, 1.5, w * h * c).astype(np.float32)
        x[:8] = [np.nan, np.inf, -np.inf, 1e10, -1e10, 0.999, 1.0, 256.0 / 255.0]
        t = L.mag_tensor_create_3d(ctx, 0, c, h, w)
        L.mag_tensor_copy_buffer_from(t, x.ctypes.data, x.nbytes)
        L.mag_tensor_save_image(t, b"synthetic.png")
        out[f"save{i}_src"] = x
        out[f"save{i}_out"] = captured.pop("u8")
        L.mag_tensor_decref(t)
    for i, (w, h, x1, y1, x2, y2, wi, rgb, bg) in enumerate(BOXES):
        img = (np.random.default_rng(300 + i).uniform(0, 1, 3 * w * h) if bg else np.zeros(3 * w * h)).astype(np.float32)
        t = L.mag_tensor_create_3d(ctx, 0, 3, h, w)
        L.mag_tensor_copy_buffer_from(t, img.ctypes.data, img.nbytes)
        L.mag_tensor_img_draw_box(t, x1, y1, x2, y2, wi, rgb)
        out[f"box{i}_src"] = img
        out[f"box{i}_out"] = read(t)
        L.mag_tensor_decref(t)
    for i, (w, h, x, y, rgb, txt) in enumerate(TEXTS):
        t = L.mag_tensor_create_3d(ctx, 0, 3, h, w)
        L.mag_tensor_img_draw_text(t, x, y, 8, rgb, txt.encode("latin-1"))
        out[f"text{i}_out"] = read(t)
        L.mag_tensor_decref(t)
    L.mag_ctx_destroy(ctx)
    np.savez_compressed(os.path.join(HERE, "images.npz"), **out)


if __name__ == "__main__":
    main()
