"""Device image pixel work against outputs of the reference's own image code
(tests/golden/images.npz): conversion, resize, save conversion, box and text drawing,
all bit-identical."""
import os
import sys

import numpy as np
import pytest

import mag_b200 as MB
from gpu_util import device

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import gen_images as G  # noqa: E402

Z = np.load(os.path.join(HERE, "golden", "images.npz"))


def same(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(np.isnan(a), np.isnan(b)) and \
        np.array_equal(a[~np.isnan(a)].view(np.uint32), b[~np.isnan(b)].view(np.uint32))


@pytest.mark.parametrize("i", range(len(G.LOADS)))
def test_image_from_u8(i):
    dev = device()
    w, h, c, rw, rh = G.LOADS[i]
    t = dev.image_from_u8(Z[f"load{i}_src"], w, h, c, rw, rh)
    assert same(t.read(), Z[f"load{i}_out"])


def test_image_from_u8_device_source():
    import torch
    dev = device()
    w, h, c, rw, rh = G.LOADS[3]
    src = torch.from_numpy(Z["load3_src"]).to(f"cuda:{dev.L.mag_cuda_device_ordinal(dev.p)}")
    torch.cuda.synchronize()
    t = dev.tensor((c, rh, rw))
    MB.check(dev.L.mag_cuda_img_from_u8(dev.p, t.ptr, src.data_ptr(), w, h, c, rw, rh), "img_from_u8")
    assert same(t.read(), Z["load3_out"])


@pytest.mark.parametrize("i", range(len(G.SAVES)))
def test_image_to_u8(i):
    dev = device()
    w, h, c = G.SAVES[i]
    t = dev.tensor((c, h, w))
    t.write(Z[f"save{i}_src"])
    assert np.array_equal(dev.image_to_u8(t), Z[f"save{i}_out"])


@pytest.mark.parametrize("i", range(len(G.BOXES)))
def test_draw_box(i):
    dev = device()
    w, h, x1, y1, x2, y2, wi, rgb, bg = G.BOXES[i]
    t = dev.tensor((3, h, w))
    if bg:
        t.write(Z[f"box{i}_src"])
    dev.draw_box(t, x1, y1, x2, y2, wi, rgb)
    assert np.array_equal(t.read(), Z[f"box{i}_out"])


@pytest.mark.parametrize("i", range(len(G.TEXTS)))
def test_draw_text(i):
    dev = device()
    w, h, x, y, rgb, txt = G.TEXTS[i]
    t = dev.tensor((3, h, w))
    dev.draw_text(t, x, y, 8, rgb, txt)
    assert np.array_equal(t.read(), Z[f"text{i}_out"])


def test_image_argument_checks():
    dev = device()
    t = dev.tensor((3, 10, 10))
    assert dev.L.mag_cuda_img_draw_box(dev.p, t.ptr, 0, 1, 5, 5, 1, 0) == MB.E_INVALID  # x1 > 0 (:2161)
    assert dev.L.mag_cuda_img_draw_box(dev.p, t.ptr, 5, 1, 5, 5, 1, 0) == MB.E_INVALID  # x2 > x1
    assert dev.L.mag_cuda_img_draw_text(dev.p, t.ptr, 0, 0, 7, 0, b"a") == MB.E_INVALID  # size >= 8
    g = dev.tensor((1, 10, 10))
    assert dev.L.mag_cuda_img_draw_text(dev.p, g.ptr, 0, 0, 8, 0, b"a") == MB.E_INVALID  # 3 channels
    src = np.zeros(10 * 10 * 3, np.uint8)
    assert dev.L.mag_cuda_img_from_u8(dev.p, t.ptr, src.ctypes.data, 10, 10, 3, 5, 5) == MB.E_INVALID  # dst shape
