"""Image pixel work on the CPU: the oracle's numpy restatement and the backend's glyph table
against outputs of the reference's own image code (tests/golden/images.npz, made by
tests/golden/gen_images.py through the reference build with image callbacks)."""
import os
import re
import sys

import numpy as np
import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import gen_images as G  # noqa: E402

Z = np.load(os.path.join(HERE, "golden", "images.npz"))
GLYPHS = os.path.join(HERE, "..", "magnetron-pre-oss-release-old_b200", "csrc", "mcu_glyphs.cuh")


def same(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(np.isnan(a), np.isnan(b)) and \
        np.array_equal(a[~np.isnan(a)].view(np.uint32), b[~np.isnan(b)].view(np.uint32))


@pytest.mark.parametrize("i", range(len(G.LOADS)))
def test_load_conversion_and_resize(i):
    w, h, c, rw, rh = G.LOADS[i]
    assert same(O.img_load(Z[f"load{i}_src"], w, h, c, rw, rh), Z[f"load{i}_out"])


@pytest.mark.parametrize("i", range(len(G.SAVES)))
def test_save_conversion(i):
    w, h, c = G.SAVES[i]
    assert np.array_equal(O.img_save(Z[f"save{i}_src"], w, h, c), Z[f"save{i}_out"])


@pytest.mark.parametrize("i", range(len(G.BOXES)))
def test_draw_box(i):
    w, h, x1, y1, x2, y2, wi, rgb, _ = G.BOXES[i]
    assert np.array_equal(O.img_draw_box(Z[f"box{i}_src"], w, h, x1, y1, x2, y2, wi, rgb), Z[f"box{i}_out"])


@pytest.mark.parametrize("i", range(len(G.TEXTS)))
def test_glyph_table_reproduces_reference_text(i):
    """The device's glyph table, blitted the way the device kernel places glyphs, gives the
    reference's text pixels."""
    rows = [int(v, 16) for v in re.findall(r"0x([0-9a-f]{2})", open(GLYPHS).read())]
    assert len(rows) == 94 * 14
    w, h, x, y, rgb, txt = G.TEXTS[i]
    img = np.zeros((3, h, w), np.float32)
    col = [np.float32((rgb >> s) & 0xFF) / np.float32(255.0) for s in (16, 8, 0)]
    lx, ly = x, y
    for ch in txt.encode("latin-1"):
        if 32 < ch < 127:
            for yy in range(14):
                for xx in range(1, 8):
                    if (rows[(ch - 33) * 14 + yy] >> (xx - 1)) & 1 and lx + xx < w and ly + yy < h:
                        img[:, ly + yy, lx + xx] = col
        lx, ly = (x, ly + 14) if ch == 10 else (lx + 8, ly)
    assert np.array_equal(img.reshape(-1), Z[f"text{i}_out"])
