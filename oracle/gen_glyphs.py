"""Recipe: extract the reference font's glyph shapes into the backend's glyph table.

The reference draws text with a 7 x 14 bitmap font (mag_glyph, magnetron/magnetron.c:2216-2242)
for the 94 printable ASCII characters 33..126.  Pixel-identical text on the device needs the
same shapes, so this renders every glyph through the reference build itself
(oracle/_ref/libmagnetron.so, mag_tensor_img_draw_text on a CPU image) and writes the set
pixels as one 7-bit row mask per glyph row (bit x-1 = column x of the 8-column cell) to
magnetron-pre-oss-release-old_b200/csrc/mcu_glyphs.cuh.  Run once from the repository root
after `make -C oracle ref`:

    python oracle/gen_glyphs.py
"""
import ctypes as C
import os

import numpy as np

from oracle import RefLib

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "..", "magnetron-pre-oss-release-old_b200", "csrc", "mcu_glyphs.cuh")


def main():
    R = RefLib()
    L = R.L
    L.mag_tensor_create_3d.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_int64]
    L.mag_tensor_create_3d.restype = C.c_void_p
    L.mag_tensor_img_draw_text.argtypes = [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_uint32, C.c_char_p]
    rows = []
    for code in range(33, 127):
        t = L.mag_tensor_create_3d(R.ctx, 0, 3, 14, 8)  # (c, h, w)
        L.mag_tensor_img_draw_text(t, 0, 0, 8, 0xFFFFFF, bytes([code]))
        red = R.read(t)[: 14 * 8].reshape(14, 8)
        assert not red[:, 0].any()
        for yy in range(14):
            rows.append(sum(1 << (xx - 1) for xx in range(1, 8) if red[yy, xx] != 0))
        R.free(t)
    R.close()
    body = ",\n".join("    " + ", ".join(f"0x{v:02x}" for v in rows[g * 14:(g + 1) * 14]) for g in range(94))
    with open(OUT, "w") as f:
        f.write("// Glyph shapes of the reference's text font (magnetron/magnetron.c:2216-2242), ASCII 33..126:\n"
                "// 14 rows per glyph, bit x-1 of a row = pixel column x of the glyph's 8-column cell\n"
                "// (column 0 is never set).  Extracted by rendering each glyph with the reference\n"
                "// (oracle/gen_glyphs.py); text drawn on the device is pixel-identical with it.\n"
                "#pragma once\n#include <stdint.h>\n\n"
                f"__constant__ uint8_t mcu_glyph_rows[94 * 14] = {{\n{body}}};\n")


if __name__ == "__main__":
    main()
