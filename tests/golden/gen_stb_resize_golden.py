"""Generate tests/golden/stb_resize.npz from the reference's legacy resize.

The reference resizes images for models whose rfdetr.preprocess.resize_mode is
legacy_stb (or absent) with stb_image_resize2's stbir_resize_uint8_linear
(src/image_io.cpp:249-275).  oracle/_ref/libstbresize.so is that library built
from the header in the reference tree (`make -C oracle ref`); this script runs
it on seeded images and stores the resized bytes.  The inputs are not stored:
image i of a case is np.random.default_rng(seed).integers(0, 256, (h, w, 3)).

Run from the repository root:  python tests/golden/gen_stb_resize_golden.py
"""
import ctypes as C
import os

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_SO = os.path.join(REPO, "oracle", "_ref", "libstbresize.so")
OUT = os.path.join(REPO, "tests", "golden", "stb_resize.npz")

# (seed, w, h, out_w, out_h): both axes shrinking, both growing, mixed, one axis kept, a 2:1
# (rational, polyphase) shrink, a tall image, a detector-size shrink and a 3 x 3 source
CASES = [(11, 90, 70, 64, 64), (12, 40, 30, 64, 64), (13, 100, 50, 64, 64), (14, 64, 40, 64, 64),
         (15, 128, 128, 64, 64), (16, 37, 300, 96, 96), (17, 333, 201, 112, 112), (18, 3, 3, 64, 64)]


def source(seed, w, h):
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


def stb_resize(img, ow, oh):
    lib = C.CDLL(REF_SO)
    lib.stb_resize_rgb.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int]
    img = np.ascontiguousarray(img)
    out = np.zeros((oh, ow, 3), np.uint8)
    assert lib.stb_resize_rgb(img.ctypes.data, img.shape[1], img.shape[0], out.ctypes.data, ow, oh) == 1
    return out


def main():
    arrays = {}
    for seed, w, h, ow, oh in CASES:
        arrays[f"case_{seed}"] = stb_resize(source(seed, w, h), ow, oh)
    np.savez_compressed(OUT, cases=np.array(CASES, np.int32), **arrays)
    print(f"wrote {OUT}: {len(CASES)} cases")


if __name__ == "__main__":
    main()
