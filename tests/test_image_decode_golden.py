"""JPEG decoding at the library boundary against the reference's decoder.

The reference decodes every input image with stb_image (src/image_io.cpp:26-35).
tests/golden/jpeg.npz holds seeded JPEG files in the flavours a caller may pass
(4:4:4 / 4:2:0 / 4:2:2 chroma, grayscale, progressive, restart markers, odd sizes)
with the RGB bytes the reference's stb_image (oracle/_ref/libstbimage.so, built
from the reference tree) produces for them (tests/golden/gen_jpeg_golden.py).
rfdetr_image_load_buffer must give the same bytes, so an image enters the
network with the reference's pixels.  Runs on the CPU (the decode is host code).
"""
import ctypes as C
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "tests", "golden"))
GOLDEN = os.path.join(REPO, "tests", "golden", "jpeg.npz")


def _load(data):
    from rfdetr_b200 import lib
    L = lib.lib()
    st = C.c_int(0)
    img = L.rfdetr_image_load_buffer(data.ctypes.data, data.size, C.byref(st))
    assert img and st.value == 0, st.value
    w, h = L.rfdetr_image_width(img), L.rfdetr_image_height(img)
    p = L.rfdetr_image_rgb_data(img)
    out = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_ubyte)), (h, w, 3)).copy()
    L.rfdetr_image_free(img)
    return out


def test_jpeg_pixels_are_the_reference_decoders():
    g = np.load(GOLDEN)
    names = [str(n) for n in g["names"]]
    assert len(names) == 8
    for name in names:
        got = _load(g[f"{name}_jpeg"])
        want = g[f"{name}_rgb"]
        assert got.shape == want.shape, name
        assert np.array_equal(got, want), (name, int(np.abs(got.astype(int) - want).max()))


def test_golden_vectors_are_the_reference_decode():
    import gen_jpeg_golden as gen

    if not os.path.exists(gen.REF_SO):
        pytest.skip("oracle/_ref/libstbimage.so is built only where the reference tree is present")
    g = np.load(GOLDEN)
    for name in (str(n) for n in g["names"]):
        assert np.array_equal(gen.stb_decode(g[f"{name}_jpeg"].tobytes()), g[f"{name}_rgb"]), name


def test_corrupt_jpeg_is_a_decode_error():
    from rfdetr_b200 import lib
    g = np.load(GOLDEN)
    data = g["q75_420_jpeg"].copy()
    L = lib.lib()
    st = C.c_int(0)
    for cut in (3, 64, data.size // 2):
        trunc = np.ascontiguousarray(data[:cut])
        img = L.rfdetr_image_load_buffer(trunc.ctypes.data, trunc.size, C.byref(st))
        if img:  # stb decodes a truncated scan as far as it goes, as the reference does
            L.rfdetr_image_free(img)
        else:
            assert st.value == -5  # RFDETR_ERR_DECODE
