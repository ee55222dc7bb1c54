"""Generate tests/golden/jpeg.npz: seeded JPEG files and their pixels as the
reference decodes them.

The reference decodes every input image with stb_image (src/image_io.cpp:26-35,
stbi_load_from_memory forcing three channels).  oracle/_ref/libstbimage.so is that
decoder built from the header in the reference tree (`make -C oracle ref`); this
script encodes seeded images with PIL in the JPEG flavours a caller may pass
(4:4:4, 4:2:0 and 4:2:2 chroma subsampling, grayscale, progressive, restart
markers, odd sizes) and stores each file with the reference decoder's RGB bytes.

Run from the repository root:  python tests/golden/gen_jpeg_golden.py
"""
import ctypes as C
import io
import os

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_SO = os.path.join(REPO, "oracle", "_ref", "libstbimage.so")
OUT = os.path.join(REPO, "tests", "golden", "jpeg.npz")

# (name, seed, width, height, PIL save options, grayscale)
CASES = [
    ("q90_444", 31, 64, 48, {"quality": 90, "subsampling": 0}, False),
    ("q75_420", 32, 64, 48, {"quality": 75, "subsampling": 2}, False),
    ("q85_422", 33, 48, 40, {"quality": 85, "subsampling": 1}, False),
    ("odd_420", 34, 37, 23, {"quality": 80, "subsampling": 2}, False),
    ("gray", 35, 40, 33, {"quality": 85}, True),
    ("progressive_420", 36, 56, 40, {"quality": 80, "subsampling": 2, "progressive": True}, False),
    ("progressive_444", 37, 33, 31, {"quality": 92, "subsampling": 0, "progressive": True}, False),
    ("restart_420", 38, 64, 32, {"quality": 70, "subsampling": 2, "restart_marker_blocks": 2}, False),
]


def source(seed, w, h, gray):
    """Smooth gradients plus noise: chroma and luma detail at every frequency."""
    rng = np.random.default_rng(seed)
    yy, xx = np.mgrid[0:h, 0:w].astype(np.float64)
    base = np.stack([128 + 100 * np.sin(xx / (3 + c) + yy / (5 + 2 * c) + c) for c in range(3)], -1)
    img = np.clip(base + rng.normal(0, 25, (h, w, 3)), 0, 255).astype(np.uint8)
    return img[..., 0] if gray else img


def encode(img, opts):
    from PIL import Image
    buf = io.BytesIO()
    Image.fromarray(img).save(buf, format="JPEG", **opts)
    return buf.getvalue()


def stb_decode(data):
    L = C.CDLL(REF_SO)
    L.ref_stbi_load_rgb.restype = C.POINTER(C.c_ubyte)
    L.ref_stbi_load_rgb.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.ref_stbi_free.argtypes = [C.POINTER(C.c_ubyte)]
    w, h = C.c_int(0), C.c_int(0)
    p = L.ref_stbi_load_rgb(data, len(data), C.byref(w), C.byref(h))
    if not p:
        raise RuntimeError("stb_image could not decode the file")
    out = np.ctypeslib.as_array(p, (h.value, w.value, 3)).copy()
    L.ref_stbi_free(p)
    return out


def main():
    if not os.path.exists(REF_SO):
        raise SystemExit("oracle/_ref/libstbimage.so is missing: make -C oracle ref REF_STB=<tree>/third_party/stb")
    arrays = {}
    for name, seed, w, h, opts, gray in CASES:
        data = encode(source(seed, w, h, gray), opts)
        arrays[f"{name}_jpeg"] = np.frombuffer(data, np.uint8)
        arrays[f"{name}_rgb"] = stb_decode(data)
    np.savez_compressed(OUT, names=np.array([c[0] for c in CASES]), **arrays)
    print(f"wrote {OUT}: {len(CASES)} files")


if __name__ == "__main__":
    main()
