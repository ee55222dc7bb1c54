"""Generate tests/golden/host_ref.npz from the reference's own host-side code.

oracle/_ref/librefhost.so is the reference's src/image_io.cpp and
src/postprocess.cpp (with src/common.cpp and src/visualize.cpp, which they call)
built from the reference tree (`make -C oracle ref REF_ROOT=<reference>`).  This
script runs, on seeded inputs:

* rfdetr_preprocess (src/image_io.cpp:184-248, the RF-DETR 1.9 bilinear path):
  the SHA-256 of each normalized float32 plane set [3][th][tw] is stored;
* rfdetr_select_detections_with_masks (src/postprocess.cpp:43-276): the records
  (class id, score and box as float32 bit patterns) in the reference's order, and
  the 0/255 masks of the mask cases.

The inputs are not stored: they are regenerated from their seeds by the
functions below, which the tests import.  The selection sorts with std::sort on
the score alone, so records of equal score may come in any order; the cases are
chosen so that top_k never cuts a run of equal scores (checked here).

Run from the repository root:  python tests/golden/gen_host_ref_golden.py
"""
import ctypes as C
import hashlib
import os

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_SO = os.path.join(REPO, "oracle", "_ref", "librefhost.so")
OUT = os.path.join(REPO, "tests", "golden", "host_ref.npz")

MEAN = np.array([0.485, 0.456, 0.406], np.float32)
STD = np.array([0.229, 0.224, 0.225], np.float32)

# (seed, w, h, out_w, out_h): the three sizes the engine's resize parity test feeds a 128 model
# (seed = w + h, as that test draws them), an odd non-square target, a 1 x 1 source, a very wide
# source (the double-precision coordinates matter there) and a camera frame to a Base model
PRE_CASES = [(190, 100, 90, 128, 128), (557, 300, 257, 128, 128), (256, 128, 128, 128, 128),
             (31, 37, 53, 64, 48), (41, 1, 1, 16, 16), (51, 2471, 5, 56, 56), (61, 640, 480, 560, 560)]

# (seed, nq, nc, threshold, top_k, class filter, img_w, img_h, mask_w, mask_h, saturated):
# top_k below / at / above the kept count and 0 (no cap), a class filter, saturated sigmoids
# (score exactly 1.0: ties), duplicated query rows (ties), boxes past the image (clamping),
# nothing above the threshold, and masks upsampled to an odd image size
SEL_CASES = [(101, 40, 91, 0.5, 10, None, 160, 200, 0, 0, True),
             (102, 300, 91, 0.3, 300, (1, 5, 17, 90), 640, 480, 0, 0, True),
             (103, 300, 91, 0.5, 0, None, 1920, 1080, 0, 0, True),
             (104, 100, 91, 0.5, 40, None, 77, 61, 24, 24, True),
             (105, 300, 91, 0.99, 100, None, 560, 560, 0, 0, True),
             (106, 50, 3, 0.9999, 20, None, 64, 64, 0, 0, False),
             (107, 60, 20, 0.4, 0, (0, 3, 7), 33, 47, 13, 9, True)]


def pre_source(seed, w, h):
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


def sel_inputs(seed, nq, nc, mask_w, mask_h, saturated):
    """logits [nq][nc], boxes [nq][4] (cx, cy, w, h), masks [nq][mask_h][mask_w] or None."""
    r = np.random.default_rng(seed)
    logits = (r.standard_normal((nq, nc)) * 3.0 - 4.0).astype(np.float32)
    dup = r.choice(nq, size=2 * max(1, nq // 20), replace=False)
    logits[dup[1::2]] = logits[dup[0::2]]  # equal rows: equal best scores
    if saturated:
        sat = r.choice(nq, size=max(2, nq // 40), replace=False)
        logits[sat, r.integers(0, nc, len(sat))] = 40.0  # sigmoid rounds to 1.0
    boxes = r.uniform(-0.1, 1.1, (nq, 4)).astype(np.float32)
    boxes[:, 2:] = (np.abs(boxes[:, 2:]) * 0.6).astype(np.float32)
    masks = (r.standard_normal((nq, mask_h, mask_w)) * 2.0).astype(np.float32) if mask_w else None
    return logits, boxes, masks


class Detection(C.Structure):
    _fields_ = [("class_id", C.c_uint32), ("class_name", C.c_char_p), ("score", C.c_float),
                ("x1", C.c_float), ("y1", C.c_float), ("x2", C.c_float), ("y2", C.c_float),
                ("mask", C.POINTER(C.c_uint8)), ("mask_width", C.c_int), ("mask_height", C.c_int)]


def _lib():
    lib = C.CDLL(REF_SO)
    lib.rfdetr_image_from_rgb_buffer.restype = C.c_void_p
    lib.rfdetr_image_from_rgb_buffer.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]
    lib.rfdetr_image_free.argtypes = [C.c_void_p]
    lib.rfdetr_preprocess.restype = C.c_int
    lib.rfdetr_preprocess.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                      C.c_bool, C.POINTER(C.POINTER(C.c_float)), C.POINTER(C.c_int),
                                      C.POINTER(C.c_int)]
    lib.rfdetr_select_detections_with_masks.restype = None
    lib.rfdetr_select_detections_with_masks.argtypes = [
        C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_size_t, C.c_size_t, C.c_float,
        C.c_uint32, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.POINTER(C.POINTER(Detection)),
        C.POINTER(C.c_size_t)]
    lib.rfdetr_detections_free.argtypes = [C.POINTER(Detection), C.c_size_t]
    return lib


def ref_preprocess(img, tw, th):
    """The reference's rfdetr_preprocess (bilinear path): float32 [3][th][tw]."""
    lib = _lib()
    libc = C.CDLL(None)
    libc.free.argtypes = [C.c_void_p]
    img = np.ascontiguousarray(img)
    st = C.c_int(0)
    h = lib.rfdetr_image_from_rgb_buffer(img.ctypes.data, img.shape[1], img.shape[0], C.byref(st))
    assert h and st.value == 0
    out = C.POINTER(C.c_float)()
    ow, oh = C.c_int(0), C.c_int(0)
    fp = C.POINTER(C.c_float)
    rc = lib.rfdetr_preprocess(h, tw, th, MEAN.ctypes.data_as(fp), STD.ctypes.data_as(fp), True, C.byref(out),
                               C.byref(ow), C.byref(oh))
    lib.rfdetr_image_free(h)
    assert rc == 0 and (ow.value, oh.value) == (tw, th)
    planes = np.ctypeslib.as_array(out, shape=(3, th, tw)).copy()
    libc.free(C.cast(out, C.c_void_p))
    return planes


def ref_select(logits, boxes, masks, thr, top_k, flt, img_w, img_h):
    """The reference's selection: list of (class, score bits, box bits (4,), mask bytes or None)."""
    lib = _lib()
    nq, nc = logits.shape
    f = None if flt is None else np.ascontiguousarray(flt, np.uint32)
    mw = masks.shape[2] if masks is not None else 0
    mh = masks.shape[1] if masks is not None else 0
    out = C.POINTER(Detection)()
    n = C.c_size_t(0)
    lib.rfdetr_select_detections_with_masks(
        logits.ctypes.data, boxes.ctypes.data, masks.ctypes.data if masks is not None else None, mw, mh, 0.5,
        nq, nc, thr, top_k, f.ctypes.data if f is not None else None, 0 if f is None else len(f), img_w, img_h,
        C.byref(out), C.byref(n))
    recs = []
    for i in range(n.value):
        d = out[i]
        box = np.array([d.x1, d.y1, d.x2, d.y2], np.float32).view(np.uint32)
        mk = np.ctypeslib.as_array(d.mask, shape=(img_h, img_w)).copy() if d.mask else None
        recs.append((int(d.class_id), int(np.float32(d.score).view(np.uint32)), box, mk))
    if n.value:
        lib.rfdetr_detections_free(out, n)
    return recs


def tie_runs(scores):
    """[start, end) ranges of equal consecutive score bits."""
    runs, s = [], 0
    for i in range(1, len(scores) + 1):
        if i == len(scores) or scores[i] != scores[s]:
            runs.append((s, i))
            s = i
    return runs


def main():
    arrays = {}
    digests = []
    for seed, w, h, tw, th in PRE_CASES:
        planes = ref_preprocess(pre_source(seed, w, h), tw, th)
        digests.append(hashlib.sha256(planes.tobytes()).hexdigest())
        arrays[f"pre_head_{seed}"] = planes.reshape(-1)[:16]
    for seed, nq, nc, thr, top_k, flt, iw, ih, mw, mh, sat in SEL_CASES:
        lg, bx, mk = sel_inputs(seed, nq, nc, mw, mh, sat)
        recs = ref_select(lg, bx, mk, thr, top_k, flt, iw, ih)
        if top_k and len(recs) == top_k:
            # top_k must not cut a run of equal scores: the record after the cut must score lower
            full = ref_select(lg, bx, None, thr, 0, flt, iw, ih)
            assert len(full) == len(recs) or full[top_k][1] != recs[-1][1], f"case {seed}: top_k cuts a tie"
        arrays[f"sel_{seed}_class"] = np.array([r[0] for r in recs], np.uint32)
        arrays[f"sel_{seed}_score"] = np.array([r[1] for r in recs], np.uint32)
        arrays[f"sel_{seed}_box"] = np.array([r[2] for r in recs], np.uint32).reshape(-1, 4)
        if mw:
            arrays[f"sel_{seed}_mask"] = np.array([r[3] for r in recs], np.uint8).reshape(-1, ih, iw)
        print(f"select case {seed}: {len(recs)} records, runs of equal score "
              f"{[e - s for s, e in tie_runs([r[1] for r in recs]) if e - s > 1]}")
    np.savez_compressed(OUT, pre_cases=np.array(PRE_CASES, np.int32), pre_sha256=np.array(digests), **arrays)
    print(f"wrote {OUT}: {len(PRE_CASES)} preprocess cases, {len(SEL_CASES)} selection cases")


if __name__ == "__main__":
    main()
