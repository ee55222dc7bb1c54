"""The oracle's pre- and post-processing pinned to the reference's own code.

tests/golden/host_ref.npz holds outputs of the reference's src/image_io.cpp
(rfdetr_preprocess, 1.9 bilinear path) and src/postprocess.cpp (selection with
masks) built from the reference tree into oracle/_ref/librefhost.so
(tests/golden/gen_host_ref_golden.py).  The oracle's restatements must equal
them bit for bit: the normalized planes (SHA-256), and the selection records
(class id, score and box bit patterns, 0/255 masks).  The reference sorts with
std::sort on the score alone, so runs of equal score are compared as sets.
Where the reference build is present, the fixtures are also re-derived from it.
The device selection is checked against the same fixtures in
tests/test_gpu_postprocess.py.
"""
import ctypes as C
import hashlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "tests", "golden"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

GOLDEN = os.path.join(REPO, "tests", "golden", "host_ref.npz")


def golden():
    return np.load(GOLDEN)


def golden_records(g, seed, with_masks):
    """Reference records of a selection case: list of (class, score bits, box bits, mask bytes)."""
    cls, sc, bx = g[f"sel_{seed}_class"], g[f"sel_{seed}_score"], g[f"sel_{seed}_box"]
    mk = g[f"sel_{seed}_mask"] if with_masks else None
    return [(int(cls[i]), int(sc[i]), tuple(int(v) for v in bx[i]), None if mk is None else mk[i].tobytes())
            for i in range(len(cls))]


def same_up_to_ties(got, want):
    """Equal lists, except that records inside a run of equal score (same bits) may be permuted."""
    import gen_host_ref_golden as gen

    if len(got) != len(want):
        return False
    for s, e in gen.tie_runs([r[1] for r in want]):
        if sorted(got[s:e]) != sorted(want[s:e]):
            return False
    return True


def test_oracle_preprocess_equals_the_reference():
    import gen_host_ref_golden as gen
    import oracle as O

    g = golden()
    assert [tuple(c) for c in g["pre_cases"]] == gen.PRE_CASES
    fp = C.POINTER(C.c_float)
    for (seed, w, h, tw, th), digest in zip(gen.PRE_CASES, g["pre_sha256"]):
        img = np.ascontiguousarray(gen.pre_source(seed, w, h))
        out = np.empty((3, th, tw), np.float32)
        O.lib().oracle_preprocess(img.ctypes.data_as(C.POINTER(C.c_uint8)), w, h, tw, th,
                                  gen.MEAN.ctypes.data_as(fp), gen.STD.ctypes.data_as(fp), out.ctypes.data_as(fp))
        assert np.array_equal(out.reshape(-1)[:16], g[f"pre_head_{seed}"]), (seed, w, h, tw, th)
        assert hashlib.sha256(out.tobytes()).hexdigest() == digest, (seed, w, h, tw, th)


def test_oracle_selection_and_masks_equal_the_reference():
    import gen_host_ref_golden as gen
    import oracle as O

    g = golden()
    for seed, nq, nc, thr, top_k, flt, iw, ih, mw, mh, sat in gen.SEL_CASES:
        lg, bx, mk = gen.sel_inputs(seed, nq, nc, mw, mh, sat)
        q, c, s, xy = O.select(lg, bx, thr, top_k, iw, ih, None if flt is None else list(flt))
        got = []
        for i in range(len(q)):
            m = O.mask_upsample(mk[q[i]], iw, ih, 0.5).tobytes() if mw else None
            got.append((int(c[i]), int(np.float32(s[i]).view(np.uint32)),
                        tuple(int(v) for v in xy[i].astype(np.float32).view(np.uint32)), m))
        assert same_up_to_ties(got, golden_records(g, seed, bool(mw))), f"selection case {seed}"


def test_golden_fixtures_are_the_reference_code():
    import gen_host_ref_golden as gen

    if not os.path.exists(gen.REF_SO):
        pytest.skip("oracle/_ref/librefhost.so is built only where the reference tree is present")
    g = golden()
    for (seed, w, h, tw, th), digest in zip(gen.PRE_CASES, g["pre_sha256"]):
        planes = gen.ref_preprocess(gen.pre_source(seed, w, h), tw, th)
        assert hashlib.sha256(planes.tobytes()).hexdigest() == digest
    for seed, nq, nc, thr, top_k, flt, iw, ih, mw, mh, sat in gen.SEL_CASES:
        lg, bx, mk = gen.sel_inputs(seed, nq, nc, mw, mh, sat)
        recs = [(r[0], r[1], tuple(int(v) for v in r[2]), None if r[3] is None else r[3].tobytes())
                for r in gen.ref_select(lg, bx, mk, thr, top_k, flt, iw, ih)]
        assert recs == golden_records(g, seed, bool(mw)), f"selection case {seed}"
