"""Device post-processing (rfdetr_b200_op_select / rfdetr_b200_op_mask_bits)
against the oracle's restatement of the reference's src/postprocess.cpp:43-181,
through the C ABI, including the edge cases of that code: score ties (saturated
sigmoids, duplicated queries: lower query first, lower class first), nothing
above the threshold, top_k larger and smaller than the kept count, class
filters, odd image sizes for the bit-packed masks."""
import ctypes as C
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

pytestmark = pytest.mark.gpu


def _lib():
    from rfdetr_b200 import lib
    return lib.lib()


def _p(t):
    return t.data_ptr() if t is not None else None


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _select(logits, boxes, thr, top_k, w, h, flt=None):
    """Device select over a batch: list of (q, c, s, xyxy) per image."""
    from rfdetr_b200 import lib
    B, NQ, NC = logits.shape
    dl = torch.from_numpy(logits).cuda()
    db = torch.from_numpy(boxes).cuda()
    df = torch.tensor(flt, dtype=torch.int32).cuda() if flt else None
    out = torch.zeros(B * NQ * 8, dtype=torch.int32, device="cuda")
    cnt = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    rc = _lib().rfdetr_b200_op_select(_p(dl), _p(db), B, NQ, NC, thr, top_k, _p(df), len(flt) if flt else 0, w, h,
                                      _p(out), _p(cnt), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    recs = (lib.B200Det * (B * NQ)).from_buffer_copy(out.cpu().numpy().tobytes())
    res = []
    for b in range(B):
        n = int(cnt[b])
        r = [recs[b * NQ + i] for i in range(n)]
        res.append((np.array([x.query for x in r], np.int32), np.array([x.class_id for x in r], np.int32),
                    np.array([x.score for x in r], np.float32),
                    np.array([[x.x1, x.y1, x.x2, x.y2] for x in r], np.float32).reshape(-1, 4)))
    return res, out, cnt


def _check(got, ref):
    q, c, s, xy = got
    rq, rc, rs, rxy = ref
    assert len(q) == len(rq)
    assert np.array_equal(q, rq) and np.array_equal(c, rc)
    assert np.allclose(s, rs, rtol=1e-6, atol=0)
    assert np.allclose(xy, rxy, atol=1e-3)


@pytest.mark.parametrize("B,NQ,NC", [(3, 300, 91), (2, 100, 91), (1, 1000, 7), (4, 37, 5)])
@pytest.mark.parametrize("thr,top_k,flt", [(0.5, 100, None), (0.3, 0, None), (0.6, 7, [1, 3, 4]),
                                           (0.9999999, 10, None)])
def test_select_matches_oracle(B, NQ, NC, thr, top_k, flt):
    import oracle as O
    rng = np.random.default_rng(B * 1000 + NQ + NC)
    logits = (rng.standard_normal((B, NQ, NC)) * 2.0).astype(np.float32)
    boxes = rng.uniform(-0.1, 1.1, (B, NQ, 4)).astype(np.float32)
    w, h = 640, 427
    got, _, _ = _select(logits, boxes, thr, top_k, w, h, flt)
    for b in range(B):
        _check(got[b], O.select(logits[b], boxes[b], thr, top_k, w, h, class_filter=flt))


def test_select_ties_follow_the_reference_order():
    """Saturated sigmoids (= 1.0f) tie across classes and across queries: the
    lowest class wins the argmax and equal scores keep query order."""
    import oracle as O
    B, NQ, NC = 2, 64, 9
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((B, NQ, NC)).astype(np.float32)
    logits[:, ::3, 2] = 30.0   # several saturated classes in these queries
    logits[:, ::3, 5] = 40.0
    logits[:, 7] = logits[:, 4]  # duplicated query rows: identical scores
    boxes = rng.uniform(0, 1, (B, NQ, 4)).astype(np.float32)
    got, _, _ = _select(logits, boxes, 0.5, 0, 100, 50)
    for b in range(B):
        ref = O.select(logits[b], boxes[b], 0.5, 0, 100, 50)
        _check(got[b], ref)
        sat = got[b][0][got[b][2] == 1.0]
        assert np.all(np.diff(sat) > 0)       # equal scores in ascending query order
        assert np.all(got[b][1][got[b][2] == 1.0] == 2)  # first of the tied classes


def test_select_nothing_above_threshold():
    logits = np.full((2, 50, 4), -8.0, np.float32)
    boxes = np.full((2, 50, 4), 0.5, np.float32)
    got, _, cnt = _select(logits, boxes, 0.5, 10, 32, 32)
    assert cnt.tolist() == [0, 0] and all(len(g[0]) == 0 for g in got)


@pytest.mark.parametrize("w,h", [(77, 50), (384, 384), (33, 1), (1000, 3)])
def test_mask_bits_match_oracle_upsample(w, h):
    import oracle as O
    B, NQ, NC, side = 2, 50, 6, 24
    rng = np.random.default_rng(w + h)
    logits = (rng.standard_normal((B, NQ, NC)) * 2).astype(np.float32)
    boxes = rng.uniform(0, 1, (B, NQ, 4)).astype(np.float32)
    masks = rng.standard_normal((B, NQ, side, side)).astype(np.float32)
    max_dets = 8
    got, d_dets, d_cnt = _select(logits, boxes, 0.5, max_dets, w, h)
    words = _lib().rfdetr_b200_mask_bits_words(w, h)
    assert words == h * ((w + 31) // 32)
    bits = torch.zeros(B * max_dets * words, dtype=torch.int32, device="cuda")
    dm = torch.from_numpy(masks).cuda()
    rc = _lib().rfdetr_b200_op_mask_bits(_p(dm), B, NQ, side, _p(d_dets), _p(d_cnt), max_dets, w, h, _p(bits),
                                         _stream())
    assert rc == 0
    torch.cuda.synchronize()
    u = bits.cpu().numpy().view(np.uint32).reshape(B, max_dets, h, -1)
    for b in range(B):
        for i, q in enumerate(got[b][0]):
            ref = O.mask_upsample(masks[b, q], w, h)
            px = np.arange(w)
            ours = ((u[b, i][:, px // 32] >> (px % 32).astype(np.uint32)) & 1) * 255
            assert (ours == ref).mean() >= 0.99999, (b, i)
    # a detection count beyond max_dets is rejected before any launch
    assert _lib().rfdetr_b200_op_mask_bits(_p(dm), B, NQ, side, _p(d_dets), _p(d_cnt), NQ + 1, w, h, _p(bits),
                                           _stream()) != 0


def test_select_and_masks_match_the_reference_code():
    """Device selection and mask bits on the seeded cases of tests/golden/host_ref.npz, which hold
    the outputs of the reference's own src/postprocess.cpp (built from the reference tree): the
    same records in the same order, except that runs of equal score (the reference sorts them with
    std::sort) are compared as sets; scores to 1e-6 relative (the device's exp), boxes to 1e-3 px,
    masks (square mask cases) pixel for pixel."""
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import gen_host_ref_golden as gen

    g = np.load(os.path.join(ROOT, "tests", "golden", "host_ref.npz"))
    for seed, nq, nc, thr, top_k, flt, iw, ih, mw, mh, sat in gen.SEL_CASES:
        lg, bx, mk = gen.sel_inputs(seed, nq, nc, mw, mh, sat)
        got, d_dets, d_cnt = _select(lg[None], bx[None], thr, top_k, iw, ih, list(flt) if flt else None)
        q, c, s, xy = got[0]
        rc_, rs = g[f"sel_{seed}_class"], g[f"sel_{seed}_score"].view(np.float32)
        rxy = g[f"sel_{seed}_box"].view(np.float32)
        assert len(q) == len(rc_), f"case {seed}: {len(q)} records, reference {len(rc_)}"
        masks_ok = mw and mw == mh
        if masks_ok:
            words = _lib().rfdetr_b200_mask_bits_words(iw, ih)
            bits = torch.zeros(max(1, len(q)) * words, dtype=torch.int32, device="cuda")
            dm = torch.from_numpy(mk[None]).cuda()
            assert _lib().rfdetr_b200_op_mask_bits(_p(dm), 1, nq, mw, _p(d_dets), _p(d_cnt), max(1, len(q)), iw,
                                                   ih, _p(bits), _stream()) == 0
            torch.cuda.synchronize()
            u = bits.cpu().numpy().view(np.uint32).reshape(max(1, len(q)), ih, -1)
            px = np.arange(iw)
            ours = [((u[i][:, px // 32] >> (px % 32).astype(np.uint32)) & 1).astype(np.uint8) * 255
                    for i in range(len(q))]
            rmk = g[f"sel_{seed}_mask"]
        for a, e in gen.tie_runs(g[f"sel_{seed}_score"].tolist()):
            key = lambda cls, box: (int(cls),) + tuple(np.round(box, 2))  # noqa: E731
            mine = sorted(range(a, e), key=lambda i: key(c[i], xy[i]))
            refs = sorted(range(a, e), key=lambda i: key(rc_[i], rxy[i]))
            for i, j in zip(mine, refs):
                assert c[i] == rc_[j], f"case {seed} record {i}"
                assert np.isclose(s[i], rs[j], rtol=1e-6, atol=0), f"case {seed} record {i}"
                assert np.allclose(xy[i], rxy[j], atol=1e-3), f"case {seed} record {i}"
                if masks_ok:
                    assert (ours[i] == rmk[j]).mean() >= 0.99999, f"case {seed} mask of record {i}"
