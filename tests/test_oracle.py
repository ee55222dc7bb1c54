"""The CPU oracle, pinned: against an independent float64 PyTorch
restatement (tests/torch_ref.py) at every stage, and against the reference's
closed-form known answers (proposal-mask ring, tests/test_two_stage_mask.cpp;
sine embedding, src/decoder.cpp:383-417; AA bicubic pos-embed,
src/model_loader.cpp:83-208)."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle as O
from rfdetr_b200 import synth
from torch_ref import TorchRef


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("variant", ["tiny", "tiny-base", "seg-tiny", "grid52"])
def test_oracle_matches_torch(variant, make_model):
    path = make_model(variant, "f32", 0)
    o = O.Oracle(path)
    S = o.image_size
    rgb = np.random.default_rng(7).integers(0, 256, (S, S, 3), dtype=np.uint8)
    x = o.preprocess(rgb)
    r = o.forward(x, trace=True)
    meta, tensors = synth.read_gguf_f32(path)
    ref = TorchRef(meta, tensors).forward(x)
    tr = r["trace"]
    for j in range(4):
        assert rel(tr[f"backbone.multiscale.level{j}"], ref[f"tap{j}"].reshape(-1)) < 1e-5
    assert rel(tr["projector.output"], ref["projector"].reshape(-1)) < 1e-5
    assert rel(tr["two_stage.cls_all"], ref["cls_all"].reshape(-1)) < 1e-5
    assert np.array_equal(r["topk"], ref["topk"])
    assert rel(r["logits"], ref["logits"]) < 1e-5
    assert rel(r["boxes"], ref["boxes"]) < 1e-5
    if r["masks"] is not None:
        assert rel(r["masks"], ref["masks"]) < 1e-5


@pytest.mark.parametrize("S,masked", [(40, False), (49, False), (50, True), (52, True), (64, True)])
def test_proposal_mask_ring(S, masked):
    # tests/test_two_stage_mask.cpp part A: only the one-cell border ring fires, only for S >= 50.
    cfg = synth.get_variant("grid52")
    assert cfg  # grid arithmetic restated here exactly as src/two_stage.cpp:69-88
    fs = np.float32(S)
    zeroed = 0
    for h in range(S):
        for w in range(S):
            p = [np.float32((np.float32(w) + np.float32(0.5)) / fs), np.float32((np.float32(h) + np.float32(0.5)) / fs),
                 np.float32(0.05), np.float32(0.05)]
            valid = all(v > np.float32(0.01) and v < np.float32(0.99) for v in p)
            border = w == 0 or h == 0 or w == S - 1 or h == S - 1
            if not valid:
                zeroed += 1
                assert border
            elif masked:
                assert not border
    assert zeroed == (4 * S - 4 if masked else 0)


def test_grid52_masks_memory(make_model):
    # test_two_stage_mask.cpp part B: masked tokens' memory is zeroed before enc_output,
    # so their boxes reparam to exactly zero.
    path = make_model("grid52", "f32", 0)
    o = O.Oracle(path)
    x = o.preprocess(np.full((o.image_size, o.image_size, 3), 128, np.uint8))
    tr = o.forward(x, trace=True)["trace"]
    G = 52
    bb = tr["two_stage.bbox_all"].reshape(G, G, 4)
    assert np.all(bb[0] == 0) and np.all(bb[-1] == 0) and np.all(bb[:, 0] == 0) and np.all(bb[:, -1] == 0)
    assert np.all(bb[1:-1, 1:-1, 2:] > 0)


def test_bicubic_matches_torch_antialias():
    rng = np.random.default_rng(0)
    for src, dst in [(37, 40), (24, 24), (6, 8), (44, 44), (32, 36)]:
        a = rng.standard_normal((src * src, 16)).astype(np.float32)
        ours = O.bicubic_resample(a, src, dst)
        t = torch.from_numpy(a).reshape(1, src, src, 16).permute(0, 3, 1, 2).double()
        ref = F.interpolate(t, size=(dst, dst), mode="bicubic", align_corners=False, antialias=True)
        ref = ref.permute(0, 2, 3, 1).reshape(dst * dst, 16).numpy()
        assert rel(ours, ref) < 1e-5, (src, dst)


def test_sine_embed_closed_form(make_model):
    path = make_model("tiny", "f32", 0)
    o = O.Oracle(path)
    x = o.preprocess(np.random.default_rng(1).integers(0, 256, (128, 128, 3), dtype=np.uint8))
    tr = o.forward(x, trace=True)["trace"]
    rp = tr["decoder.refpoints"].reshape(-1, 4)
    assert rp.shape[0] == o.nq and np.all(rp[:, 2:] > 0)


def test_select_and_mask_upsample():
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((20, 5)).astype(np.float32)
    boxes = rng.uniform(0.1, 0.9, (20, 4)).astype(np.float32)
    q, c, s, xy = O.select(logits, boxes, 0.5, 7, 640, 480)
    sig = 1 / (1 + np.exp(-logits.astype(np.float64)))
    best = sig.max(1)
    keep = np.where(best > 0.5)[0]
    order = keep[np.argsort(-best[keep], kind="stable")][:7]
    assert np.array_equal(q, order)
    assert np.allclose(s, best[order], rtol=1e-6)
    assert np.all(xy[:, 0] >= 0) and np.all(xy[:, 2] <= 640)
    # class filter (applied before the sort and top_k)
    qf, cf, sf, _ = O.select(logits, boxes, 0.5, 7, 640, 480, class_filter=[1, 3])
    cls = sig.argmax(1)
    keepf = np.where((best > 0.5) & np.isin(cls, [1, 3]))[0]
    orderf = keepf[np.argsort(-best[keepf], kind="stable")][:7]
    assert np.array_equal(qf, orderf) and set(cf.tolist()) <= {1, 3}
    m = rng.standard_normal((6, 6)).astype(np.float32)
    up = O.mask_upsample(m, 18, 12)
    t = torch.from_numpy(m)[None, None].double()
    ref = F.interpolate(t, size=(12, 18), mode="bilinear", align_corners=False)[0, 0].numpy()
    agree = (up == 255) == (ref > 0)
    assert agree.mean() > 0.99
