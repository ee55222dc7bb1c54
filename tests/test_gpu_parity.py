"""End-to-end parity on the B200: the CUDA engine (through the C ABI) against
the CPU oracle on the same seeded synthetic models and images.

Metrics, per output tensor (class logits, boxes):
  rel       max|gpu - oracle| / max|oracle|                                   <= tol
  el_p50    median over elements of |gpu - oracle| / max(|oracle|, tol * max|oracle|)  <= tol
  el_p90, el_max   the same ratio's 90th percentile and maximum (reported)
with tol = 1e-3 for F32/F16 weights and 2e-2 for Q8_0/Q4_K.  The element-wise
figures measure each value against its own magnitude; the floor (tol x the
tensor's largest magnitude) keeps a value that is zero in the oracle from
dividing by zero.  Their tail is not held to tol: rounding the activations to
f16 gives errors of absolute, not relative, size, so logits near zero carry a
large relative error, and the reference's own arithmetic does the same (the
oracle's mode ii against its mode i on Nano F16: p50 2.3e-4, p90 1.4e-3, max
0.16; on a Q8_0 model: p50 5.9e-3, p90 3.4e-2).  The engine computes GEMM operands in f16 with
f32 accumulation and an f32 residual stream; the oracle is f32 throughout
(mode i).  For Q8_0 / Q4_K models the oracle is also run in mode ii, which
rounds activations before each weight product the way ggml's CPU vec-dot does
(F16 / Q8_0 / Q8_K blocks), and the distances to both are printed and checked.

Top-K: the selected token must be the oracle's at every rank, except where
the two tokens' oracle class scores differ by at most tol x the largest
score (a near-tie the tolerance cannot order).  The decoder and heads are then
compared with the oracle forced onto the engine's selection, so both see the
same queries.  Masks: mean IoU of the thresholded masks (logit > 0, i.e.
sigmoid > 0.5) per query >= 0.99, queries empty in both counting as 1.
Intermediate stages (projector output, two-stage class logits) are checked at
3x the output tolerance as diagnostics that localize a regression.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-3, "f16": 1e-3, "q8_0": 2e-2, "q4_K": 2e-2}


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def rel_elementwise(a, b, tol):
    """(median, 90th percentile, max) over elements of |a - b| / max(|b|, tol * max|b|)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.maximum(np.abs(b), tol * max(np.abs(b).max(), 1e-30))
    r = np.abs(a - b) / den
    p50, p90 = np.percentile(r, [50, 90])
    return float(p50), float(p90), float(r.max())


def mask_iou(gpu, ref):
    """(mean, min) over queries of the IoU of the masks thresholded at logit > 0."""
    g = np.asarray(gpu).reshape(gpu.shape[0], -1) > 0
    r = np.asarray(ref).reshape(ref.shape[0], -1) > 0
    inter = (g & r).sum(1)
    union = (g | r).sum(1)
    iou = np.where(union > 0, inter / np.maximum(union, 1), 1.0)
    return float(iou.mean()), float(iou.min())


def _images(S, n, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (n, S, S, 3), dtype=np.uint8)


def check_topk(gpu_idx, ora_idx, scores, tol):
    """Same token at each rank as the oracle's own selection, except where the two
    tokens' oracle scores differ by at most tol x max|score| (a near-tie).

    Returns (swaps, largest gap / max|score|)."""
    gpu_idx = np.asarray(gpu_idx, np.int64)
    ora_idx = np.asarray(ora_idx, np.int64)
    smax = np.abs(scores).max()
    diff = gpu_idx != ora_idx
    gap = 0.0
    if diff.any():
        gap = float(np.abs(scores[gpu_idx[diff]] - scores[ora_idx[diff]]).max() / smax)
        assert gap <= tol, f"top-K differs beyond near-ties: gap {gap:.3g} x max score > {tol}"
    return int(diff.sum()), gap


def compare_image(ora, x, lg, bx, mk, topk, cls_gpu, cls_o, own_topk, tol, mode2=False):
    """Every parity figure of one image; asserts the contract and returns the report."""
    r = {}
    r["topk_swaps"], r["topk_gap"] = check_topk(topk, own_topk, cls_o.max(1), tol)
    r["cls_all"] = rel(cls_gpu, cls_o)
    forced = ora.forward(x, force_topk=topk)
    for name, got, want in (("logits", lg, forced["logits"]), ("boxes", bx, forced["boxes"])):
        r[name] = rel(got, want)
        r[name + "_el_p50"], r[name + "_el_p90"], r[name + "_el_max"] = rel_elementwise(got, want, tol)
    if mk is not None:
        r["masks"] = rel(mk, forced["masks"])
        r["mask_iou_mean"], r["mask_iou_min"] = mask_iou(mk, forced["masks"])
    if mode2:
        # oracle mode ii (ggml-like activation rounding) on the same queries
        f2 = ora.forward(x, act_round=1, force_topk=topk)
        r["logits_mode2"] = rel(lg, f2["logits"])
        r["boxes_mode2"] = rel(bx, f2["boxes"])
        r["mode2_vs_mode1_logits"] = rel(f2["logits"], forced["logits"])
    assert r["cls_all"] < 3 * tol, r
    for name in ("logits", "boxes"):
        assert r[name] < tol and r[name + "_el_p50"] < tol, (name, r)
        if mode2:
            assert r[name + "_mode2"] < tol, (name, r)
    if mk is not None:
        assert r["mask_iou_mean"] >= 0.99, r
    return r


CASES = [("tiny", "f32", 2), ("tiny", "f16", 1), ("tiny", "q8_0", 1), ("tiny", "q4_K", 1),
         ("tiny-base", "f16", 2), ("seg-tiny", "f16", 2), ("grid52", "f16", 1)]


@pytest.mark.parametrize("variant,dtype,batch", CASES)
def test_engine_matches_oracle(variant, dtype, batch, make_model):
    import oracle as O
    from rfdetr_b200 import lib

    path = make_model(variant, dtype, 0)
    ora = O.Oracle(path)
    eng = lib.Engine(path, device=0, max_batch=batch)
    S = eng.image_size
    imgs = _images(S, batch, 100 + batch)
    lg, bx, mk = eng.forward_rgb(imgs)
    NQ, NC = eng.nq, eng.nc
    G = S // int(ora.meta["rfdetr.patch_size"])
    cls_gpu = eng.trace("two_stage.cls_all", batch).reshape(batch, G * G, NC)
    topk_gpu = eng.trace("topk", batch).reshape(batch, NQ).astype(np.int64)
    proj_gpu = eng.trace("projector.output", batch).reshape(batch, G * G, -1)
    eng.close()
    tol = TOL[dtype]
    report = []
    for b in range(batch):
        x = ora.preprocess(imgs[b])
        own = ora.forward(x, trace=True)
        tr = own["trace"]
        cls_o = tr["two_stage.cls_all"].reshape(G * G, NC)
        r = compare_image(ora, x, lg[b], bx[b], None if mk is None else mk[b], topk_gpu[b], cls_gpu[b], cls_o,
                          own["topk"], tol, mode2=dtype in ("q8_0", "q4_K"))
        r["projector"] = rel(proj_gpu[b], tr["projector.output"].reshape(G * G, -1))
        assert r["projector"] < 3 * tol, r
        report.append(r)
    print(f"\n{variant}/{dtype}: {report}")


def test_rgb_and_planar_paths_agree(make_model):
    import oracle as O
    from rfdetr_b200 import lib

    path = make_model("tiny", "f16", 0)
    ora = O.Oracle(path)
    eng = lib.Engine(path)
    img = _images(eng.image_size, 1, 5)
    lg1, bx1, _ = eng.forward_rgb(img)
    planar = ora.preprocess(img[0])
    lg2, bx2, _ = eng.forward_planar(planar)
    assert rel(lg1, lg2) < 1e-5 and rel(bx1, bx2) < 1e-5
    eng.close()


def test_nano_batch1_parity(make_model):
    """Nano F16, batch 1 at 384 x 384 (the reference's CPU-runnable config)."""
    import oracle as O
    from rfdetr_b200 import lib

    path = make_model("nano", "f16", 0)
    ora = O.Oracle(path)
    eng = lib.Engine(path)
    img = _images(384, 1, 1000)
    lg, bx, _ = eng.forward_rgb(img)
    topk = eng.trace("topk", 1).astype(np.int64)
    cls_gpu = eng.trace("two_stage.cls_all", 1).reshape(-1, 91)
    eng.close()
    x = ora.preprocess(img[0])
    own = ora.forward(x, trace=True)
    cls_o = own["trace"]["two_stage.cls_all"].reshape(-1, 91)
    r = compare_image(ora, x, lg[0], bx[0], None, topk, cls_gpu, cls_o, own["topk"], 1e-3)
    print(f"\nnano/f16 batch 1: {r}")


def test_graph_replay_matches_direct_launches(make_model, monkeypatch):
    """The second and later forwards of a shape replay a captured CUDA graph;
    they must reproduce the directly launched forward bit for bit."""
    from rfdetr_b200 import lib

    path = make_model("tiny", "f16", 0)
    S = 128
    a, b = _images(S, 2, 21), _images(S, 2, 22)
    eng = lib.Engine(path, max_batch=2)
    la1, ba1, _ = eng.forward_rgb(a)      # direct launches (+ capture)
    lb_graph, bb_graph, _ = eng.forward_rgb(b)  # graph replay, new input
    la2, ba2, _ = eng.forward_rgb(a)      # graph replay again
    eng.close()
    assert np.array_equal(la1, la2) and np.array_equal(ba1, ba2)
    monkeypatch.setenv("RFDETR_NO_GRAPH", "1")
    direct = lib.Engine(path, max_batch=2)
    lb_direct, bb_direct, _ = direct.forward_rgb(b)
    lb_direct2, _, _ = direct.forward_rgb(b)
    direct.close()
    assert np.array_equal(lb_graph, lb_direct) and np.array_equal(bb_graph, bb_direct)
    assert np.array_equal(lb_direct, lb_direct2)


@pytest.mark.parametrize("variant,dtype,S", [("tiny", "f16", 128), ("base", "q8_0", 560)])
def test_fused_norm1_and_tap_match_separate_launches(variant, dtype, S, make_model, monkeypatch):
    """A tapped block's output is normalised once for the backbone tap and the next block's norm1
    (one launch reading x once); the forward must equal, bit for bit, the one with the two
    separate LayerNorm launches (RFDETR_LN_TAP=0), including the projector input the taps feed."""
    from rfdetr_b200 import lib

    path = make_model(variant, dtype, 0)
    imgs = _images(S, 2, 31)
    outs = []
    for env in ("1", "0"):
        monkeypatch.setenv("RFDETR_LN_TAP", env)
        eng = lib.Engine(path, max_batch=2)
        lg, bx, _ = eng.forward_rgb(imgs)
        proj = eng.trace("projector.output", 2)
        eng.close()
        outs.append((lg, bx, proj))
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a, b)


def test_split_k_layernorm_gemms_match_the_oracle(make_model):
    """With few row blocks (batch 1: 300 decoder rows, one 24 x 24 grid) the LayerNorm GEMMs run as
    split-K f32 partial sums plus an in-order row reduction: the forward repeats bit for bit and
    matches the oracle (with the engine's top-K indices forced, since the changed summation order
    may swap near-tied proposals)."""
    import oracle as O
    from rfdetr_b200 import lib

    path = make_model("nano", "f16", 0)
    eng = lib.Engine(path, max_batch=1)
    S = eng.image_size
    img = _images(S, 1, 41)
    l1, b1, _ = eng.forward_rgb(img)
    l2, b2, _ = eng.forward_rgb(img)
    topk = eng.trace("topk", 1).astype(np.int32)
    eng.close()
    assert np.array_equal(l1, l2) and np.array_equal(b1, b2)
    ora = O.Oracle(path)
    ref = ora.forward(ora.preprocess(img[0]), force_topk=topk)
    assert rel(l1[0], ref["logits"]) < 1e-3 and rel(b1[0], ref["boxes"]) < 1e-3


def test_pipelined_submissions_match_forward_rgb(make_model):
    """rfdetr_b200_submit_rgb / rfdetr_b200_wait: several batches in flight
    (uploads on a copy stream into two alternating device slots, forwards on
    the engine stream, outputs copied into two alternating device slots and
    downloaded on a third stream) give, batch for batch, the outputs of the
    synchronous rfdetr_b200_forward_rgb; a larger batch and another image size
    in the middle of the stream regrow the slots."""
    import torch
    from rfdetr_b200 import lib

    path = make_model("tiny", "f16", 0)
    S = 128
    eng = lib.Engine(path, max_batch=2)
    batches = [_images(S, 2, 31), _images(S, 2, 32), _images(S, 1, 33), _images(S + 40, 3, 34), _images(S, 2, 35)]
    want = [eng.forward_rgb(x)[:2] for x in batches]
    pinned = [torch.from_numpy(x).pin_memory() for x in batches]
    outs = []
    for x in pinned:
        B = x.shape[0]
        lg = torch.empty((B, eng.nq, eng.nc), dtype=torch.float32).pin_memory()
        bx = torch.empty((B, eng.nq, 4), dtype=torch.float32).pin_memory()
        eng.submit_rgb(x.numpy(), lg.numpy(), bx.numpy())
        outs.append((lg, bx))
    eng.wait()
    for (lg, bx), (wl, wb) in zip(outs, want):
        assert np.array_equal(lg.numpy(), wl) and np.array_equal(bx.numpy(), wb)
    eng.close()


def test_pipelined_submissions_with_masks(make_model):
    """Segmentation outputs through rfdetr_b200_submit_rgb (logits, boxes and masks through the
    device output slots and the download stream) equal rfdetr_b200_forward_rgb's, batch for
    batch; a submission that asks for the logits only writes nothing else."""
    import torch
    from rfdetr_b200 import lib

    path = make_model("seg-tiny", "f16", 0)
    eng = lib.Engine(path, max_batch=2)
    S, m = eng.image_size, eng.mask_side
    assert m > 0
    batches = [_images(S, 2, 61 + i) for i in range(4)]
    want = [eng.forward_rgb(x) for x in batches]
    outs = []
    for x in batches:
        o = (torch.empty((2, eng.nq, eng.nc)).pin_memory(), torch.empty((2, eng.nq, 4)).pin_memory(),
             torch.empty((2, eng.nq, m, m)).pin_memory())
        eng.submit_rgb(x, o[0].numpy(), o[1].numpy(), o[2].numpy())
        outs.append(o)
    only = torch.empty((2, eng.nq, eng.nc)).pin_memory()
    eng.submit_rgb(batches[1], only.numpy(), None)
    eng.wait()
    for o, w in zip(outs, want):
        for got, ref in zip(o, w):
            assert np.array_equal(got.numpy(), ref)
    assert np.array_equal(only.numpy(), want[1][0])
    eng.close()


def test_streaming_submissions_wait_oldest(make_model):
    """A streaming loop with rfdetr_b200_wait_oldest: submit batch i+1, wait for the oldest, read
    batch i while i+1 runs; every batch equals the synchronous rfdetr_b200_forward_rgb."""
    import torch
    from rfdetr_b200 import lib

    path = make_model("tiny", "f16", 0)
    S = 128
    eng = lib.Engine(path, max_batch=2)
    batches = [_images(S, 2, 51 + i) for i in range(4)]
    want = [eng.forward_rgb(x)[:2] for x in batches]
    pinned = [torch.from_numpy(x).pin_memory() for x in batches]
    outs = [(torch.empty((2, eng.nq, eng.nc), dtype=torch.float32).pin_memory(),
             torch.empty((2, eng.nq, 4), dtype=torch.float32).pin_memory()) for _ in batches]
    eng.submit_rgb(pinned[0].numpy(), outs[0][0].numpy(), outs[0][1].numpy())
    for i in range(len(batches)):
        if i + 1 < len(batches):
            eng.submit_rgb(pinned[i + 1].numpy(), outs[i + 1][0].numpy(), outs[i + 1][1].numpy())
        eng.wait_oldest()  # batch i is complete
        assert np.array_equal(outs[i][0].numpy(), want[i][0]) and np.array_equal(outs[i][1].numpy(), want[i][1])
    eng.wait_oldest()  # nothing outstanding: returns at once
    eng.wait()
    eng.close()


# Every configuration the benchmark description names, at its real model size
# (batch 2: the oracle checks both images; the full batches run through the
# same kernels, only more rows).
FULL = [("nano", "f16"), ("base", "q8_0"), ("medium", "q4_K"), ("seg-small", "f16"), ("large", "f16")]


def _check_variant(variant, dtype, batch, make_model, sample=None):
    """Engine vs oracle at the variant's full size: class scores and top-K,
    then logits / boxes / masks with the oracle forced onto the engine's top-K.
    `sample` lists the images of the batch the oracle checks (default: all)."""
    import oracle as O
    from rfdetr_b200 import lib

    path = make_model(variant, dtype, 0)
    ora = O.Oracle(path)
    eng = lib.Engine(path, max_batch=batch)
    S = eng.image_size
    imgs = _images(S, batch, 500 + S)
    lg, bx, mk = eng.forward_rgb(imgs)
    NQ, NC = eng.nq, eng.nc
    G = S // int(ora.meta["rfdetr.patch_size"])
    topk = eng.trace("topk", batch).reshape(batch, NQ).astype(np.int64)
    cls_gpu = eng.trace("two_stage.cls_all", batch).reshape(batch, G * G, NC)
    eng.close()
    tol = TOL[dtype]
    report = []
    for b in (sample if sample is not None else range(batch)):
        x = ora.preprocess(imgs[b])
        own = ora.forward(x, trace=True)
        cls_o = own["trace"]["two_stage.cls_all"].reshape(G * G, NC)
        r = compare_image(ora, x, lg[b], bx[b], None if mk is None else mk[b], topk[b], cls_gpu[b], cls_o,
                          own["topk"], tol, mode2=dtype in ("q8_0", "q4_K"))
        r["image"] = b
        report.append(r)
    print(f"\n{variant}/{dtype} batch {batch}: {report}")


@pytest.mark.parametrize("variant,dtype", FULL)
def test_full_size_configs(variant, dtype, make_model):
    _check_variant(variant, dtype, 2, make_model)


@pytest.mark.parametrize("variant,dtype,batch,sample", [("base", "q8_0", 32, (0, 17, 31)),
                                                        ("base", "q8_0", 64, (0, 63)),
                                                        ("large", "f16", 256, (0, 137, 255))])
def test_benchmarked_batches(variant, dtype, batch, sample, make_model):
    """The batches the benchmark times (Base Q8_0 at 32 and 64 images, Large F16 at 256), checked
    against the oracle on sampled images of the full batch: the GEMM tiling, split choices and
    row counts are those of the timed forward."""
    _check_variant(variant, dtype, batch, make_model, sample)


# The remaining variants of the converter's table (scripts/convert_rfdetr_to_gguf.py:125-205)
# through the same kernels: Small; Seg-Nano (num_windows = 1: every block attends over the
# whole 26 x 26 grid); Seg-Medium / Large; Seg-XLarge (G = 52) and Seg-2XLarge (G = 64, the
# largest grid the top-K kernel takes), where the two-stage proposal mask fires
# (src/two_stage.cpp:34-89).
REST = [("small", "f16"), ("seg-nano", "f16"), ("seg-medium", "q8_0"), ("seg-large", "q4_K"),
        ("seg-xlarge", "f16"), ("seg-2xlarge", "f16")]


@pytest.mark.parametrize("variant,dtype", REST)
def test_remaining_variants(variant, dtype, make_model):
    _check_variant(variant, dtype, 1, make_model)


def test_batch_position_invariance(make_model, monkeypatch):
    """An image's outputs do not depend on its position in the batch or on the other images of the
    batch (bit for bit).  Across batch sizes they are bit-identical when the LayerNorm GEMMs keep
    full-row tiles (RFDETR_GEMM_SPLITK=0); by default small batches split K (another f32 summation
    order), which the split-K oracle test covers."""
    from rfdetr_b200 import lib

    path = make_model("tiny-base", "f16", 0)
    eng = lib.Engine(path, max_batch=4)
    imgs = _images(eng.image_size, 4, 77)
    lg, bx, _ = eng.forward_rgb(imgs)
    perm = imgs[[2, 0, 3, 1]]
    lg2, bx2, _ = eng.forward_rgb(perm)
    eng.close()
    assert np.array_equal(lg[[2, 0, 3, 1]], lg2) and np.array_equal(bx[[2, 0, 3, 1]], bx2)
    monkeypatch.setenv("RFDETR_GEMM_SPLITK", "0")
    eng = lib.Engine(path, max_batch=4)
    lg, bx, _ = eng.forward_rgb(imgs)
    one, bone, _ = eng.forward_rgb(imgs[3:4])
    eng.close()
    assert np.array_equal(lg[3], one[0]) and np.array_equal(bx[3], bone[0])


@pytest.mark.parametrize("src", [(100, 90), (300, 257), (128, 128)])
def test_resize_path_matches_oracle_preprocess(src, make_model):
    """Images not at the model resolution are resized on the GPU exactly like
    rfdetr_preprocess (bilinear, half-pixel, double coordinates)."""
    import oracle as O
    from rfdetr_b200 import lib

    path = make_model("tiny", "f32", 0)
    ora = O.Oracle(path)
    eng = lib.Engine(path)
    w, h = src
    img = np.random.default_rng(w + h).integers(0, 256, (1, h, w, 3), dtype=np.uint8)
    lg, bx, _ = eng.forward_rgb(img)
    lg2, bx2, _ = eng.forward_planar(ora.preprocess(img[0]))
    eng.close()
    assert rel(lg, lg2) < 1e-5 and rel(bx, bx2) < 1e-5


def test_detect_api_matches_oracle_selection(make_model):
    """rfdetr_detect end to end (C ABI): same detections as the oracle's
    postprocess of the engine's raw outputs (src/postprocess.cpp rules)."""
    import ctypes as C

    import oracle as O
    from rfdetr_b200 import lib

    path = make_model("tiny", "f16", 0)
    L = lib.lib()
    st = C.c_int(0)
    p = lib.Params(path.encode(), 1, lib.LOG_CB(), None)
    ctx = L.rfdetr_init(C.byref(p), C.byref(st))
    assert ctx and st.value == 0
    assert L.rfdetr_context_num_queries(ctx) == 40 and L.rfdetr_context_image_size(ctx) == 128
    img_np = np.random.default_rng(9).integers(0, 256, (200, 160, 3), dtype=np.uint8)
    img = L.rfdetr_image_from_rgb_buffer(img_np.ctypes.data, 160, 200, C.byref(st))
    dp = lib.DetectParams(0.5, 10, None, 0)
    out = C.POINTER(lib.Detection)()
    n = C.c_size_t(0)
    assert L.rfdetr_detect(ctx, img, C.byref(dp), C.byref(out), C.byref(n)) == 0
    dets = [(out[i].class_id, out[i].score, out[i].x1, out[i].y1, out[i].x2, out[i].y2, out[i].class_name)
            for i in range(n.value)]
    L.rfdetr_detections_free(out, n)
    L.rfdetr_image_free(img)
    L.rfdetr_free(ctx)
    eng = lib.Engine(path)
    lg, bx, _ = eng.forward_rgb(img_np[None])
    eng.close()
    q, c, s, xy = O.select(lg[0], bx[0], 0.5, 10, 160, 200)
    assert len(dets) == len(q) and len(dets) > 0
    for d, ci, si, box in zip(dets, c, s, xy):
        assert d[0] == ci and abs(d[1] - si) < 1e-6
        assert np.allclose(d[2:6], box, atol=1e-3)
        assert d[6] is not None


def test_detect_batch_matches_per_run_forwards(make_model):
    """rfdetr_b200_detect_batch over images of two sizes (a run of two, then one): each image's
    records equal the oracle's selection from the forward of its run; an empty list returns OK,
    and a missing image returns RFDETR_ERR_INVALID_ARG with every output cleared."""
    import ctypes as C

    import oracle as O
    from rfdetr_b200 import lib

    path = make_model("tiny", "f16", 0)
    L = lib.lib()
    eng = lib.Engine(path, max_batch=2)
    rng = np.random.default_rng(17)
    arrs = [rng.integers(0, 256, (200, 160, 3), dtype=np.uint8) for _ in range(2)]
    arrs.append(rng.integers(0, 256, (96, 144, 3), dtype=np.uint8))
    st = C.c_int(0)
    imgs = [L.rfdetr_image_from_rgb_buffer(a.ctypes.data, a.shape[1], a.shape[0], C.byref(st)) for a in arrs]
    assert all(imgs)
    dp = lib.DetectParams(0.3, 10, None, 0)
    dets = (C.POINTER(lib.Detection) * 3)()
    counts = (C.c_size_t * 3)()
    assert L.rfdetr_b200_detect_batch(eng.ctx, (C.c_void_p * 3)(*imgs), 3, C.byref(dp), dets, counts) == 0
    got = [[(dets[b][i].class_id, dets[b][i].score, dets[b][i].x1, dets[b][i].y1, dets[b][i].x2, dets[b][i].y2)
            for i in range(counts[b])] for b in range(3)]
    for b in range(3):
        L.rfdetr_detections_free(dets[b], counts[b])

    lg2, bx2, _ = eng.forward_rgb(np.stack(arrs[:2]))
    lg1, bx1, _ = eng.forward_rgb(arrs[2][None])
    want = [O.select(lg2[0], bx2[0], 0.3, 10, 160, 200), O.select(lg2[1], bx2[1], 0.3, 10, 160, 200),
            O.select(lg1[0], bx1[0], 0.3, 10, 144, 96)]
    assert sum(len(g) for g in got) > 0
    for g, (q, c, s, xy) in zip(got, want):
        assert len(g) == len(q)
        for d, ci, si, box in zip(g, c, s, xy):
            assert d[0] == ci and abs(d[1] - si) < 1e-6
            assert np.allclose(d[2:6], box, atol=1e-3)

    assert L.rfdetr_b200_detect_batch(eng.ctx, (C.c_void_p * 1)(), 0, C.byref(dp), dets, counts) == 0
    bad_dets = (C.POINTER(lib.Detection) * 2)()
    bad_counts = (C.c_size_t * 2)(7, 7)
    assert L.rfdetr_b200_detect_batch(eng.ctx, (C.c_void_p * 2)(imgs[0], None), 2, C.byref(dp), bad_dets,
                                      bad_counts) == -1
    assert not bad_dets[0] and not bad_dets[1] and list(bad_counts) == [0, 0]
    for im in imgs:
        L.rfdetr_image_free(im)
    eng.close()


def test_legacy_resize_mode(tmp_path):
    """A model whose rfdetr.preprocess.resize_mode is legacy_stb resizes images that are not at the
    model size with the library's resize (src/image_io.cpp:249-275): its forward of a 200 x 160
    image equals, bit for bit, its forward of that image resized by rfdetr_b200_op_resize_legacy,
    and differs from the 1.9 bilinear model's; at the model size both modes are the identity."""
    import torch
    from rfdetr_b200 import lib, synth

    paths = {}
    for mode in ("legacy_stb", "bilinear_no_antialias"):
        cfg = synth.get_variant("tiny")
        cfg["resize_mode"] = mode
        paths[mode] = str(tmp_path / f"{mode}.gguf")
        synth.write_gguf(paths[mode], "tiny", cfg, synth.make_state(synth.get_variant("tiny"), 0), "f16")
    legacy = lib.Engine(paths["legacy_stb"], max_batch=2)
    bilinear = lib.Engine(paths["bilinear_no_antialias"], max_batch=2)
    S = legacy.image_size
    img = np.random.default_rng(77).integers(0, 256, (2, 160, 200, 3), dtype=np.uint8)
    lg, bx, _ = legacy.forward_rgb(img)
    src = torch.from_numpy(img).cuda()
    dst = torch.zeros((2, S, S, 3), dtype=torch.uint8, device="cuda:0")
    L = lib.lib()
    assert L.rfdetr_b200_op_resize_legacy(src.data_ptr(), 2, 200, 160, dst.data_ptr(), S, S,
                                          torch.cuda.current_stream().cuda_stream) == 0
    lg2, bx2, _ = legacy.forward_rgb(dst.cpu().numpy())
    assert np.array_equal(lg, lg2) and np.array_equal(bx, bx2)
    lg3, _, _ = bilinear.forward_rgb(img)
    assert not np.array_equal(lg, lg3)
    same = _images(S, 2, 78)
    assert np.array_equal(legacy.forward_rgb(same)[0], bilinear.forward_rgb(same)[0])
    legacy.close()
    bilinear.close()


def test_flat_capi_with_png_and_seg_masks(make_model, tmp_path):
    """LocalAI's flat API (rfdetr_capi_*) on a segmentation model: JSON
    envelope, accessors, two-call sizing, PNG masks at the image size, and
    clearing of the previous batch on a failed detect (tests/test_capi_flat.cpp,
    tests/test_capi_accessors.cpp)."""
    import ctypes as C
    import json
    import struct
    import zlib

    from rfdetr_b200 import lib

    path = make_model("seg-tiny", "f16", 0)
    L = lib.lib()
    h = C.c_size_t(0)
    assert L.rfdetr_capi_load(path.encode(), 1, C.byref(h)) == 0 and h.value
    rgb = np.random.default_rng(3).integers(0, 256, (64, 80, 3), dtype=np.uint8)
    rows = b"".join(b"\x00" + rgb[y].tobytes() for y in range(64))

    def chunk(t, d):
        return struct.pack(">I", len(d)) + t + d + struct.pack(">I", zlib.crc32(t + d) & 0xFFFFFFFF)
    png = (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", 80, 64, 8, 2, 0, 0, 0)) +
           chunk(b"IDAT", zlib.compress(rows)) + chunk(b"IEND", b""))
    out = C.c_void_p()
    assert L.rfdetr_capi_detect_buffer(h, png, len(png), 0.3, 5, C.byref(out)) == 0
    js = json.loads(C.string_at(out).decode())
    L.rfdetr_capi_free_string(out)
    assert js["status"] == "ok" and js["image"] == {"width": 80, "height": 64}
    n = L.rfdetr_capi_get_n_detections(h)
    assert n == len(js["detections"]) and 0 < n <= 5
    xy = (C.c_float * 4)()
    for i in range(n):
        assert L.rfdetr_capi_get_detection_box(h, i, xy) == 0
        assert abs(xy[0] - js["detections"][i]["x1"]) < 1e-2
        need = L.rfdetr_capi_get_detection_class_name(h, i, None, 0)
        buf = C.create_string_buffer(need)
        assert L.rfdetr_capi_get_detection_class_name(h, i, buf, need) == need
        msz = L.rfdetr_capi_get_detection_mask_png(h, i, None, 0)
        assert msz > 0
        mbuf = (C.c_ubyte * msz)()
        assert L.rfdetr_capi_get_detection_mask_png(h, i, mbuf, msz) == msz
        mp = bytes(mbuf)
        assert mp[:8] == b"\x89PNG\r\n\x1a\n" and struct.unpack(">II", mp[16:24]) == (80, 64)
    assert L.rfdetr_capi_get_detection_class_id(h, n) == -1
    # a failed detect clears the previous batch
    assert L.rfdetr_capi_detect_buffer(h, b"not an image", 12, 0.3, 5, C.byref(out)) != 0
    assert L.rfdetr_capi_get_n_detections(h) == 0
    assert L.rfdetr_capi_unload(h) == 0


_FAULT_CHILD = r'''
import ctypes as C, sys
import numpy as np
sys.path.insert(0, sys.argv[2])
from rfdetr_b200 import lib
L = lib.lib()
eng = lib.Engine(sys.argv[1], max_batch=2)
rng = np.random.default_rng(5)
arrs = [rng.integers(0, 256, (200, 160, 3), dtype=np.uint8), rng.integers(0, 256, (96, 144, 3), dtype=np.uint8)]
st = C.c_int(0)
imgs = [L.rfdetr_image_from_rgb_buffer(a.ctypes.data, a.shape[1], a.shape[0], C.byref(st)) for a in arrs]
dp = lib.DetectParams(0.0, 5, None, 0)   # threshold 0: every image has detections
dets = (C.POINTER(lib.Detection) * 2)()
counts = (C.c_size_t * 2)(7, 7)
# two runs (two sizes): the first run's post-processing succeeds, the second throws after handing out an array
rc = L.rfdetr_b200_detect_batch(eng.ctx, (C.c_void_p * 2)(*imgs), 2, C.byref(dp), dets, counts)
print("batch", rc, bool(dets[0]), bool(dets[1]), list(counts))
out = C.POINTER(lib.Detection)()
n = C.c_size_t(9)
rc1 = L.rfdetr_detect(eng.ctx, imgs[0], C.byref(dp), C.byref(out), C.byref(n))   # third call: no fault
print("detect", rc1, bool(out), n.value)
L.rfdetr_detections_free(out, n.value)
for im in imgs:
    L.rfdetr_image_free(im)
eng.close()
'''


def test_postprocess_allocation_failure_releases_every_array(make_model, tmp_path):
    """An allocation failure thrown while detection arrays are being built (injected on the host:
    RFDETR_FAULT_INJECT=postprocess_alloc:2 makes the second post-processing call of the process throw
    std::bad_alloc after its first array is handed out) ends rfdetr_b200_detect_batch with
    RFDETR_ERR_OUT_OF_MEMORY and every output cleared, the arrays of the run before it included, and
    the context keeps working (a later rfdetr_detect succeeds).  Runs in a child process so the
    injection counter starts at zero."""
    import subprocess
    import sys

    path = make_model("tiny", "f16", 0)
    script = tmp_path / "fault_child.py"
    script.write_text(_FAULT_CHILD)
    env = dict(os.environ, RFDETR_FAULT_INJECT="postprocess_alloc:2")
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rf-detr.cpp_b200")
    r = subprocess.run([sys.executable, str(script), path, pkg], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = dict(line.split(" ", 1) for line in r.stdout.strip().splitlines())
    assert lines["batch"] == "-4 False False [0, 0]", r.stdout   # RFDETR_ERR_OUT_OF_MEMORY
    rc1, has, n = lines["detect"].split()
    assert rc1 == "0" and has == "True" and int(n) > 0
