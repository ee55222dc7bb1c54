"""Seeded synthetic RF-DETR models written as GGUF (format v2).

There are no real checkpoints on this machine, so every model the engine is
tested or timed on is generated here: a seeded random state dict with the exact
tensor inventory, shapes and dtype rules of the reference converter, written
with the same `gguf` package calls in the same order.

Reference behaviour restated here (paths are within localai-org/rf-detr.cpp):

* variant table .................. scripts/convert_rfdetr_to_gguf.py:76-205
* tensor name map + transforms ... scripts/convert_rfdetr_to_gguf.py:265-460
* which tensors get quantized .... scripts/convert_rfdetr_to_gguf.py:463-498
* metadata keys and order ........ scripts/convert_rfdetr_to_gguf.py:509-679
* Q4_K files (F32 file re-quantized, K-quant -> Q8_0 fallback for rows whose
  length is not a multiple of 256) examples/cli/main.cpp:344-541, with the
  Q4_K block quantizer of ggml (quantize_row_q4_K_ref / make_qkx2_quants,
  ggml-quants.c; ggml itself is an un-vendored submodule of the reference, so
  the algorithm is restated from its published source, see `quantize_q4_K`).

Weight initialisation (fixed by the benchmark description): linear weights
N(0, 0.02), biases 0, LayerNorm gamma 1 / beta 0; conv kernels, cls token,
pos-embed, query features and refpoints N(0, 0.02); layer scales 1.0; the
segmentation scalar bias 0.
"""
from __future__ import annotations

import copy
from collections import OrderedDict

import numpy as np

FORMAT_VERSION = "2"


def _variant(*, image_size, patch_size, num_windows, global_attn_indices,
             out_feature_indices, pos_embed_train_size, dec_layers,
             num_queries=300, segmentation_head=False, mask_downsample_ratio=4):
    return {
        "image_size": image_size,
        "patch_size": patch_size,
        "num_queries": num_queries,
        "group_detr": 13,
        "num_classes": 91,
        "segmentation_head": segmentation_head,
        "mask_downsample_ratio": mask_downsample_ratio,
        "backbone": {
            "dim": 384, "depth": 12, "heads": 6, "ffn_dim": 1536,
            "num_windows": num_windows,
            "global_attn_indices": list(global_attn_indices),
            "out_feature_indices": list(out_feature_indices),
            "pos_embed_train_size": pos_embed_train_size,
        },
        "projector": {"in_dim": 1536, "out_dim": 256, "bottleneck_dim": 128,
                      "n_bottlenecks": 3},
        "decoder": {"layers": dec_layers, "model_dim": 256, "ffn_dim": 2048,
                    "self_attn_heads": 8, "cross_attn_heads": 16,
                    "cross_attn_n_levels": 1, "cross_attn_n_points": 2},
        "two_stage": {"n_groups": 13},
    }


_G369 = [3, 6, 9]
_O3612 = [3, 6, 9, 12]

# The published variants (scripts/convert_rfdetr_to_gguf.py:125-205).
VARIANTS = {
    "nano": _variant(image_size=384, patch_size=16, num_windows=2, global_attn_indices=_G369,
                     out_feature_indices=_O3612, pos_embed_train_size=24, dec_layers=2),
    "small": _variant(image_size=512, patch_size=16, num_windows=2, global_attn_indices=_G369,
                      out_feature_indices=_O3612, pos_embed_train_size=32, dec_layers=3),
    "base": _variant(image_size=560, patch_size=14, num_windows=4,
                     global_attn_indices=[2, 5, 8, 11], out_feature_indices=[2, 5, 8, 11],
                     pos_embed_train_size=37, dec_layers=3),
    "medium": _variant(image_size=576, patch_size=16, num_windows=2, global_attn_indices=_G369,
                       out_feature_indices=_O3612, pos_embed_train_size=36, dec_layers=4),
    "large": _variant(image_size=704, patch_size=16, num_windows=2, global_attn_indices=_G369,
                      out_feature_indices=_O3612, pos_embed_train_size=44, dec_layers=4),
    "seg-nano": _variant(image_size=312, patch_size=12, num_windows=1, global_attn_indices=_G369,
                         out_feature_indices=_O3612, pos_embed_train_size=26, dec_layers=4,
                         num_queries=100, segmentation_head=True),
    "seg-small": _variant(image_size=384, patch_size=12, num_windows=2, global_attn_indices=_G369,
                          out_feature_indices=_O3612, pos_embed_train_size=32, dec_layers=4,
                          num_queries=100, segmentation_head=True),
    "seg-medium": _variant(image_size=432, patch_size=12, num_windows=2, global_attn_indices=_G369,
                           out_feature_indices=_O3612, pos_embed_train_size=36, dec_layers=5,
                           num_queries=200, segmentation_head=True),
    "seg-large": _variant(image_size=504, patch_size=12, num_windows=2, global_attn_indices=_G369,
                          out_feature_indices=_O3612, pos_embed_train_size=42, dec_layers=5,
                          num_queries=200, segmentation_head=True),
    "seg-xlarge": _variant(image_size=624, patch_size=12, num_windows=2, global_attn_indices=_G369,
                           out_feature_indices=_O3612, pos_embed_train_size=52, dec_layers=6,
                           num_queries=300, segmentation_head=True),
    "seg-2xlarge": _variant(image_size=768, patch_size=12, num_windows=2, global_attn_indices=_G369,
                            out_feature_indices=_O3612, pos_embed_train_size=64, dec_layers=6,
                            num_queries=300, segmentation_head=True),
}

# Small test-only variants with the real channel widths and head sizes but
# tiny grids, so the CPU oracle finishes in well under a second.
TEST_VARIANTS = {
    # 128 px / 16 -> 8x8 grid, 2x2 windows of 4x4 (+CLS = 17 tokens).
    "tiny": _variant(image_size=128, patch_size=16, num_windows=2, global_attn_indices=_G369,
                     out_feature_indices=_O3612, pos_embed_train_size=6, dec_layers=2,
                     num_queries=40),
    # Base-like: 4x4 windows and Base's taps, 112 px / 14 -> 8x8 grid.
    "tiny-base": _variant(image_size=112, patch_size=14, num_windows=4,
                          global_attn_indices=[2, 5, 8, 11], out_feature_indices=[2, 5, 8, 11],
                          pos_embed_train_size=10, dec_layers=3, num_queries=48),
    # Segmentation: 96 px / 12 -> 8x8 grid, 24x24 masks.
    "seg-tiny": _variant(image_size=96, patch_size=12, num_windows=2, global_attn_indices=_G369,
                         out_feature_indices=_O3612, pos_embed_train_size=8, dec_layers=2,
                         num_queries=30, segmentation_head=True),
    # 52x52 grid: the only size class where the two-stage proposal mask fires.
    "grid52": _variant(image_size=624, patch_size=12, num_windows=2, global_attn_indices=_G369,
                       out_feature_indices=_O3612, pos_embed_train_size=16, dec_layers=2,
                       num_queries=100),
}


def get_variant(name: str) -> dict:
    if name in VARIANTS:
        return copy.deepcopy(VARIANTS[name])
    if name in TEST_VARIANTS:
        return copy.deepcopy(TEST_VARIANTS[name])
    raise KeyError(f"unknown variant {name!r}")


# 91-slot COCO logit table (scripts/convert_rfdetr_to_gguf.py:207-239).
_COCO = {1: "person", 2: "bicycle", 3: "car", 4: "motorcycle", 5: "airplane", 6: "bus",
         7: "train", 8: "truck", 9: "boat", 10: "traffic light", 11: "fire hydrant",
         13: "stop sign", 14: "parking meter", 15: "bench", 16: "bird", 17: "cat", 18: "dog",
         19: "horse", 20: "sheep", 21: "cow", 22: "elephant", 23: "bear", 24: "zebra",
         25: "giraffe", 27: "backpack", 28: "umbrella", 31: "handbag", 32: "tie",
         33: "suitcase", 34: "frisbee", 35: "skis", 36: "snowboard", 37: "sports ball",
         38: "kite", 39: "baseball bat", 40: "baseball glove", 41: "skateboard",
         42: "surfboard", 43: "tennis racket", 44: "bottle", 46: "wine glass", 47: "cup",
         48: "fork", 49: "knife", 50: "spoon", 51: "bowl", 52: "banana", 53: "apple",
         54: "sandwich", 55: "orange", 56: "broccoli", 57: "carrot", 58: "hot dog",
         59: "pizza", 60: "donut", 61: "cake", 62: "chair", 63: "couch", 64: "potted plant",
         65: "bed", 67: "dining table", 70: "toilet", 72: "tv", 73: "laptop", 74: "mouse",
         75: "remote", 76: "keyboard", 77: "cell phone", 78: "microwave", 79: "oven",
         80: "toaster", 81: "sink", 82: "refrigerator", 84: "book", 85: "clock", 86: "vase",
         87: "scissors", 88: "teddy bear", 89: "hair drier", 90: "toothbrush"}
COCO_CLASS_NAMES = [_COCO.get(i, "") for i in range(91)]


# --------------------------------------------------------------------------
# Tensor inventory.  Each entry: gguf name -> (torch shape, init kind, transform)
# init kinds: "w" N(0,0.02), "zero", "one".  Transforms follow the converter:
# slice_first_300, squeeze_cls, squeeze_pos.
# --------------------------------------------------------------------------

def tensor_specs(cfg: dict) -> "OrderedDict[str, tuple]":
    bb = cfg["backbone"]
    pj = cfg["projector"]
    dc = cfg["decoder"]
    D, F = bb["dim"], bb["ffn_dim"]
    p = cfg["patch_size"]
    ts = bb["pos_embed_train_size"]
    C, Cb = pj["out_dim"], pj["bottleneck_dim"]
    Dm, Fd = dc["model_dim"], dc["ffn_dim"]
    NC = cfg["num_classes"]
    nq_all = 300 * cfg["group_detr"]
    so = dc["cross_attn_heads"] * dc["cross_attn_n_levels"] * dc["cross_attn_n_points"] * 2
    aw = dc["cross_attn_heads"] * dc["cross_attn_n_levels"] * dc["cross_attn_n_points"]

    s: "OrderedDict[str, tuple]" = OrderedDict()

    def lin(name, out_f, in_f):
        s[name + ".weight"] = ((out_f, in_f), "w", None)
        s[name + ".bias"] = ((out_f,), "zero", None)

    def ln(name, n):
        s[name + ".weight"] = ((n,), "one", None)
        s[name + ".bias"] = ((n,), "zero", None)

    s["backbone.patch_embed.weight"] = ((D, 3, p, p), "w", None)
    s["backbone.patch_embed.bias"] = ((D,), "zero", None)
    s["backbone.cls_token"] = ((1, 1, D), "w", "squeeze_cls")
    s["backbone.pos_embed"] = ((1, ts * ts + 1, D), "w", "squeeze_pos")
    for i in range(bb["depth"]):
        b = f"backbone.blocks.{i}."
        ln(b + "norm1", D)
        lin(b + "attn.q", D, D)
        lin(b + "attn.k", D, D)
        lin(b + "attn.v", D, D)
        lin(b + "attn.proj", D, D)
        s[b + "layer_scale1"] = ((D,), "one", None)
        ln(b + "norm2", D)
        lin(b + "mlp.fc1", F, D)
        lin(b + "mlp.fc2", D, F)
        s[b + "layer_scale2"] = ((D,), "one", None)
    ln("backbone.norm", D)

    n_levels = len(bb["out_feature_indices"])
    s["projector.cv1.conv.weight"] = ((C, n_levels * D, 1, 1), "w", None)
    ln("projector.cv1.norm", C)
    s["projector.cv2.conv.weight"] = ((C, (2 + pj["n_bottlenecks"]) * Cb, 1, 1), "w", None)
    ln("projector.cv2.norm", C)
    for j in range(pj["n_bottlenecks"]):
        b = f"projector.bottleneck.{j}."
        s[b + "cv1.conv.weight"] = ((Cb, Cb, 3, 3), "w", None)
        ln(b + "cv1.norm", Cb)
        s[b + "cv2.conv.weight"] = ((Cb, Cb, 3, 3), "w", None)
        ln(b + "cv2.norm", Cb)
    ln("projector.final_norm", C)

    for g in range(cfg["two_stage"]["n_groups"]):
        lin(f"two_stage.enc_output.{g}", Dm, Dm)
        ln(f"two_stage.enc_output_norm.{g}", Dm)
        lin(f"two_stage.enc_out_class_embed.{g}", NC, Dm)
        lin(f"two_stage.enc_out_bbox_embed.{g}.layers.0", Dm, Dm)
        lin(f"two_stage.enc_out_bbox_embed.{g}.layers.1", Dm, Dm)
        lin(f"two_stage.enc_out_bbox_embed.{g}.layers.2", 4, Dm)

    s["decoder.queries.feat"] = ((nq_all, Dm), "w", "slice_first_300")
    s["decoder.queries.refpoints"] = ((nq_all, 4), "w", "slice_first_300")
    lin("decoder.ref_point_head.layers.0", Dm, 2 * Dm)
    lin("decoder.ref_point_head.layers.1", Dm, Dm)
    for i in range(dc["layers"]):
        b = f"decoder.layers.{i}."
        s[b + "self_attn.in_proj.weight"] = ((3 * Dm, Dm), "w", None)
        s[b + "self_attn.in_proj.bias"] = ((3 * Dm,), "zero", None)
        lin(b + "self_attn.out_proj", Dm, Dm)
        ln(b + "norm1", Dm)
        lin(b + "cross_attn.sampling_offsets", so, Dm)
        lin(b + "cross_attn.attention_weights", aw, Dm)
        lin(b + "cross_attn.value_proj", Dm, Dm)
        lin(b + "cross_attn.output_proj", Dm, Dm)
        ln(b + "norm2", Dm)
        lin(b + "linear1", Fd, Dm)
        lin(b + "linear2", Dm, Fd)
        ln(b + "norm3", Dm)
    ln("decoder.norm", Dm)

    lin("heads.class_embed", NC, Dm)
    lin("heads.bbox_embed.layers.0", Dm, Dm)
    lin("heads.bbox_embed.layers.1", Dm, Dm)
    lin("heads.bbox_embed.layers.2", 4, Dm)

    if cfg.get("segmentation_head", False):
        for b in range(dc["layers"]):
            sp = f"segmentation_head.blocks.{b}."
            s[sp + "dwconv.weight"] = ((Dm, 1, 3, 3), "w", None)
            s[sp + "dwconv.bias"] = ((Dm,), "zero", None)
            ln(sp + "norm", Dm)
            lin(sp + "pwconv1", Dm, Dm)
        s["segmentation_head.spatial_features_proj.weight"] = ((Dm, Dm, 1, 1), "w", None)
        s["segmentation_head.spatial_features_proj.bias"] = ((Dm,), "zero", None)
        ln("segmentation_head.query_features_block.norm_in", Dm)
        lin("segmentation_head.query_features_block.layers.0", 4 * Dm, Dm)
        lin("segmentation_head.query_features_block.layers.2", Dm, 4 * Dm)
        lin("segmentation_head.query_features_proj", Dm, Dm)
        s["segmentation_head.bias"] = ((1,), "zero", None)
    return s


def apply_transform(arr: np.ndarray, tag):
    if tag is None:
        return arr
    if tag == "slice_first_300":
        return arr[:300]
    if tag == "squeeze_cls":
        return arr.reshape(-1)
    if tag == "squeeze_pos":
        return arr[0]
    raise ValueError(tag)


def make_torch_state(cfg: dict, seed: int) -> "OrderedDict[str, np.ndarray]":
    """Seeded tensors in torch (pre-transform) shapes, keyed by GGUF name."""
    rng = np.random.default_rng(seed)
    out: "OrderedDict[str, np.ndarray]" = OrderedDict()
    for name, (shape, kind, _t) in tensor_specs(cfg).items():
        if kind == "w":
            a = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        elif kind == "one":
            a = np.ones(shape, np.float32)
        else:
            a = np.zeros(shape, np.float32)
        out[name] = a
    return out


def make_state(cfg: dict, seed: int) -> "OrderedDict[str, np.ndarray]":
    """Seeded tensors after the converter transforms (what gets written)."""
    specs = tensor_specs(cfg)
    return OrderedDict((k, np.ascontiguousarray(apply_transform(v, specs[k][2])))
                       for k, v in make_torch_state(cfg, seed).items())


_SKIP = {"backbone.pos_embed", "decoder.queries.feat", "decoder.queries.refpoints"}


def should_quantize(name: str, arr: np.ndarray) -> bool:
    """2-D `.weight` tensors with both dims >= 64, embeddings excluded
    (scripts/convert_rfdetr_to_gguf.py:463-498)."""
    if not name.endswith(".weight"):
        return False
    if arr.ndim != 2:
        return False
    if arr.shape[0] < 64 or arr.shape[1] < 64:
        return False
    if name in _SKIP:
        return False
    return arr.shape[-1] % 32 == 0


# --------------------------------------------------------------------------
# Q4_K block quantizer (ggml quantize_row_q4_K_ref without an importance
# matrix).  Vectorised over all 32-element sub-blocks; every float operation is
# float32 and sums run in the same sequential order as the C loops.
# Block layout (144 bytes per 256 values): f16 d, f16 dmin, 12 bytes of packed
# 6-bit sub-block scales/mins, 128 bytes of 4-bit quants.
# --------------------------------------------------------------------------

def _nearest_int(v: np.ndarray) -> np.ndarray:
    return np.rint(v).astype(np.int32)


def _make_qkx2(x: np.ndarray, w: np.ndarray, nmax=15, rmin=-1.0, rdelta=0.1, nstep=20):
    f32 = np.float32
    n = x.shape[1]
    mn = x.min(axis=1).astype(f32)
    mx = x.max(axis=1).astype(f32)
    sum_w = w[:, 0].copy()
    sum_x = (sum_w * x[:, 0]).astype(f32)
    for i in range(1, n):
        sum_w = (sum_w + w[:, i]).astype(f32)
        sum_x = (sum_x + w[:, i] * x[:, i]).astype(f32)
    mn = np.minimum(mn, f32(0))
    flat = mx == mn
    rng_ = np.where(flat, f32(1), mx - mn).astype(f32)
    iscale = (f32(nmax) / rng_).astype(f32)
    scale = (f32(1) / iscale).astype(f32)
    L = np.clip(_nearest_int(iscale[:, None] * (x - mn[:, None])), 0, nmax)
    diff = (scale[:, None] * L.astype(f32) + mn[:, None] - x).astype(f32)
    best = np.zeros(x.shape[0], f32)
    for i in range(n):
        best = (best + w[:, i] * (diff[:, i] * diff[:, i])).astype(f32)
    the_min = mn.copy()
    for st in range(nstep + 1):
        isc = ((f32(rmin) + f32(rdelta) * f32(st) + f32(nmax)) / rng_).astype(f32)
        La = np.clip(_nearest_int(isc[:, None] * (x - mn[:, None])), 0, nmax)
        Lf = La.astype(f32)
        sl = np.zeros(x.shape[0], f32)
        sl2 = np.zeros(x.shape[0], f32)
        sxl = np.zeros(x.shape[0], f32)
        for i in range(n):
            wl = (w[:, i] * Lf[:, i]).astype(f32)
            sl = (sl + wl).astype(f32)
            sl2 = (sl2 + wl * Lf[:, i]).astype(f32)
            sxl = (sxl + wl * x[:, i]).astype(f32)
        D = (sum_w * sl2 - sl * sl).astype(f32)
        ok = D > 0
        Ds = np.where(ok, D, f32(1)).astype(f32)
        this_scale = ((sum_w * sxl - sum_x * sl) / Ds).astype(f32)
        this_min = ((sl2 * sum_x - sl * sxl) / Ds).astype(f32)
        pos = this_min > 0
        sl2s = np.where(sl2 == 0, f32(1), sl2).astype(f32)
        this_scale = np.where(pos, (sxl / sl2s).astype(f32), this_scale)
        this_min = np.where(pos, f32(0), this_min)
        d2 = (this_scale[:, None] * Lf + this_min[:, None] - x).astype(f32)
        mad = np.zeros(x.shape[0], f32)
        for i in range(n):
            mad = (mad + w[:, i] * (d2[:, i] * d2[:, i])).astype(f32)
        upd = ok & (mad < best)
        L = np.where(upd[:, None], La, L)
        best = np.where(upd, mad, best)
        scale = np.where(upd, this_scale, scale)
        the_min = np.where(upd, this_min, the_min)
    scale = np.where(flat, f32(0), scale)
    the_min = np.where(flat, mn, the_min)
    return scale.astype(f32), (-the_min).astype(f32)


def quantize_q4_K(a: np.ndarray) -> np.ndarray:
    """Quantize rows (last dim multiple of 256) to Q4_K bytes, shape (..., n/256*144)."""
    f32 = np.float32
    a = np.ascontiguousarray(a, dtype=f32)
    n = a.shape[-1]
    assert n % 256 == 0
    sb = a.reshape(-1, 32)  # sub-blocks in order
    sum_x2 = np.zeros(sb.shape[0], f32)
    for i in range(32):
        sum_x2 = (sum_x2 + sb[:, i] * sb[:, i]).astype(f32)
    av = np.sqrt((sum_x2 / f32(32)).astype(f32)).astype(f32)
    w = (av[:, None] + np.abs(sb)).astype(f32)
    scales, mins = _make_qkx2(sb, w)
    nblk = sb.shape[0] // 8
    scales = scales.reshape(nblk, 8)
    mins = mins.reshape(nblk, 8)
    max_scale = np.zeros(nblk, f32)
    max_min = np.zeros(nblk, f32)
    for j in range(8):
        max_scale = np.where(scales[:, j] > max_scale, scales[:, j], max_scale)
        max_min = np.where(mins[:, j] > max_min, mins[:, j], max_min)
    inv_scale = np.where(max_scale > 0, f32(63) / np.where(max_scale > 0, max_scale, f32(1)), f32(0)).astype(f32)
    inv_min = np.where(max_min > 0, f32(63) / np.where(max_min > 0, max_min, f32(1)), f32(0)).astype(f32)
    ls = np.minimum(63, _nearest_int((inv_scale[:, None] * scales).astype(f32))).astype(np.uint8)
    lm = np.minimum(63, _nearest_int((inv_min[:, None] * mins).astype(f32))).astype(np.uint8)
    sc = np.zeros((nblk, 12), np.uint8)
    for j in range(8):
        if j < 4:
            sc[:, j] = ls[:, j]
            sc[:, j + 4] = lm[:, j]
        else:
            sc[:, j + 4] = (ls[:, j] & 0xF) | ((lm[:, j] & 0xF) << 4)
            sc[:, j - 4] |= (ls[:, j] >> 4) << 6
            sc[:, j] |= (lm[:, j] >> 4) << 6
    d16 = (max_scale / f32(63)).astype(np.float16)
    dmin16 = (max_min / f32(63)).astype(np.float16)
    d = d16.astype(f32)
    dmin = dmin16.astype(f32)
    xb = sb.reshape(nblk, 8, 32)
    L = np.zeros((nblk, 8, 32), np.uint8)
    for j in range(8):
        if j < 4:
            s_ = sc[:, j] & 63
            m_ = sc[:, j + 4] & 63
        else:
            s_ = (sc[:, j + 4] & 0xF) | ((sc[:, j - 4] >> 6) << 4)
            m_ = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
        dj = (d * s_.astype(f32)).astype(f32)
        dmj = (dmin * m_.astype(f32)).astype(f32)
        nz = dj != 0
        djs = np.where(nz, dj, f32(1))
        l = _nearest_int(((xb[:, j, :] + dmj[:, None]) / djs[:, None]).astype(f32))
        l = np.clip(l, 0, 15).astype(np.uint8)
        L[:, j, :] = np.where(nz[:, None], l, 0)
    Lf = L.reshape(nblk, 256)
    qs = np.zeros((nblk, 128), np.uint8)
    for t in range(4):
        lo = Lf[:, 64 * t: 64 * t + 32]
        hi = Lf[:, 64 * t + 32: 64 * t + 64]
        qs[:, 32 * t: 32 * t + 32] = lo | (hi << 4)
    out = np.concatenate([d16.view(np.uint8).reshape(nblk, 2), dmin16.view(np.uint8).reshape(nblk, 2),
                          sc, qs], axis=1)
    return out.reshape(*a.shape[:-1], (n // 256) * 144)


def dequantize_q4_K(q: np.ndarray, n: int) -> np.ndarray:
    """Reference-style Q4_K dequantization (inverse of the layout above)."""
    f32 = np.float32
    b = q.reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(f32)[:, 0]
    dmin = b[:, 2:4].copy().view(np.float16).astype(f32)[:, 0]
    sc = b[:, 4:16]
    qs = b[:, 16:144]
    out = np.zeros((b.shape[0], 256), f32)
    for j in range(8):
        if j < 4:
            s_ = sc[:, j] & 63
            m_ = sc[:, j + 4] & 63
        else:
            s_ = (sc[:, j + 4] & 0xF) | ((sc[:, j - 4] >> 6) << 4)
            m_ = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
        t, half = divmod(j, 2)
        nib = (qs[:, 32 * t: 32 * t + 32] >> (4 * half)) & 0xF
        out[:, 32 * j: 32 * j + 32] = (d * s_.astype(f32))[:, None] * nib.astype(f32) - (dmin * m_.astype(f32))[:, None]
    return out.reshape(-1)[: q.size // 144 * 256]


# --------------------------------------------------------------------------
# GGUF writing
# --------------------------------------------------------------------------

DTYPES = ("f32", "f16", "q8_0", "q4_K")


def _tensor_type_for(dtype: str, name: str, arr: np.ndarray):
    """Return one of 'f32', 'f16', 'q8_0', 'q4_K' for a tensor under a file dtype."""
    if dtype == "f32":
        return "f32"
    q = should_quantize(name, arr)
    if dtype == "f16":
        return "f16" if q else "f32"
    if dtype == "q8_0":
        return "q8_0" if q else "f32"
    if dtype == "q4_K":
        # rfdetr-cli quantize: ne[0] (= numpy last dim) % 256 == 0 -> Q4_K,
        # else Q8_0 when it is a multiple of 32 (examples/cli/main.cpp:466-515).
        if not q:
            return "f32"
        return "q4_K" if arr.shape[-1] % 256 == 0 else "q8_0"
    raise ValueError(dtype)


def write_gguf(path: str, variant_name: str, cfg: dict, state: "OrderedDict[str, np.ndarray]",
               dtype: str) -> dict:
    """Write `state` as an RF-DETR format-v2 GGUF. Returns {name: tensor type}."""
    import gguf as G

    w = G.GGUFWriter(path, arch="rfdetr")
    w.add_string("rfdetr.format.version", FORMAT_VERSION)
    w.add_string("rfdetr.variant", variant_name)
    w.add_uint32("rfdetr.image_size", cfg["image_size"])
    w.add_uint32("rfdetr.patch_size", cfg["patch_size"])
    w.add_uint32("rfdetr.num_queries", cfg["num_queries"])
    w.add_uint32("rfdetr.group_detr", cfg["group_detr"])
    w.add_uint32("rfdetr.num_classes", cfg["num_classes"])
    names = COCO_CLASS_NAMES if cfg["num_classes"] == 91 else [f"class_{i}" for i in range(cfg["num_classes"])]
    w.add_array("rfdetr.class_names", names)
    w.add_array("rfdetr.preprocess.mean", np.array([0.485, 0.456, 0.406], np.float32).tolist())
    w.add_array("rfdetr.preprocess.std", np.array([0.229, 0.224, 0.225], np.float32).tolist())
    mode = cfg.get("resize_mode", "bilinear_no_antialias")
    if mode is not None:  # None: no key, as in files converted before it existed
        w.add_string("rfdetr.preprocess.resize_mode", mode)
    bb = cfg["backbone"]
    for k in ("dim", "depth", "heads", "ffn_dim", "num_windows"):
        w.add_uint32(f"rfdetr.backbone.{k}", bb[k])
    w.add_array("rfdetr.backbone.global_attn_indices", bb["global_attn_indices"])
    w.add_array("rfdetr.backbone.out_feature_indices", bb["out_feature_indices"])
    w.add_uint32("rfdetr.backbone.pos_embed_train_size", bb["pos_embed_train_size"])
    for k in ("in_dim", "out_dim", "bottleneck_dim", "n_bottlenecks"):
        w.add_uint32(f"rfdetr.projector.{k}", cfg["projector"][k])
    for k in ("layers", "model_dim", "ffn_dim", "self_attn_heads", "cross_attn_heads",
              "cross_attn_n_levels", "cross_attn_n_points"):
        w.add_uint32(f"rfdetr.decoder.{k}", cfg["decoder"][k])
    w.add_uint32("rfdetr.two_stage.n_groups", cfg["two_stage"]["n_groups"])
    is_seg = bool(cfg.get("segmentation_head", False))
    w.add_bool("rfdetr.has_segmentation_head", is_seg)
    if is_seg:
        w.add_uint32("rfdetr.mask_downsample_ratio", cfg["mask_downsample_ratio"])

    types = {}
    for name, arr in state.items():
        t = _tensor_type_for(dtype, name, arr)
        types[name] = t
        a32 = np.ascontiguousarray(arr, dtype=np.float32)
        if t == "f32":
            w.add_tensor(name, a32, raw_dtype=G.GGMLQuantizationType.F32)
        elif t == "f16":
            w.add_tensor(name, a32.astype(np.float16), raw_dtype=G.GGMLQuantizationType.F16)
        elif t == "q8_0":
            w.add_tensor(name, G.quants.quantize(a32, G.GGMLQuantizationType.Q8_0),
                         raw_dtype=G.GGMLQuantizationType.Q8_0)
        elif t == "q4_K":
            w.add_tensor(name, quantize_q4_K(a32), raw_dtype=G.GGMLQuantizationType.Q4_K)
        else:
            raise ValueError(t)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file(progress=False)
    w.close()
    return types


def write_model(path: str, variant: str, dtype: str = "f32", seed: int = 0,
                cfg_overrides: dict | None = None) -> dict:
    cfg = get_variant(variant)
    if cfg_overrides:
        cfg.update(cfg_overrides)
    state = make_state(cfg, seed)
    return write_gguf(path, variant, cfg, state, dtype)


# --------------------------------------------------------------------------
# Reading back (for the oracle): name -> float32 array in ggml ne order
# --------------------------------------------------------------------------

def read_gguf_f32(path: str):
    """Return (metadata dict, {name: (type_name, float32 ndarray in numpy/torch order)})."""
    import gguf as G
    r = G.GGUFReader(path)
    meta = {}
    for f in r.fields.values():
        if not f.name.startswith("rfdetr."):
            continue
        tp = f.types[0]
        if tp == G.GGUFValueType.STRING:
            meta[f.name] = bytes(f.parts[f.data[0]]).decode()
        elif tp == G.GGUFValueType.ARRAY:
            sub = f.types[1]
            if sub == G.GGUFValueType.STRING:
                meta[f.name] = [bytes(f.parts[i]).decode() for i in f.data]
            else:
                meta[f.name] = [f.parts[i].tolist()[0] for i in f.data]
        else:
            meta[f.name] = f.parts[f.data[0]].tolist()[0]
    tensors = {}
    for t in r.tensors:
        shape = tuple(int(x) for x in reversed(t.shape.tolist()))
        tn = t.tensor_type.name
        if tn == "Q4_K":
            arr = dequantize_q4_K(np.asarray(t.data).reshape(-1), int(np.prod(shape))).reshape(shape)
        else:
            arr = G.quants.dequantize(np.asarray(t.data), t.tensor_type).reshape(shape)
        tensors[t.name] = (tn, np.ascontiguousarray(arr, dtype=np.float32))
    return meta, tensors
