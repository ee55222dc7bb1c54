"""ctypes front-end of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Loads oracle/liboracle.so (a plain C++ restatement of the reference forward,
see oracle.h) and feeds it the dequantized tensors of a GGUF file.  Only the
test-suite, the smoke check and the CPU-baseline leg of bench.py use this; the
product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(REPO, "rf-detr.cpp_b200"))
from rfdetr_b200 import synth  # noqa: E402

# Weight storage type -> the oracle's activation-rounding class (mode 1): ggml's
# CPU dot products round activations to f16 for F16 weights, to Q8_0 blocks for
# Q8_0 weights and to Q8_K blocks for every K-quant (Q4_K, Q5_K, Q6_K).
TYPE_CODES = {"F32": 0, "F16": 1, "Q8_0": 2, "Q4_K": 3, "Q5_K": 3, "Q6_K": 3}


class OracleConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "image_size", "patch_size", "num_queries", "num_classes",
        "dim", "depth", "heads", "ffn_dim", "num_windows", "pos_train")] + [
        ("n_global", C.c_int), ("global_idx", C.c_int * 16),
        ("n_taps", C.c_int), ("tap_stage", C.c_int * 8)] + [(n, C.c_int) for n in (
            "proj_out", "proj_bneck", "proj_nb",
            "dec_layers", "dec_dim", "dec_ffn", "sa_heads", "ca_heads", "ca_points",
            "has_seg", "mask_ratio", "act_round", "n_threads")]


class OracleTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("data", C.POINTER(C.c_float)),
                ("n", C.c_int64), ("type", C.c_int)]


PUBLISH = C.CFUNCTYPE(None, C.c_char_p, C.POINTER(C.c_float), C.c_int64, C.c_void_p)

_lib = None


def lib():
    global _lib
    if _lib is None:
        so = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(so):
            subprocess.check_call(["make", "-s", "-C", HERE])
        L = C.CDLL(so)
        L.oracle_forward.restype = C.c_int
        L.oracle_forward.argtypes = [C.POINTER(OracleConfig), C.POINTER(OracleTensor), C.c_int,
                                     C.POINTER(C.c_float), C.POINTER(C.c_int32),
                                     C.POINTER(C.c_float), C.POINTER(C.c_float),
                                     C.POINTER(C.c_int32), C.POINTER(C.c_float), PUBLISH, C.c_void_p]
        L.oracle_preprocess.argtypes = [C.POINTER(C.c_uint8), C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_float)]
        L.oracle_bicubic_resample.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int,
                                              C.POINTER(C.c_float), C.c_int]
        L.oracle_select.restype = C.c_int
        L.oracle_select.argtypes = [C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_int, C.c_int,
                                    C.c_float, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_uint32), C.c_int,
                                    C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_float),
                                    C.POINTER(C.c_float)]
        L.oracle_mask_upsample.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.c_float, C.POINTER(C.c_uint8)]
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def config_from_meta(meta: dict, act_round: int = 0, n_threads: int = 0) -> OracleConfig:
    c = OracleConfig()
    g = lambda k: int(meta["rfdetr." + k])  # noqa: E731
    c.image_size, c.patch_size = g("image_size"), g("patch_size")
    c.num_queries, c.num_classes = g("num_queries"), g("num_classes")
    c.dim, c.depth, c.heads = g("backbone.dim"), g("backbone.depth"), g("backbone.heads")
    c.ffn_dim, c.num_windows = g("backbone.ffn_dim"), g("backbone.num_windows")
    c.pos_train = g("backbone.pos_embed_train_size")
    gi = meta["rfdetr.backbone.global_attn_indices"]
    c.n_global = len(gi)
    for i, v in enumerate(gi):
        c.global_idx[i] = int(v)
    ti = meta["rfdetr.backbone.out_feature_indices"]
    c.n_taps = len(ti)
    for i, v in enumerate(ti):
        c.tap_stage[i] = int(v)
    c.proj_out, c.proj_bneck = g("projector.out_dim"), g("projector.bottleneck_dim")
    c.proj_nb = g("projector.n_bottlenecks")
    c.dec_layers, c.dec_dim, c.dec_ffn = g("decoder.layers"), g("decoder.model_dim"), g("decoder.ffn_dim")
    c.sa_heads, c.ca_heads = g("decoder.self_attn_heads"), g("decoder.cross_attn_heads")
    c.ca_points = g("decoder.cross_attn_n_points")
    c.has_seg = int(bool(meta.get("rfdetr.has_segmentation_head", False)))
    c.mask_ratio = int(meta.get("rfdetr.mask_downsample_ratio", 4))
    c.act_round = act_round
    c.n_threads = n_threads
    return c


class Oracle:
    """CPU oracle bound to one GGUF file."""

    def __init__(self, gguf_path: str):
        self.meta, tensors = synth.read_gguf_f32(gguf_path)
        self.tensors = {k: (t, np.ascontiguousarray(a.reshape(-1))) for k, (t, a) in tensors.items()}
        names = list(self.tensors)
        self._names = [n.encode() for n in names]
        arr = (OracleTensor * len(names))()
        for i, n in enumerate(names):
            t, a = self.tensors[n]
            arr[i].name = self._names[i]
            arr[i].data = _fp(a)
            arr[i].n = a.size
            arr[i].type = TYPE_CODES[t]
        self._arr = arr
        m = self.meta
        self.image_size = int(m["rfdetr.image_size"])
        self.nq = int(m["rfdetr.num_queries"])
        self.nc = int(m["rfdetr.num_classes"])
        self.has_seg = bool(m.get("rfdetr.has_segmentation_head", False))
        self.mask_side = self.image_size // int(m.get("rfdetr.mask_downsample_ratio", 4))
        self.mean = np.array(m["rfdetr.preprocess.mean"], np.float32)
        self.std = np.array(m["rfdetr.preprocess.std"], np.float32)

    def preprocess(self, rgb: np.ndarray) -> np.ndarray:
        """uint8 HWC -> planar float [3][S][S] (bilinear, no antialias)."""
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        h, w = rgb.shape[:2]
        S = self.image_size
        out = np.empty((3, S, S), np.float32)
        lib().oracle_preprocess(rgb.ctypes.data_as(C.POINTER(C.c_uint8)), w, h, S, S,
                                _fp(self.mean), _fp(self.std), _fp(out))
        return out

    def forward(self, planar: np.ndarray, act_round: int = 0, trace: bool = False, n_threads: int = 0,
                force_topk=None):
        cfg = config_from_meta(self.meta, act_round, n_threads)
        planar = np.ascontiguousarray(planar, dtype=np.float32)
        logits = np.zeros((self.nq, self.nc), np.float32)
        boxes = np.zeros((self.nq, 4), np.float32)
        topk = np.zeros(self.nq, np.int32)
        masks = np.zeros((self.nq, self.mask_side, self.mask_side), np.float32) if self.has_seg else None
        store = {}

        def _pub(name, data, n, _u):
            store[name.decode()] = np.ctypeslib.as_array(data, shape=(n,)).copy()

        cb = PUBLISH(_pub) if trace else PUBLISH()
        ft = None
        if force_topk is not None:
            force_topk = np.ascontiguousarray(force_topk, np.int32)
            ft = force_topk.ctypes.data_as(C.POINTER(C.c_int32))
        rc = lib().oracle_forward(C.byref(cfg), self._arr, len(self._names), _fp(planar), ft,
                                  _fp(logits), _fp(boxes), topk.ctypes.data_as(C.POINTER(C.c_int32)),
                                  _fp(masks) if masks is not None else None, cb, None)
        if rc != 0:
            raise RuntimeError(f"oracle_forward failed: {rc}")
        return {"logits": logits, "boxes": boxes, "topk": topk, "masks": masks, "trace": store}


def select(logits, boxes, threshold, top_k, img_w, img_h, class_filter=None):
    nq, nc = logits.shape
    q = np.zeros(nq, np.int32)
    c = np.zeros(nq, np.int32)
    s = np.zeros(nq, np.float32)
    xy = np.zeros((nq, 4), np.float32)
    lg = np.ascontiguousarray(logits, np.float32)
    bx = np.ascontiguousarray(boxes, np.float32)
    flt = None if class_filter is None else np.ascontiguousarray(class_filter, np.uint32)
    n = lib().oracle_select(_fp(lg), _fp(bx), nq, nc, threshold, top_k, img_w, img_h,
                            None if flt is None else flt.ctypes.data_as(C.POINTER(C.c_uint32)),
                            0 if flt is None else len(flt),
                            q.ctypes.data_as(C.POINTER(C.c_int32)), c.ctypes.data_as(C.POINTER(C.c_int32)),
                            _fp(s), _fp(xy))
    return q[:n], c[:n], s[:n], xy[:n]


def mask_upsample(src: np.ndarray, dw: int, dh: int, thr: float = 0.5) -> np.ndarray:
    src = np.ascontiguousarray(src, np.float32)
    out = np.zeros((dh, dw), np.uint8)
    lib().oracle_mask_upsample(_fp(src), src.shape[1], src.shape[0], dw, dh, thr,
                               out.ctypes.data_as(C.POINTER(C.c_uint8)))
    return out


def bicubic_resample(src: np.ndarray, src_side: int, dst_side: int) -> np.ndarray:
    src = np.ascontiguousarray(src, np.float32)
    dim = src.shape[-1]
    out = np.zeros((dst_side * dst_side, dim), np.float32)
    lib().oracle_bicubic_resample(_fp(src), src_side, dim, _fp(out), dst_side)
    return out
