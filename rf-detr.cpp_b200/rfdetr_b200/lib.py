"""ctypes binding of librfdetr.so (the B200 engine's C ABI).

This is the host-side mirror of the reference's public interface
(include/rfdetr.h, include/rfdetr_capi.h) plus the additive batch / operator
entry points of include/rfdetr_b200.h.  There is no Python fallback: if the
shared library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("RFDETR_LIB", os.path.join(PKG, "lib", "librfdetr.so"))

RFDETR_OK = 0
STATUS = {0: "ok", -1: "invalid argument", -2: "file not found", -3: "i/o error", -4: "out of memory",
          -5: "image decode error", -6: "model format error", -7: "model load error", -8: "inference error",
          -99: "not implemented"}

LOG_CB = C.CFUNCTYPE(None, C.c_int, C.c_char_p, C.c_void_p)


class Params(C.Structure):
    _fields_ = [("model_path", C.c_char_p), ("n_threads", C.c_int), ("log_cb", LOG_CB), ("log_user_data", C.c_void_p)]


class DetectParams(C.Structure):
    _fields_ = [("threshold", C.c_float), ("top_k", C.c_uint32), ("class_filter", C.POINTER(C.c_uint32)),
                ("class_filter_len", C.c_size_t)]


class Detection(C.Structure):
    _fields_ = [("class_id", C.c_uint32), ("class_name", C.c_char_p), ("score", C.c_float),
                ("x1", C.c_float), ("y1", C.c_float), ("x2", C.c_float), ("y2", C.c_float),
                ("mask", C.POINTER(C.c_uint8)), ("mask_width", C.c_int), ("mask_height", C.c_int)]


class B200Det(C.Structure):
    """rfdetr_b200_det: one selected detection written by rfdetr_b200_op_select (32 bytes)."""
    _fields_ = [("query", C.c_int32), ("class_id", C.c_int32), ("score", C.c_float), ("x1", C.c_float),
                ("y1", C.c_float), ("x2", C.c_float), ("y2", C.c_float), ("pad", C.c_float)]


class B200Params(C.Structure):
    _fields_ = [("device", C.c_int), ("max_batch", C.c_int), ("weight_type", C.c_int)]


class ModelInfo(C.Structure):
    _fields_ = [("image_size", C.c_uint32), ("patch_size", C.c_uint32), ("num_queries", C.c_uint32),
                ("num_classes", C.c_uint32), ("dim", C.c_uint32), ("depth", C.c_uint32),
                ("num_windows", C.c_uint32), ("dec_layers", C.c_uint32), ("has_segmentation_head", C.c_int),
                ("n_tensors", C.c_size_t), ("variant", C.c_char * 32), ("legacy_resize", C.c_int32)]


# name -> (restype, argtypes); every symbol declared in include/*.h
SIGNATURES = {
    # rfdetr.h
    "rfdetr_status_str": (C.c_char_p, [C.c_int]),
    "rfdetr_set_log_callback": (None, [LOG_CB, C.c_void_p]),
    "rfdetr_init": (C.c_void_p, [C.POINTER(Params), C.POINTER(C.c_int)]),
    "rfdetr_free": (None, [C.c_void_p]),
    "rfdetr_context_variant": (C.c_char_p, [C.c_void_p]),
    "rfdetr_context_image_size": (C.c_uint32, [C.c_void_p]),
    "rfdetr_context_num_queries": (C.c_uint32, [C.c_void_p]),
    "rfdetr_context_num_classes": (C.c_uint32, [C.c_void_p]),
    "rfdetr_context_n_tensors": (C.c_size_t, [C.c_void_p]),
    "rfdetr_image_load_file": (C.c_void_p, [C.c_char_p, C.POINTER(C.c_int)]),
    "rfdetr_image_load_buffer": (C.c_void_p, [C.c_void_p, C.c_size_t, C.POINTER(C.c_int)]),
    "rfdetr_image_from_rgb_buffer": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "rfdetr_image_free": (None, [C.c_void_p]),
    "rfdetr_image_width": (C.c_int, [C.c_void_p]),
    "rfdetr_image_height": (C.c_int, [C.c_void_p]),
    "rfdetr_image_rgb_data": (C.POINTER(C.c_uint8), [C.c_void_p]),
    "rfdetr_visualize_draw_box": (None, [C.c_void_p, Detection, C.c_int]),
    "rfdetr_visualize_overlay_mask": (None, [C.c_void_p, Detection, C.c_float]),
    "rfdetr_detect": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(DetectParams), C.POINTER(C.POINTER(Detection)),
                                C.POINTER(C.c_size_t)]),
    "rfdetr_detections_free": (None, [C.POINTER(Detection), C.c_size_t]),
    "rfdetr_render": (C.c_int, [C.c_void_p, C.POINTER(Detection), C.c_size_t, C.c_char_p]),
    # rfdetr_capi.h
    "rfdetr_capi_load": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(C.c_size_t)]),
    "rfdetr_capi_unload": (C.c_int, [C.c_size_t]),
    "rfdetr_capi_detect_path": (C.c_int, [C.c_size_t, C.c_char_p, C.c_float, C.c_uint32, C.POINTER(C.c_void_p)]),
    "rfdetr_capi_detect_buffer": (C.c_int, [C.c_size_t, C.c_void_p, C.c_size_t, C.c_float, C.c_uint32,
                                            C.POINTER(C.c_void_p)]),
    "rfdetr_capi_free_string": (None, [C.c_void_p]),
    "rfdetr_capi_get_n_detections": (C.c_int, [C.c_size_t]),
    "rfdetr_capi_get_detection_class_id": (C.c_int, [C.c_size_t, C.c_int]),
    "rfdetr_capi_get_detection_box": (C.c_int, [C.c_size_t, C.c_int, C.POINTER(C.c_float)]),
    "rfdetr_capi_get_detection_score": (C.c_float, [C.c_size_t, C.c_int]),
    "rfdetr_capi_get_detection_class_name": (C.c_int, [C.c_size_t, C.c_int, C.c_char_p, C.c_int]),
    "rfdetr_capi_get_detection_mask_png": (C.c_int, [C.c_size_t, C.c_int, C.c_void_p, C.c_int]),
    # rfdetr_b200.h
    "rfdetr_b200_init": (C.c_void_p, [C.POINTER(Params), C.POINTER(B200Params), C.POINTER(C.c_int)]),
    "rfdetr_b200_forward_rgb": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                          C.c_void_p, C.c_void_p]),
    "rfdetr_b200_forward_planar": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "rfdetr_b200_enqueue_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "rfdetr_b200_sync": (C.c_int, [C.c_void_p]),
    "rfdetr_b200_submit_rgb": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                         C.c_void_p, C.c_void_p]),
    "rfdetr_b200_wait": (C.c_int, [C.c_void_p]),
    "rfdetr_b200_wait_oldest": (C.c_int, [C.c_void_p]),
    "rfdetr_b200_device_outputs": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                             C.POINTER(C.c_void_p)]),
    "rfdetr_b200_detect_batch": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.c_size_t, C.POINTER(DetectParams),
                                           C.POINTER(C.POINTER(Detection)), C.POINTER(C.c_size_t)]),
    "rfdetr_b200_device": (C.c_int, [C.c_void_p]),
    "rfdetr_b200_mask_side": (C.c_int, [C.c_void_p]),
    "rfdetr_b200_kernels_per_forward": (C.c_int, [C.c_void_p]),
    "rfdetr_b200_stream": (C.c_void_p, [C.c_void_p]),
    "rfdetr_b200_trace": (C.c_longlong, [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_size_t]),
    "rfdetr_b200_profile_enable": (None, [C.c_void_p, C.c_int]),
    "rfdetr_b200_profile_read": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_int]),
    "rfdetr_b200_inspect": (C.c_int, [C.c_char_p, C.POINTER(ModelInfo)]),
    "rfdetr_b200_dequantize": (C.c_int, [C.c_uint32, C.c_void_p, C.c_longlong, C.c_void_p]),
    "rfdetr_b200_op_gemm": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                      C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
    "rfdetr_b200_op_attention": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                           C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                           C.c_void_p]),
    "rfdetr_b200_quantize_gguf": (C.c_int, [C.c_char_p, C.c_char_p, C.c_int, C.c_int]),
    "rfdetr_b200_op_quantize": (C.c_int, [C.c_int, C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p]),
    "rfdetr_b200_op_resize_legacy": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                               C.c_void_p]),
    "rfdetr_b200_op_topk": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "rfdetr_b200_op_select": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                                        C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "rfdetr_b200_mask_bits_words": (C.c_size_t, [C.c_int, C.c_int]),
    "rfdetr_b200_op_mask_bits": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                           C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "rfdetr_b200_op_deform": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "rfdetr_b200_op_conv3x3_workspace": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "rfdetr_b200_op_conv3x3": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                         C.c_int, C.c_void_p, C.c_void_p, C.c_float, C.c_int, C.c_void_p, C.c_int,
                                         C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "rfdetr_b200_op_conv3x3_noalloc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                 C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_float, C.c_int,
                                                 C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
}

_lib = None


def lib():
    """Load librfdetr.so (raises if it is absent: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"librfdetr.so not built ({LIB_PATH}); run `make -C rf-detr.cpp_b200`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str):
    if status != RFDETR_OK:
        raise RuntimeError(f"{what}: {STATUS.get(status, status)} ({status})")


def _ptr(a):
    return C.c_void_p(a.ctypes.data) if a is not None else None


class Engine:
    """One rfdetr_context on one GPU (rfdetr_b200_init)."""

    def __init__(self, model_path: str, device: int = 0, max_batch: int = 1, weight_type: int = 0):
        """weight_type: 0 = weights as stored, else re-quantize them at load (GGUF type id)."""
        L = lib()
        st = C.c_int(0)
        p = Params(model_path.encode(), 1, LOG_CB(), None)
        b = B200Params(device, max_batch, weight_type)
        self._ctx = L.rfdetr_b200_init(C.byref(p), C.byref(b), C.byref(st))
        if not self._ctx:
            raise RuntimeError(f"rfdetr_b200_init failed: {STATUS.get(st.value, st.value)} ({st.value})")
        self.image_size = L.rfdetr_context_image_size(self._ctx)
        self.nq = L.rfdetr_context_num_queries(self._ctx)
        self.nc = L.rfdetr_context_num_classes(self._ctx)
        self.mask_side = L.rfdetr_b200_mask_side(self._ctx)

    @property
    def ctx(self):
        return self._ctx

    def close(self):
        if self._ctx:
            lib().rfdetr_free(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _outputs(self, batch):
        lg = np.zeros((batch, self.nq, self.nc), np.float32)
        bx = np.zeros((batch, self.nq, 4), np.float32)
        mk = np.zeros((batch, self.nq, self.mask_side, self.mask_side), np.float32) if self.mask_side else None
        return lg, bx, mk

    def forward_planar(self, planar: np.ndarray):
        planar = np.ascontiguousarray(planar, np.float32)
        if planar.ndim == 3:
            planar = planar[None]
        B = planar.shape[0]
        lg, bx, mk = self._outputs(B)
        check(lib().rfdetr_b200_forward_planar(self._ctx, _ptr(planar), B, _ptr(lg), _ptr(bx), _ptr(mk)),
              "forward_planar")
        return lg, bx, mk

    def forward_rgb(self, rgb: np.ndarray):
        rgb = np.ascontiguousarray(rgb, np.uint8)
        if rgb.ndim == 3:
            rgb = rgb[None]
        B, H, W, _ = rgb.shape
        lg, bx, mk = self._outputs(B)
        check(lib().rfdetr_b200_forward_rgb(self._ctx, _ptr(rgb), B, W, H, _ptr(lg), _ptr(bx), _ptr(mk)),
              "forward_rgb")
        return lg, bx, mk

    def submit_rgb(self, rgb: np.ndarray, logits: np.ndarray, boxes: np.ndarray, masks=None):
        """Pipelined forward from host images into caller-owned output arrays
        (kept alive and untouched until wait()); returns at once."""
        B, H, W, _ = rgb.shape
        assert rgb.flags.c_contiguous and rgb.dtype == np.uint8
        check(lib().rfdetr_b200_submit_rgb(self._ctx, _ptr(rgb), B, W, H, _ptr(logits), _ptr(boxes),
                                           _ptr(masks) if masks is not None else None), "submit_rgb")

    def wait(self):
        check(lib().rfdetr_b200_wait(self._ctx), "wait")

    def wait_oldest(self):
        check(lib().rfdetr_b200_wait_oldest(self._ctx), "wait_oldest")

    def trace(self, name: str, batch: int, size_hint: int = 1 << 26) -> np.ndarray:
        out = np.zeros(size_hint, np.float32)
        n = lib().rfdetr_b200_trace(self._ctx, name.encode(), batch, _ptr(out), out.size)
        if n < 0:
            raise KeyError(name)
        return out[:n].copy()

    def enqueue_device(self, d_rgb_ptr: int, batch: int, width: int, height: int):
        check(lib().rfdetr_b200_enqueue_device(self._ctx, C.c_void_p(d_rgb_ptr), batch, width, height),
              "enqueue_device")

    def sync(self):
        check(lib().rfdetr_b200_sync(self._ctx), "sync")

    def profile_enable(self, on: bool = True):
        lib().rfdetr_b200_profile_enable(self._ctx, 1 if on else 0)

    def profile_read(self, cap: int = 4096, name_len: int = 48):
        names = C.create_string_buffer(cap * name_len)
        ms = np.zeros(cap, np.float32)
        n = lib().rfdetr_b200_profile_read(self._ctx, names, name_len, _ptr(ms), cap)
        raw = names.raw
        out = []
        for i in range(min(n, cap)):
            nm = raw[i * name_len:(i + 1) * name_len].split(b"\0", 1)[0].decode()
            out.append((nm, float(ms[i])))
        return out

    def kernels_per_forward(self) -> int:
        return lib().rfdetr_b200_kernels_per_forward(self._ctx)

    def stream(self) -> int:
        return lib().rfdetr_b200_stream(self._ctx) or 0


def inspect(model_path: str):
    info = ModelInfo()
    st = lib().rfdetr_b200_inspect(model_path.encode(), C.byref(info))
    return st, info


def dequantize(ggml_type: int, raw: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    raw = np.ascontiguousarray(raw)
    rc = lib().rfdetr_b200_dequantize(ggml_type, _ptr(raw), n, _ptr(out))
    if rc != 0:
        raise ValueError(f"unsupported ggml type {ggml_type}")
    return out
