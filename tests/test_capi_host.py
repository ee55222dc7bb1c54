"""Host-side checks of librfdetr.so that need no GPU: the library loads and
exports every symbol the headers declare; the GGUF loader's contract and
error codes (reference tests/test_model_loader.cpp, src/model_loader.cpp:
212-371, 703-750); the block dequantizers against gguf-py; image decoding;
and the flat C API's invalid-handle behaviour (tests/test_capi_flat.cpp,
tests/test_capi_accessors.cpp)."""
import ctypes as C
import os
import re
import struct
import zlib

import numpy as np
import pytest

from rfdetr_b200 import lib, synth

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("rfdetr.h", "rfdetr_capi.h", "rfdetr_b200.h"):
        src = open(os.path.join(REPO, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(rfdetr_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    names.discard("rfdetr_log_cb")
    return names


def test_library_exports_every_declared_symbol():
    L = lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 45
    for s in sorted(syms):
        assert hasattr(L, s), s
    assert syms <= set(lib.SIGNATURES), sorted(syms - set(lib.SIGNATURES))


def test_status_strings():
    L = lib.lib()
    assert L.rfdetr_status_str(0) == b"ok"
    assert L.rfdetr_status_str(-7) == b"model load error"
    assert L.rfdetr_status_str(-99) == b"not implemented"
    assert L.rfdetr_status_str(12345) == b"unknown error"


@pytest.mark.parametrize("variant", ["tiny", "seg-tiny", "base", "grid52"])
def test_inspect_valid(variant, make_model):
    path = make_model(variant, "f16", 0)
    st, info = lib.inspect(path)
    cfg = synth.get_variant(variant)
    assert st == 0
    assert info.image_size == cfg["image_size"] and info.num_queries == cfg["num_queries"]
    assert info.num_windows == cfg["backbone"]["num_windows"]
    assert info.has_segmentation_head == int(cfg["segmentation_head"])
    assert info.n_tensors == len(synth.tensor_specs(cfg))
    assert info.variant.decode() == variant


def _write(tmp_path, name, variant="tiny", drop=None, meta_override=None, dtype="f32"):
    cfg = synth.get_variant(variant)
    st = synth.make_state(cfg, 0)
    if drop:
        st.pop(drop)
    if meta_override:
        cfg.update(meta_override)
    p = str(tmp_path / name)
    synth.write_gguf(p, variant, cfg, st, dtype)
    return p


def test_inspect_errors(tmp_path):
    assert lib.inspect(str(tmp_path / "nope.gguf"))[0] == -2
    p = _write(tmp_path, "missing.gguf", drop="decoder.layers.1.norm3.bias")
    assert lib.inspect(p)[0] == -7  # missing tensor -> RFDETR_ERR_MODEL_LOAD
    p = _write(tmp_path, "seg_missing.gguf", variant="seg-tiny", drop="segmentation_head.blocks.1.dwconv.weight")
    assert lib.inspect(p)[0] == -7
    good = _write(tmp_path, "good.gguf")
    data = open(good, "rb").read()
    (tmp_path / "trunc.gguf").write_bytes(data[: len(data) // 2])
    assert lib.inspect(str(tmp_path / "trunc.gguf"))[0] == -6
    (tmp_path / "garbage.gguf").write_bytes(b"NOTAGGUF" + bytes(64))
    assert lib.inspect(str(tmp_path / "garbage.gguf"))[0] == -6
    p = _write(tmp_path, "mode.gguf", meta_override={"resize_mode": "bogus"})
    assert lib.inspect(p)[0] == -6


def test_inspect_survives_corrupted_files(tmp_path):
    """The GGUF reader on damaged input (src/model_loader.cpp reads untrusted files): seeded byte
    flips and 8-byte overwrites (string lengths, counts, offsets, types) in the header, metadata
    and tensor-info region, and truncations at random offsets.  Every call returns OK or one of
    the status codes; none may crash (the sanitize build of the Makefile runs this under ASan +
    UBSan)."""
    good = _write(tmp_path, "good.gguf", dtype="f16")
    data = open(good, "rb").read()
    head = min(len(data), 16384)
    rng = np.random.default_rng(1234)
    statuses = set(lib.STATUS)
    p = str(tmp_path / "bad.gguf")
    for i in range(90):
        b = bytearray(data)
        if i % 3 == 0:
            b = b[: int(rng.integers(0, len(data)))]
        elif i % 3 == 1:
            for _ in range(int(rng.integers(1, 4))):
                b[int(rng.integers(0, head))] ^= 1 << int(rng.integers(0, 8))
        else:
            at = int(rng.integers(0, head - 8))
            b[at:at + 8] = rng.integers(0, 256, 8, dtype=np.uint8).tobytes()
        open(p, "wb").write(bytes(b))
        st, _ = lib.inspect(p)
        assert st in statuses, (i, st)


def test_gguf_reader_checks_lengths_against_the_file(tmp_path):
    """Lengths and offsets read from a GGUF file are checked against the file itself: a tensor
    offset near 2^64 (whose end would wrap around past the bounds check) is rejected, and so are
    a metadata string length and an array count larger than the bytes left in the file, before
    anything is allocated for them."""
    good = _write(tmp_path, "good.gguf", dtype="f16")
    data = bytes(open(good, "rb").read())
    assert lib.inspect(good)[0] == 0

    def status(b):
        p = tmp_path / "bad.gguf"
        p.write_bytes(bytes(b))
        return lib.inspect(str(p))[0]

    name = b"decoder.layers.1.norm3.bias"
    at = data.find(struct.pack("<Q", len(name)) + name)
    assert at > 0
    n_dims = struct.unpack_from("<I", data, at + 8 + len(name))[0]
    b = bytearray(data)
    struct.pack_into("<Q", b, at + 8 + len(name) + 4 + 8 * n_dims + 4, 2**64 - 16)  # the tensor's offset
    assert status(b) == -6
    b = bytearray(data)
    struct.pack_into("<Q", b, 24, (1 << 30) - 1)  # length of the first metadata key
    assert status(b) == -6
    key = b"rfdetr.class_names"
    at = data.find(struct.pack("<Q", len(key)) + key)
    assert at > 0
    b = bytearray(data)
    struct.pack_into("<Q", b, at + 8 + len(key) + 8, 1 << 25)  # element count of the string array
    assert status(b) == -6


def test_resize_mode_key(tmp_path):
    """rfdetr.preprocess.resize_mode (tests/test_model_loader.cpp:41-46,133-163 of the reference):
    an absent key means the legacy stb resize, as in every file converted before the key existed;
    the two values a converter writes select their path; an unknown value is
    RFDETR_ERR_MODEL_FORMAT with a logged message that names the key."""
    cases = {None: 1, "legacy_stb": 1, "bilinear_no_antialias": 0}
    for mode, legacy in cases.items():
        p = _write(tmp_path, f"mode-{mode}.gguf", meta_override={"resize_mode": mode}, dtype="f16")
        st, info = lib.inspect(p)
        assert st == 0 and info.legacy_resize == legacy, (mode, st, info.legacy_resize)
    msgs = []
    cb = lib.LOG_CB(lambda level, msg, user: msgs.append(msg.decode()))
    L = lib.lib()
    L.rfdetr_set_log_callback(cb, None)
    try:
        st, _ = lib.inspect(_write(tmp_path, "mode-bogus.gguf", meta_override={"resize_mode": "bogus"}, dtype="f16"))
    finally:
        L.rfdetr_set_log_callback(lib.LOG_CB(), None)
    assert st == -6 and any("resize_mode" in m for m in msgs), (st, msgs)


def test_inspect_rejects_unsupported_config(tmp_path):
    cfg = synth.get_variant("tiny")
    cfg["backbone"]["heads"] = 8  # head_dim 48: not implemented by the kernels
    p = str(tmp_path / "h8.gguf")
    synth.write_gguf(p, "tiny", cfg, synth.make_state(synth.get_variant("tiny"), 0), "f32")
    assert lib.inspect(p)[0] == -6


@pytest.mark.parametrize("qt", ["F16", "Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "BF16"])
def test_dequantizers_match_gguf_py(qt):
    import gguf
    T = gguf.GGMLQuantizationType[qt]
    a = (np.random.default_rng(1).standard_normal((8, 512)) * 0.05).astype(np.float32)
    if qt == "F16":
        raw = a.astype(np.float16).view(np.uint8)
    else:
        raw = gguf.quants.quantize(a, T)
    ours = lib.dequantize(int(T), raw, a.size)
    ref = gguf.quants.dequantize(raw, T).reshape(-1)
    assert np.array_equal(ours, ref.astype(np.float32))


@pytest.mark.parametrize("qt", ["Q4_K", "Q5_K", "Q6_K"])
def test_kquant_dequantizers_match_gguf_py(qt):
    import gguf
    T = gguf.GGMLQuantizationType[qt]
    bs = {"Q4_K": 144, "Q5_K": 176, "Q6_K": 210}[qt]
    rng = np.random.default_rng(2)
    raw = rng.integers(0, 256, (16, bs), dtype=np.uint8)
    # keep the f16 scales finite and small
    for off in ((0, 2) if qt != "Q6_K" else (208,)):
        raw[:, off:off + 2] = np.frombuffer(
            (rng.uniform(-0.01, 0.01, 16).astype(np.float16)).tobytes(), np.uint8).reshape(16, 2)
    ours = lib.dequantize(int(T), raw, 16 * 256)
    ref = gguf.quants.dequantize(raw, T).reshape(-1).astype(np.float32)
    assert np.allclose(ours, ref, rtol=0, atol=0)


def _png(rgb, color_type=2, filt=0):
    h, w = rgb.shape[:2]
    rows = b"".join(bytes([filt]) + rgb[y].tobytes() for y in range(h))
    if filt == 1:  # Sub filter for 3-channel
        out = bytearray()
        for y in range(h):
            r = rgb[y].reshape(-1).astype(np.int32)
            sub = (r - np.concatenate([np.zeros(3, np.int32), r[:-3]])) & 0xFF
            out += bytes([1]) + sub.astype(np.uint8).tobytes()
        rows = bytes(out)

    def chunk(t, d):
        return struct.pack(">I", len(d)) + t + d + struct.pack(">I", zlib.crc32(t + d) & 0xFFFFFFFF)
    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, color_type, 0, 0, 0)) +
            chunk(b"IDAT", zlib.compress(rows)) + chunk(b"IEND", b""))


@pytest.mark.parametrize("filt", [0, 1])
def test_png_and_ppm_decode(filt):
    L = lib.lib()
    rgb = np.random.default_rng(4).integers(0, 256, (17, 23, 3), dtype=np.uint8)
    for blob in (_png(rgb, filt=filt), b"P6\n23 17\n255\n" + rgb.tobytes()):
        st = C.c_int(0)
        img = L.rfdetr_image_load_buffer(blob, len(blob), C.byref(st))
        assert img and st.value == 0
        assert L.rfdetr_image_width(img) == 23 and L.rfdetr_image_height(img) == 17
        data = np.ctypeslib.as_array(L.rfdetr_image_rgb_data(img), shape=(17 * 23 * 3,))
        assert np.array_equal(data.reshape(17, 23, 3), rgb)
        L.rfdetr_image_free(img)
    st = C.c_int(0)
    assert not L.rfdetr_image_load_buffer(b"\x00\x01garbage", 9, C.byref(st))
    assert st.value == -5
    assert not L.rfdetr_image_load_file(b"/nonexistent/x.png", C.byref(st))
    assert st.value == -2


def _png_chunks(w, h, depth, ctype, rows):
    def chunk(t, d):
        return struct.pack(">I", len(d)) + t + d + struct.pack(">I", zlib.crc32(t + d) & 0xFFFFFFFF)
    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, depth, ctype, 0, 0, 0)) +
            chunk(b"IDAT", zlib.compress(rows)) + chunk(b"IEND", b""))


def test_png_bit_depths():
    """Gray PNGs of the specification's sub-byte depths (1, 2, 4) decode to the expected levels;
    depths 3, 5, 6 and 7 (not in the specification) are RFDETR_ERR_DECODE, not unpacked past the
    end of each row."""
    L = lib.lib()
    W, H = 100, 2
    rng = np.random.default_rng(8)
    for depth in range(1, 8):
        stride = (W * depth + 7) // 8
        raw = rng.integers(0, 256, (H, stride), dtype=np.uint8)
        blob = _png_chunks(W, H, depth, 0, b"".join(b"\x00" + raw[y].tobytes() for y in range(H)))
        st = C.c_int(0)
        img = L.rfdetr_image_load_buffer(blob, len(blob), C.byref(st))
        if depth in (1, 2, 4):
            assert img and st.value == 0
            got = np.ctypeslib.as_array(L.rfdetr_image_rgb_data(img), shape=(H * W * 3,)).reshape(H, W, 3)
            bits = np.unpackbits(raw, axis=1)[:, : W * depth].reshape(H, W, depth)
            level = (bits * (1 << np.arange(depth - 1, -1, -1))).sum(-1)
            assert np.array_equal(got[..., 0], level * 255 // ((1 << depth) - 1))
            L.rfdetr_image_free(img)
        else:
            assert not img and st.value == -5, depth


def test_png_rejects_sizes_its_data_cannot_hold():
    """An IHDR of 65535 x 65535 16-bit RGBA pixels over a few bytes of IDAT is RFDETR_ERR_DECODE
    at once: deflate expands at most 1032:1, so no buffer of the declared size is allocated."""
    L = lib.lib()
    blob = _png_chunks(65535, 65535, 16, 6, bytes(64))
    st = C.c_int(0)
    assert not L.rfdetr_image_load_buffer(blob, len(blob), C.byref(st)) and st.value == -5


def test_image_decoders_survive_corrupted_input():
    """PNG (two filters) and PPM decoding of damaged buffers: seeded byte flips, 4-byte overwrites
    (chunk lengths, dimensions, header numbers) and truncations give an image whose pixel buffer
    matches its dimensions, or RFDETR_ERR_DECODE; none may crash (clean under the sanitize build)."""
    L = lib.lib()
    rgb = np.random.default_rng(9).integers(0, 256, (17, 23, 3), dtype=np.uint8)
    rng = np.random.default_rng(4321)
    for blob in (_png(rgb), _png(rgb, filt=1), b"P6\n23 17\n255\n" + rgb.tobytes()):
        for i in range(120):
            b = bytearray(blob)
            if i % 3 == 0:
                b = b[: int(rng.integers(1, len(blob)))]
            elif i % 3 == 1:
                for _ in range(int(rng.integers(1, 4))):
                    b[int(rng.integers(0, min(len(b), 64)))] ^= 1 << int(rng.integers(0, 8))
            else:
                at = int(rng.integers(0, min(len(b), 64) - 4))
                b[at:at + 4] = rng.integers(0, 256, 4, dtype=np.uint8).tobytes()
            st = C.c_int(0)
            img = L.rfdetr_image_load_buffer(bytes(b), len(b), C.byref(st))
            if img:
                w, h = L.rfdetr_image_width(img), L.rfdetr_image_height(img)
                assert st.value == 0 and w > 0 and h > 0
                L.rfdetr_image_free(img)
            else:
                assert st.value == -5, (i, st.value)


def test_image_from_rgb_copies():
    L = lib.lib()
    rgb = np.arange(4 * 5 * 3, dtype=np.uint8).reshape(4, 5, 3)
    st = C.c_int(0)
    img = L.rfdetr_image_from_rgb_buffer(rgb.ctypes.data, 5, 4, C.byref(st))
    rgb[:] = 0
    data = np.ctypeslib.as_array(L.rfdetr_image_rgb_data(img), shape=(60,))
    assert data[5] == 5
    L.rfdetr_image_free(img)
    assert not L.rfdetr_image_from_rgb_buffer(None, 5, 4, C.byref(st)) and st.value == -1
    # dimensions whose byte count no buffer can have are an invalid argument (nothing is read)
    assert not L.rfdetr_image_from_rgb_buffer(rgb.ctypes.data, 2**31 - 1, 2**31 - 1, C.byref(st)) and st.value == -1


def test_visualize_any_box(tmp_path):
    """rfdetr_visualize_draw_box with caller boxes outside the image, inverted, NaN or infinite
    writes inside the image only; a sane box gets its edges in the class colour and keeps its
    interior; rfdetr_render rejects a NULL detection array with n > 0."""
    L = lib.lib()
    rgb = np.zeros((40, 50, 3), np.uint8)
    st = C.c_int(0)
    img = L.rfdetr_image_from_rgb_buffer(rgb.ctypes.data, 50, 40, C.byref(st))
    d = lib.Detection()
    d.class_id = 1
    inf, nan = float("inf"), float("nan")
    for box in [(-100, -100, 1e9, 1e9), (30, 20, 5, 5), (nan, nan, nan, nan), (-inf, 0, inf, 40),
                (1e30, -1e30, 3, 3), (49.9, 39.9, 60, 60)]:
        d.x1, d.y1, d.x2, d.y2 = box
        L.rfdetr_visualize_draw_box(img, d, 3)
        L.rfdetr_visualize_draw_box(img, d, -7)
    L.rfdetr_image_free(img)
    img = L.rfdetr_image_from_rgb_buffer(rgb.ctypes.data, 50, 40, C.byref(st))
    d.x1, d.y1, d.x2, d.y2 = 5, 18, 30, 35
    L.rfdetr_visualize_draw_box(img, d, 3)
    px = np.ctypeslib.as_array(L.rfdetr_image_rgb_data(img), shape=(40 * 50 * 3,)).reshape(40, 50, 3)
    assert px[18, 5].tolist() == [60, 180, 75] and px[34, 29].tolist() == [60, 180, 75]
    assert px[26, 17].tolist() == [0, 0, 0]
    assert L.rfdetr_render(img, None, 2, str(tmp_path / "r.png").encode()) == -1
    assert L.rfdetr_render(img, None, 0, str(tmp_path / "r.png").encode()) == 0
    L.rfdetr_image_free(img)


def test_flat_capi_invalid_handles():
    L = lib.lib()
    assert L.rfdetr_capi_unload(0) == 0
    assert L.rfdetr_capi_get_n_detections(0) == -1
    assert L.rfdetr_capi_get_detection_class_id(0, 0) == -1
    xy = (C.c_float * 4)()
    assert L.rfdetr_capi_get_detection_box(0, 0, xy) == -1
    assert L.rfdetr_capi_get_detection_score(0, 0) == -1.0
    assert L.rfdetr_capi_get_detection_class_name(0, 0, None, 0) == -1
    assert L.rfdetr_capi_get_detection_mask_png(0, 0, None, 0) == -1
    out = C.c_void_p()
    assert L.rfdetr_capi_detect_path(0, b"x.png", 0.5, 10, C.byref(out)) == -1
    h = C.c_size_t(0)
    assert L.rfdetr_capi_load(None, 1, C.byref(h)) == -1
    assert L.rfdetr_capi_load(b"/nonexistent.gguf", 1, C.byref(h)) == -2 and h.value == 0


def test_b200_entry_points_reject_null_handles():
    """Host-side argument checks of the batch / pipelined entry points: a null
    context or buffer is RFDETR_ERR_INVALID_ARG before any CUDA call."""
    L = lib.lib()
    buf = (C.c_uint8 * 12)()
    out = (C.c_float * 4)()
    assert L.rfdetr_b200_submit_rgb(None, buf, 1, 2, 2, out, out, None) == -1
    assert L.rfdetr_b200_wait(None) == -1
    assert L.rfdetr_b200_wait_oldest(None) == -1
    assert L.rfdetr_b200_forward_rgb(None, buf, 1, 2, 2, out, out, None) == -1
    assert L.rfdetr_b200_enqueue_device(None, buf, 1, 2, 2) == -1
    assert L.rfdetr_b200_sync(None) == -1
    # operator argument checks come before any launch: cudaErrorInvalidValue (1)
    assert L.rfdetr_b200_op_topk(None, 1, 1600, 91, 300, None, None) == 1
    assert L.rfdetr_b200_op_resize_legacy(None, 1, 200, 160, None, 128, 128, None) == 1
    assert L.rfdetr_b200_detect_batch(None, None, 0, None, None, None) == -1


def test_init_errors_without_touching_the_gpu(tmp_path):
    L = lib.lib()
    st = C.c_int(0)
    p = lib.Params(None, 1, lib.LOG_CB(), None)
    assert not L.rfdetr_init(C.byref(p), C.byref(st)) and st.value == -1
    p = lib.Params(b"/nonexistent.gguf", 1, lib.LOG_CB(), None)
    assert not L.rfdetr_init(C.byref(p), C.byref(st)) and st.value == -2
    bad = _write(tmp_path, "missing.gguf", drop="heads.class_embed.bias")
    msgs = []
    cb = lib.LOG_CB(lambda lvl, msg, ud: msgs.append(msg.decode()))
    p = lib.Params(bad.encode(), 1, cb, None)
    assert not L.rfdetr_init(C.byref(p), C.byref(st)) and st.value == -7
    assert any("missing tensor" in m for m in msgs)
    L.rfdetr_set_log_callback(lib.LOG_CB(), None)


@pytest.mark.parametrize("noalloc", [False, True])
def test_conv3x3_rejects_misaligned_source_before_any_launch(noalloc):
    """The im2col path of both ConvX entry points reads `src` 8 channels (16 bytes) at a
    time: a source that is not 16-byte aligned, a pixel pitch shorter than the channel
    count, or a channel count that is not a multiple of 8 is refused with
    cudaErrorInvalidValue (1) before any device work.  The pointers are fake addresses that
    nothing may touch (c = 96 selects the im2col path of the workspace variant)."""
    L = lib.lib()
    src, w, g, out = C.c_void_p(0x100000), C.c_void_p(0x200000), C.c_void_p(0x300000), C.c_void_p(0x400000)
    ws = C.c_void_p(0x500000)
    B, H, W, Cin = 1, 8, 8, 96
    ws_bytes = L.rfdetr_b200_op_conv3x3_workspace(B, H, W, Cin)

    def call(s, lds, c):
        if noalloc:
            return L.rfdetr_b200_op_conv3x3_noalloc(s, lds, B, H, W, c, w, 128, g, g, 1e-6, 0, out, 128, None, 0,
                                                    None)
        return L.rfdetr_b200_op_conv3x3(s, lds, B, H, W, c, w, 128, g, g, 1e-6, 0, out, 128, None, 0, ws,
                                        ws_bytes, None)

    assert call(C.c_void_p(0x100002), Cin, Cin) == 1   # src one f16 element past a 16-byte boundary
    assert call(src, Cin - 8, Cin) == 1                  # lds < c
    assert call(src, Cin + 4, Cin) == 1                  # lds not a multiple of 8
    assert call(src, 100, 100) == 1                      # c not a multiple of 8
    if not noalloc:
        # a misaligned workspace is refused as well
        assert L.rfdetr_b200_op_conv3x3(src, Cin, B, H, W, Cin, w, 128, g, g, 1e-6, 0, out, 128, None, 0,
                                        C.c_void_p(0x500008), ws_bytes, None) == 1

