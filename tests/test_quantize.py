"""GGUF re-quantization (rfdetr_b200_quantize_gguf = the reference's
`rfdetr-cli quantize`, examples/cli/main.cpp:387-640; and load-time
re-quantization through rfdetr_b200_params.weight_type).

CPU: the GGUF writer (metadata copied byte for byte, tensors re-laid out) and
the argument checks.  GPU: the block quantizers produce exactly the bytes of
the converter path (gguf-py's Q8_0, the Q4_K restatement in synth.py, f16),
Q5_K / Q6_K round-trip through gguf-py's dequantizers within their error
bounds, and an engine loading F32 weights with weight_type = Q8_0 / Q4_K
computes exactly what it computes from the converter's Q8_0 / Q4_K file."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "rf-detr.cpp_b200"))

from rfdetr_b200 import lib, synth  # noqa: E402

F16, Q8_0, Q4_K, Q5_K, Q6_K = 1, 8, 12, 13, 14


def _quantize(src, dst, t, device=0):
    return lib.lib().rfdetr_b200_quantize_gguf(str(src).encode(), str(dst).encode(), t, device)


@pytest.mark.parametrize("dtype,t", [("f16", F16), ("q8_0", Q8_0), ("q4_K", Q4_K)])
def test_rewrite_without_conversion_is_byte_identical(make_model, tmp_path, dtype, t):
    """A file already in the requested type: every tensor is copied, so the
    writer must reproduce the converter's file exactly (no GPU involved)."""
    src = make_model("tiny", dtype, 0)
    out = tmp_path / "out.gguf"
    assert _quantize(src, out, t) == 0
    assert open(src, "rb").read() == open(out, "rb").read()


def test_quantize_rejects_bad_arguments(make_model, tmp_path):
    src = make_model("tiny", "f32", 0)
    assert _quantize(src, tmp_path / "x.gguf", 2) == -1           # Q4_0 is not a target type
    assert _quantize(tmp_path / "missing.gguf", tmp_path / "y.gguf", Q8_0) == -2
    assert lib.lib().rfdetr_b200_quantize_gguf(None, b"x", Q8_0, 0) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("t", [F16, Q8_0, Q4_K])
def test_block_quantizers_match_host_restatements(t):
    """Raw blocks from rfdetr_b200_op_quantize against gguf-py (F16 via numpy, Q8_0) and synth.py (Q4_K)."""
    import gguf as G
    import torch
    rng = np.random.default_rng(t)
    x = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    x[3, :32] = 0.0                  # an all-zero block
    x[5, 100] = 1.0                  # an outlier
    if t == F16:
        ref = x.astype(np.float16).view(np.uint8).ravel()
    elif t == Q8_0:
        ref = G.quants.quantize(x, G.GGMLQuantizationType.Q8_0).ravel()
    else:
        ref = synth.quantize_q4_K(x).ravel()
    d_x = torch.from_numpy(x).cuda()
    d_o = torch.zeros(ref.size, dtype=torch.uint8, device="cuda")
    rc = lib.lib().rfdetr_b200_op_quantize(t, d_x.data_ptr(), x.size, d_o.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    got = d_o.cpu().numpy()
    diff = np.nonzero(got != ref)[0]
    assert diff.size == 0, f"{diff.size} bytes differ, first at {diff[:8]}: {got[diff[:8]]} vs {ref[diff[:8]]}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,t", [("f16", F16), ("q8_0", Q8_0), ("q4_K", Q4_K)])
@pytest.mark.parametrize("variant", ["tiny", "tiny-base"])
def test_quantize_matches_converter_bytes(make_model, tmp_path, variant, dtype, t):
    src = make_model(variant, "f32", 0)
    ref = make_model(variant, dtype, 0)
    out = tmp_path / "q.gguf"
    assert _quantize(src, out, t) == 0
    a, b = open(out, "rb").read(), open(ref, "rb").read()
    assert len(a) == len(b)
    if a != b:
        diff = np.nonzero(np.frombuffer(a, np.uint8) != np.frombuffer(b, np.uint8))[0]
        pytest.fail(f"{len(diff)} bytes differ, first at {diff[0]}")


@pytest.mark.gpu
@pytest.mark.parametrize("t,tol", [(Q5_K, 0.05), (Q6_K, 0.025)])
def test_k_quants_round_trip(make_model, tmp_path, t, tol):
    import gguf as G
    src = make_model("tiny-base", "f32", 0)
    out = tmp_path / "k.gguf"
    assert _quantize(src, out, t) == 0
    want = G.GGMLQuantizationType(t)
    orig = {x.name: np.array(x.data, np.float32) for x in G.GGUFReader(src).tensors}
    n_k = 0
    for x in G.GGUFReader(out).tensors:
        if x.tensor_type in (want, G.GGMLQuantizationType.Q8_0):
            deq = G.quants.dequantize(x.data, x.tensor_type).reshape(orig[x.name].shape)
            e = np.linalg.norm(deq - orig[x.name]) / np.linalg.norm(orig[x.name])
            assert e < (tol if x.tensor_type == want else 0.01), (x.name, e)
            n_k += x.tensor_type == want
    assert n_k > 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,t", [("q8_0", Q8_0), ("q4_K", Q4_K)])
def test_load_time_requantization_matches_file(make_model, dtype, t):
    """weight_type at load == loading the converter's quantized file: same outputs bit for bit."""
    f32 = make_model("tiny", "f32", 0)
    qf = make_model("tiny", dtype, 0)
    a = lib.Engine(f32, weight_type=t)
    b = lib.Engine(qf)
    imgs = np.random.default_rng(4).integers(0, 256, (2, a.image_size, a.image_size, 3), dtype=np.uint8)
    la, ba, _ = a.forward_rgb(imgs)
    lb, bb, _ = b.forward_rgb(imgs)
    a.close()
    b.close()
    assert np.array_equal(la, lb) and np.array_equal(ba, bb)


@pytest.mark.gpu
def test_q6_K_engine_matches_oracle(make_model, tmp_path):
    """An engine on a Q6_K re-quantized file against the oracle on the same file."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    src = make_model("tiny-base", "f32", 0)
    out = tmp_path / "q6.gguf"
    assert _quantize(src, out, Q6_K) == 0
    eng = lib.Engine(str(out))
    ora = O.Oracle(str(out))
    img = np.random.default_rng(8).integers(0, 256, (1, eng.image_size, eng.image_size, 3), dtype=np.uint8)
    lg, bx, _ = eng.forward_rgb(img)
    topk = eng.trace("topk", 1).astype(np.int64)
    eng.close()
    own = ora.forward(ora.preprocess(img[0]), force_topk=topk)
    rel = np.abs(lg[0] - own["logits"]).max() / np.abs(own["logits"]).max()
    assert rel < 2e-2
