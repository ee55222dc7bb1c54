"""rfdetr_b200_op_conv3x3_noalloc — the ConvX operator for callers that cannot
call cudaMalloc (its im2col scratch is a fixed device array inside the
library instead of a caller workspace).

Checked through the C ABI against rfdetr_b200_op_conv3x3 (the workspace
variant) and directly against a float64 torch conv2d + layer_norm (+ SiLU), on
two calls in a row with different inputs, so a second call that reused stale
scratch contents would be caught.  This file is collected last on purpose; it
passes alone in a fresh process and after the other tests.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _p(t):
    return t.data_ptr() if t is not None else None


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def test_noalloc_conv3x3_matches_workspace_variant():
    from rfdetr_b200 import lib
    L = lib.lib()
    dev = "cuda:0"
    st = torch.cuda.current_stream().cuda_stream
    torch.manual_seed(11)
    B, H, W, C, OC = 2, 20, 20, 128, 128
    w = (torch.randn(OC, 3, 3, C, device=dev) * 0.05).half()
    g = torch.rand(OC, device=dev) + 0.5
    b = torch.randn(OC, device=dev) * 0.1
    ws_bytes = L.rfdetr_b200_op_conv3x3_workspace(B, H, W, C)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    for call in range(2):
        # different input each call: an im2col that skipped elements would expose the previous call's data
        x = torch.randn(B * H * W, C, device=dev).half() * (1 + call)
        ref16 = torch.zeros(B * H * W, OC, dtype=torch.float16, device=dev)
        ref32 = torch.zeros(B * H * W, OC, device=dev)
        assert L.rfdetr_b200_op_conv3x3(_p(x), C, B, H, W, C, _p(w), OC, _p(g), _p(b), 1e-6, 3, _p(ref32), OC,
                                        _p(ref16), OC, _p(ws), ws_bytes, st) == 0
        out16 = torch.full((B * H * W, OC), float("nan"), dtype=torch.float16, device=dev)
        out32 = torch.full((B * H * W, OC), float("nan"), device=dev)
        assert L.rfdetr_b200_op_conv3x3_noalloc(_p(x), C, B, H, W, C, _p(w), OC, _p(g), _p(b), 1e-6, 3,
                                                _p(out32), OC, _p(out16), OC, st) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(out32).all() and torch.isfinite(out16.float()).all()
        assert rel(out32, ref32) < 1e-6, call
        assert rel(out16, ref16) < 1e-3, call
        # the same ConvX block in float64: 3x3 convolution, channel LayerNorm (eps 1e-6), SiLU
        xd = x.double().reshape(B, H, W, C).permute(0, 3, 1, 2)
        wd = w.double().permute(0, 3, 1, 2)  # [oc][ky][kx][c] -> [oc][c][ky][kx]
        y = F.conv2d(xd, wd, padding=1).permute(0, 2, 3, 1)
        y = F.silu(F.layer_norm(y, (OC,), g.double(), b.double(), 1e-6)).reshape(-1, OC)
        assert rel(out32, y) < 1e-4, call
        assert rel(out16, y) < 2e-3, call


def test_noalloc_conv3x3_rejects_oversize():
    from rfdetr_b200 import lib
    L = lib.lib()
    dev = "cuda:0"
    x = torch.zeros(8, 128, dtype=torch.float16, device=dev)
    w = torch.zeros(128, 9 * 128, dtype=torch.float16, device=dev)
    g = torch.ones(128, device=dev)
    out = torch.zeros(8, 128, device=dev)
    # 64 x 64 x 64 pixels x 9 x 128 channels = 302 M values > the 8 Mi fixed scratch: rejected before any launch
    rc = L.rfdetr_b200_op_conv3x3_noalloc(_p(x), 128, 64, 64, 64, 128, _p(w), 128, _p(g), _p(g), 1e-6, 0,
                                          _p(out), 128, None, 0, torch.cuda.current_stream().cuda_stream)
    assert rc != 0
