"""Kernel-level numerics on the B200: each sm_100a operator of librfdetr.so,
called through its C-ABI entry point, against a plain PyTorch fp32 (float64
accumulate) reference of the same op.  Inputs are f16 (what the kernels
consume); the tolerance covers f16 output rounding and f32 accumulation order.
"""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _lib():
    from rfdetr_b200 import lib
    return lib.lib()


def _p(t):
    return t.data_ptr() if t is not None else None


def _stream():
    return torch.cuda.current_stream().cuda_stream


def rel(a, b):
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


GEMM_SHAPES = [(300, 256, 256), (1000, 1152, 384), (517, 91, 256), (200, 4, 256), (4097, 1536, 384),
               (333, 384, 1536), (4097, 384, 768), (129, 256, 592), (64, 512, 512), (2000, 2048, 256), (1, 128, 64)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("epi,act", [(0, 0), (1, 0), (0, 1), (0, 2), (2, 0), (1, 1)])
def test_gemm(M, N, K, epi, act):
    torch.manual_seed(M * 7 + N + K)
    dev = "cuda:0"
    lda = (K + 7) // 8 * 8
    A = torch.zeros(M, lda, dtype=torch.float16, device=dev)
    A[:, :K] = torch.randn(M, K, device=dev).half()
    B = torch.zeros(N, lda, dtype=torch.float16, device=dev)
    B[:, :K] = (torch.randn(N, K, device=dev) * 0.05).half()
    bias = torch.randn(N, device=dev) * 0.1
    scale = torch.rand(N, device=dev) + 0.5
    ref = A[:, :K].double() @ B[:, :K].double().T + bias.double()
    if act == 1:
        ref = F.gelu(ref)
    elif act == 2:
        ref = F.relu(ref)
    out16 = torch.zeros(M, N, dtype=torch.float16, device=dev) if epi == 0 else None
    out32 = torch.randn(M, N, device=dev) if epi in (1, 2) else None
    base = out32.clone() if epi == 2 else None
    rc = _lib().rfdetr_b200_op_gemm(_p(A), lda, _p(B), lda, M, N, K, epi, act, _p(bias),
                                    _p(scale) if epi == 2 else None, None, None, 0.0, None, 0,
                                    _p(out32), N, _p(out16), N, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    if epi == 0:
        assert rel(out16, ref) < 2e-3
    elif epi == 1:
        assert rel(out32, ref) < 1e-4
    else:
        assert rel(out32, base.double() + scale.double() * ref) < 1e-4


def test_gelu_epilogue_accuracy():
    """The erf-GELU of the GEMM epilogue on exact accumulators: A holds 65536 f16 values v in
    [-8, 8] in its first column and every row of B selects that column, so the accumulator is v
    exactly; the f32 output must be GELU(v) within 3.5e-7 (the bound of the evaluation) for
    every v, and the f16 output within one f16 spacing of it."""
    dev = "cuda:0"
    vals = torch.linspace(-8, 8, 65536, dtype=torch.float64).half()
    M, N, K = vals.numel(), 8, 16
    A = torch.zeros(M, K, dtype=torch.float16, device=dev)
    A[:, 0] = vals.to(dev)
    B = torch.zeros(N, K, dtype=torch.float16, device=dev)
    B[:, 0] = 1.0
    bias = torch.zeros(N, device=dev)
    ref = F.gelu(vals.double(), approximate="none")
    out32 = torch.zeros(M, N, device=dev)
    assert _lib().rfdetr_b200_op_gemm(_p(A), K, _p(B), K, M, N, K, 1, 1, _p(bias), None, None, None, 0.0, None, 0,
                                      _p(out32), N, None, N, _stream()) == 0
    out16 = torch.zeros(M, N, dtype=torch.float16, device=dev)
    assert _lib().rfdetr_b200_op_gemm(_p(A), K, _p(B), K, M, N, K, 0, 1, _p(bias), None, None, None, 0.0, None, 0,
                                      None, N, _p(out16), N, _stream()) == 0
    torch.cuda.synchronize()
    err32 = (out32.double().cpu() - ref[:, None]).abs().max().item()
    assert err32 < 3.5e-7, err32
    spacing = torch.from_numpy(np.spacing(np.abs(ref.half().numpy())).astype(np.float64))
    err16 = (out16.double().cpu() - ref[:, None]).abs() / spacing[:, None]
    assert err16.max().item() <= 1.0


def _gemm_case(M, N, K, epi, act):
    """One rfdetr_b200_op_gemm call on seeded data against float64 torch."""
    torch.manual_seed(M * 7 + N + K)
    dev = "cuda:0"
    A = (torch.randn(M, K, device=dev)).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    bias = torch.randn(N, device=dev) * 0.1
    scale = torch.rand(N, device=dev) + 0.5
    ref = A.double() @ B.double().T + bias.double()
    if act == 1:
        ref = F.gelu(ref)
    out16 = torch.zeros(M, N, dtype=torch.float16, device=dev) if epi == 0 else None
    out32 = torch.randn(M, N, device=dev) if epi == 2 else None
    base = out32.clone() if epi == 2 else None
    rc = _lib().rfdetr_b200_op_gemm(_p(A), K, _p(B), K, M, N, K, epi, act, _p(bias), _p(scale) if epi == 2 else None,
                                    None, None, 0.0, None, 0, _p(out32), N, _p(out16), N, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    if epi == 0:
        assert rel(out16, ref) < 2e-3
    else:
        assert rel(out32, base.double() + scale.double() * ref) < 1e-4


@pytest.mark.parametrize("M,N,K,epi,act", [(300, 256, 256, 0, 0), (4097, 1536, 384, 0, 1), (1000, 1152, 384, 0, 0),
                                           (4097, 384, 1536, 2, 0), (333, 384, 768, 2, 0), (2000, 256, 512, 2, 0)])
def test_gemm_two_sm_tiles(M, N, K, epi, act, monkeypatch):
    """Two-SM tiles (cta_group::2 over a cluster of two CTAs) forced on for every eligible shape: 192-,
    256- and 384-wide tiles (the last as two N = 192 pair MMAs, each CTA holding half of each slab)."""
    monkeypatch.setenv("RFDETR_GEMM_2SM", "1")
    _gemm_case(M, N, K, epi, act)


def test_gemm_large_residual_default_tiles():
    """The MLP output GEMM at batch-32 scale (M = 40000, N = 384, K = 1536): by default it runs as
    384-wide two-SM tiles."""
    _gemm_case(40000, 384, 1536, 2, 0)


# SiLU is instantiated for the 128 / 256-wide projector LayerNorms only
@pytest.mark.parametrize("N,act,with_resid", [(128, 0, True), (256, 0, True), (384, 0, True),
                                              (128, 3, False), (256, 3, False)])
@pytest.mark.parametrize("M", [777, 40000])
def test_gemm_layernorm_epilogue(N, act, with_resid, M):
    torch.manual_seed(N + act)
    dev = "cuda:0"
    K = 640
    A = torch.randn(M, K, device=dev).half()
    B = (torch.randn(N, K, device=dev) * 0.05).half()
    bias = torch.randn(N, device=dev) * 0.1
    g = torch.rand(N, device=dev) + 0.5
    b = torch.randn(N, device=dev) * 0.1
    resid = torch.randn(M, N, device=dev) if with_resid else None
    v = A.double() @ B.double().T + bias.double()
    if with_resid:
        v = v + resid.double()
    ref = F.layer_norm(v, (N,), g.double(), b.double(), 1e-5)
    if act == 3:
        ref = F.silu(ref)
    out32 = torch.zeros(M, N, device=dev)
    out16 = torch.zeros(M, N, dtype=torch.float16, device=dev)
    rc = _lib().rfdetr_b200_op_gemm(_p(A), K, _p(B), K, M, N, K, 4, act, _p(bias), None, _p(g), _p(b), 1e-5,
                                    _p(resid), N if with_resid else 0, _p(out32), N, _p(out16), N, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert rel(out32, ref) < 1e-4
    assert rel(out16, ref) < 2e-3


@pytest.mark.parametrize("L,groups,heads,hd", [(101, 8, 6, 64), (580, 2, 6, 64), (1616, 1, 6, 64),
                                               (300, 3, 8, 32), (17, 5, 6, 64), (64, 2, 8, 32),
                                               (150, 3, 6, 64), (129, 2, 6, 64), (256, 2, 6, 64)])
def test_attention(L, groups, heads, hd):
    torch.manual_seed(L + groups)
    dev = "cuda:0"
    D = heads * hd
    qkv = torch.randn(groups * L, 3 * D, device=dev).half()
    o = torch.zeros(groups * L, D, dtype=torch.float16, device=dev)
    scale = 1.0 / math.sqrt(hd)
    rc = _lib().rfdetr_b200_op_attention(_p(qkv), _p(qkv[:, D:]), _p(qkv[:, 2 * D:]), 3 * D, 3 * D, 3 * D, _p(o), D,
                                         L, groups, heads, hd, scale, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    x = qkv.double().view(groups, L, 3, heads, hd)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    ref = torch.softmax(q @ k.transpose(-1, -2) * scale, -1) @ v
    ref = ref.transpose(1, 2).reshape(groups * L, D)
    assert rel(o, ref) < 4e-3


@pytest.mark.parametrize("L", [1616, 150, 129])
def test_attention_64_key_blocks(L, monkeypatch):
    """Sequences longer than 128 keys run in 128-key blocks with P in TMEM by default; the 64-key
    kernel (P in shared memory) stays selectable with RFDETR_ATTN_KB=64 and gives the same softmax."""
    monkeypatch.setenv("RFDETR_ATTN_KB", "64")
    test_attention(L, 2, 6, 64)
    test_attention_growing_max(L)


@pytest.mark.parametrize("L", [1616, 150, 700])
def test_attention_growing_max(L):
    """Scores whose row maximum keeps growing along the keys, so the lazily
    raised reference max moves several times and O is rescaled in TMEM."""
    torch.manual_seed(L)
    dev = "cuda:0"
    groups, heads, hd = 2, 6, 64
    D = heads * hd
    qkv = torch.randn(groups * L, 3 * D, device=dev)
    ramp = torch.linspace(0.2, 3.0, L, device=dev).repeat(groups)[:, None]
    qkv[:, D:2 * D] *= ramp  # later keys score higher: the block maxima rise by several log2 units
    qkv = qkv.half()
    o = torch.zeros(groups * L, D, dtype=torch.float16, device=dev)
    scale = 1.0 / math.sqrt(hd)
    rc = _lib().rfdetr_b200_op_attention(_p(qkv), _p(qkv[:, D:]), _p(qkv[:, 2 * D:]), 3 * D, 3 * D, 3 * D, _p(o), D,
                                         L, groups, heads, hd, scale, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    x = qkv.double().view(groups, L, 3, heads, hd)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    ref = torch.softmax(q @ k.transpose(-1, -2) * scale, -1) @ v
    ref = ref.transpose(1, 2).reshape(groups * L, D)
    assert rel(o, ref) < 4e-3


@pytest.mark.parametrize("B,G,NQ,H,P", [(2, 12, 37, 16, 2), (64, 40, 300, 16, 2), (2, 9, 20, 8, 3), (1, 5, 1, 16, 1)])
def test_deform_matches_grid_sample(B, G, NQ, H, P):
    """Deformable sampling (k_deform) against float64 grid_sample: the converter's 16 heads x 2 points
    (the compile-time path that issues both points' corner loads together), at a small and at the
    Base batch-64 decoder shape, and other head / point counts (the run-time path)."""
    torch.manual_seed(B + G + P)
    dev = "cuda:0"
    Dm = 256
    value = torch.randn(B * G * G, Dm, device=dev).half()
    so_aw = torch.randn(B * NQ, H * P * 3, device=dev)
    refp = torch.cat([torch.rand(B * NQ, 2, device=dev), torch.rand(B * NQ, 2, device=dev) * 0.5 + 0.05], 1)
    out = torch.zeros(B * NQ, Dm, dtype=torch.float16, device=dev)
    rc = _lib().rfdetr_b200_op_deform(_p(value), _p(so_aw), H * P * 3, _p(refp), B, NQ, G, H, P, Dm, _p(out),
                                      _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert rel(out, _deform_ref(value, so_aw, refp, B, G, NQ, H, P, Dm)) < 2e-3


def _deform_ref(value, so_aw, refp, B, G, NQ, H, P, Dm):
    """def_attn_op (src/decoder.cpp:127-207) in float64 through grid_sample (zero padding,
    align_corners=False), from the offsets / attention logits rows so_aw."""
    so = so_aw[:, :H * P * 2].double().view(B, NQ, H, P, 2)
    aw = torch.softmax(so_aw[:, H * P * 2:].double().view(B, NQ, H, P), -1)
    rp = refp.double().view(B, NQ, 1, 1, 4)
    loc = rp[..., :2] + so / P * rp[..., 2:] * 0.5
    hd = Dm // H
    vmap = value.double().view(B, G, G, H, hd).permute(0, 3, 4, 1, 2).reshape(B * H, hd, G, G)
    grid = (2 * loc - 1).permute(0, 2, 1, 3, 4).reshape(B * H, NQ, P, 2)
    s = F.grid_sample(vmap, grid, mode="bilinear", padding_mode="zeros", align_corners=False)  # (B*H, hd, NQ, P)
    s = (s * aw.permute(0, 2, 1, 3).reshape(B * H, 1, NQ, P)).sum(-1)
    return s.view(B, H, hd, NQ).permute(0, 3, 1, 2).reshape(B * NQ, Dm)


@pytest.mark.parametrize("oc,act", [(128, 3), (256, 0)])
@pytest.mark.parametrize("B,H,W,Cin,lds", [(2, 9, 7, 128, 128), (3, 40, 40, 128, 640), (2, 24, 24, 64, 64),
                                           (1, 44, 44, 128, 128), (1, 5, 130, 64, 64), (2, 6, 6, 96, 96)])
def test_conv3x3_layernorm(oc, act, B, H, W, Cin, lds):
    """ConvX block (3x3 conv, channel LN, SiLU) against torch conv2d.

    Cin % 64 == 0 and W <= 128 take the implicit GEMM (image rows per 128-row
    tile: 18, 3 with a partial last tile, 5, 2); W = 130 and Cin = 96 take the
    im2col path.  lds > Cin reads the input out of a wider channel-concat map.
    """
    torch.manual_seed(oc + H)
    dev = "cuda:0"
    xw = torch.randn(B, H, W, lds, device=dev).half()
    x = xw[..., :Cin]
    w = (torch.randn(oc, Cin, 3, 3, device=dev) * 0.05)
    wk = w.permute(0, 2, 3, 1).contiguous().half()  # [oc][ky][kx][c]
    g = torch.rand(oc, device=dev) + 0.5
    b = torch.randn(oc, device=dev) * 0.1
    ref = F.conv2d(x.double().permute(0, 3, 1, 2), wk.double().permute(0, 3, 1, 2), padding=1)
    ref = F.layer_norm(ref.permute(0, 2, 3, 1), (oc,), g.double(), b.double(), 1e-6)
    if act == 3:
        ref = F.silu(ref)
    L = _lib()
    ws_bytes = L.rfdetr_b200_op_conv3x3_workspace(B, H, W, Cin)
    assert ws_bytes == B * H * W * 9 * Cin * 2
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    out16 = torch.zeros(B * H * W, oc, dtype=torch.float16, device=dev)
    out32 = torch.zeros(B * H * W, oc, device=dev)
    rc = L.rfdetr_b200_op_conv3x3(_p(xw), lds, B, H, W, Cin, _p(wk), oc, _p(g), _p(b), 1e-6, act, _p(out32), oc,
                                  _p(out16), oc, _p(ws), ws_bytes, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert rel(out32, ref.reshape(-1, oc)) < 1e-4
    assert rel(out16, ref.reshape(-1, oc)) < 2e-3
    # a workspace that is too small is rejected before any launch
    assert L.rfdetr_b200_op_conv3x3(_p(xw), lds, B, H, W, Cin, _p(wk), oc, _p(g), _p(b), 1e-6, act, _p(out32), oc,
                                    _p(out16), oc, _p(ws), ws_bytes - 1, _stream()) != 0



@pytest.mark.parametrize("B,N,NC,K", [(1, 1600, 91, 300), (3, 1225, 91, 300), (2, 4096, 91, 300), (2, 1600, 120, 300),
                                      (1, 50, 91, 50), (2, 20, 91, 7), (1, 1, 91, 1), (2, 700, 1, 300)])
def test_topk_by_max_class(B, N, NC, K):
    """Two-stage token selection (src/rfdetr_model.cpp:39-62) through rfdetr_b200_op_topk: the K
    tokens of largest class maximum in descending order, ties to the lower token.  Logits are
    multiples of 1/8 in a narrow range, so most maxima tie and the tie order is exercised; no
    logit is zero, so signed zeros cannot tie."""
    rng = np.random.default_rng(N + NC)
    cls = ((rng.integers(-40, 40, (B, N, NC)) + 0.5) / 8).astype(np.float32)
    m = cls.max(-1)
    want = np.stack([np.lexsort((np.arange(N), -m[b]))[:K] for b in range(B)]).astype(np.int32)
    d_cls = torch.from_numpy(cls).cuda()
    d_idx = torch.full((B, K), -1, dtype=torch.int32, device="cuda:0")
    L = _lib()
    assert L.rfdetr_b200_op_topk(_p(d_cls), B, N, NC, K, _p(d_idx), _stream()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(d_idx.cpu().numpy(), want)
    # sizes the kernel does not take are rejected before any launch
    assert L.rfdetr_b200_op_topk(_p(d_cls), B, 4097, NC, K, _p(d_idx), _stream()) != 0
    assert L.rfdetr_b200_op_topk(_p(d_cls), B, N, NC, N + 1, _p(d_idx), _stream()) != 0


def test_resize_legacy_matches_the_reference_resize():
    """The legacy preprocess resize (rfdetr_b200_op_resize_legacy) against the reference's own
    stb_image_resize2 output (tests/golden/stb_resize.npz, pinned by
    tests/test_stb_resize_golden.py): growing, shrinking, mixed, kept and 2:1 axes, a batch of two.
    Bytes differ by at most one, and only where a value lies within float rounding of a half (the
    library's SIMD sums run in another order): at least 99.9 % are identical."""
    import os
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import gen_stb_resize_golden as gen

    golden = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "stb_resize.npz"))
    L = _lib()
    for seed, w, h, ow, oh in gen.CASES:
        img = gen.source(seed, w, h)
        src = torch.from_numpy(np.stack([img, img])).cuda()
        dst = torch.zeros((2, oh, ow, 3), dtype=torch.uint8, device="cuda:0")
        assert L.rfdetr_b200_op_resize_legacy(_p(src), 2, w, h, _p(dst), ow, oh, _stream()) == 0
        got = dst.cpu().numpy().astype(np.int32)
        want = golden[f"case_{seed}"].astype(np.int32)
        for b in range(2):
            d = np.abs(got[b] - want)
            assert d.max() <= 1 and (d == 0).mean() >= 0.999, (seed, d.max(), (d == 0).mean())
    assert L.rfdetr_b200_op_resize_legacy(None, 1, 4, 4, None, 2, 2, _stream()) != 0
