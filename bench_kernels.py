"""Micro-benchmark of single engine operators at model shapes.

    python bench_kernels.py gemm --m 51712 --n 1536 --k 384 [--epi 0 --act 1] [--cublas]
    python bench_kernels.py attn --seq 1616 --groups 32 --heads 6 --hd 64
    python bench_kernels.py deform --batch 32 --grid 40 --nq 300 --heads 16 --points 2
    python bench_kernels.py topk --batch 1 --grid 40 --nc 91 --nq 300

Times `--iters` launches with CUDA events on the current stream (after
`--warmup` launches) and prints one JSON line: ms per launch and achieved
TFLOP/s (algorithmic FLOPs: 2*M*N*K for a GEMM, 4*L^2*hd per (group, head)
for attention) or GB/s for the deformable sampling (algorithmic bytes: the
value map read once, the offset/logit rows, the reference points and the f16
output) and the two-stage top-K (the grid x grid x nc f32 class logits of each
image read once, the nq int32 indices written).  Used for ncu captures of one
kernel in isolation.  `gemm --cublas` times the library GEMM of the same shape
instead (torch.matmul, f16 in and out, no bias or activation) as a point of
comparison; it is not part of the engine.
"""
import argparse
import json
import math
import os
import sys

import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "rf-detr.cpp_b200"))
from rfdetr_b200 import lib  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["gemm", "attn", "deform", "topk"])
    ap.add_argument("--m", type=int, default=51712)
    ap.add_argument("--n", type=int, default=1536)
    ap.add_argument("--k", type=int, default=384)
    ap.add_argument("--epi", type=int, default=0)
    ap.add_argument("--act", type=int, default=1)
    ap.add_argument("--seq", type=int, default=1616)
    ap.add_argument("--groups", type=int, default=32)
    ap.add_argument("--heads", type=int, default=6)
    ap.add_argument("--hd", type=int, default=64)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--grid", type=int, default=40)
    ap.add_argument("--nq", type=int, default=300)
    ap.add_argument("--points", type=int, default=2)
    ap.add_argument("--dm", type=int, default=256)
    ap.add_argument("--nc", type=int, default=91)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--cublas", action="store_true")
    ap.add_argument("--ln", type=int, default=0, help="gemm: LayerNorm epilogue (epi 4): 1 = plain, 2 = with a "
                                                         "residual and f32 + f16 outputs (the decoder's form)")
    a = ap.parse_args()
    L = lib.lib()
    dev = "cuda:0"
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=dev).manual_seed(0)
    if a.op == "gemm":
        A = torch.randn(a.m, a.k, device=dev, generator=g).half()
        B = (torch.randn(a.n, a.k, device=dev, generator=g) * 0.05).half()
        bias = torch.zeros(a.n, device=dev)
        out16 = torch.empty(a.m, a.n, dtype=torch.float16, device=dev)
        out32 = torch.empty(a.m, a.n, device=dev) if a.epi in (1, 2) or a.ln == 2 else None
        lng = torch.ones(a.n, device=dev)
        lnb = torch.zeros(a.n, device=dev)
        resid = torch.randn(a.m, a.n, device=dev, generator=g) if a.ln == 2 else None
        epi = 4 if a.ln else a.epi

        def run():
            rc = L.rfdetr_b200_op_gemm(A.data_ptr(), a.k, B.data_ptr(), a.k, a.m, a.n, a.k, epi, a.act,
                                       bias.data_ptr(), None, lng.data_ptr() if a.ln else None,
                                       lnb.data_ptr() if a.ln else None, 1e-5,
                                       resid.data_ptr() if resid is not None else None, a.n,
                                       out32.data_ptr() if out32 is not None else None, a.n, out16.data_ptr(),
                                       a.n, st)
            assert rc == 0, rc
        flops = 2.0 * a.m * a.n * a.k
        name = f"gemm M={a.m} N={a.n} K={a.k} epi={epi} act={a.act}" + (f" ln={a.ln}" if a.ln else "")
        if a.cublas:
            Bt = B.t()

            def run():
                torch.matmul(A, Bt, out=out16)
            name = f"cublas gemm M={a.m} N={a.n} K={a.k} (f16 out, no epilogue)"
    elif a.op == "deform":
        H, P, Dm, NQ, G, B = a.heads, a.points, a.dm, a.nq, a.grid, a.batch
        ld = H * P * 3
        value = (torch.randn(B * G * G, Dm, device=dev, generator=g)).half()
        so_aw = torch.randn(B * NQ, ld, device=dev, generator=g)
        refp = torch.rand(B * NQ, 4, device=dev, generator=g) * 0.5 + 0.25
        out = torch.empty(B * NQ, Dm, dtype=torch.float16, device=dev)

        def run():
            rc = L.rfdetr_b200_op_deform(value.data_ptr(), so_aw.data_ptr(), ld, refp.data_ptr(), B, NQ, G, H, P,
                                         Dm, out.data_ptr(), st)
            assert rc == 0, rc
        nbytes = value.numel() * 2 + so_aw.numel() * 4 + refp.numel() * 4 + out.numel() * 2
        name = f"deform batch={B} grid={G} nq={NQ} heads={H} points={P} dm={Dm}"
    elif a.op == "topk":
        B, N, NC, K = a.batch, a.grid * a.grid, a.nc, a.nq
        cls = torch.randn(B, N, NC, device=dev, generator=g)
        idx = torch.empty(B, K, dtype=torch.int32, device=dev)

        def run():
            rc = L.rfdetr_b200_op_topk(cls.data_ptr(), B, N, NC, K, idx.data_ptr(), st)
            assert rc == 0, rc
        nbytes = cls.numel() * 4 + idx.numel() * 4
        name = f"topk batch={B} tokens={N} classes={NC} k={K}"
    else:
        D = a.heads * a.hd
        qkv = torch.randn(a.groups * a.seq, 3 * D, device=dev, generator=g).half()
        o = torch.empty(a.groups * a.seq, D, dtype=torch.float16, device=dev)

        def run():
            rc = L.rfdetr_b200_op_attention(qkv.data_ptr(), qkv[:, D:].data_ptr(), qkv[:, 2 * D:].data_ptr(),
                                            3 * D, 3 * D, 3 * D, o.data_ptr(), D, a.seq, a.groups, a.heads, a.hd,
                                            1.0 / math.sqrt(a.hd), st)
            assert rc == 0, rc
        flops = 4.0 * a.seq * a.seq * a.hd * a.groups * a.heads
        name = f"attention L={a.seq} groups={a.groups} heads={a.heads} hd={a.hd}"
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    if a.op in ("deform", "topk"):
        print(json.dumps({"op": name, "ms": round(ms, 5), "gbs": round(nbytes / ms / 1e6, 1),
                          "bytes": nbytes}))
    else:
        print(json.dumps({"op": name, "ms": round(ms, 5), "tflops": round(flops / ms / 1e9, 1)}))


if __name__ == "__main__":
    main()
