"""Independent PyTorch restatement of the RF-DETR forward (test infrastructure).

Written against the PyTorch operators whose semantics the reference engine
(localai-org/rf-detr.cpp) documents as its own parity target: F.interpolate
bicubic antialias for the pos-embed (src/model_loader.cpp:83-116),
grid_sample-style bilinear sampling for MSDeformAttn (src/decoder.cpp:103-207,
ms_deform_attn_core_pytorch), F.interpolate bilinear align_corners=False for the
segmentation resize (src/segmentation.cpp:187-199).  It shares no code with the
C++ oracle, so agreement between the two pins the oracle.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).double()


class TorchRef:
    def __init__(self, meta: dict, tensors: dict):
        self.m = meta
        self.w = {k: _t(a) for k, (_ty, a) in tensors.items()}

    def g(self, k):
        return int(self.m["rfdetr." + k])

    def lin(self, x, name):
        return F.linear(x, self.w[name + ".weight"], self.w[name + ".bias"])

    def ln(self, x, name, eps):
        return F.layer_norm(x, (x.shape[-1],), self.w[name + ".weight"], self.w[name + ".bias"], eps)

    def forward(self, planar: np.ndarray):
        g = self.g
        S, p = g("image_size"), g("patch_size")
        G = S // p
        D, H = g("backbone.dim"), g("backbone.heads")
        nw = g("backbone.num_windows")
        ws = G // nw
        T = ws * ws + 1
        glob = set(self.m["rfdetr.backbone.global_attn_indices"])
        taps = list(self.m["rfdetr.backbone.out_feature_indices"])
        out = {}

        x = _t(planar)[None]  # (1,3,S,S)
        emb = F.conv2d(x, self.w["backbone.patch_embed.weight"], self.w["backbone.patch_embed.bias"], stride=p)
        tok = emb.flatten(2).transpose(1, 2)[0]  # (G*G, D)
        pe = self.w["backbone.pos_embed"]
        ts = g("backbone.pos_embed_train_size")
        grid = pe[1:].reshape(1, ts, ts, D).permute(0, 3, 1, 2)
        if ts != G:
            grid = F.interpolate(grid, size=(G, G), mode="bicubic", align_corners=False, antialias=True)
        pos_p = grid.permute(0, 2, 3, 1).reshape(G * G, D)
        tok = tok + pos_p
        cls = self.w["backbone.cls_token"] + pe[0]
        # windowing: (G,G,D) -> (nw, ws, nw, ws, D) -> (nw*nw, ws*ws, D)
        wt = tok.reshape(nw, ws, nw, ws, D).permute(0, 2, 1, 3, 4).reshape(nw * nw, ws * ws, D)
        xw = torch.cat([cls.expand(nw * nw, 1, D), wt], 1)  # (NW, T, D)
        hd = D // H
        for i in range(g("backbone.depth")):
            b = f"backbone.blocks.{i}."
            h = self.ln(xw, b + "norm1", 1e-6)
            if i in glob:
                h = h.reshape(1, -1, D)
            q, k, v = self.lin(h, b + "attn.q"), self.lin(h, b + "attn.k"), self.lin(h, b + "attn.v")
            B_, L_ = q.shape[:2]
            q = q.reshape(B_, L_, H, hd).transpose(1, 2)
            k = k.reshape(B_, L_, H, hd).transpose(1, 2)
            v = v.reshape(B_, L_, H, hd).transpose(1, 2)
            a = torch.softmax((q / math.sqrt(hd)) @ k.transpose(-1, -2), -1) @ v
            a = a.transpose(1, 2).reshape(B_, L_, D).reshape(nw * nw, T, D)
            xw = xw + self.lin(a, b + "attn.proj") * self.w[b + "layer_scale1"]
            y = self.ln(xw, b + "norm2", 1e-6)
            y = self.lin(F.gelu(self.lin(y, b + "mlp.fc1")), b + "mlp.fc2")
            xw = xw + y * self.w[b + "layer_scale2"]
            if (i + 1) in taps:
                n = self.ln(xw, "backbone.norm", 1e-6)[:, 1:]
                sp = n.reshape(nw, nw, ws, ws, D).permute(0, 2, 1, 3, 4).reshape(G * G, D)
                out[f"tap{taps.index(i + 1)}"] = sp

        # projector (channels-first conv semantics)
        def convx(x, name, k):
            y = F.conv2d(x, self.w[name + ".conv.weight"], None, padding=k // 2)
            y = F.layer_norm(y.permute(0, 2, 3, 1), (y.shape[1],), self.w[name + ".norm.weight"],
                             self.w[name + ".norm.bias"], 1e-6).permute(0, 3, 1, 2)
            return F.silu(y)

        feat = torch.cat([out[f"tap{j}"] for j in range(len(taps))], 1)
        feat = feat.reshape(1, G, G, -1).permute(0, 3, 1, 2)
        hcv = convx(feat, "projector.cv1", 1)
        c = hcv.shape[1] // 2
        ys = [hcv[:, :c], hcv[:, c:]]
        cur = ys[1]
        for j in range(g("projector.n_bottlenecks")):
            cur = convx(convx(cur, f"projector.bottleneck.{j}.cv1", 3), f"projector.bottleneck.{j}.cv2", 3)
            ys.append(cur)
        pr = convx(torch.cat(ys, 1), "projector.cv2", 1)
        pr = F.layer_norm(pr.permute(0, 2, 3, 1), (pr.shape[1],), self.w["projector.final_norm.weight"],
                          self.w["projector.final_norm.bias"], 1e-6)  # (1,G,G,C)
        mem = pr.reshape(G * G, -1)
        out["projector"] = mem

        # two-stage
        gy, gx = torch.meshgrid(torch.arange(G, dtype=torch.float64), torch.arange(G, dtype=torch.float64),
                                indexing="ij")
        prop = torch.stack([(gx + 0.5) / G, (gy + 0.5) / G, torch.full_like(gx, 0.05),
                            torch.full_like(gx, 0.05)], -1).reshape(-1, 4)
        valid = ((prop > 0.01) & (prop < 0.99)).all(-1, keepdim=True)
        prop = prop.masked_fill(~valid, 0.0)
        om = mem.masked_fill(~valid, 0.0)
        y = self.ln(self.lin(om, "two_stage.enc_output.0"), "two_stage.enc_output_norm.0", 1e-5)
        cls_all = self.lin(y, "two_stage.enc_out_class_embed.0")
        bb = "two_stage.enc_out_bbox_embed.0.layers."
        d = self.lin(F.relu(self.lin(F.relu(self.lin(y, bb + "0")), bb + "1")), bb + "2")
        bbox_all = torch.cat([d[:, :2] * prop[:, 2:] + prop[:, :2], d[:, 2:].exp() * prop[:, 2:]], -1)
        out["cls_all"], out["bbox_all"] = cls_all, bbox_all

        NQ = g("num_queries")
        score = cls_all.max(-1)[0]
        # descending score, ties by lower index (stable sort of the negated score)
        idx = torch.sort(-score, stable=True)[1][:NQ]
        out["topk"] = idx
        box = bbox_all[idx]
        lrn = self.w["decoder.queries.refpoints"][:NQ]
        rp = torch.cat([lrn[:, :2] * box[:, 2:] + box[:, :2], lrn[:, 2:].exp() * box[:, 2:]], -1)
        out["refpoints"] = rp

        Dm = g("decoder.model_dim")
        half = Dm // 2
        dim_t = 10000 ** (2 * (torch.arange(half, dtype=torch.float64) // 2) / half)

        def emb1(v):
            pv = v[:, None] * 2 * math.pi / dim_t
            return torch.stack([pv[:, 0::2].sin(), pv[:, 1::2].cos()], -1).flatten(1)

        sine = torch.cat([emb1(rp[:, 1]), emb1(rp[:, 0]), emb1(rp[:, 2]), emb1(rp[:, 3])], -1)
        qpos = self.lin(F.relu(self.lin(sine, "decoder.ref_point_head.layers.0")), "decoder.ref_point_head.layers.1")

        tgt = self.w["decoder.queries.feat"][:NQ]
        sh, ch_, npt = g("decoder.self_attn_heads"), g("decoder.cross_attn_heads"), g("decoder.cross_attn_n_points")
        per_layer = []
        for li in range(g("decoder.layers")):
            b = f"decoder.layers.{li}."
            W_ip, b_ip = self.w[b + "self_attn.in_proj.weight"], self.w[b + "self_attn.in_proj.bias"]
            qk = tgt + qpos
            q = F.linear(qk, W_ip[:Dm], b_ip[:Dm])
            k = F.linear(qk, W_ip[Dm:2 * Dm], b_ip[Dm:2 * Dm])
            v = F.linear(tgt, W_ip[2 * Dm:], b_ip[2 * Dm:])
            hd = Dm // sh
            qh = q.reshape(NQ, sh, hd).transpose(0, 1)
            kh = k.reshape(NQ, sh, hd).transpose(0, 1)
            vh = v.reshape(NQ, sh, hd).transpose(0, 1)
            a = torch.softmax(qh @ kh.transpose(-1, -2) / math.sqrt(hd), -1) @ vh
            sa = self.lin(a.transpose(0, 1).reshape(NQ, Dm), b + "self_attn.out_proj")
            x = self.ln(tgt + sa, b + "norm1", 1e-5)
            cq = x + qpos
            so = self.lin(cq, b + "cross_attn.sampling_offsets").reshape(NQ, ch_, npt, 2)
            aw = torch.softmax(self.lin(cq, b + "cross_attn.attention_weights").reshape(NQ, ch_, npt), -1)
            loc = rp[:, None, None, :2] + so / npt * rp[:, None, None, 2:] * 0.5
            val = self.lin(mem, b + "cross_attn.value_proj")  # (G*G, Dm)
            chd = Dm // ch_
            vmap = val.reshape(G, G, ch_, chd).permute(2, 3, 0, 1)  # (heads, chd, G, G)
            grid_ = (2 * loc - 1).permute(1, 0, 2, 3)  # (heads, NQ, npt, 2)
            smp = F.grid_sample(vmap, grid_, mode="bilinear", padding_mode="zeros", align_corners=False)
            smp = (smp * aw.permute(1, 0, 2)[:, None]).sum(-1)  # (heads, chd, NQ)
            smp = smp.permute(2, 0, 1).reshape(NQ, Dm)
            ca = self.lin(smp, b + "cross_attn.output_proj")
            x = self.ln(x + ca, b + "norm2", 1e-5)
            f = self.lin(F.relu(self.lin(x, b + "linear1")), b + "linear2")
            x = self.ln(x + f, b + "norm3", 1e-5)
            tgt = x
            per_layer.append(self.ln(x, "decoder.norm", 1e-5))
        dec = self.ln(tgt, "decoder.norm", 1e-5)
        out["decoder"] = dec
        logits = self.lin(dec, "heads.class_embed")
        hb = "heads.bbox_embed.layers."
        bd = self.lin(F.relu(self.lin(F.relu(self.lin(dec, hb + "0")), hb + "1")), hb + "2")
        boxes = torch.cat([bd[:, :2] * rp[:, 2:] + rp[:, :2], bd[:, 2:].exp() * rp[:, 2:]], -1)
        out["logits"], out["boxes"] = logits, boxes

        if self.m.get("rfdetr.has_segmentation_head", False):
            r = g("mask_downsample_ratio")
            Ht = S // r
            sp = F.interpolate(pr.permute(0, 3, 1, 2), size=(Ht, Ht), mode="bilinear", align_corners=False)
            for bi in range(g("decoder.layers")):
                b = f"segmentation_head.blocks.{bi}."
                y = F.conv2d(sp, self.w[b + "dwconv.weight"], self.w[b + "dwconv.bias"], padding=1, groups=Dm)
                y = self.ln(y.permute(0, 2, 3, 1), b + "norm", 1e-6)
                y = F.gelu(self.lin(y, b + "pwconv1")).permute(0, 3, 1, 2)
                sp = y + sp
            spp = F.conv2d(sp, self.w["segmentation_head.spatial_features_proj.weight"],
                           self.w["segmentation_head.spatial_features_proj.bias"])
            qf = per_layer[-1]
            qb = "segmentation_head.query_features_block."
            qn = self.ln(qf, qb + "norm_in", 1e-6)
            qf = self.lin(F.gelu(self.lin(qn, qb + "layers.0")), qb + "layers.2") + qf
            qf = self.lin(qf, "segmentation_head.query_features_proj")
            masks = torch.einsum("chw,nc->nhw", spp[0], qf) + self.w["segmentation_head.bias"]
            out["masks"] = masks
        return {k: (v.numpy() if isinstance(v, torch.Tensor) else v) for k, v in out.items()}
