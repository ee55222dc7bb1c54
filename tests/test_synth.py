"""Synthetic model fixtures: the writer reproduces the reference converter's
bytes (golden digests from tests/golden/gen_converter_golden.py), and the
per-dtype tensor census follows the reference's quantization rules
(tests/test_kquant.cpp:86-121, tests/test_q8_quant.cpp:93-115)."""
import hashlib
import json
import os

import numpy as np
import pytest

from rfdetr_b200 import synth

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "converter_digests.json")


@pytest.mark.parametrize("case", sorted(json.load(open(GOLDEN))))
def test_writer_matches_reference_converter(case, tmp_path):
    variant, dtype, seed = case.split("/")
    p = tmp_path / "m.gguf"
    synth.write_model(str(p), variant, dtype, int(seed))
    assert hashlib.sha256(p.read_bytes()).hexdigest() == json.load(open(GOLDEN))[case]


def test_inventory_counts():
    # gen_model_gguf.cpp:1-15 — a base-structured model has 486 tensors.
    assert len(synth.tensor_specs(synth.get_variant("base"))) == 486
    seg = synth.get_variant("seg-small")
    n_det = len(synth.tensor_specs(synth.get_variant("nano")))
    # seg adds 6 per decoder layer + 11 shared (src/model_loader.hpp:72-76)
    assert len(synth.tensor_specs(seg)) - (n_det + 22 * (4 - 2)) == 6 * 4 + 11


def test_q4k_census(tmp_path):
    cfg = synth.get_variant("tiny")
    st = synth.make_state(cfg, 0)
    types = synth.write_gguf(str(tmp_path / "q.gguf"), "tiny", cfg, st, "q4_K")
    # dim-384 rows fall back to Q8_0; K = 256/512/1536 rows are Q4_K
    assert types["backbone.blocks.0.attn.q.weight"] == "q8_0"
    assert types["backbone.blocks.0.mlp.fc1.weight"] == "q8_0"
    assert types["backbone.blocks.0.mlp.fc2.weight"] == "q4_K"
    assert types["two_stage.enc_output.0.weight"] == "q4_K"
    assert types["decoder.ref_point_head.layers.0.weight"] == "q4_K"
    # stays F32: conv kernels, attention_weights (N=32), bbox last layer (N=4), embeddings
    for n in ("backbone.patch_embed.weight", "projector.cv1.conv.weight",
              "decoder.layers.0.cross_attn.attention_weights.weight",
              "heads.bbox_embed.layers.2.weight", "backbone.pos_embed", "decoder.queries.feat"):
        assert types[n] == "f32", n
    n_q8 = sum(t == "q8_0" for t in types.values())
    n_f32 = sum(t == "f32" for t in types.values())
    assert n_q8 > 50 and n_f32 > 100


def test_q4k_roundtrip_matches_gguf_py():
    import gguf
    a = (np.random.default_rng(3).standard_normal((16, 768)) * 0.02).astype(np.float32)
    q = synth.quantize_q4_K(a)
    assert q.shape == (16, 3 * 144)
    d_ours = synth.dequantize_q4_K(q, a.size).reshape(a.shape)
    d_ref = gguf.quants.dequantize(q, gguf.GGMLQuantizationType.Q4_K).reshape(a.shape)
    assert np.array_equal(d_ours, d_ref)
    # 4-bit with 6-bit sub-block scales: error well under one quant step of the block range
    err = np.abs(d_ours - a).reshape(-1, 32).max(1)
    rng = (a.reshape(-1, 32).max(1) - np.minimum(a.reshape(-1, 32).min(1), 0))
    assert np.all(err <= rng / 15 + 1e-6)
