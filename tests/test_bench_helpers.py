"""The benchmark's measurement arithmetic, on the CPU: the backbone GEMM FLOP
count behind the roofline (68.63 GFLOP per RF-DETR Base image), the parsing of
the clock samples that flags throttled runs, and the profile-derived DRAM
traffic of the roofline object."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "rf-detr.cpp_b200"))


def test_backbone_gemm_flops_of_base():
    import bench
    from rfdetr_b200 import synth

    cfg = synth.get_variant("base")
    per = bench.backbone_gemm_flops(cfg, 1)
    total = cfg["backbone"]["depth"] * (per["qkv"] + per["proj"] + per["fc1"] + per["fc2"])
    assert abs(total / 1e9 - 68.63) < 0.01
    assert bench.backbone_gemm_flops(cfg, 32)["qkv"] == 32 * per["qkv"]


def test_backbone_gemm_bytes_and_bounds_of_base():
    """Base batch 64 (M = 103424 rows): qkv and fc1 are bound by the tensor peak, proj by
    HBM (its f32 residual read-modify-write), and the per-launch fractions recombine."""
    import bench
    from rfdetr_b200 import synth

    cfg = synth.get_variant("base")
    by = bench.backbone_gemm_bytes(cfg, 64)
    M, D, F = 103424, 384, 1536
    assert by["proj"] == 2 * (M * D + D * D) + 8 * M * D
    assert by["fc2"] == 2 * (M * F + D * F) + 8 * M * D
    fl = bench.backbone_gemm_flops(cfg, 64)
    g_ms = {"qkv": 0.105, "proj": 0.0736, "fc1": 0.155, "fc2": 0.135}
    g_n = {k: 1 for k in g_ms}
    parts, own = bench.gemm_parts(fl, by, g_ms, g_n, 6545.0, 1368.8)
    assert parts["qkv"]["bound"] == "tensor" and parts["fc1"]["bound"] == "tensor"
    assert parts["proj"]["bound"] == "hbm" and parts["fc2"]["bound"] == "hbm"
    t_bound = sum(max(parts[k]["frac_tensor"], parts[k]["frac_hbm"]) * g_ms[k] for k in g_ms)
    assert abs(own - t_bound / sum(g_ms.values())) < 1e-3
    assert 0.5 < parts["proj"]["frac_hbm"] < 1.0


def _clocks(rows):
    import bench

    c = bench.Clocks(0)
    c.f.write("\n".join(rows) + "\n")
    c.f.flush()
    return c.stop()


def test_clock_samples_median_under_load_and_power_cap():
    busy = "0, 1965, 1965, 900.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active"
    idle = "0, 345, 1965, 120.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"
    out = _clocks([idle] + [busy] * 4 + ["0, 1830, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active"])
    assert out["sm_mhz"] == 1965 and out["sm_max_mhz"] == 1965 and out["samples"] == 6
    assert out["reasons"] == ["sw_power_cap"]


def test_clock_samples_flag_thermal_slowdown():
    rows = ["0, 1500, 1965, 700.0, 0x40, Not Active, Active, Not Active, Not Active"] * 3
    assert _clocks(rows)["reasons"] == ["hw_thermal_slowdown"]


def test_clock_samples_absent():
    assert _clocks([])["reasons"] == ["unsampled"]


def test_roofline_traffic_from_the_committed_profile():
    import bench

    t = bench.traffic_from_profiles()
    assert t["bytes_per_launch"] == t["dram_read_bytes"] + t["dram_write_bytes"]
    assert 0 < t["bytes_per_launch"] <= t["algorithmic_bytes"]


def test_clock_sampler_names_the_visible_gpu(monkeypatch):
    import bench

    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert bench.smi_device(1) == "5"
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-aaaa, GPU-bbbb")
    assert bench.smi_device(0) == "GPU-aaaa"
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.smi_device(2) == "2"
