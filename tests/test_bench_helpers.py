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
