"""The kernels' division-free index arithmetic (div_small in
rf-detr.cpp_b200/csrc/kernels.cu): for 0 <= x < 2^21, trunc((x + 1/2) * fl(1/d))
evaluated in float32 equals x // d.  Checked exhaustively for every divisor the
patch extraction and the backbone tap use (patch sizes, window widths, tokens
per window and grid areas of every variant, and all d <= 128)."""
import numpy as np


def test_div_small_exact_below_2_pow_21():
    x = np.arange(0, 1 << 21, dtype=np.int64)
    xf = x.astype(np.float32) + np.float32(0.5)
    divisors = sorted(set(range(1, 129)) | {g * g for g in (24, 32, 36, 40, 44, 48, 50, 64)} |
                      {3 * p * p for p in (12, 14, 16)} | {(g // 2) ** 2 for g in (24, 32, 36, 40, 44, 48)} |
                      {(g // 4) ** 2 for g in (24, 32, 36, 40, 44, 48)} | {256, 400, 484, 576, 1024, 1936})
    for d in divisors:
        inv = np.float32(1.0) / np.float32(d)
        q = np.trunc(xf * inv).astype(np.int64)
        assert np.array_equal(q, x // d), d
