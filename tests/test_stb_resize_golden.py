"""The legacy-resize golden vectors (tests/golden/stb_resize.npz) against the
reference's own resize: oracle/_ref/libstbresize.so is stb_image_resize2 built
from the reference tree (`make -C oracle ref`, run by the build when the tree
is present); regenerating every case from its seed gives the committed bytes.
The GPU kernel is checked against the same vectors in tests/test_gpu_ops.py."""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "tests", "golden"))


def test_golden_vectors_are_the_reference_resize():
    import gen_stb_resize_golden as gen

    if not os.path.exists(gen.REF_SO):
        pytest.skip("oracle/_ref/libstbresize.so is built only where the reference tree is present")
    golden = np.load(os.path.join(REPO, "tests", "golden", "stb_resize.npz"))
    assert [tuple(c) for c in golden["cases"]] == gen.CASES
    for seed, w, h, ow, oh in gen.CASES:
        assert np.array_equal(gen.stb_resize(gen.source(seed, w, h), ow, oh), golden[f"case_{seed}"])
