"""Generate tests/golden/converter_digests.json from the reference converter.

Runs the reference's own `write_gguf` + `build_tensor_name_map`
(scripts/convert_rfdetr_to_gguf.py:265-679) on the seeded synthetic state
dict and records the SHA-256 of each written file.  The repository's writer
(rfdetr_b200.synth) must reproduce these bytes exactly.

Needs a checkout of localai-org/rf-detr.cpp named by RFDETR_REFERENCE; run
from the repository root:
    RFDETR_REFERENCE=<checkout> python tests/golden/gen_converter_golden.py
"""
import hashlib
import json
import os
import sys
import tempfile

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(REPO, "rf-detr.cpp_b200"))
REF = os.environ.get("RFDETR_REFERENCE")
if not REF or not os.path.isfile(os.path.join(REF, "scripts", "convert_rfdetr_to_gguf.py")):
    raise SystemExit("set RFDETR_REFERENCE to a checkout of localai-org/rf-detr.cpp "
                     "(scripts/convert_rfdetr_to_gguf.py is read from it)")
sys.path.insert(0, os.path.join(REF, "scripts"))

import torch  # noqa: E402
import convert_rfdetr_to_gguf as ref  # noqa: E402
from rfdetr_b200 import synth  # noqa: E402

CASES = [("tiny", "f32", 0), ("tiny", "f16", 1), ("tiny", "q8_0", 2),
         ("seg-tiny", "f16", 3), ("tiny-base", "q8_0", 4)]


def sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def main():
    out = {}
    for variant, dtype, seed in CASES:
        cfg = synth.get_variant(variant)
        torch_state = synth.make_torch_state(cfg, seed)
        name_map = ref.build_tensor_name_map(cfg)
        assert list(name_map.keys()) == list(torch_state.keys()), "tensor inventory differs"
        sd = {src: torch.from_numpy(torch_state[g]) for g, (src, _t) in name_map.items()}
        with tempfile.TemporaryDirectory() as td:
            p = os.path.join(td, "m.gguf")
            ref.write_gguf(p, variant, cfg, name_map, sd, dtype)
            out[f"{variant}/{dtype}/{seed}"] = sha(p)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "converter_digests.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
