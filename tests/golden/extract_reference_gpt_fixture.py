"""Extracts the Stage-1 GPT tensors of the reference's golden fixture
(crates/core/fixtures/golden_ref.safetensors, written by the reference's
`make generate-fixtures` from the Python MLX package with the real checkpoint) into
reference_gpt_fixture.npz beside this script:

  conds F32[1, 3, 1280], token_ids_0..5 I32, prefill_logits F32[8194] (CP-10 target),
  greedy_codes I32[32] (CP-11 target).

The reference's CP-10 / CP-11 tests (crates/core/src/models/gpt.rs:931-979,
crates/core/src/models/sampler.rs:488-536) prefill token_ids_0 with `conds` and language
zh (token id 1), then compare the logits and 32 greedy codes.  Run once where the
reference is checked out:  python tests/golden/extract_reference_gpt_fixture.py <reference root>
"""
import json
import struct
import sys
from pathlib import Path

import numpy as np

NAMES = ["conds", "prefill_logits", "greedy_codes"] + [f"token_ids_{i}" for i in range(6)]
DT = {"F32": np.float32, "I32": np.int32}


def main(root: str) -> None:
    src = Path(root) / "crates/core/fixtures/golden_ref.safetensors"
    with open(src, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name in NAMES:
            h = header[name]
            lo, hi = h["data_offsets"]
            f.seek(base + lo)
            out[name] = np.frombuffer(f.read(hi - lo), DT[h["dtype"]]).reshape(h["shape"])
    dst = Path(__file__).resolve().parent / "reference_gpt_fixture.npz"
    np.savez_compressed(dst, **out)
    print("wrote", dst, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else ".")
