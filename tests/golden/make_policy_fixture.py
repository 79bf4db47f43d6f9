"""Write a policy directory with the REFERENCE's own policy code.

Run from the repository root where the GASSFY/Logitfill sources are
importable (``--reference-src``, default ``$LOGITFILL_REFERENCE_SRC``):

    python tests/golden/make_policy_fixture.py --reference-src <logitfill>/src

It builds a Key tier map for the tiny Qwen2 shape the adapter tests use
(2 layers, 2 KV heads, head_dim 128; the seeded water-filling policy at
target_bit 2.5 of ``logitfill_b200.synthetic``) and saves it with the
reference's ``build_policy(...).save(...)`` (``src/logitfill/allocators/policy.py``)
into ``tests/golden/policy_ref/``: ``policy.npz`` + ``metadata.json`` exactly
as LogitFill's offline calibration writes them.  The GPU test
``tests/test_policy_gpu.py`` loads that directory through
``DeepSeekQwenKVAdapter.load_policy`` and decodes through it; nothing at test
time imports the reference.
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

OUT = HERE / "policy_ref"
MODEL_ID = "tiny-qwen2-test"


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reference-src", default=os.environ.get("LOGITFILL_REFERENCE_SRC"))
    args = ap.parse_args()
    if not args.reference_src:
        raise SystemExit("give --reference-src (the reference's src/ directory)")
    sys.path.insert(0, args.reference_src)
    from logitfill.allocators.policy import build_policy

    from logitfill_b200.synthetic import synthetic_levels

    levels = np.asarray(synthetic_levels(2, 2, 128, 2.5, seed=3), np.int64)
    curves = {"d2": np.linspace(0.0, 1.0, levels.size).reshape(levels.shape)}
    policy = build_policy(levels, model_id=MODEL_ID, target_bit=2.5, bit_v=2, curves=curves)
    if OUT.exists():
        shutil.rmtree(OUT)
    policy.save(OUT)
    print(f"wrote {OUT}: levels {levels.shape}, metadata keys {sorted(policy.metadata)}")


if __name__ == "__main__":
    main()
