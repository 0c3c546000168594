"""Regenerates tests/golden/golden.npz from the reference itself.

Runs the reference's own ``torch.ops.assignment.jonker_dense_batch`` and
``jonker_compact_batch`` (CPU backend of tue-p8n/torchmatch, cpu/ops.cpp:176-289)
on every recipe of cases.py and stores their int64 outputs (as int16, the
compact ones under ``compact__<case>``) plus the input digests.
Needs the reference source tree: ``REF`` names its ``sources`` directory,
by default the checkout beside this repository's (``<parent>/reference``):

    REF=/path/to/torchmatch/sources TORCHMATCH_FORCE_JIT=1 \
        TORCH_EXTENSIONS_DIR=/tmp/tm_ext python tests/golden/make_golden.py
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, os.environ.get("REF", str(HERE.parents[2] / "reference" / "sources")))
sys.path.insert(0, str(HERE))

import torch  # noqa: E402
import torchmatch  # noqa: E402,F401  (loads the reference CPU extension)

from cases import CASES, digest  # noqa: E402


def main() -> None:
    op = torch.ops.assignment.jonker_dense_batch
    op_compact = torch.ops.assignment.jonker_compact_batch
    arrays, meta = {}, {}
    for name, make in CASES.items():
        x = make()
        out = op(x)
        arrays[name] = out.numpy().astype(np.int16)
        arrays["compact__" + name] = op_compact(x).numpy().astype(np.int16)
        meta[name] = {"shape": list(x.shape), "sha256": digest(x)}
        print(name, tuple(x.shape))
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
