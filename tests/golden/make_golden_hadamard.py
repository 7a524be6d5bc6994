"""Golden vectors of the reference's Hadamard16 transform and of the weight-gradient
operand quantisation of ``_NVFP4Linear.backward`` (src/mcl4_coe/nvfp4.py:337-355,
:454-459), computed by the REFERENCE's own functions on the CPU:

    python tests/golden/make_golden_hadamard.py --reference-src PATH

(``PATH`` the reference checkout's ``src/`` folder, or set MCL4_REFERENCE_SRC.)
Writes ``hadamard.npz``: the reference's ``_hadamard16_matrix`` and, per case of
``inputs.hadamard_cases``, the input, ``_hadamard16(y.t())`` and the round-to-nearest
quantisation ``_quantize_nvfp4_core`` of that matrix zero-padded to 32 columns (what
``nvfp4_mm`` does with its B operand): packed codes, E4M3 scale bits and global scale.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

from inputs import hadamard_cases  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("MCL4_REFERENCE_SRC"),
                    help="the reference checkout's src/ folder (or set MCL4_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("pass --reference-src PATH (the reference's src/ folder) or set MCL4_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)
    import torch
    from torch.nn import functional as F

    import mcl4_coe.nvfp4 as nv

    out = {"h16": nv._hadamard16_matrix("cpu").numpy()}
    for name, y in hadamard_cases():
        t = torch.from_numpy(np.ascontiguousarray(y))
        ht = nv._hadamard16(t.t())
        cols = ht.shape[1]
        pad = (cols + 31) // 32 * 32 - cols
        rows_pad = (ht.shape[0] + 31) // 32 * 32 - ht.shape[0]
        hp = F.pad(ht, (0, pad, 0, rows_pad)) if (pad or rows_pad) else ht
        packed, scales, g = nv._quantize_nvfp4_core(hp.contiguous(), False, False, False)
        out[f"{name}/y"] = y
        out[f"{name}/ht"] = ht.numpy()
        out[f"{name}/packed"] = packed.numpy()
        out[f"{name}/scales"] = scales.view(torch.uint8).numpy()
        out[f"{name}/g"] = g.numpy()
    np.savez_compressed(HERE / "hadamard.npz", **out)
    print("wrote", HERE / "hadamard.npz", sorted(out))


if __name__ == "__main__":
    main()
