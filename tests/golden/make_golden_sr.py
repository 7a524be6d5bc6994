"""Golden vectors of the reference's stochastic-rounding NVFP4 gradient quantiser.

Runs the REFERENCE's own Triton kernel ``_nvfp4_quantize_1d_kernel`` with
``STOCHASTIC=True`` (src/mcl4_coe/nvfp4.py:735-790, launched by the grouped
backward at :1128-1151) on the CPU through Triton's interpreter, so no GPU is
needed:

    TRITON_INTERPRET=1 python tests/golden/make_golden_sr.py --reference-src PATH

(``PATH`` the reference checkout's ``src/`` folder, or set MCL4_REFERENCE_SRC.)
The global scale follows the reference backward (:1129-1134):
``max(amax/2688 if amax > 0 else 1, FLT_MIN)`` over the whole matrix.  Writes
``sr_quant.npz``: per case the bf16 input bits, the seed, the global scale, the
packed codes [M, K/2] and the E4M3 scales [M, K/16] (row-major), plus
``rn_scales``: the same block scales converted by torch's round-to-nearest
``.to(float8_e4m3fn)``.  On a GPU the kernel's ``.to(tl.float8e4nv)`` is the
hardware's round-to-nearest conversion; the interpreter emulates it in numpy and
truncates subnormal scales and loses the exponent carry of values just below a
power of two, so where ``scales`` and ``rn_scales`` differ the interpreter's bytes
are not the GPU's (the tests compare every other block bit for bit).
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

from inputs import sr_quant_cases  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("MCL4_REFERENCE_SRC"),
                    help="the reference checkout's src/ folder (or set MCL4_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("pass --reference-src PATH (the reference's src/ folder) or set MCL4_REFERENCE_SRC")
    if os.environ.get("TRITON_INTERPRET") != "1":
        ap.error("run with TRITON_INTERPRET=1 (the reference's Triton kernel runs on the CPU interpreter)")
    sys.path.insert(0, args.reference_src)
    import torch
    import triton

    import mcl4_coe.nvfp4 as nv

    out = {}
    for name, bits, seed in sr_quant_cases():
        m, k = bits.shape
        x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
        amax = x.float().abs().amax()
        one = torch.ones(1, dtype=torch.float32)
        g = torch.where(amax > 0, amax / 2688.0, one).clamp_min(1.17549435e-38).reshape(1)
        qa = torch.empty((m, k // 2), dtype=torch.uint8)
        sa = torch.empty((m, k // 16), dtype=torch.float8_e4m3fn)
        nv._nvfp4_quantize_1d_kernel[(triton.cdiv(m, 32), k // 128)](
            x, g, qa, sa, m, K=k, seed=seed, BLOCK_M=32, BLOCK_K=128, STOCHASTIC=True)
        out[f"{name}__x_bits"] = bits
        out[f"{name}__seed"] = np.array(seed, np.int64)
        out[f"{name}__g"] = g.numpy().astype(np.float32)
        out[f"{name}__packed"] = qa.numpy()
        out[f"{name}__scales"] = sa.view(torch.uint8).numpy()
        blocks = x.float().reshape(m, k // 16, 16).abs().amax(dim=-1)
        rn = torch.clamp(blocks / (6.0 * g), max=448.0).to(torch.float8_e4m3fn)
        out[f"{name}__rn_scales"] = rn.view(torch.uint8).numpy()
    np.savez_compressed(HERE / "sr_quant.npz", **out)
    print("wrote", HERE / "sr_quant.npz", sorted(out)[:3], "...")


if __name__ == "__main__":
    main()
