"""CPU oracle for the NVFP4 SwiGLU MoE hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithms of the reference
(mESmaC/MCL4-COE, ``src/mcl4_coe/nvfp4.py`` and ``src/mcl4_coe/backbone.py``)
that the B200 kernels must reproduce:

* ``nvfp4_ref``: E2M1 code rounding, E4M3 scale conversion, the per-row
  activation quantiser, the 16x16-tile grouped weight quantiser, the cuBLASLt /
  tcgen05 scale swizzle and the dequantiser.
* ``moe_ref``: fp32 router, softmax, top-k (+ renormalisation), routing
  statistics (counts, aux loss, z loss, selection mask), the stable
  expert-major permutation and the dequantised-FP4 layer forward.

Parity status: PINNED.  ``tests/golden/make_golden.py`` ran the reference's
own functions on CPU and committed their outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks every function here against them.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline.  The product path (the
``mcl4-coe_b200`` package and its CUDA library) never imports it.
"""

from . import nvfp4_ref, moe_ref  # noqa: F401
