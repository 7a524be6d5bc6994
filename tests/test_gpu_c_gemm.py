"""tcgen05 grouped NVFP4 GEMM (the reference's ``nvfp4_grouped_linear`` seam)
vs the dequantised-FP4 product computed in fp32."""

import numpy as np
import pytest
import torch

from gpu_ref import rel_l2
from inputs import bf16_values, rng
from oracle import nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _Experts(torch.nn.Module):
    def __init__(self, weights):
        super().__init__()
        self.experts = torch.nn.ModuleList()
        for w in weights:
            m = torch.nn.Module()
            m.proj = torch.nn.Linear(w.shape[1], w.shape[0], bias=False)
            with torch.no_grad():
                m.proj.weight.copy_(torch.from_numpy(w))
            self.experts.append(m)


def _reference(x: np.ndarray, counts, w: np.ndarray) -> np.ndarray:
    """bf16(quant(x_e) . deq(W_e)^T) per expert segment (src/mcl4_coe/nvfp4.py:848-873)."""
    b_fwd, bs_fwd, bg, _, _ = nr.quantize_grouped_weights(w)
    out = np.zeros((x.shape[0], w.shape[1]), np.float32)
    start = 0
    for e, c in enumerate(counts):
        if c:
            wd = nr.dequantize_grouped_weight(b_fwd, bs_fwd, bg, e)
            xq = nr.fake_quantize_activations(x[start:start + c])
            out[start:start + c] = nr.round_bf16((xq.astype(np.float64) @ wd.T.astype(np.float64)).astype(np.float32))
        start += c
    return out


@pytest.mark.parametrize("counts,K,N", [
    ([128], 256, 256),                                  # one full tile
    ([1, 0, 127, 128, 129, 300, 0, 513], 512, 512),     # ragged, empty experts, partial tiles
    ([700, 5, 64], 1024, 768),                          # K = 4 k-blocks, N = 3 tiles
])
def test_grouped_linear_matches_dequantised_product(moe_pkg, counts, K, N):
    r = rng(1000 + K + N)
    M = int(sum(counts))
    x = bf16_values(r.standard_normal((M, K), dtype=np.float32))
    w = (r.standard_normal((len(counts), N, K), dtype=np.float32) * 0.02).astype(np.float32)
    mod = _Experts(list(w)).to(DEV)
    offs = torch.tensor(np.cumsum(counts), dtype=torch.int32, device=DEV)
    xt = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    out = moe_pkg.nvfp4_grouped_linear(xt, mod.experts, "proj", offs)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    ref = _reference(x, counts, w)
    # Only the fp32 accumulation order differs: results agree to a bf16 ulp.
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < 2e-3, rel_l2(got, ref)
    tol = np.abs(ref) * 2.0 ** -7 + 1e-4
    bad = np.abs(got - ref) > tol
    assert bad.mean() < 1e-3, f"{bad.sum()} of {bad.size} elements off by more than a bf16 ulp"


def test_grouped_linear_empty_input(moe_pkg):
    w = np.zeros((2, 256, 256), np.float32)
    mod = _Experts(list(w)).to(DEV)
    x = torch.zeros((0, 256), dtype=torch.bfloat16, device=DEV)
    out = moe_pkg.nvfp4_grouped_linear(x, mod.experts, "proj", torch.zeros(2, dtype=torch.int32, device=DEV))
    assert out.shape == (0, 256)
