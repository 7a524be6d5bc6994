"""Single-matrix NVFP4 operators (reference signatures) on the GPU.

* ``quantize_nvfp4`` in all three modes (causal 1-D, tensor-wise 1-D,
  16x16 tiles) from bf16 or fp32 input: bit-exact against the reference's bytes
  (``quant_act.npz``: packed codes, ``_swizzle_scales`` output, global scale).
* ``nvfp4_mm`` (src/mcl4_coe/nvfp4.py:285-334): fp32 result against the product
  of the oracle's dequantised operands (the GEMM sums exact FP4 products in
  fp32; only the summation order differs), padded and unpadded shapes,
  prequantised B.
* ``NVFP4Linear`` (:474-542): bias, 2:4 sparsity, the weight cache.
"""

import numpy as np
import pytest
import torch
from torch import nn

from inputs import act_quant_cases, rng
from oracle import nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("case", act_quant_cases(), ids=lambda c: c[0])
@pytest.mark.parametrize("as_bf16", [False, True])
def test_quantize_nvfp4_matches_reference_bytes(moe_pkg, golden, case, as_bf16):
    name, x, mode = case
    g = golden("quant_act")
    xt = torch.from_numpy(x).to(DEV)
    if as_bf16:
        if not np.array_equal(nr.round_bf16(x), x):
            pytest.skip("values not representable in bf16")
        xt = xt.to(torch.bfloat16)
    packed, scales, gs = moe_pkg.quantize_nvfp4(xt, two_dimensional=mode == "tile2d",
                                                causal_row_scale=mode == "act")
    torch.cuda.synchronize()
    assert packed.dtype == getattr(torch, "float4_e2m1fn_x2", torch.uint8)
    np.testing.assert_array_equal(packed.view(torch.uint8).cpu().numpy(), g[f"{name}__packed"])
    np.testing.assert_array_equal(scales.view(torch.uint8).cpu().numpy(), g[f"{name}__swizzled"])
    np.testing.assert_array_equal(gs.cpu().numpy().reshape(-1), g[f"{name}__g"].reshape(-1))


def _deq(x: np.ndarray, mode: str) -> np.ndarray:
    """Oracle dequantisation of one operand quantised in ``mode``."""
    rows, cols = x.shape
    packed, scales, g = nr.quantize_nvfp4_core(x, mode == "tile2d", mode == "act")
    return nr.dequantize(packed, scales, g, rows, cols).astype(np.float64)


def _pad32(x: np.ndarray) -> np.ndarray:
    r, c = x.shape
    return np.pad(x, ((0, (-r) % 32), (0, (-c) % 32)))


@pytest.mark.parametrize("m,k,n", [(300, 512, 256), (64, 2048, 768), (37, 80, 100)])
@pytest.mark.parametrize("causal_a,weight_b", [(True, True), (False, True), (False, False)])
@pytest.mark.parametrize("a_dtype", [torch.bfloat16, torch.float32])
def test_nvfp4_mm_matches_dequantised_product(moe_pkg, m, k, n, causal_a, weight_b, a_dtype):
    r = rng(m * 7 + k + n)
    a = r.standard_normal((m, k), dtype=np.float32)
    b = (r.standard_normal((n, k), dtype=np.float32) * 0.05).astype(np.float32)
    if a_dtype == torch.bfloat16:
        a = nr.round_bf16(a)
    got = moe_pkg.nvfp4_mm(torch.from_numpy(a).to(DEV, a_dtype), torch.from_numpy(b).to(DEV), weight_b=weight_b,
                           causal_a=causal_a)
    torch.cuda.synchronize()
    assert got.dtype == torch.float32 and got.shape == (m, n)
    # the reference pads both operands to multiples of 32 before quantising (:305-316)
    da = _deq(_pad32(a), "act" if causal_a else "tensor1d")[:m, :k]
    db = _deq(_pad32(b), "tile2d" if weight_b else "tensor1d")[:n, :k]
    ref = da @ db.T
    err = np.linalg.norm(got.cpu().numpy() - ref) / np.linalg.norm(ref)
    assert err < 1e-5, err


def test_nvfp4_mm_prequantized_b_equals_weight_b(moe_pkg):
    r = rng(77)
    a = torch.from_numpy(nr.round_bf16(r.standard_normal((200, 320), dtype=np.float32))).to(DEV, torch.bfloat16)
    b = torch.from_numpy((r.standard_normal((96, 320), dtype=np.float32) * 0.05).astype(np.float32)).to(DEV)
    pre = moe_pkg.quantize_nvfp4(b, two_dimensional=True)  # 96 and 320 are multiples of 32
    x = moe_pkg.nvfp4_mm(a, b, weight_b=True, causal_a=True)
    y = moe_pkg.nvfp4_mm(a, b, weight_b=True, causal_a=True, prequantized_b=pre)
    torch.cuda.synchronize()
    assert torch.equal(x, y)


def test_nvfp4_mm_rejects_bad_operands(moe_pkg):
    a = torch.zeros((4, 32), device=DEV)
    with pytest.raises(ValueError):
        moe_pkg.nvfp4_mm(a, torch.zeros((4, 16), device=DEV))
    with pytest.raises(ValueError):
        moe_pkg.nvfp4_mm(a, torch.zeros((4, 32)))
    with pytest.raises(NotImplementedError):  # two-dimensional stochastic rounding: no reference caller
        moe_pkg.nvfp4_mm(a, torch.zeros((4, 32), device=DEV), weight_b=True, stochastic_b=True)


@pytest.mark.parametrize("sparsity", ["none", "2to4_transposable", "2to4_row"])
@pytest.mark.parametrize("bias", [False, True])
def test_nvfp4_linear_matches_oracle(moe_pkg, sparsity, bias):
    r = rng(5 if bias else 6)
    lin = nn.Linear(512, 384, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy((r.standard_normal((384, 512), dtype=np.float32) * 0.03).astype(np.float32)))
        if bias:
            lin.bias.copy_(torch.from_numpy(r.standard_normal(384, dtype=np.float32)))
    mod = moe_pkg.NVFP4Linear.from_linear(lin, sparsity_mode=sparsity).to(DEV)
    x = torch.from_numpy(nr.round_bf16(r.standard_normal((3, 50, 512), dtype=np.float32))).to(DEV, torch.bfloat16)
    with torch.no_grad():
        y = mod(x)
        y2 = mod(x)  # served from the weight cache
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16 and y.shape == (3, 50, 384) and torch.equal(y, y2)
    w = lin.weight.detach().numpy()
    if sparsity != "none":
        w = (w * nr.mask_2to4(w, sparsity)).astype(np.float32)
        assert torch.equal(mod.active_2to4_mask().cpu(), torch.from_numpy(nr.mask_2to4(lin.weight.detach().numpy(),
                                                                                       sparsity)))
    xf = x.float().cpu().numpy().reshape(-1, 512)
    ref = _deq(_pad32(xf), "act")[:150, :512] @ _deq(_pad32(w), "tile2d")[:384, :512].T
    if bias:
        ref = ref + lin.bias.detach().numpy()
    ref = nr.round_bf16(ref.astype(np.float32))
    got = y.float().cpu().numpy().reshape(-1, 384)
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 2 ** -7 + 1e-6
    # a weight update invalidates the cache
    with torch.no_grad():
        mod.weight.mul_(0.5)
        y3 = mod(x)
    torch.cuda.synchronize()
    assert not torch.equal(y3, y)
