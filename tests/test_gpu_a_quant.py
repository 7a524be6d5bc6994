"""NVFP4 quantiser kernels vs the reference's bytes (bit-exact)."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_ref import build_module
from inputs import act_quant_cases, bf16_values, moe_case, rng, weight_quant_cases
from oracle import nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _act_bf16_cases():
    return [c for c in act_quant_cases() if c[2] == "act" and np.array_equal(bf16_values(c[1]), c[1])]


@pytest.mark.parametrize("case", _act_bf16_cases(), ids=lambda c: c[0])
def test_activation_quantiser_matches_reference_golden(moe_pkg, golden, case):
    name, x, _ = case
    g = golden("quant_act")
    xt = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    packed, scales, gs = moe_pkg.quantize_activations(xt)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(packed.cpu().numpy(), g[f"{name}__packed"])
    np.testing.assert_array_equal(scales.view(torch.uint8).cpu().numpy(), g[f"{name}__scales"])
    assert float(gs) == 1.0
    _, sw, _ = moe_pkg.quantize_activations(xt, swizzled=True)
    np.testing.assert_array_equal(sw.view(torch.uint8).cpu().numpy().reshape(g[f"{name}__swizzled"].shape),
                                  g[f"{name}__swizzled"])


@pytest.mark.parametrize("rows,cols", [(1, 64), (1000, 2048), (333, 1536)])
def test_activation_quantiser_random_vs_oracle(moe_pkg, rows, cols):
    r = rng(7 + rows)
    x = bf16_values((r.standard_normal((rows, cols), dtype=np.float32)
                     * np.power(10.0, r.uniform(-3, 3, size=(rows, 1))).astype(np.float32)))
    xt = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    packed, scales, _ = moe_pkg.quantize_activations(xt)
    _, sw, _ = moe_pkg.quantize_activations(xt, swizzled=True)
    op, os_ = nr.quantize_activations(x)
    np.testing.assert_array_equal(packed.cpu().numpy(), op)
    np.testing.assert_array_equal(scales.view(torch.uint8).cpu().numpy(), os_)
    np.testing.assert_array_equal(sw.view(torch.uint8).cpu().numpy().reshape(-1), nr.swizzle_scales(os_).reshape(-1))


def _quantize_case(moe_pkg, w):
    """Quantise a numpy [D, N, K] stack through the C ABI into both layouts."""
    d, n, k = w.shape
    wt = [torch.from_numpy(w[i]).to(DEV).contiguous() for i in range(d)]
    cache = moe_pkg.GroupedNVFP4Cache(d, n, k, torch.device(DEV))
    ref = {
        "B_fwd": torch.zeros((d, k // 2, n), dtype=torch.uint8, device=DEV),
        "Bs_fwd": torch.zeros((d, n, k // 16), dtype=torch.uint8, device=DEV),
        "B_bwd": torch.zeros((d, n // 2, k), dtype=torch.uint8, device=DEV),
        "Bs_bwd": torch.zeros((d, k, n // 16), dtype=torch.uint8, device=DEV),
    }
    from mcl4coe_b200.nvfp4 import quantize_weight_slots

    quantize_weight_slots(wt, list(range(d)), cache, ref)
    torch.cuda.synchronize()
    return cache, {key: v.cpu().numpy() for key, v in ref.items()}


@pytest.mark.parametrize("case", weight_quant_cases(), ids=lambda c: c[0])
def test_weight_quantiser_matches_reference_golden(moe_pkg, golden, case):
    name, w = case
    g = golden("quant_w")
    cache, ref = _quantize_case(moe_pkg, w)
    np.testing.assert_array_equal(ref["B_fwd"], g[f"{name}__b_fwd"])
    np.testing.assert_array_equal(ref["Bs_fwd"], g[f"{name}__bs_fwd"])
    np.testing.assert_array_equal(ref["B_bwd"], g[f"{name}__b_bwd"])
    np.testing.assert_array_equal(ref["Bs_bwd"], g[f"{name}__bs_bwd"])
    np.testing.assert_array_equal(cache.g.cpu().numpy().view(np.uint32), g[f"{name}__bg"].view(np.uint32))
    # kernel layout == the same bytes, transposed / swizzled
    packed, sw = nr.weights_to_mma_layout(g[f"{name}__b_fwd"], g[f"{name}__bs_fwd"])
    np.testing.assert_array_equal(cache.packed.cpu().numpy(), packed)
    n = w.shape[1]
    np.testing.assert_array_equal(cache.scales.cpu().numpy()[:, : sw.shape[1]], sw)


def test_weight_quantiser_full_size_vs_oracle(moe_pkg):
    r = rng(11)
    w = (r.standard_normal((2, 2048, 1024), dtype=np.float32) * 0.02).astype(np.float32)
    cache, ref = _quantize_case(moe_pkg, w)
    b_fwd, bs_fwd, bg, b_bwd, bs_bwd = nr.quantize_grouped_weights(w)
    np.testing.assert_array_equal(ref["B_fwd"], b_fwd)
    np.testing.assert_array_equal(ref["Bs_fwd"], bs_fwd)
    np.testing.assert_array_equal(ref["B_bwd"], b_bwd)
    np.testing.assert_array_equal(cache.g.cpu().numpy(), bg)


def test_cache_requantises_only_dirty_experts(moe_pkg):
    c = moe_case(12, 16, 256, 4, 2, 256)
    moe = build_module(moe_pkg, c, DEV)
    entry = moe_pkg.get_or_build_grouped_cache(moe.experts, "up_proj")
    before = entry.packed.clone()
    with torch.no_grad():
        moe.experts[2].up_proj.weight.mul_(2.0)  # bumps weight._version of expert 2 only
    entry2 = moe_pkg.get_or_build_grouped_cache(moe.experts, "up_proj")
    assert entry2 is entry
    after = entry2.packed
    torch.cuda.synchronize()
    assert torch.equal(before[[0, 1, 3]], after[[0, 1, 3]])
    # doubling the weights doubles g and keeps the codes and tile scales
    assert torch.equal(before[2], after[2])
    w = np.stack([m.up_proj.weight.detach().cpu().numpy() for m in moe.experts])
    _, _, bg, _, _ = nr.quantize_grouped_weights(w)
    np.testing.assert_array_equal(entry2.g.cpu().numpy(), bg)
