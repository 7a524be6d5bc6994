"""Pin the CPU oracle to the reference: every oracle function must reproduce
the golden outputs recorded from the reference's own code (make_golden.py)."""

import numpy as np
import pytest

from inputs import act_quant_cases, layer_case, routing_cases, weight_quant_cases
from make_golden import digest
from oracle import moe_ref, nvfp4_ref as nr


@pytest.mark.parametrize("case", act_quant_cases(), ids=lambda c: c[0])
def test_activation_and_core_quantiser_bytes(golden, case):
    name, x, mode = case
    g = golden("quant_act")
    np.testing.assert_array_equal(g[f"{name}__in"].view(np.uint32), x.view(np.uint32))
    two_d = mode == "tile2d"
    causal = mode == "act"
    packed, scales, gs = nr.quantize_nvfp4_core(x, two_d, causal)
    np.testing.assert_array_equal(packed, g[f"{name}__packed"])
    np.testing.assert_array_equal(scales, g[f"{name}__scales"])
    np.testing.assert_array_equal(gs.view(np.uint32), g[f"{name}__g"].view(np.uint32))
    sw = nr.swizzle_scales(scales)
    np.testing.assert_array_equal(sw, g[f"{name}__swizzled"])
    np.testing.assert_array_equal(nr.unswizzle_scales(sw, *scales.shape), scales)


@pytest.mark.parametrize("case", weight_quant_cases(), ids=lambda c: c[0])
def test_grouped_weight_quantiser_bytes(golden, case):
    name, w = case
    g = golden("quant_w")
    assert str(g[f"{name}__digest"]) == digest(w)
    b_fwd, bs_fwd, bg, b_bwd, bs_bwd = nr.quantize_grouped_weights(w)
    np.testing.assert_array_equal(b_fwd, g[f"{name}__b_fwd"])
    np.testing.assert_array_equal(bs_fwd, g[f"{name}__bs_fwd"])
    np.testing.assert_array_equal(bg.view(np.uint32), g[f"{name}__bg"].view(np.uint32))
    np.testing.assert_array_equal(b_bwd, g[f"{name}__b_bwd"])
    np.testing.assert_array_equal(bs_bwd, g[f"{name}__bs_bwd"])
    # grouped core == per-matrix two-dimensional core (src/mcl4_coe/nvfp4.py:206-213 vs :923-952)
    np.testing.assert_array_equal(b_fwd[0].T, g[f"{name}__core2d_packed0"])
    np.testing.assert_array_equal(bs_fwd[0], g[f"{name}__core2d_scales0"])


def _near_tie_tokens(logits: np.ndarray, k: int, eps: float = 1e-5) -> np.ndarray:
    """Tokens whose k-th and (k+1)-th largest logits are within eps."""
    if logits.shape[1] <= k:
        return np.zeros(logits.shape[0], bool)
    s = -np.sort(-logits, axis=1)
    return (s[:, k - 1] - s[:, k]) <= eps


@pytest.mark.parametrize("case", routing_cases(), ids=lambda c: c[0])
def test_routing_matches_reference(golden, case):
    name, c = case
    g = golden("routing")
    assert str(g[f"{name}__digest"]) == digest(c["x_bf16_bits"], c["wr"])
    x = nr.bf16_bits_to_f32(c["x_bf16_bits"]).reshape(c["t"], c["d"])
    valid = c["valid"]
    # (1) given the reference's logits, everything downstream is exact
    ref_logits = g[f"{name}__logits"]
    full_logits = np.zeros((c["t"], c["e"]), np.float32)
    active = np.arange(c["t"]) if valid is None else np.nonzero(valid)[0]
    full_logits[active] = ref_logits
    r = moe_ref.route(x, c["wr"], c["k"], c["norm_topk_prob"], valid, c["logit_bias"], logits=full_logits)
    np.testing.assert_array_equal(r.selected, g[f"{name}__topk_indices"])
    np.testing.assert_array_equal(r.perm, g[f"{name}__perm"])
    np.testing.assert_array_equal(r.sel_mask.astype(np.uint8), g[f"{name}__sel_mask"])
    np.testing.assert_allclose(r.counts, g[f"{name}__counts"], rtol=0, atol=0)
    topv = g[f"{name}__topk_values"]
    np.testing.assert_allclose(np.take_along_axis(r.probs, r.selected, 1), topv, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(r.aux_loss, g[f"{name}__aux"], rtol=1e-5)
    np.testing.assert_allclose(r.z_loss, g[f"{name}__z"], rtol=1e-5)
    # (2) with the oracle's own fp32 logits: identical except near-tie tokens
    r2 = moe_ref.route(x, c["wr"], c["k"], c["norm_topk_prob"], valid, c["logit_bias"])
    np.testing.assert_allclose(r2.logits, ref_logits, rtol=1e-5, atol=1e-5)
    tie = _near_tie_tokens(ref_logits, c["k"])
    same = np.all(np.sort(r2.selected, 1) == np.sort(g[f"{name}__topk_indices"], 1), axis=1)
    assert np.all(same | tie)


def test_layer_output_matches_reference(golden):
    name, c = layer_case()
    g = golden("layer")
    assert str(g[f"{name}__digest"]) == digest(c["x_bf16_bits"], c["wr"], c["w_up"], c["w_dn"])
    x = nr.bf16_bits_to_f32(c["x_bf16_bits"]).reshape(c["t"], c["d"])
    experts = moe_ref.QuantizedExperts(c["w_up"], c["w_dn"])
    out, aux, z, counts, r = moe_ref.moe_forward(x, c["wr"], experts, c["k"], c["norm_topk_prob"])
    ref = nr.bf16_bits_to_f32(g[f"{name}__out_bf16"]).reshape(out.shape)
    np.testing.assert_array_equal(r.selected, g[f"{name}__topk_indices"])
    np.testing.assert_array_equal(r.perm, g[f"{name}__perm"])
    # Same math in a different BLAS summation order: bf16 outputs agree to
    # within a couple of bf16 ulps, far inside the product tolerance.
    rel_l2 = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel_l2 < 2e-3, rel_l2
    assert np.abs(out - ref).max() < 2e-2
    np.testing.assert_allclose(aux, g[f"{name}__aux"], rtol=1e-5)
    np.testing.assert_allclose(z, g[f"{name}__z"], rtol=1e-5)
    np.testing.assert_array_equal(counts, g[f"{name}__counts"])


def test_swizzle_is_the_tcgen05_scale_atom():
    """Element (r, c) of the swizzled scales sits at the byte the tcgen05
    32x128b scale copy reads for row r, scale c."""
    rows, cols = 256, 8
    s = (np.arange(rows * cols) % 251).astype(np.uint8).reshape(rows, cols)
    sw = nr.swizzle_scales(s).reshape(-1)
    for r in range(0, rows, 7):
        for c in range(cols):
            off = ((r // 128) * (cols // 4) + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4
            assert sw[off] == s[r, c]


def test_sr_quantiser_matches_reference_kernel(golden):
    """The stochastic-rounding gradient quantiser (Philox noise, codes, scales) against the
    reference's own Triton kernel run on the CPU interpreter (tests/golden/make_golden_sr.py).
    Blocks whose scale the interpreter's numpy fp8 emulation rounds differently from the
    hardware's round-to-nearest (``rn_scales``) are the only ones allowed to differ."""
    from inputs import sr_quant_cases

    g = golden("sr_quant")
    total_blocks = compared = 0
    for name, bits, seed in sr_quant_cases():
        np.testing.assert_array_equal(g[f"{name}__x_bits"], bits)
        x = nr.bf16_bits_to_f32(bits)
        gs = nr.sr_global_scale(x)
        assert gs == g[f"{name}__g"][0]
        packed, scales = nr.quantize_sr(x, gs, int(g[f"{name}__seed"]))
        np.testing.assert_array_equal(scales, g[f"{name}__rn_scales"])
        same = g[f"{name}__scales"] == g[f"{name}__rn_scales"]
        np.testing.assert_array_equal(scales[same], g[f"{name}__scales"][same])
        keep = np.repeat(same, 8, axis=1)
        np.testing.assert_array_equal(packed[keep], g[f"{name}__packed"][keep])
        total_blocks += same.size
        compared += int(same.sum())
    assert compared > 0.98 * total_blocks  # the emulation differences are rare edge blocks


def test_philox_matches_published_known_answer():
    """Philox4x32-10 known-answer vector of Salmon et al. (Random123 kat_vectors):
    counter 0, key 0 -> first word 0x6627e8d5."""
    assert int(nr.philox_first_word(np.array([0], np.uint64), 0)[0]) == 0x6627E8D5


def test_hadamard16_matches_reference(golden):
    """The Hadamard16 matrix, the transform of ``y.T`` and the round-to-nearest
    quantisation of the transformed, 32-padded matrix (the weight-gradient operand of
    ``_NVFP4Linear.backward``) against the reference's own functions
    (tests/golden/make_golden_hadamard.py).  The transform sums 16 signed terms: the
    oracle's butterfly order and the reference's matmul agree exactly on bf16-valued
    inputs and to float32 rounding on fp32 inputs; the bytes agree exactly."""
    from inputs import hadamard_cases

    g = golden("hadamard")
    np.testing.assert_array_equal(nr.hadamard16_matrix().view(np.uint32), g["h16"].view(np.uint32))
    h = nr.hadamard16_matrix().astype(np.float64)
    np.testing.assert_allclose(h @ h.T, np.eye(16), atol=1e-7)
    for name, y in hadamard_cases():
        np.testing.assert_array_equal(g[f"{name}/y"], y)
        ht = nr.hadamard16(y.T)
        ref = g[f"{name}/ht"]
        assert ht.shape == ref.shape
        np.testing.assert_allclose(ht, ref, rtol=0, atol=4e-7 * float(np.abs(ref).max()))
        if name != "ht_f32_150x64":  # bf16-valued inputs: every partial sum is exact
            np.testing.assert_array_equal(ht.view(np.uint32), ref.view(np.uint32))
        m, c = y.shape
        packed, scales, gs = nr.linear_wgrad_operand(y, nr.round_up(m, 32), nr.round_up(c, 32), stochastic=False)
        np.testing.assert_array_equal(packed, g[f"{name}/packed"])
        np.testing.assert_array_equal(scales, g[f"{name}/scales"])
        np.testing.assert_array_equal(gs.view(np.uint32), g[f"{name}/g"].view(np.uint32))


def test_single_matrix_sr_codes_bracket_the_value():
    """quantize_nvfp4(stochastic=True) oracle: scales and global scale are the
    round-to-nearest ones, every code is the floor or the ceiling of the scaled
    magnitude's E2M1 position, and the mean over seeds converges to the value."""
    r = np.random.default_rng(5)
    x = nr.round_bf16((r.standard_normal((8, 64)) * 0.01).astype(np.float32))
    p_rn, s_rn, g_rn = nr.quantize_nvfp4_core(x, False, False)
    acc = np.zeros_like(x, dtype=np.float64)
    n = 400
    for seed in range(n):
        p, s, gs = nr.quantize_nvfp4_sr(x, seed)
        np.testing.assert_array_equal(s, s_rn)
        assert gs[0] == g_rn[0]
        deq = nr.dequantize(p, s, gs[0], 8, 64)
        acc += deq
        lo = nr.dequantize(p_rn, s_rn, g_rn[0], 8, 64)
        step = np.repeat(nr.e4m3_to_f32(s).astype(np.float64) * gs[0], 16, axis=1) * 2.0
        assert np.all(np.abs(deq.astype(np.float64) - lo) <= step * (1 + 1e-6))
    mean = acc / n
    scale = np.repeat(nr.e4m3_to_f32(s_rn).astype(np.float64) * g_rn[0], 16, axis=1)
    assert np.abs(mean - x).max() <= 0.25 * scale.max()
