"""2:4 sparsity: the oracle's masks and masked-weight bytes against the reference.

``tests/golden/sparse.npz`` holds the reference's ``compute_2to4_mask``
(src/mcl4_coe/nvfp4.py:70-110) in both modes, the grouped quantiser's bytes of
the masked weights (:1017-1024) and the dequantised-FP4 layer whose experts
carry masked weights.  Masks must agree bit for bit except where the reference
itself leaves the choice to ``topk``'s tie order (row mode, equal 2nd / 3rd
magnitudes) or to BLAS summation order (transposable mode, pattern scores within
fp32 rounding); the bytes and the layer follow from the masks.
"""

import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

from inputs import sparse_cases, sparse_layer_cases  # noqa: E402
from make_golden import digest  # noqa: E402
from oracle import moe_ref  # noqa: E402
from oracle import nvfp4_ref as nr  # noqa: E402

GOLD = np.load(HERE / "golden" / "sparse.npz")
MODES = ("2to4_row", "2to4_transposable")


def test_catalog_is_the_doubly_2to4_set():
    cat = nr.catalog_2to4().reshape(-1, 4, 4)
    assert cat.shape[0] == 90 and len({c.tobytes() for c in cat}) == 90
    assert np.all(cat.sum(axis=1) == 2) and np.all(cat.sum(axis=2) == 2)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", [n for n, _ in sparse_cases()])
def test_oracle_masks_match_reference(name, mode):
    w = dict(sparse_cases())[name]
    assert str(GOLD[f"{name}__digest"]) == digest(w)
    gold = GOLD[f"{name}__{mode}__mask"].astype(bool)
    for i in range(len(w)):
        m = nr.mask_2to4(w[i], mode)
        free = ~nr.mask_tie_groups(w[i], mode)
        np.testing.assert_array_equal(m[free], gold[i][free])
        # every 4-group / tile keeps exactly half
        if mode == "2to4_row":
            assert np.all(m.reshape(m.shape[0], -1, 4).sum(-1) == 2)
        else:
            t = m.reshape(m.shape[0] // 4, 4, m.shape[1] // 4, 4)
            assert np.all(t.sum(axis=1) == 2) and np.all(t.sum(axis=3) == 2)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", [n for n, w in sparse_cases() if w.shape[1] % 16 == 0 and w.shape[2] % 64 == 0])
def test_masked_weight_bytes_match_reference(name, mode):
    """The grouped quantiser on w * mask (dropped negative weights become -0 and
    quantise to code 8, as in the reference)."""
    w = dict(sparse_cases())[name]
    masked = w * GOLD[f"{name}__{mode}__mask"].astype(np.float32)
    b_fwd, bs_fwd, bg, _, _ = nr.quantize_grouped_weights(masked, with_bwd=False)
    np.testing.assert_array_equal(b_fwd, GOLD[f"{name}__{mode}__b_fwd"])
    np.testing.assert_array_equal(bs_fwd, GOLD[f"{name}__{mode}__bs_fwd"])
    np.testing.assert_array_equal(bg, GOLD[f"{name}__{mode}__bg"])


@pytest.mark.parametrize("name", [n for n, _, _ in sparse_layer_cases()])
def test_oracle_layer_with_sparse_experts(name):
    case, mode = {n: (c, m) for n, c, m in sparse_layer_cases()}[name]
    assert str(GOLD[f"{name}__digest"]) == digest(case["x_bf16_bits"], case["wr"], case["w_up"], case["w_dn"])
    w_up = np.stack([w * nr.mask_2to4(w, mode) for w in case["w_up"]]).astype(np.float32)
    w_dn = np.stack([w * nr.mask_2to4(w, mode) for w in case["w_dn"]]).astype(np.float32)
    x = nr.bf16_bits_to_f32(case["x_bf16_bits"]).reshape(case["t"], case["d"])
    out, aux, z, counts, _ = moe_ref.moe_forward(x, case["wr"], moe_ref.QuantizedExperts(w_up, w_dn), case["k"],
                                                 case["norm_topk_prob"], case["valid"])
    ref = nr.bf16_bits_to_f32(GOLD[f"{name}__out_bf16"]).reshape(out.shape)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 2e-3
    assert np.abs(out - ref).max() < 2e-2
    np.testing.assert_array_equal(counts, GOLD[f"{name}__counts"])
