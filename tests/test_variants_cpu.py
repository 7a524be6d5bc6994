"""Routing variants: the host-side selection against the reference's own outputs.

``tests/golden/variants.npz`` holds what the reference ``SparseMoE``
(src/mcl4_coe/backbone.py) returned with mitotic twins, lineage families, the
coverage penalty, dense subsets and the extra auxiliary losses switched on.
The selection, statistics and losses of ``routing_variants`` run here on CPU
torch from the same fp32 router logits the reference computes
(``F.linear(active_x.float(), W_r)``, :929), so they must agree exactly:
``last_selected_mask`` and counts bit for bit, aux / z losses to the last bit.
The layer outputs are checked on the GPU (test_gpu_g_variants.py).
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch
from torch.nn import functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

from inputs import variant_cases, variant_prior  # noqa: E402

GOLD = np.load(HERE / "golden" / "variants.npz")
CASES = {name: (case, opt) for name, case, opt in variant_cases()}


def _module(pkg, case, opt):
    cfg = pkg.MoEConfig(d_model=case["d"], expert_hidden_dim=case["f"], num_experts=case["e"], top_k=case["k"],
                        norm_topk_prob=case["norm_topk_prob"], recurrent_coverage_penalty=opt["coverage"],
                        mitotic_ortho_coef=opt["ortho"], sequence_diversity_coef=opt["seq_div"],
                        dense_subset_k=opt["dense_k"], combine_dense_and_sparse=opt["combine"])
    moe = pkg.SparseMoE(cfg)
    with torch.no_grad():
        moe.router.weight.copy_(torch.from_numpy(case["wr"]))
        for i, ex in enumerate(moe.experts):
            ex.up_proj.weight.copy_(torch.from_numpy(case["w_up"][i]))
            ex.down_proj.weight.copy_(torch.from_numpy(case["w_dn"][i]))
    moe.mitotic_pairs = [tuple(p) for p in opt["pairs"]]
    if opt["lineage"] is not None:
        roots, fams, share = opt["lineage"]
        moe.configure_lineage_family_routing(roots, top_families=fams, child_share=share)
    return moe


@pytest.mark.parametrize("name", sorted(CASES))
def test_variant_selection_matches_reference(moe_pkg, name):
    rv = moe_pkg.routing_variants
    case, opt = CASES[name]
    moe = _module(moe_pkg, case, opt)
    T, E = case["t"], case["e"]
    if opt["lineage"] is not None:
        np.testing.assert_array_equal(moe.lineage_root_ids.numpy(), GOLD[f"{name}__lineage_root_ids"])
        np.testing.assert_array_equal(moe.lineage_logit_prior.numpy(), GOLD[f"{name}__lineage_logit_prior"])
    x = torch.from_numpy(case["x_bf16_bits"].view(np.int16).copy()).view(torch.bfloat16).reshape(T, case["d"])
    valid = torch.ones(T, dtype=torch.bool) if case["valid"] is None else torch.from_numpy(case["valid"].astype(bool))
    active = valid.nonzero(as_tuple=False).squeeze(-1)
    logits = F.linear(x.index_select(0, active).float(), moe.router.weight.float())
    prior = variant_prior(name, T, E, opt["prior_frac"])
    prior_a = None
    if prior is not None and moe.recurrent_coverage_penalty > 0.0:
        prior_a = torch.from_numpy(prior).index_select(0, active)
    x_shape = (T, case["d"]) if opt["shape"] is None else (*opt["shape"], case["d"])
    valid_arg = None if case["valid"] is None else valid.reshape(x_shape[:-1])
    if opt["dense_idx"] is not None or opt["dense_k"] > 0:
        sel = rv.dense_selection(moe, logits, prior_a, list(opt["dense_idx"] or ()), opt["dense_k"])
        mask, aux, z, counts = rv.dense_statistics(moe, logits, sel["probs"], sel["chosen"], sel["chosen_t"])
        probs = sel["probs"]
    else:
        probs, weights, selected = rv.sparse_selection(moe, logits, prior_a)
        aux, z, counts = rv.sparse_statistics(moe, logits, probs, selected)
        mask = F.one_hot(selected, num_classes=E).sum(dim=1).float()
        assert torch.all(weights >= 0)
    aux = rv.add_extra_aux(moe, aux, x_shape, probs, active, T, valid_arg)
    full = torch.zeros((T, E))
    full.index_copy_(0, active, mask)
    np.testing.assert_array_equal(full.numpy(), GOLD[f"{name}__sel_mask"])
    np.testing.assert_array_equal(counts.numpy(), GOLD[f"{name}__counts"])
    assert np.float32(aux.item()) == GOLD[f"{name}__aux"], (aux.item(), GOLD[f"{name}__aux"])
    assert np.float32(z.item()) == GOLD[f"{name}__z"]


def test_variant_fixtures_match_their_inputs():
    """The stored digests pin the inputs the fixtures were made from."""
    sys.path.insert(0, str(HERE / "golden"))
    from make_golden import digest

    for name, (case, _) in CASES.items():
        assert str(GOLD[f"{name}__digest"]) == digest(case["x_bf16_bits"], case["wr"], case["w_up"], case["w_dn"])
