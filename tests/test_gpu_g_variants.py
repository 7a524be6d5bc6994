"""Routing variants on the GPU against the reference's own layer outputs.

Each case of ``tests/golden/variants.npz`` was produced by the reference
``SparseMoE`` (src/mcl4_coe/backbone.py) with dequantised-FP4 experts and a
routing variant switched on.  Here the same layer runs through the library:
the variant's selection on the tcgen05 router's logits, then
``mcl4moe_moe_forward_routed`` (permutation, NVFP4 quantisation, grouped
GEMMs, combine).  Routing (``last_selected_mask``) must be identical, the
counts and losses equal to fp32 rounding, and the outputs within the
layer tolerance; the reference sums dense-subset outputs in bf16 step by step,
the library in fp32, so those cases carry one extra bf16 rounding per expert.
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

from inputs import bf16_bits_to_f32, variant_cases, variant_prior  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"
REL_L2, MAX_ABS = 2e-2, 1e-1  # the layer tolerance of the parity contract
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
    moe = moe.to(DEV)
    moe.mitotic_pairs = [tuple(p) for p in opt["pairs"]]
    if opt["lineage"] is not None:
        roots, fams, share = opt["lineage"]
        moe.configure_lineage_family_routing(roots, top_families=fams, child_share=share)
        # the family tree of the reference: with random weights the child -> root cosine
        # similarities are noise (~1e-3), so the GPU's fp32 summation order may pick other
        # parents; the configuration itself is pinned bit for bit on CPU (test_variants_cpu)
        name = next(n for n, (c, _) in CASES.items() if c is case)
        moe.lineage_root_ids = torch.from_numpy(GOLD[f"{name}__lineage_root_ids"]).to(DEV)
        moe.lineage_logit_prior = torch.from_numpy(GOLD[f"{name}__lineage_logit_prior"]).to(DEV)
    return moe


def _lineage_live_mask(moe, case, name):
    """1 where an expert has nonzero lineage-routing probability for the token (its family
    is among the token's top families), from the reference's logits on CPU."""
    from torch.nn import functional as F

    x = torch.from_numpy(case["x_bf16_bits"].view(np.int16).copy()).view(torch.bfloat16).reshape(case["t"], case["d"])
    logits = F.linear(x.float(), torch.from_numpy(case["wr"]))
    root_ids = torch.from_numpy(GOLD[f"{name}__lineage_root_ids"])
    probs = F.softmax(logits + torch.from_numpy(GOLD[f"{name}__lineage_logit_prior"]).unsqueeze(0), dim=-1)
    fam = torch.zeros((logits.shape[0], moe.lineage_num_roots)).scatter_add_(
        1, root_ids.unsqueeze(0).expand(logits.shape[0], -1), probs)
    _, top = fam.topk(moe.lineage_top_families, dim=-1)
    fam_mask = torch.zeros_like(fam).scatter_(1, top, 1.0)
    return (fam_mask.index_select(1, root_ids) * probs > 0).float().numpy()


def _rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", sorted(CASES))
def test_variant_layer_matches_reference(moe_pkg, name):
    case, opt = CASES[name]
    T, d, E = case["t"], case["d"], case["e"]
    moe = _module(moe_pkg, case, opt)
    x = torch.from_numpy(case["x_bf16_bits"].view(np.int16).copy()).view(torch.bfloat16).reshape(T, d).to(DEV)
    valid = None if case["valid"] is None else torch.from_numpy(case["valid"].astype(bool)).to(DEV)
    if opt["shape"] is not None:
        x = x.reshape(*opt["shape"], d)
        valid = None if valid is None else valid.reshape(*opt["shape"])
    prior = variant_prior(name, T, E, opt["prior_frac"])
    prior = None if prior is None else torch.from_numpy(prior).to(DEV)
    with torch.no_grad():
        out, aux, z, counts = moe(x, valid=valid, prior_expert_mask=prior,
                                  dense_expert_indices=None if opt["dense_idx"] is None else list(opt["dense_idx"]))
    torch.cuda.synchronize()
    mask = moe.last_selected_mask.reshape(T, E).cpu().numpy()
    gold_mask = GOLD[f"{name}__sel_mask"]
    if opt["lineage"] is None:
        np.testing.assert_array_equal(mask, gold_mask)
        # integer slot counts / slot total: CUDA's division may differ from the CPU's in the last bit
        np.testing.assert_allclose(counts.cpu().numpy(), GOLD[f"{name}__counts"], rtol=1e-6, atol=0)
        np.testing.assert_allclose(float(aux), GOLD[f"{name}__aux"], rtol=1e-5, atol=1e-7)
    else:
        # lineage routing fills k_sel slots with zero-weight experts where a token's families
        # are small; which zero-weight experts is torch.topk's tie order (CPU and CUDA differ,
        # in the reference too).  Every selection that carries weight must match exactly.
        live = _lineage_live_mask(moe, case, name)
        np.testing.assert_array_equal(mask * live, gold_mask * live)
        np.testing.assert_array_equal(mask.sum(axis=1), gold_mask.sum(axis=1))
    np.testing.assert_allclose(float(z), GOLD[f"{name}__z"], rtol=1e-5, atol=1e-7)
    got = out.reshape(T, d).float().cpu().numpy()
    ref = bf16_bits_to_f32(GOLD[f"{name}__out_bf16"]).reshape(T, d)
    err, mx = _rel_l2(got, ref), float(np.abs(got - ref).max())
    assert err < REL_L2 and mx < MAX_ABS, (err, mx)
    if case["valid"] is not None:
        assert np.all(got[case["valid"] == 0] == 0)


def test_forward_dense_subset_matches_routed_layer(moe_pkg):
    """forward_dense_subset(x, ids, expert_weights=w) equals the layer routed to those
    experts with those weights (src/mcl4_coe/backbone.py:307-398)."""
    case, opt = CASES["v_dense_idx"]
    moe = _module(moe_pkg, case, opt)
    T, d = case["t"], case["d"]
    x = torch.from_numpy(case["x_bf16_bits"].view(np.int16).copy()).view(torch.bfloat16).reshape(T, d).to(DEV)
    w = torch.rand((T, 3), device=DEV)
    with torch.no_grad():
        a = moe.forward_dense_subset(x, [6, 2, 4], expert_weights=w)
        idx = torch.tensor([2, 4, 6], dtype=torch.int32, device=DEV).expand(T, 3).contiguous()
        b = moe._forward_routed(x, None, idx, w[:, [1, 2, 0]].contiguous())
        shared = moe.forward_dense_subset(x, [2, 4], expert_weights=torch.tensor([0.25, 0.75], device=DEV))
        c = moe._forward_routed(x, None, torch.tensor([2, 4], dtype=torch.int32, device=DEV).expand(T, 2).contiguous(),
                                torch.tensor([0.25, 0.75], device=DEV).expand(T, 2).contiguous())
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(shared, c)


def test_routed_forward_skips_out_of_range_ids(moe_pkg):
    """Slots whose id is outside [0, E) are not routed: the result equals the routing
    without them, and nothing outside the buffers is touched."""
    case, opt = CASES["v_coverage"]
    moe = _module(moe_pkg, case, opt)
    T, d, E = case["t"], case["d"], case["e"]
    x = torch.from_numpy(case["x_bf16_bits"].view(np.int16).copy()).view(torch.bfloat16).reshape(T, d).to(DEV)
    g = torch.Generator(device="cpu").manual_seed(7)
    idx = torch.stack([torch.randperm(E, generator=g)[:3] for _ in range(T)]).to(torch.int32)
    w = torch.rand((T, 3), generator=g)
    bad = idx.clone()
    bad[::3, 2] = -1
    bad[1::3, 2] = E + 5
    keep = torch.ones_like(idx, dtype=torch.bool)
    keep[::3, 2] = False
    keep[1::3, 2] = False
    w_keep = torch.where(keep, w, torch.zeros_like(w))
    with torch.no_grad():
        a = moe._forward_routed(x, None, bad.to(DEV), w.to(DEV))
        b = moe._forward_routed(x, None, idx.to(DEV), w_keep.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_dense_subset_without_valid_ids(moe_pkg):
    """Only out-of-range dense ids: the subset contributes nothing (zeros), and with
    combine_dense_and_sparse the sparse remainder alone is mixed in."""
    case, opt = CASES["v_dense_idx"]
    moe = _module(moe_pkg, case, opt)
    T, d = case["t"], case["d"]
    x = torch.from_numpy(case["x_bf16_bits"].view(np.int16).copy()).view(torch.bfloat16).reshape(T, d).to(DEV)
    with torch.no_grad():
        out, aux, z, counts = moe(x, dense_expert_indices=[99, -1])
        assert torch.all(out == 0)
        moe.combine_dense_and_sparse = True
        mixed, _, _, _ = moe(x, dense_expert_indices=[99])
    torch.cuda.synchronize()
    assert torch.isfinite(mixed.float()).all() and mixed.abs().sum() > 0
