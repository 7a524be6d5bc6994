"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run from the repository root, in a container that has the reference checkout:

    python tests/golden/make_golden.py --reference-src PATH   (or MCL4_REFERENCE_SRC=PATH)

It imports ``mcl4_coe`` from the reference's ``src/`` folder and records the
outputs of the reference's own functions on seeded inputs:

* ``quant_act.npz``   — ``_quantize_nvfp4_core(x, False, False, True)``
  (activation mode, src/mcl4_coe/nvfp4.py:197-225) and the non-causal /
  two-dimensional modes, plus ``_swizzle_scales`` (:131-144).
* ``quant_w.npz``     — ``_quantize_grouped_weights_core`` (:923-952).
* ``routing.npz``     — ``SparseMoE.forward`` (src/mcl4_coe/backbone.py:618)
  instrumented to record the router logits, ``topk`` and stable ``argsort``
  results, plus the returned aux / z / counts and ``last_selected_mask``.
* ``layer.npz``       — the layer output of the unmodified ``SparseMoE.forward``
  whose expert projections were replaced by dequantised-FP4 linears built
  from the reference's ``_quantize_nvfp4_core`` / ``_dequantize_nvfp4``.
* ``sparse.npz``      — ``compute_2to4_mask`` (:70-110) in both modes, the grouped
  quantiser's bytes of the masked weights (:1017-1024), and the dequantised-FP4
  layer whose experts carry 2:4-masked weights.
* ``variants.npz``    — the same dequantised-FP4 layer with the routing
  variants switched on (mitotic twins, lineage families, coverage penalty,
  dense subsets, sequence-diversity / orthogonality losses): outputs, losses,
  counts, ``last_selected_mask``, and the lineage configuration.

Inputs come from numpy's PCG64 generator (platform independent); their
SHA-256 digests are stored so the tests can regenerate and verify them
instead of storing large weight arrays.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
from contextlib import contextmanager
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

from inputs import (  # noqa: E402  (shared with the tests)
    act_quant_cases,
    layer_case,
    routing_cases,
    sparse_cases,
    sparse_layer_cases,
    variant_cases,
    variant_prior,
    weight_quant_cases,
)


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("MCL4_REFERENCE_SRC"),
                    help="the reference checkout's src/ folder (or set MCL4_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("pass --reference-src PATH (the reference's src/ folder) or set MCL4_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)
    import torch
    from torch import nn
    from torch.nn import functional as F

    import mcl4_coe.backbone as bb
    import mcl4_coe.nvfp4 as nv

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # ---------------------------------------------------------------- quantisers
    out = {}
    for name, x, mode in act_quant_cases():
        xt = torch.from_numpy(x)
        if mode == "act":
            packed, scales, g = nv._quantize_nvfp4_core(xt, False, False, True)
        elif mode == "tensor1d":
            packed, scales, g = nv._quantize_nvfp4_core(xt, False, False, False)
        else:  # "tile2d"
            packed, scales, g = nv._quantize_nvfp4_core(xt, True, False, False)
        out[f"{name}__in"] = x
        out[f"{name}__packed"] = packed.numpy()
        out[f"{name}__scales"] = scales.view(torch.uint8).numpy()
        out[f"{name}__g"] = g.numpy().astype(np.float32)
        out[f"{name}__swizzled"] = nv._swizzle_scales(scales).view(torch.uint8).numpy()
    np.savez_compressed(HERE / "quant_act.npz", **out)

    out = {}
    for name, w in weight_quant_cases():
        b_fwd, bs_fwd, bg, b_bwd, bs_bwd = nv._quantize_grouped_weights_core(torch.from_numpy(w))
        out[f"{name}__digest"] = np.array(digest(w))
        out[f"{name}__b_fwd"] = b_fwd.numpy()
        out[f"{name}__bs_fwd"] = bs_fwd.view(torch.uint8).numpy()
        out[f"{name}__bg"] = bg.numpy()
        out[f"{name}__b_bwd"] = b_bwd.numpy()
        out[f"{name}__bs_bwd"] = bs_bwd.view(torch.uint8).numpy()
        # the per-matrix two-dimensional core must agree with the grouped one
        p2, s2, g2 = nv._quantize_nvfp4_core(torch.from_numpy(w[0]), True, False, False)
        out[f"{name}__core2d_packed0"] = p2.numpy()
        out[f"{name}__core2d_scales0"] = s2.view(torch.uint8).numpy()
        out[f"{name}__core2d_g0"] = g2.numpy()
    np.savez_compressed(HERE / "quant_w.npz", **out)

    # ---------------------------------------------------------------- routing
    @contextmanager
    def recording(router_weight, bias):
        rec = {}
        orig_linear = F.linear
        orig_topk = torch.Tensor.topk
        orig_argsort = torch.Tensor.argsort

        def linear(inp, weight, b=None):
            res = orig_linear(inp, weight, b)
            if weight.data_ptr() == router_weight.data_ptr():
                if bias is not None:
                    res = res + bias
                rec["logits"] = res.detach().clone()
            return res

        def topk(self, *a, **kw):
            res = orig_topk(self, *a, **kw)
            if "topk_values" not in rec:
                rec["topk_values"] = res[0].detach().clone()
                rec["topk_indices"] = res[1].detach().clone()
            return res

        def argsort(self, *a, **kw):
            res = orig_argsort(self, *a, **kw)
            rec.setdefault("perm", res.detach().clone())
            return res

        F.linear = linear
        bb.F.linear = linear
        torch.Tensor.topk = topk
        torch.Tensor.argsort = argsort
        try:
            yield rec
        finally:
            F.linear = orig_linear
            bb.F.linear = orig_linear
            torch.Tensor.topk = orig_topk
            torch.Tensor.argsort = orig_argsort

    class FakeQuantLinear(nn.Module):
        """Dequantised-FP4 projection: NVFP4 1x16 activations, 16x16-tile weights."""

        def __init__(self, weight: np.ndarray):
            super().__init__()
            wt = torch.from_numpy(weight)
            packed, scales, g = nv._quantize_nvfp4_core(wt, True, False, False)
            self.register_buffer("w_deq", nv._dequantize_nvfp4(
                packed, nv._swizzle_scales(scales), g, wt.shape[0], wt.shape[1]))
            self.register_buffer("weight", wt.clone())  # read by the orthogonality loss

        def forward(self, x):
            xf = x.float()
            rows, cols = xf.shape
            packed, scales, g = nv._quantize_nvfp4_core(xf, False, False, True)
            xd = nv._dequantize_nvfp4(packed, nv._swizzle_scales(scales), g, rows, cols)
            return F.linear(xd, self.w_deq).to(x.dtype)

    def build_moe(case, fake_experts: bool):
        cfg = bb.MCL4CEDConfig(d_model=case["d"], n_heads=4, expert_hidden_dim=case["f"],
                               num_experts=case["e"], top_k=case["k"],
                               norm_topk_prob=case["norm_topk_prob"])
        moe = bb.SparseMoE(cfg).eval()
        with torch.no_grad():
            moe.router.weight.copy_(torch.from_numpy(case["wr"]))
            for i, ex in enumerate(moe.experts):
                ex.up_proj.weight.copy_(torch.from_numpy(case["w_up"][i]))
                ex.down_proj.weight.copy_(torch.from_numpy(case["w_dn"][i]))
                if fake_experts:
                    ex.up_proj = FakeQuantLinear(case["w_up"][i])
                    ex.down_proj = FakeQuantLinear(case["w_dn"][i])
        return moe

    def run(case, fake_experts):
        moe = build_moe(case, fake_experts)
        x = torch.from_numpy(case["x_bf16_bits"].view(np.int16)).view(torch.bfloat16).reshape(case["t"], case["d"])
        valid = None if case["valid"] is None else torch.from_numpy(case["valid"].astype(bool))
        bias = None if case["logit_bias"] is None else torch.from_numpy(case["logit_bias"])
        with torch.no_grad(), recording(moe.router.weight, bias) as rec:
            y, aux, z, counts = moe(x, valid=valid)
        return moe, y, aux, z, counts, rec

    out = {}
    for name, case in routing_cases():
        moe, y, aux, z, counts, rec = run(case, fake_experts=True)
        out[f"{name}__digest"] = np.array(digest(case["x_bf16_bits"], case["wr"]))
        out[f"{name}__logits"] = rec["logits"].numpy()
        out[f"{name}__topk_values"] = rec["topk_values"].numpy()
        out[f"{name}__topk_indices"] = rec["topk_indices"].numpy()
        out[f"{name}__perm"] = rec["perm"].numpy()
        out[f"{name}__aux"] = np.float32(aux.item())
        out[f"{name}__z"] = np.float32(z.item())
        out[f"{name}__counts"] = counts.numpy()
        out[f"{name}__sel_mask"] = moe.last_selected_mask.reshape(case["t"], case["e"]).numpy().astype(np.uint8)
    np.savez_compressed(HERE / "routing.npz", **out)

    out = {}
    for name, case in [layer_case()]:
        moe, y, aux, z, counts, rec = run(case, fake_experts=True)
        out[f"{name}__digest"] = np.array(digest(case["x_bf16_bits"], case["wr"], case["w_up"], case["w_dn"]))
        out[f"{name}__out_bf16"] = y.view(torch.int16).numpy().view(np.uint16)
        out[f"{name}__aux"] = np.float32(aux.item())
        out[f"{name}__z"] = np.float32(z.item())
        out[f"{name}__counts"] = counts.numpy()
        out[f"{name}__topk_indices"] = rec["topk_indices"].numpy()
        out[f"{name}__perm"] = rec["perm"].numpy()
    np.savez_compressed(HERE / "layer.npz", **out)

    # ---------------------------------------------------------------- 2:4 sparsity
    out = {}
    for name, w in sparse_cases():
        out[f"{name}__digest"] = np.array(digest(w))
        for mode in ("2to4_row", "2to4_transposable"):
            masks = np.stack([nv.compute_2to4_mask(torch.from_numpy(w[i]), mode=mode).numpy() for i in range(len(w))])
            out[f"{name}__{mode}__mask"] = masks.astype(np.uint8)
            if w.shape[1] % 16 == 0 and w.shape[2] % 64 == 0:
                masked = torch.from_numpy(w) * torch.from_numpy(masks).float()
                b_fwd, bs_fwd, bg, _, _ = nv._quantize_grouped_weights_core(masked)
                out[f"{name}__{mode}__b_fwd"] = b_fwd.numpy()
                out[f"{name}__{mode}__bs_fwd"] = bs_fwd.view(torch.uint8).numpy()
                out[f"{name}__{mode}__bg"] = bg.numpy()
    for name, case, mode in sparse_layer_cases():
        masked = {}
        for proj, key in (("up_proj", "w_up"), ("down_proj", "w_dn")):
            masked[key] = np.stack([(torch.from_numpy(case[key][i])
                                     * nv.compute_2to4_mask(torch.from_numpy(case[key][i]), mode=mode).float()).numpy()
                                    for i in range(case["e"])])
        mcase = dict(case, w_up=masked["w_up"], w_dn=masked["w_dn"])
        moe, y, aux, z, counts, rec = run(mcase, fake_experts=True)
        out[f"{name}__digest"] = np.array(digest(case["x_bf16_bits"], case["wr"], case["w_up"], case["w_dn"]))
        out[f"{name}__out_bf16"] = y.view(torch.int16).numpy().view(np.uint16)
        out[f"{name}__aux"] = np.float32(aux.item())
        out[f"{name}__z"] = np.float32(z.item())
        out[f"{name}__counts"] = counts.numpy()
    np.savez_compressed(HERE / "sparse.npz", **out)

    # ---------------------------------------------------------------- routing variants
    out = {}
    for name, case, o in variant_cases():
        cfg = bb.MCL4CEDConfig(d_model=case["d"], n_heads=4, expert_hidden_dim=case["f"], num_experts=case["e"],
                               top_k=case["k"], norm_topk_prob=case["norm_topk_prob"],
                               recurrent_coverage_penalty=o["coverage"], mitotic_ortho_coef=o["ortho"],
                               sequence_diversity_coef=o["seq_div"], dense_subset_k=o["dense_k"],
                               combine_dense_and_sparse=o["combine"])
        moe = bb.SparseMoE(cfg).eval()
        with torch.no_grad():
            moe.router.weight.copy_(torch.from_numpy(case["wr"]))
            for i, ex in enumerate(moe.experts):
                ex.up_proj.weight.copy_(torch.from_numpy(case["w_up"][i]))
                ex.down_proj.weight.copy_(torch.from_numpy(case["w_dn"][i]))
        if o["pairs"]:
            moe.mitotic_pairs = [tuple(p) for p in o["pairs"]]
        if o["lineage"] is not None:
            roots, fams, share = o["lineage"]
            moe.configure_lineage_family_routing(roots, top_families=fams, child_share=share)
            out[f"{name}__lineage_root_ids"] = moe.lineage_root_ids.numpy()
            out[f"{name}__lineage_logit_prior"] = moe.lineage_logit_prior.numpy()
        for i, ex in enumerate(moe.experts):
            ex.up_proj = FakeQuantLinear(case["w_up"][i])
            ex.down_proj = FakeQuantLinear(case["w_dn"][i])
        x = torch.from_numpy(case["x_bf16_bits"].view(np.int16)).view(torch.bfloat16).reshape(case["t"], case["d"])
        valid = None if case["valid"] is None else torch.from_numpy(case["valid"].astype(bool))
        if o["shape"] is not None:
            x = x.reshape(*o["shape"], case["d"])
            valid = None if valid is None else valid.reshape(*o["shape"])
        prior = variant_prior(name, case["t"], case["e"], o["prior_frac"])
        prior_t = None if prior is None else torch.from_numpy(prior)
        with torch.no_grad():
            y, aux, z, counts = moe(x, valid=valid, prior_expert_mask=prior_t,
                                    dense_expert_indices=None if o["dense_idx"] is None else list(o["dense_idx"]))
        out[f"{name}__digest"] = np.array(digest(case["x_bf16_bits"], case["wr"], case["w_up"], case["w_dn"]))
        out[f"{name}__out_bf16"] = y.reshape(case["t"], case["d"]).view(torch.int16).numpy().view(np.uint16)
        out[f"{name}__aux"] = np.float32(aux.item())
        out[f"{name}__z"] = np.float32(z.item())
        out[f"{name}__counts"] = counts.numpy().astype(np.float32)
        out[f"{name}__sel_mask"] = moe.last_selected_mask.reshape(case["t"], case["e"]).numpy().astype(np.float32)
    np.savez_compressed(HERE / "variants.npz", **out)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
