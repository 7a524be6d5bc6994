"""Routing variants of ``SparseMoE`` that feed the native layer with a precomputed routing.

The reference decides, per token, which experts run and with which weights in
several ways besides plain top-k (src/mcl4_coe/backbone.py):

* mitotic twin pairs: a parent / child pair shares one routing slot, the
  higher logit wins it (:791-832, loop branch :935-969);
* lineage families: top families of a root-anchored expert tree, then top-k
  inside them, k possibly larger than ``top_k`` (:274-305, :833-841);
* recurrent coverage penalty: experts already used by the previous pass are
  down-weighted for selection only (:843-851);
* dense subsets: a fixed or pooled-top-k set of experts runs on every active
  token, optionally mixed with a sparse remainder (:640-785, :307-398);
* two auxiliary-loss terms: sequence diversity (:452-469) and mitotic
  orthogonality (:400-450).

These functions compute exactly the reference's probabilities, selections,
weights and losses with torch on the router logits (the selection logic is a
few [T, E] elementwise / top-k operations); the expert work then runs through
``mcl4moe_moe_forward_routed`` (stable expert-major permutation, NVFP4
quantisation, tcgen05 grouped GEMMs, combine).  Everything here is
device-agnostic, so the CPU tests check it against the reference's own
outputs.  Statistics follow the reference's loop branch (:913-1047): masked
tokens are dropped before routing.
"""

from __future__ import annotations

from typing import Any, Sequence

import torch
from torch import Tensor
from torch.nn import functional as F

LN2 = 0.6931471805599453
SQRT2 = 1.4142135623730951


def pair_tensors(moe: Any, device: torch.device) -> tuple[Tensor, Tensor] | None:
    """Parent and child index tensors of the valid mitotic pairs, or None
    (src/mcl4_coe/backbone.py:471-488)."""
    pairs = [(p, c) for p, c in getattr(moe, "mitotic_pairs", [])
             if 0 <= p < moe.num_experts and 0 <= c < moe.num_experts and p != c]
    if not pairs:
        return None
    key = (tuple(pairs), moe.num_experts, str(device))
    cached = getattr(moe, "_pair_index_cache", None)
    if cached is not None and cached[0] == key:
        return cached[1], cached[2]
    p_t = torch.tensor([p for p, _ in pairs], dtype=torch.long, device=device)
    c_t = torch.tensor([c for _, c in pairs], dtype=torch.long, device=device)
    moe._pair_index_cache = (key, p_t, c_t)
    return p_t, c_t


def lineage_active(moe: Any, pairs) -> bool:
    return (moe.lineage_top_families > 0 and moe.lineage_root_ids is not None
            and moe.lineage_logit_prior is not None and pairs is None)


def _twin_probabilities(moe: Any, logits: Tensor, pairs, adjust_norm_false: bool) -> tuple[Tensor, Tensor]:
    """Softmax probabilities and the routed probabilities after the twin rule.

    ``adjust_norm_false``: with ``norm_topk_prob`` off the sparse path shifts both
    twins' logits by -ln 2 and gives the winner the pair's mass
    (src/mcl4_coe/backbone.py:791-817); otherwise (and always in the dense-subset
    path, :654-670) the winner keeps its own probability and the loser gets 0."""
    if pairs is not None and adjust_norm_false and not moe.norm_topk_prob:
        p_t, c_t = pairs
        adj = logits.clone()
        adj[:, p_t] = adj[:, p_t] - LN2
        adj[:, c_t] = adj[:, c_t] - LN2
        probs = F.softmax(adj, dim=-1)
    else:
        probs = F.softmax(logits, dim=-1)
    if pairs is None:
        return probs, probs
    p_t, c_t = pairs
    routed = probs.clone()
    parent_wins = logits.index_select(1, p_t) >= logits.index_select(1, c_t)
    zero = torch.zeros_like(parent_wins, dtype=routed.dtype)
    if adjust_norm_false and not moe.norm_topk_prob:
        mass = probs.index_select(1, p_t) + probs.index_select(1, c_t)
        routed[:, c_t] = torch.where(parent_wins, zero, mass)
        routed[:, p_t] = torch.where(parent_wins, mass, zero)
    else:
        routed[:, c_t] = torch.where(parent_wins, zero, probs.index_select(1, c_t))
        routed[:, p_t] = torch.where(parent_wins, probs.index_select(1, p_t), zero)
    return probs, routed


def _coverage_scores(moe: Any, routed: Tensor, prior: Tensor | None) -> Tensor:
    """Selection scores with the recurrent coverage penalty (src/mcl4_coe/backbone.py:843-851)."""
    if prior is None or moe.recurrent_coverage_penalty <= 0.0:
        return routed
    return routed * (1.0 - moe.recurrent_coverage_penalty * prior.to(routed.dtype)).clamp_min(0.05)


def lineage_selection(moe: Any, logits: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Family-calibrated probabilities, weights and selection (src/mcl4_coe/backbone.py:274-305)."""
    dev = logits.device
    root_ids = moe.lineage_root_ids.to(dev)
    probs = F.softmax(logits + moe.lineage_logit_prior.to(dev).unsqueeze(0), dim=-1)
    n = logits.shape[0]
    fam = logits.new_zeros((n, moe.lineage_num_roots))
    fam.scatter_add_(1, root_ids.unsqueeze(0).expand(n, -1), probs)
    _, top_fams = fam.topk(moe.lineage_top_families, dim=-1)
    fam_mask = logits.new_zeros((n, moe.lineage_num_roots))
    fam_mask.scatter_(1, top_fams, 1.0)
    exp_mask = fam_mask.index_select(1, root_ids)
    max_active = int(exp_mask.sum(dim=-1).max().item()) if n > 0 else moe.top_k
    k_sel = max(moe.top_k, min(moe.num_experts, max_active))
    # tokens whose families hold fewer than k_sel experts fill the rest with zero-weight
    # (family-masked) experts; which ones is torch.topk's tie order, which differs between
    # CPU and CUDA, as in the reference.  They change last_selected_mask, not the output.
    weights, selected = (probs * exp_mask).topk(k_sel, dim=-1)
    if moe.norm_topk_prob:
        weights = weights / weights.sum(dim=-1, keepdim=True).clamp_min(1e-9)
    return probs, weights, selected


def sparse_selection(moe: Any, logits: Tensor, prior: Tensor | None) -> tuple[Tensor, Tensor, Tensor]:
    """(probabilities, weights [n, k_eff], selected [n, k_eff]) of the sparse routing
    of the active tokens (src/mcl4_coe/backbone.py:928-994)."""
    pairs = pair_tensors(moe, logits.device)
    probs, routed = _twin_probabilities(moe, logits, pairs, adjust_norm_false=True)
    if lineage_active(moe, pairs):
        return lineage_selection(moe, logits)
    if prior is not None and moe.recurrent_coverage_penalty > 0.0:
        _, selected = _coverage_scores(moe, routed, prior).topk(moe.top_k, dim=-1)
        weights = routed.gather(-1, selected)
    else:
        weights, selected = routed.topk(moe.top_k, dim=-1)
    if moe.norm_topk_prob:
        weights = weights / weights.sum(dim=-1, keepdim=True).clamp_min(1e-9)
    return probs, weights, selected


def dense_selection(moe: Any, logits: Tensor, prior: Tensor | None, dense_indices: Sequence[int],
                    dense_k: int) -> dict[str, Any]:
    """Chosen experts, their per-token weights and the scores the sparse remainder
    uses (src/mcl4_coe/backbone.py:650-700)."""
    pairs = pair_tensors(moe, logits.device)
    probs, routed = _twin_probabilities(moe, logits, pairs, adjust_norm_false=False)
    scores = _coverage_scores(moe, routed, prior)
    if dense_indices:
        chosen = [i for i in dense_indices if 0 <= i < moe.num_experts]
        chosen_t = torch.tensor(chosen, dtype=torch.long, device=logits.device)
    else:
        _, chosen_t = scores.mean(dim=0).topk(min(max(1, dense_k), moe.num_experts), dim=-1)
        chosen = [int(i) for i in chosen_t.detach().cpu().tolist()]
    w = probs.index_select(1, chosen_t)
    w = w / w.sum(dim=-1, keepdim=True).clamp_min(1e-9)
    return dict(probs=probs, routed=routed, scores=scores, chosen=chosen, chosen_t=chosen_t, weights=w)


def dense_remainder(moe: Any, sel: dict[str, Any], dtype: torch.dtype) -> dict[str, Tensor] | None:
    """Sparse remainder of a dense subset and the mixing coefficients
    (src/mcl4_coe/backbone.py:733-752), or None when nothing remains."""
    chosen_t = sel["chosen_t"]
    rem_k = min(moe.top_k, moe.num_experts - len(sel["chosen"]))
    if not moe.combine_dense_and_sparse or len(sel["chosen"]) >= moe.num_experts or rem_k <= 0:
        return None
    dense_mass = sel["probs"].index_select(1, chosen_t).sum(dim=-1, keepdim=True).clamp_min(1e-9)
    rem_scores = sel["scores"].clone()
    rem_scores[:, chosen_t] = -1.0
    _, rem_sel = rem_scores.topk(rem_k, dim=-1)
    rem_raw = sel["routed"].gather(-1, rem_sel)
    rem_mass = rem_raw.sum(dim=-1, keepdim=True).clamp_min(0.0)
    total = (dense_mass + rem_mass).clamp_min(1e-9)
    return dict(selected=rem_sel, weights=rem_raw / rem_mass.clamp_min(1e-9),
                alpha_dense=(dense_mass / total).to(dtype), alpha_rem=(rem_mass / total).to(dtype))


def mitotic_ortho_loss(moe: Any, device: torch.device) -> Tensor:
    """Chordal orthogonality of the twin pairs' weights (src/mcl4_coe/backbone.py:400-450)."""
    pairs = [(p, c) for p, c in getattr(moe, "mitotic_pairs", [])
             if 0 <= p < moe.num_experts and 0 <= c < moe.num_experts and p != c]
    if not pairs:
        return torch.zeros((), dtype=torch.float32, device=device)
    max_pairs = 2 if moe.num_experts * moe.router.in_features >= 65536 else 16
    if len(pairs) > max_pairs:  # a rotating window of pairs per call
        offset = int(getattr(moe, "_ortho_pair_cursor", 0)) % len(pairs)
        moe._ortho_pair_cursor = offset + max_pairs
        pairs = (pairs + pairs)[offset:offset + max_pairs]

    def chordal(proj: str, dim: int) -> Tensor:
        a = F.normalize(torch.stack([getattr(moe.experts[p], proj).weight for p, _ in pairs]).float(),
                        p=2.0, dim=dim, eps=1e-8)
        b = F.normalize(torch.stack([getattr(moe.experts[c], proj).weight for _, c in pairs]).float(),
                        p=2.0, dim=dim, eps=1e-8)
        return ((SQRT2 - (a - b).norm(p=2.0, dim=dim)) / SQRT2).clamp_min(0.0).mean()

    return 0.5 * (chordal("up_proj", -1) + chordal("down_proj", 1))


def sequence_diversity_loss(moe: Any, probs_bt: Tensor, valid: Tensor | None) -> Tensor:
    """Within-sequence expert-collision penalty (src/mcl4_coe/backbone.py:452-469)."""
    if probs_bt.ndim != 3 or probs_bt.shape[1] <= 1:
        return probs_bt.new_zeros(())
    if valid is None:
        seq = probs_bt.mean(dim=1)
        return (moe.num_experts * seq.square().sum(dim=-1).mean() - 1.0).clamp_min(0.0)
    v = valid.to(probs_bt.dtype).unsqueeze(-1)
    seq = (probs_bt * v).sum(dim=1) / v.sum(dim=1).clamp_min(1.0)
    row_valid = valid.any(dim=1).to(probs_bt.dtype)
    collision = (moe.num_experts * seq.square().sum(dim=-1) - 1.0).clamp_min(0.0)
    return (collision * row_valid).sum() / row_valid.sum().clamp_min(1.0)


def add_extra_aux(moe: Any, aux: Tensor, x_shape, probs_active: Tensor, active: Tensor, n_tokens: int,
                  valid: Tensor | None) -> Tensor:
    """``aux`` plus the sequence-diversity and mitotic-orthogonality terms, added in
    the reference's order (src/mcl4_coe/backbone.py:1004-1015)."""
    if moe.sequence_diversity_coef > 0.0 and len(x_shape) == 3 and x_shape[1] > 1:
        full = probs_active.new_zeros((n_tokens, moe.num_experts))
        full.index_copy_(0, active, probs_active)
        aux = aux + moe.sequence_diversity_coef * sequence_diversity_loss(
            moe, full.view(x_shape[0], x_shape[1], moe.num_experts), valid)
    if moe.mitotic_ortho_coef > 0.0 and getattr(moe, "mitotic_pairs", None):
        aux = aux + moe.mitotic_ortho_coef * mitotic_ortho_loss(moe, aux.device)
    return aux


def sparse_statistics(moe: Any, logits: Tensor, probs: Tensor, selected: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """(aux_loss, router_z_loss, counts) of the active tokens' sparse routing
    (src/mcl4_coe/backbone.py:1001-1004)."""
    counts = F.one_hot(selected, num_classes=moe.num_experts).sum(dim=(0, 1)).float() / max(1, selected.numel())
    aux = moe.num_experts * (counts * probs.mean(dim=0)).sum()
    z = torch.logsumexp(logits, dim=-1).square().mean()
    return aux, z, counts


def dense_statistics(moe: Any, logits: Tensor, probs: Tensor, chosen: list[int],
                     chosen_t: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """(selection mask of the active tokens, aux_loss, router_z_loss, counts) of a
    dense subset (src/mcl4_coe/backbone.py:701-711)."""
    mask = logits.new_zeros((logits.shape[0], moe.num_experts), dtype=torch.float32)
    mask[:, chosen_t] = 1.0
    counts = mask.sum(dim=0) / max(1, logits.shape[0] * len(chosen))
    aux = moe.num_experts * (counts * probs.mean(dim=0)).sum()
    z = torch.logsumexp(logits, dim=-1).square().mean()
    return mask, aux, z, counts
