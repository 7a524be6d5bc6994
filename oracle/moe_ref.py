"""numpy restatement of the reference MoE routing and dequantised-FP4 layer
(test infrastructure only).

Restates ``SparseMoE.forward`` (src/mcl4_coe/backbone.py:618-1047) for the
routing configuration the hot path serves: no mitotic pairs, no lineage
families, no coverage penalty, no dense subset.  ``valid`` follows the loop
branch (:913-1047): masked-out tokens are not routed, produce zeros and a zero
row in the selection mask.  The expert projections are the "dequantised-FP4
CPU path": every activation entering a projection is quantised to NVFP4 with
1x16 row scales and dequantised (src/mcl4_coe/nvfp4.py:197-225, :263-281), the
weights are the 16x16-tile NVFP4 weights of
src/mcl4_coe/nvfp4.py:923-952 dequantised, the product is accumulated in
float32 and rounded to bfloat16 (src/mcl4_coe/nvfp4.py:429, :869-873).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import nvfp4_ref as nr


@dataclass
class Routing:
    logits: np.ndarray        # float32 [Ta, E]  (Ta = routed tokens)
    probs: np.ndarray         # float32 [Ta, E]
    selected: np.ndarray      # int64   [Ta, k]
    weights: np.ndarray       # float32 [Ta, k]  (after optional renormalisation)
    active: np.ndarray        # int64   [Ta]  token ids routed
    counts_int: np.ndarray    # int64   [E]
    counts: np.ndarray        # float32 [E]  (the layer's 4th output)
    aux_loss: np.float32
    z_loss: np.float32
    sel_mask: np.ndarray      # float32 [T, E]
    perm: np.ndarray          # int64   [Ta*k]  stable expert-major order of flat slots
    offs: np.ndarray          # int32   [E]  inclusive ends (cumsum of counts_int)


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    """``F.softmax(dim=-1)`` in float32 (src/mcl4_coe/backbone.py:800, :939):
    subtract the row max, exponentiate, scale by the reciprocal of the sum."""
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp((logits - m).astype(np.float32)).astype(np.float32)
    s = e.sum(axis=-1, keepdims=True, dtype=np.float32)
    return (e * (np.float32(1.0) / s)).astype(np.float32)


def logsumexp_f32(logits: np.ndarray) -> np.ndarray:
    m = logits.max(axis=-1)
    return (m + np.log(np.exp(logits - m[:, None]).sum(axis=-1, dtype=np.float32))).astype(np.float32)


def topk_desc(values: np.ndarray, k: int):
    """``Tensor.topk(k)`` (src/mcl4_coe/backbone.py:853): descending values,
    ties broken towards the lower expert index."""
    order = np.argsort(-values, axis=-1, kind="stable")[:, :k]
    return np.take_along_axis(values, order, axis=-1), order.astype(np.int64)


def route(x: np.ndarray, wr: np.ndarray, top_k: int, norm_topk_prob: bool = True,
          valid: np.ndarray | None = None, logit_bias: np.ndarray | None = None,
          logits: np.ndarray | None = None) -> Routing:
    """Router, top-k and routing statistics.

    src/mcl4_coe/backbone.py:913-1004 (loop branch; identical per-token math
    to the grouped branch :787-883): fp32 logits ``x @ Wr^T`` (:929), softmax
    (:939), top-k (:992), renormalisation ``w / max(sum w, 1e-9)`` when
    ``norm_topk_prob`` (:993-994), one-hot selection mask (:995-1000), counts
    ``bincount/(Ta*k)`` (:1001-1002), ``aux = E * sum(counts * mean probs)``
    (:1003) and ``z = mean(logsumexp^2)`` (:1004); stable argsort permutation
    (:1017-1019).  ``logit_bias`` models a caller-side additive router bias
    (the Zipf skew of the benchmark's skewed configuration).  ``logits``
    overrides the router product (to check the rest bit for bit).
    """
    t_total = x.shape[0] if logits is None else logits.shape[0]
    e_count = wr.shape[0]
    if valid is None:
        active = np.arange(t_total, dtype=np.int64)
    else:
        active = np.nonzero(np.asarray(valid).reshape(-1))[0].astype(np.int64)
    if logits is None:
        xa = np.asarray(x, dtype=np.float32)[active]
        logits = (xa @ np.asarray(wr, dtype=np.float32).T).astype(np.float32)
        if logit_bias is not None:
            logits = (logits + np.asarray(logit_bias, dtype=np.float32)[None, :]).astype(np.float32)
    else:
        logits = np.asarray(logits, dtype=np.float32)[active]
    probs = softmax_f32(logits)
    weights, selected = topk_desc(probs, top_k)
    if norm_topk_prob:
        denom = np.maximum(weights.sum(axis=-1, keepdims=True, dtype=np.float32), np.float32(1e-9))
        weights = (weights / denom).astype(np.float32)
    sel_mask = np.zeros((t_total, e_count), dtype=np.float32)
    if active.size:
        sel_mask[active[:, None], selected] = 1.0
    counts_int = np.bincount(selected.reshape(-1), minlength=e_count).astype(np.int64)
    n_sel = max(1, selected.size)
    counts = (counts_int.astype(np.float32) / np.float32(n_sel)).astype(np.float32)
    if active.size:
        aux = np.float32(e_count) * np.float32((counts * probs.mean(axis=0, dtype=np.float32)).sum(dtype=np.float32))
        z = np.float32((logsumexp_f32(logits) ** 2).mean(dtype=np.float32))
    else:
        aux = np.float32(0.0)
        z = np.float32(0.0)
        counts = np.zeros(e_count, dtype=np.float32)
    perm = np.argsort(selected.reshape(-1), kind="stable").astype(np.int64)
    offs = np.cumsum(counts_int).astype(np.int32)
    return Routing(logits, probs, selected, weights.astype(np.float32), active, counts_int, counts,
                   np.float32(aux), np.float32(z), sel_mask, perm, offs)


def silu_bf16(gate: np.ndarray) -> np.ndarray:
    """``F.silu`` on a bfloat16 tensor: ``g / (1 + exp(-g))`` in float32, rounded."""
    g = gate.astype(np.float32)
    return nr.round_bf16((g / (np.float32(1.0) + np.exp(-g))).astype(np.float32))


def expert_forward(xe: np.ndarray, w_up: np.ndarray, w_dn: np.ndarray) -> np.ndarray:
    """One ``SwiGLUExpert`` on the dequantised-FP4 path (src/mcl4_coe/backbone.py:185-187).

    ``xe`` are bfloat16 values (float32 array); ``w_up`` ``[2F, d]`` (gate
    rows first) and ``w_dn`` ``[d, F]`` are the dequantised weights.
    """
    if xe.shape[0] == 0:
        return np.zeros((0, w_dn.shape[0]), dtype=np.float32)
    f = w_up.shape[0] // 2
    up = nr.round_bf16((nr.fake_quantize_activations(xe) @ w_up.T).astype(np.float32))
    gate, val = up[:, :f], up[:, f:]
    h = nr.round_bf16((silu_bf16(gate) * val).astype(np.float32))
    return nr.round_bf16((nr.fake_quantize_activations(h) @ w_dn.T).astype(np.float32))


class QuantizedExperts:
    """Dequantised NVFP4 weights of every expert (the quantised-weight cache of
    src/mcl4_coe/nvfp4.py:962-1048, built once and reused)."""

    def __init__(self, w_up: np.ndarray, w_dn: np.ndarray):
        self.up_q = nr.quantize_grouped_weights(np.asarray(w_up, dtype=np.float32), with_bwd=False)
        self.dn_q = nr.quantize_grouped_weights(np.asarray(w_dn, dtype=np.float32), with_bwd=False)
        n_exp = w_up.shape[0]
        self.up = [nr.dequantize_grouped_weight(self.up_q[0], self.up_q[1], self.up_q[2], e) for e in range(n_exp)]
        self.dn = [nr.dequantize_grouped_weight(self.dn_q[0], self.dn_q[1], self.dn_q[2], e) for e in range(n_exp)]


def moe_forward(x: np.ndarray, wr: np.ndarray, experts: QuantizedExperts, top_k: int,
                norm_topk_prob: bool = True, valid: np.ndarray | None = None,
                logit_bias: np.ndarray | None = None, routing: Routing | None = None):
    """The MoE layer on the dequantised-FP4 CPU path.

    Returns ``(out float32-held bf16 [T, d], aux, z, counts [E], routing)``.
    Combine follows src/mcl4_coe/backbone.py:1032-1041: ``bf16(y * bf16(w))``
    per slot, un-permuted, summed over the k slots of a token in float32 and
    rounded once to bfloat16.
    """
    x = nr.round_bf16(np.asarray(x, dtype=np.float32))
    t_total, d = x.shape
    r = routing if routing is not None else route(x, wr, top_k, norm_topk_prob, valid, logit_bias)
    out = np.zeros((t_total, d), dtype=np.float32)
    if r.active.size == 0:
        return out, np.float32(0.0), np.float32(0.0), np.zeros(wr.shape[0], np.float32), r
    k_eff = r.selected.shape[1]
    xa = x[r.active]
    sorted_tokens = r.perm // k_eff
    sorted_w = r.weights.reshape(-1)[r.perm]
    weighted = np.zeros((r.perm.size, d), dtype=np.float32)
    start = 0
    for e, cnt in enumerate(r.counts_int):
        cnt = int(cnt)
        if cnt == 0:
            continue
        rows = sorted_tokens[start:start + cnt]
        y = expert_forward(xa[rows], experts.up[e], experts.dn[e])
        weighted[start:start + cnt] = nr.round_bf16((y * nr.round_bf16(sorted_w[start:start + cnt])[:, None]).astype(np.float32))
        start += cnt
    unpermed = np.empty_like(weighted)
    unpermed[r.perm] = weighted
    acc = np.zeros((r.active.size, d), dtype=np.float32)
    u = unpermed.reshape(r.active.size, k_eff, d)
    for j in range(k_eff):
        acc = (acc + u[:, j, :]).astype(np.float32)
    out[r.active] = nr.round_bf16(acc)
    return out, r.aux_loss, r.z_loss, r.counts, r
