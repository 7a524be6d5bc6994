"""Helpers for the GPU parity tests: build a module from numpy weights, and a
per-token reference of the dequantised-FP4 layer for sizes where the full
numpy oracle would be too slow (weights dequantised on the GPU in torch fp32
from bytes whose bit-exactness is checked separately)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import nvfp4_ref as nr

E2M1_LUT = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                         -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)


def build_module(pkg, case: dict, device) -> torch.nn.Module:
    moe = pkg.SparseMoE(pkg.MoEConfig(d_model=case["d"], expert_hidden_dim=case["f"], num_experts=case["e"],
                                      top_k=case["k"], norm_topk_prob=case["norm_topk_prob"])).to(device)
    with torch.no_grad():
        moe.router.weight.copy_(torch.from_numpy(case["wr"]))
        for i, ex in enumerate(moe.experts):
            ex.up_proj.weight.copy_(torch.from_numpy(case["w_up"][i]))
            ex.down_proj.weight.copy_(torch.from_numpy(case["w_dn"][i]))
    if case.get("logit_bias") is not None:
        moe.router_logit_bias = torch.from_numpy(case["logit_bias"]).to(device)
    return moe


def x_tensor(case: dict, device) -> torch.Tensor:
    bits = torch.from_numpy(case["x_bf16_bits"].view(np.int16).copy())
    return bits.view(torch.bfloat16).reshape(case["t"], case["d"]).to(device)


def dequant_reference_layout(b_fwd: torch.Tensor, bs_fwd: torch.Tensor, bg: torch.Tensor) -> torch.Tensor:
    """Reference cache layout (B_fwd [E,K/2,N], Bs_fwd [E,N,K/16], Bg [E]) -> fp32 [E, N, K]."""
    e, kh, n = b_fwd.shape
    b = b_fwd.transpose(1, 2).contiguous()  # [E, N, K/2]
    codes = torch.stack(((b & 0xF), (b >> 4)), dim=-1).reshape(e, n, 2 * kh).long()
    vals = E2M1_LUT.to(b.device)[codes]
    scale = bs_fwd.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=-1)
    return vals * scale * bg.view(e, 1, 1)


def token_reference(x_bf16: torch.Tensor, topk_idx: np.ndarray, topk_w: np.ndarray,
                    w_up: torch.Tensor, w_dn: torch.Tensor) -> np.ndarray:
    """Dequantised-FP4 layer output for the given tokens and routing.

    ``x_bf16`` [Ts, d] on the GPU; ``topk_idx``/``topk_w`` numpy [Ts, k];
    ``w_up`` [E, 2F, d] / ``w_dn`` [E, d, F] dequantised fp32 on the GPU.
    Same numerics as ``oracle.moe_ref.expert_forward`` + combine.
    """
    dev = x_bf16.device
    xs = x_bf16.float().cpu().numpy()
    ts, d = xs.shape
    k = topk_idx.shape[1]
    f = w_up.shape[1] // 2
    xq = torch.from_numpy(nr.fake_quantize_activations(xs)).to(dev)
    acc = np.zeros((ts, d), dtype=np.float32)
    for j in range(k):
        for e in np.unique(topk_idx[:, j]):
            rows = np.nonzero(topk_idx[:, j] == e)[0]
            up = nr.round_bf16((xq[rows] @ w_up[e].T).cpu().numpy())
            gate, val = up[:, :f], up[:, f:]
            g = gate.astype(np.float32)
            silu = nr.round_bf16((g / (np.float32(1.0) + np.exp(-g))).astype(np.float32))
            h = nr.round_bf16((silu * val).astype(np.float32))
            hq = torch.from_numpy(nr.fake_quantize_activations(h)).to(dev)
            y = nr.round_bf16((hq @ w_dn[e].T).cpu().numpy())
            wv = nr.round_bf16(topk_w[rows, j].astype(np.float32))[:, None]
            acc[rows] = (acc[rows] + nr.round_bf16((y * wv).astype(np.float32))).astype(np.float32)
    return nr.round_bf16(acc)


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def near_tie_tokens(logits: np.ndarray, k: int, eps: float = 1e-5) -> np.ndarray:
    if logits.shape[1] <= k:
        return np.zeros(logits.shape[0], bool)
    s = -np.sort(-logits, axis=1)
    return (s[:, k - 1] - s[:, k]) <= eps


def order_tie_tokens(logits: np.ndarray, k: int, eps: float = 1e-5) -> np.ndarray:
    """Tokens whose top-k ORDER (not only membership) can flip under logit
    rounding: two adjacent values among the k+1 largest lie within ``eps``."""
    s = -np.sort(-logits, axis=1)
    m = min(k + 1, logits.shape[1])
    if m < 2:
        return np.zeros(logits.shape[0], bool)
    gaps = s[:, : m - 1] - s[:, 1:m]
    return np.any(gaps <= eps, axis=1)


def compare_routing_in_order(got_idx: np.ndarray, ref_idx: np.ndarray, logits: np.ndarray, k: int,
                             eps: float = 1e-5) -> dict:
    """Slot-by-slot comparison of two top-k selections [T, k] (same slot order
    required) with the tokens excused as order ties counted separately."""
    same = np.all(got_idx == ref_idx, axis=1)
    ties = order_tie_tokens(logits, k, eps)
    return dict(tokens=int(got_idx.shape[0]), mismatched=int((~same).sum()), order_ties=int(ties.sum()),
                mismatched_outside_ties=int((~same & ~ties).sum()), mismatched_in_ties=int((~same & ties).sum()))
