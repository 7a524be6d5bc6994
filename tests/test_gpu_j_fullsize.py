"""The benchmarked configurations at FULL size on B200, against the oracle.

For c1 (T=16384), c2 (the headline, T=32768) and c3 (T=65536, Zipf-skewed
router, experts growing 32 -> 40 between two calls), through the same
``forward_details`` path the bench times:

* routing: every token's top-k expert ids compared slot by slot (order
  included) with the oracle's fp32 router; the only tokens allowed to differ
  are order ties (two of the k+1 largest logits within 1e-5), and their
  number is printed;
* NVFP4 activation bytes: for every routed slot, the packed codes and the
  E4M3 scales the fused permute kernel wrote into the first GEMM's operand
  equal the reference quantiser's bytes of that token's row, and every
  padding row's scales are zero;
* SwiGLU re-quantisation: a sample of h rows re-quantised by the oracle gives
  the bytes the gate/up epilogue wrote (c2);
* layer output: 4096 tokens (c3: 2048 per call) against the dequantised-FP4
  reference on the kernel's routing, rel-L2 < 5e-3 and max-abs < 1e-1 (the
  north-star tolerance is 2e-2 / 1e-1);
* permutation and offsets: exactly the stable argsort of the selections.
"""

import numpy as np
import pytest
import torch

from gpu_ref import build_module, compare_routing_in_order, dequant_reference_layout, rel_l2, token_reference, x_tensor
from inputs import moe_case
from oracle import moe_ref, nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"
REL_L2, MAX_ABS = 2e-2, 1e-1


def _x_np(case):
    return nr.bf16_bits_to_f32(case["x_bf16_bits"]).reshape(case["t"], case["d"])


def _dequant_weights(pkg, moe):
    ref = {p: pkg.export_reference_cache(moe.experts, p) for p in ("up_proj", "down_proj")}
    return tuple(dequant_reference_layout(ref[p]["B_fwd"], ref[p]["Bs_fwd"].view(torch.uint8), ref[p]["Bg"])
                 for p in ("up_proj", "down_proj"))


def _check_routing(det, case, label):
    r = moe_ref.route(_x_np(case), case["wr"], case["k"], case["norm_topk_prob"], None, case["logit_bias"])
    got_idx = det["topk_idx"].cpu().numpy()
    rep = compare_routing_in_order(got_idx, r.selected, r.logits, case["k"])
    print(f"\n[{label}] routing in slot order: {rep}")
    assert rep["mismatched_outside_ties"] == 0, rep
    ok = np.all(got_idx == r.selected, axis=1)
    np.testing.assert_allclose(det["topk_w"].cpu().numpy()[ok], r.weights[ok], rtol=2e-5, atol=1e-7)
    return got_idx


def _check_permutation(det, got_idx, E):
    perm = det["perm"].cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(perm, np.argsort(got_idx.reshape(-1), kind="stable"))
    np.testing.assert_array_equal(det["offs"].cpu().numpy(),
                                  np.cumsum(np.bincount(got_idx.reshape(-1), minlength=E)))


def _check_activation_bytes(det, case, label):
    """Every routed slot row of the first GEMM's operand against the reference quantiser."""
    T, k, d, E = case["t"], case["k"], case["d"], case["e"]
    ref_q, ref_s = nr.quantize_activations(_x_np(case))
    slot = det["slot_pos"].cpu().numpy().astype(np.int64)
    assert np.all(slot >= 0)
    xq = det["xq"].cpu().numpy()
    xs = det["xs"].cpu().numpy()
    for j in range(k):  # one slot column at a time keeps host memory at one [T, d/2] copy
        np.testing.assert_array_equal(xq[slot[:, j]], ref_q, err_msg=f"{label}: codes of slot {j}")
        np.testing.assert_array_equal(xs[slot[:, j]], ref_s, err_msg=f"{label}: scales of slot {j}")
    pad = det["pad_start"].cpu().numpy().astype(np.int64)
    counts = np.bincount(det["topk_idx"].cpu().numpy().reshape(-1), minlength=E)
    pad_rows = np.concatenate([np.arange(pad[e] + counts[e], pad[e + 1]) for e in range(E)])
    assert np.all(xs[pad_rows] == 0), f"{label}: padding rows carry nonzero scales"
    used = np.zeros(xq.shape[0], bool)
    used[slot.reshape(-1)] = True
    assert used.sum() == T * k and not np.any(used[pad_rows])
    print(f"[{label}] NVFP4 activation bytes: {T * k} slot rows ({T} tokens x {k}) bit-exact, "
          f"{pad_rows.size} padding rows with zero scales")


def _check_output(pkg, moe, det, x, n_sample, seed, label):
    w_up, w_dn = _dequant_weights(pkg, moe)
    T = x.shape[0]
    sample = np.sort(np.random.default_rng(seed).choice(T, size=min(n_sample, T), replace=False))
    idx = det["topk_idx"].cpu().numpy()[sample]
    ref = token_reference(x[sample], idx, det["topk_w"].cpu().numpy()[sample], w_up, w_dn)
    got = det["out"][sample].float().cpu().numpy()
    err, mx = rel_l2(got, ref), float(np.abs(got - ref).max())
    print(f"[{label}] output on {sample.size} tokens: rel-L2 {err:.2e}, max-abs {mx:.2e}")
    assert err < REL_L2 and mx < MAX_ABS
    assert err < 5e-3


@pytest.mark.parametrize("name,cfg", [("c1", dict(seed=1, t=16384, d=1024, e=32, k=4, f=512)),
                                      ("c2", dict(seed=2, t=32768, d=2048, e=64, k=8, f=1024))])
def test_full_size_config(moe_pkg, name, cfg):
    c = moe_case(**cfg)
    moe = build_module(moe_pkg, c, DEV)
    moe.debug_capture_h = name == "c2"
    x = x_tensor(c, DEV)
    det = moe.forward_details(x, quant_bytes=True)
    torch.cuda.synchronize()
    assert moe.read_device_error() == 0
    got_idx = _check_routing(det, c, name)
    _check_permutation(det, got_idx, c["e"])
    _check_activation_bytes(det, c, name)
    if name == "c2":
        # the gate/up epilogue's NVFP4 bytes of h against the reference quantiser, on a row sample
        pad = det["pad_start"].cpu().numpy()
        counts = np.bincount(got_idx.reshape(-1), minlength=c["e"])
        rows = np.concatenate([np.arange(pad[e], pad[e] + counts[e]) for e in range(c["e"])])
        rows = np.sort(np.random.default_rng(7).choice(rows, size=16384, replace=False))
        h = det["h"][torch.from_numpy(rows).to(DEV)].float().cpu().numpy()
        op, os_ = nr.quantize_activations(h)
        mcap, F = det["hq"].shape[0], c["f"]
        np.testing.assert_array_equal(det["hq"].cpu().numpy()[rows], op)
        hs = nr.unswizzle_scales(det["hs"].cpu().numpy().reshape(mcap, F // 16), mcap, F // 16)[rows]
        np.testing.assert_array_equal(hs, os_)
    moe.debug_capture_h = False
    _check_output(moe_pkg, moe, det, x, 4096, 11, name)
    with torch.no_grad():
        again = moe(x)[0]
    torch.cuda.synchronize()
    assert torch.equal(again, det["out"]), "forward is not deterministic"


def test_full_size_skewed_growth_32_to_40(moe_pkg):
    """c3 at full size: T=65536, d=1536, k=8, F=512, router logits + 2 log(1/rank),
    E = 32 on the first call and 40 on the second (experts appended, router rows
    appended, ``num_experts`` updated, as ExpertLifecycle does)."""
    c = moe_case(3, 65536, 1536, 40, 8, 512, zipf_bias=True)
    c32 = dict(c, e=32, wr=c["wr"][:32], w_up=c["w_up"][:32], w_dn=c["w_dn"][:32], logit_bias=c["logit_bias"][:32])
    moe = build_module(moe_pkg, c32, DEV)
    x = x_tensor(c, DEV)
    det = moe.forward_details(x, quant_bytes=True)
    torch.cuda.synchronize()
    assert moe.read_device_error() == 0
    got_idx = _check_routing(det, c32, "c3 E=32")
    _check_permutation(det, got_idx, 32)
    _check_activation_bytes(det, c32, "c3 E=32")
    _check_output(moe_pkg, moe, det, x, 2048, 12, "c3 E=32")
    counts32 = np.bincount(got_idx.reshape(-1), minlength=32)
    print(f"[c3 E=32] rows per expert: max {counts32.max()}, min {counts32.min()} (Zipf skew)")
    with torch.no_grad():
        new = [moe_pkg.SwiGLUExpert(c["d"], c["f"]).to(DEV) for _ in range(8)]
        for i, ex in enumerate(new):
            ex.up_proj.weight.copy_(torch.from_numpy(c["w_up"][32 + i]))
            ex.down_proj.weight.copy_(torch.from_numpy(c["w_dn"][32 + i]))
        moe.experts = torch.nn.ModuleList(list(moe.experts) + new)
        router = torch.nn.Linear(c["d"], 40, bias=False).to(DEV)
        router.weight.copy_(torch.from_numpy(c["wr"]))
        moe.router = router
        moe.num_experts = 40
        moe.router_logit_bias = torch.from_numpy(c["logit_bias"]).to(DEV)
    del det
    det = moe.forward_details(x, quant_bytes=True)
    torch.cuda.synchronize()
    assert moe.read_device_error() == 0
    assert det["counts"].shape == (40,)
    got_idx = _check_routing(det, c, "c3 E=40")
    _check_permutation(det, got_idx, 40)
    _check_activation_bytes(det, c, "c3 E=40")
    _check_output(moe_pkg, moe, det, x, 2048, 13, "c3 E=40")
