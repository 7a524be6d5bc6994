"""The full MoE layer on B200 vs the reference's dequantised-FP4 CPU path.

2e-2 relative L2 and 1e-1 max-abs on the layer output;
routing indices, permutation and quantised bytes bit-exact.
"""

import numpy as np
import pytest
import torch

from gpu_ref import (build_module, dequant_reference_layout, near_tie_tokens, order_tie_tokens, rel_l2,
                     token_reference, x_tensor)
from inputs import layer_case, moe_case
from oracle import moe_ref, nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"
REL_L2, MAX_ABS = 2e-2, 1e-1


def _x_np(case):
    return nr.bf16_bits_to_f32(case["x_bf16_bits"]).reshape(case["t"], case["d"])


def test_layer_matches_reference_golden(moe_pkg, golden):
    name, c = layer_case()
    g = golden("layer")
    moe = build_module(moe_pkg, c, DEV)
    with torch.no_grad():
        out, aux, z, counts = moe(x_tensor(c, DEV))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    ref = nr.bf16_bits_to_f32(g[f"{name}__out_bf16"]).reshape(got.shape)
    assert rel_l2(got, ref) < REL_L2 and np.abs(got - ref).max() < MAX_ABS
    assert rel_l2(got, ref) < 5e-3  # far inside: same quantised bytes, fp32 order only
    np.testing.assert_allclose(float(aux), g[f"{name}__aux"], rtol=1e-4)
    np.testing.assert_allclose(float(z), g[f"{name}__z"], rtol=1e-4)
    np.testing.assert_array_equal(counts.cpu().numpy(), g[f"{name}__counts"])


SMALL_CONFIGS = {
    # the five benchmark configurations, token count reduced where the CPU oracle would be slow
    "c0": dict(seed=0, t=2048, d=256, e=8, k=2, f=512),
    "c1": dict(seed=1, t=256, d=1024, e=32, k=4, f=512),
    "c3_zipf": dict(seed=3, t=256, d=1536, e=32, k=8, f=512, zipf_bias=True),
    "c0_nonorm_valid": dict(seed=5, t=512, d=256, e=8, k=2, f=512, norm_topk_prob=False, valid_frac=0.7),
}


@pytest.mark.parametrize("name", list(SMALL_CONFIGS))
def test_layer_matches_oracle(moe_pkg, name):
    c = moe_case(**SMALL_CONFIGS[name])
    moe = build_module(moe_pkg, c, DEV)
    valid = None if c["valid"] is None else torch.from_numpy(c["valid"].astype(bool)).to(DEV)
    det = moe.forward_details(x_tensor(c, DEV), valid)
    torch.cuda.synchronize()
    assert moe.read_device_error() == 0
    experts = moe_ref.QuantizedExperts(c["w_up"], c["w_dn"])
    r = moe_ref.route(_x_np(c), c["wr"], c["k"], c["norm_topk_prob"], c["valid"], c["logit_bias"])
    act = r.active
    got_idx = det["topk_idx"].cpu().numpy()
    tie = order_tie_tokens(r.logits, c["k"])
    same = np.all(got_idx[act] == r.selected, axis=1)  # slot order included
    assert np.all(same | tie)
    # use the kernel's routing for the oracle layer so a near-tie flip cannot mask a GEMM error
    r.selected = got_idx[act].astype(np.int64)
    r.weights = det["topk_w"].cpu().numpy()[act]
    r.counts_int = np.bincount(r.selected.reshape(-1), minlength=c["e"])
    r.perm = np.argsort(r.selected.reshape(-1), kind="stable")
    ref, _, _, _, _ = moe_ref.moe_forward(_x_np(c), c["wr"], experts, c["k"], c["norm_topk_prob"], c["valid"],
                                          c["logit_bias"], routing=r)
    got = det["out"].float().cpu().numpy()
    assert rel_l2(got, ref) < REL_L2 and np.abs(got - ref).max() < MAX_ABS, (rel_l2(got, ref), np.abs(got - ref).max())
    assert rel_l2(got, ref) < 5e-3
    # permutation: exactly the stable argsort of the kernel's selections (flat ids t*k + j)
    flat = np.full(c["t"] * c["k"], 1 << 20, np.int64)
    for i, t in enumerate(act):
        flat[t * c["k"]:(t + 1) * c["k"]] = got_idx[t]
    ref_perm = np.argsort(flat, kind="stable")[: len(act) * c["k"]]
    np.testing.assert_array_equal(det["perm"].cpu().numpy(), ref_perm)
    np.testing.assert_array_equal(det["offs"].cpu().numpy(), np.cumsum(r.counts_int))
    if c["valid"] is not None:
        dead = np.nonzero(c["valid"] == 0)[0]
        assert np.all(got[dead] == 0)
        assert np.all(moe.last_selected_mask.cpu().numpy()[dead] == 0)


def test_swiglu_requantisation_bit_exact(moe_pkg):
    """The down GEMM's NVFP4 input equals the reference quantiser applied to the kernel's own h."""
    c = moe_case(21, 512, 1024, 16, 4, 512)
    moe = build_module(moe_pkg, c, DEV)
    moe.debug_capture_h = True
    det = moe.forward_details(x_tensor(c, DEV))
    torch.cuda.synchronize()
    pad = det["pad_start"].cpu().numpy()
    counts = np.diff(np.concatenate([[0], det["offs"].cpu().numpy()]))
    rows = np.concatenate([np.arange(pad[e], pad[e] + counts[e]) for e in range(c["e"])])
    h = det["h"].float().cpu().numpy()[rows]
    hq = det["hq"].cpu().numpy()[rows]
    F = c["f"]
    sw = det["hs"].cpu().numpy()
    mcap = det["hq"].shape[0]
    hs = nr.unswizzle_scales(sw.reshape(mcap, F // 16), mcap, F // 16)[rows]
    op, os_ = nr.quantize_activations(h)
    np.testing.assert_array_equal(hq, op)
    np.testing.assert_array_equal(hs, os_)


def test_causal_row_scaling_isolates_tokens(moe_pkg):
    """Changing later tokens leaves earlier outputs bit-identical (src/mcl4_coe/nvfp4.py causal row
    scaling; reference test tests/test_mcl4_coe.py:380-388)."""
    c = moe_case(22, 256, 256, 8, 2, 512)
    moe = build_module(moe_pkg, c, DEV)
    xa = x_tensor(c, DEV)
    xb = xa.clone()
    xb[128:] = xb[128:] * 25.0 - 10.0
    with torch.no_grad():
        oa = moe(xa)[0]
        ob = moe(xb)[0]
    torch.cuda.synchronize()
    assert torch.equal(oa[:128], ob[:128])


def test_expert_growth_between_calls(moe_pkg):
    """ExpertLifecycle contract: E grows 32 -> 40 between two calls (skewed routing)."""
    c = moe_case(3, 512, 1536, 40, 8, 512, zipf_bias=True)
    c32 = dict(c, e=32, wr=c["wr"][:32], w_up=c["w_up"][:32], w_dn=c["w_dn"][:32], logit_bias=c["logit_bias"][:32])
    moe = build_module(moe_pkg, c32, DEV)
    x = x_tensor(c, DEV)
    with torch.no_grad():
        out32 = moe(x)[0].float().cpu().numpy()
        # grow like grow_experts / in-place mitosis: new ModuleList, new router rows, num_experts
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
        before = dict(moe_pkg.nvfp4.CACHE_STATS)
        det = moe.forward_details(x)
    torch.cuda.synchronize()
    assert det["counts"].shape == (40,)
    # only the 8 new experts are quantised (up and down); the 32 kept ones bring their bytes
    assert moe_pkg.nvfp4.CACHE_STATS["quantized"] - before["quantized"] == 2 * 8
    assert moe_pkg.nvfp4.CACHE_STATS["carried"] - before["carried"] == 2 * 32
    for cc, got in ((c32, out32), (c, det["out"].float().cpu().numpy())):
        experts = moe_ref.QuantizedExperts(cc["w_up"], cc["w_dn"])
        ref, _, _, counts, _ = moe_ref.moe_forward(_x_np(cc), cc["wr"], experts, cc["k"], True, None,
                                                   cc["logit_bias"])
        assert rel_l2(got, ref) < REL_L2 and np.abs(got - ref).max() < MAX_ABS


def test_expert_prune_between_calls(moe_pkg):
    """ExpertLifecycle's prune_experts (src/mcl4_coe/ornith_rl.py:536-593; the reference's
    tests/test_mcl4_coe.py:353-365 grows 4 -> 5 and prunes back): E 40 -> 39 by removing
    expert 17 from the middle (router rows and experts of the others kept in order), then
    40 again by appending a copy of expert 3 (grow_experts' mitosis: same weights, router row
    duplicated).  Outputs and statistics follow the oracle at every step, and the surviving
    experts' NVFP4 bytes are carried over instead of re-quantised."""
    c = moe_case(31, 512, 1024, 40, 8, 512)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)

    def check(case, det):
        experts = moe_ref.QuantizedExperts(case["w_up"], case["w_dn"])
        ref, aux, z, counts, r = moe_ref.moe_forward(_x_np(case), case["wr"], experts, case["k"], True, None, None)
        got = det["out"].float().cpu().numpy()
        assert rel_l2(got, ref) < 5e-3 and np.abs(got - ref).max() < MAX_ABS
        tie = order_tie_tokens(r.logits, case["k"])
        same = np.all(det["topk_idx"].cpu().numpy() == r.selected, axis=1)
        assert np.all(same | tie)
        np.testing.assert_allclose(float(det["aux_loss"]), aux, rtol=1e-4)
        np.testing.assert_allclose(det["counts"].cpu().numpy(), counts, rtol=0, atol=2.0 / (case["t"] * case["k"]))

    with torch.no_grad():
        check(c, moe.forward_details(x))
        keep = [i for i in range(40) if i != 17]
        moe.experts = torch.nn.ModuleList([moe.experts[i] for i in keep])
        router = torch.nn.Linear(c["d"], 39, bias=False).to(DEV)
        router.weight.copy_(moe.router.weight.detach()[keep])
        moe.router = router
        moe.num_experts = 39
        before = dict(moe_pkg.nvfp4.CACHE_STATS)
        det = moe.forward_details(x)
        torch.cuda.synchronize()
        assert det["counts"].shape == (39,)
        assert moe_pkg.nvfp4.CACHE_STATS["quantized"] == before["quantized"]
        assert moe_pkg.nvfp4.CACHE_STATS["carried"] - before["carried"] == 2 * 39
        c39 = dict(c, e=39, wr=c["wr"][keep], w_up=c["w_up"][keep], w_dn=c["w_dn"][keep])
        check(c39, det)
        # grow back by mitosis of expert 3: a deep copy (new parameters, same values)
        twin = moe_pkg.SwiGLUExpert(c["d"], c["f"]).to(DEV)
        twin.load_state_dict(moe.experts[3].state_dict())
        moe.experts = torch.nn.ModuleList(list(moe.experts) + [twin])
        router = torch.nn.Linear(c["d"], 40, bias=False).to(DEV)
        router.weight.copy_(torch.cat([moe.router.weight.detach(), moe.router.weight.detach()[3:4]]))
        moe.router = router
        moe.num_experts = 40
        before = dict(moe_pkg.nvfp4.CACHE_STATS)
        det = moe.forward_details(x)
        torch.cuda.synchronize()
        assert moe_pkg.nvfp4.CACHE_STATS["quantized"] - before["quantized"] == 2
        assert moe_pkg.nvfp4.CACHE_STATS["carried"] - before["carried"] == 2 * 39
        grown = [*keep, keep[3]]
        c40 = dict(c, wr=c["wr"][grown], w_up=c["w_up"][grown], w_dn=c["w_dn"][grown])
        check(c40, det)
    assert moe.read_device_error() == 0


def test_full_size_headline_config(moe_pkg):
    """Config 2 at full size (T=32768, d=2048, E=64, k=8, F=1024): deterministic,
    a valid stable permutation, and a sample of tokens vs the dequantised-FP4 reference."""
    c = moe_case(2, 32768, 2048, 64, 8, 1024)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    det = moe.forward_details(x)
    with torch.no_grad():
        out2 = moe(x)[0]
    torch.cuda.synchronize()
    out = det["out"]
    assert moe.read_device_error() == 0
    assert torch.equal(out, out2), "forward is not deterministic"
    assert torch.isfinite(out.float()).all()
    counts = det["counts"].cpu().numpy()
    assert abs(counts.sum() - 1.0) < 1e-5
    idx = det["topk_idx"].cpu().numpy()
    perm = det["perm"].cpu().numpy().astype(np.int64)
    assert np.array_equal(np.sort(perm), np.arange(32768 * 8))
    assert np.array_equal(perm, np.argsort(idx.reshape(-1), kind="stable"))
    # sampled tokens vs the reference math on the same routing
    ref_cache = {p: moe_pkg.export_reference_cache(moe.experts, p) for p in ("up_proj", "down_proj")}
    w_up = dequant_reference_layout(ref_cache["up_proj"]["B_fwd"], ref_cache["up_proj"]["Bs_fwd"].view(torch.uint8),
                                    ref_cache["up_proj"]["Bg"])
    w_dn = dequant_reference_layout(ref_cache["down_proj"]["B_fwd"],
                                    ref_cache["down_proj"]["Bs_fwd"].view(torch.uint8), ref_cache["down_proj"]["Bg"])
    sample = np.random.default_rng(0).choice(32768, size=96, replace=False)
    ref = token_reference(x[sample], idx[sample], det["topk_w"].cpu().numpy()[sample], w_up, w_dn)
    got = out[sample].float().cpu().numpy()
    assert rel_l2(got, ref) < 5e-3 and np.abs(got - ref).max() < MAX_ABS
    # the routing of the sampled tokens agrees with the oracle's fp32 router (except near ties)
    r = moe_ref.route(_x_np(c)[sample], c["wr"], 8)
    tie = order_tie_tokens(r.logits, 8)
    same = np.all(idx[sample] == r.selected, axis=1)  # slot order included
    assert np.all(same | tie)


def test_decode_config(moe_pkg):
    """Config 4 (T=64 decode) against the per-token reference."""
    c = moe_case(4, 64, 2048, 64, 8, 1024)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    det = moe.forward_details(x)
    torch.cuda.synchronize()
    assert moe.read_device_error() == 0
    ref_cache = {p: moe_pkg.export_reference_cache(moe.experts, p) for p in ("up_proj", "down_proj")}
    w_up = dequant_reference_layout(ref_cache["up_proj"]["B_fwd"], ref_cache["up_proj"]["Bs_fwd"].view(torch.uint8),
                                    ref_cache["up_proj"]["Bg"])
    w_dn = dequant_reference_layout(ref_cache["down_proj"]["B_fwd"],
                                    ref_cache["down_proj"]["Bs_fwd"].view(torch.uint8), ref_cache["down_proj"]["Bg"])
    ref = token_reference(x, det["topk_idx"].cpu().numpy(), det["topk_w"].cpu().numpy(), w_up, w_dn)
    got = det["out"].float().cpu().numpy()
    assert rel_l2(got, ref) < 5e-3 and np.abs(got - ref).max() < MAX_ABS


def test_empty_and_fully_masked_batches(moe_pkg):
    c = moe_case(23, 32, 256, 8, 2, 512)
    moe = build_module(moe_pkg, c, DEV)
    with torch.no_grad():
        out, aux, z, counts = moe(torch.zeros((0, 256), dtype=torch.bfloat16, device=DEV))
        assert out.shape == (0, 256) and float(aux) == 0.0 and float(counts.sum()) == 0.0
        x = x_tensor(c, DEV)
        out, aux, z, counts = moe(x, valid=torch.zeros(32, dtype=torch.bool, device=DEV))
    torch.cuda.synchronize()
    assert torch.all(out == 0) and float(aux) == 0.0 and float(z) == 0.0
    assert torch.all(moe.last_selected_mask == 0)


def test_routing_variants_are_forward_only(moe_pkg):
    """Plain top-k routing trains (tests/test_gpu_k_backward.py); a routing variant under
    autograd is refused rather than run without its gradient."""
    c = moe_case(24, 16, 256, 8, 2, 512)
    moe = build_module(moe_pkg, c, DEV)
    moe.dense_subset_k = 2
    with pytest.raises(NotImplementedError):
        moe(x_tensor(c, DEV))


def test_garbage_workspace_does_not_leak_into_results(moe_pkg):
    """A recycled (non-zero) workspace must not change anything: every region the
    kernels read is written first, and the device error word is cleared per call."""
    c = moe_case(25, 64, 2048, 64, 8, 1024)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    with torch.no_grad():
        ref = moe(x)[0].clone()
        moe._ws.fill_(0xA5)
        got = moe(x)[0]
    torch.cuda.synchronize()
    assert moe.read_device_error() == 0
    assert torch.equal(ref, got)


def test_cuda_graph_replay_matches_eager(moe_pkg):
    """enable_cuda_graph: repeated same-shape calls replay a captured graph and give the
    eager outputs bit for bit, for new inputs on every call."""
    c = moe_case(51, 64, 512, 16, 4, 512)
    moe = build_module(moe_pkg, c, DEV)
    xs = [x_tensor(c, DEV) * s for s in (1.0, 0.5, 2.0)]
    with torch.no_grad():
        eager = [moe(x) for x in xs]
        moe.enable_cuda_graph()
        graphed = [moe(x) for x in xs]
        moe.enable_cuda_graph(False)
    torch.cuda.synchronize()
    for (o1, a1, z1, c1), (o2, a2, z2, c2) in zip(eager, graphed):
        assert torch.equal(o1, o2) and torch.equal(c1, c2)
        assert float(a1) == float(a2) and float(z1) == float(z2)


@pytest.mark.parametrize("shape", [(64, 2048, 64, 8, 1024, False), (200, 512, 16, 4, 256, True),
                                   (700, 512, 8, 2, 256, False)], ids=["decode_c4", "zipf_dead", "over128"])
def test_expert_tilings_agree(moe_pkg, shape):
    """Single-CTA 128-row tiles (decode: padding-only blocks skipped) and CTA-pair 256-row
    tiles give the same layer output and the same h / NVFP4 h bytes on every routed row;
    shapes with empty experts and experts of more than 128 rows included."""
    t, d, e, k, f, zipf = shape
    c = moe_case(31 + t, t, d, e, k, f, zipf_bias=zipf, dead_experts=2 if zipf else 0)
    moe = build_module(moe_pkg, c, DEV)
    moe.debug_capture_h = True
    x = x_tensor(c, DEV)
    lib = moe_pkg.library()
    res = {}
    try:
        for mode in (1, 2):
            lib.mcl4moe_set_expert_tiling(mode)
            det = moe.forward_details(x)
            torch.cuda.synchronize()
            assert moe.read_device_error() == 0
            res[mode] = {key: v.clone() for key, v in det.items() if isinstance(v, torch.Tensor)}
    finally:
        lib.mcl4moe_set_expert_tiling(0)
    a, b = res[1], res[2]
    assert torch.equal(a["out"], b["out"])
    pad = a["pad_start"].cpu().numpy()
    counts = np.diff(np.concatenate([[0], a["offs"].cpu().numpy()]))
    rows = torch.from_numpy(np.concatenate([np.arange(pad[i], pad[i] + counts[i]) for i in range(e)])).to(DEV)
    for key in ("h", "hq"):
        assert torch.equal(a[key][rows], b[key][rows]), key
    if t * k > e * 128:  # some expert exceeds one 128-row block
        assert counts.max() > 128
