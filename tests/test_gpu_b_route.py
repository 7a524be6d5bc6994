"""Router / top-k / statistics kernel vs the reference's recorded routing."""

import numpy as np
import pytest
import torch

from gpu_ref import order_tie_tokens, x_tensor
from inputs import routing_cases, to_bf16_bits
from oracle import moe_ref, nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _route(pkg, case, logits_in=None):
    lib = pkg.library()
    T, d, E, k = case["t"], case["d"], case["e"], case["k"]
    x = x_tensor(case, DEV)
    wr = torch.from_numpy(case["wr"]).to(DEV)
    bias = None if case["logit_bias"] is None else torch.from_numpy(case["logit_bias"]).to(DEV)
    valid = None if case["valid"] is None else torch.from_numpy(case["valid"]).to(DEV)
    lg_in = None if logits_in is None else torch.from_numpy(logits_in).to(DEV).contiguous()
    topk_idx = torch.empty((T, k), dtype=torch.int32, device=DEV)
    topk_w = torch.empty((T, k), dtype=torch.float32, device=DEV)
    logits = torch.empty((T, E), dtype=torch.float32, device=DEV)
    sel = torch.empty((T, E), dtype=torch.float32, device=DEV)
    counts = torch.empty((E,), dtype=torch.int32, device=DEV)
    stats = torch.empty((3 + E,), dtype=torch.float32, device=DEV)
    ws_bytes = lib.mcl4moe_route_workspace_size(T, E, k, d)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=DEV)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    st = lib.mcl4moe_route(x.data_ptr(), wr.data_ptr(), p(bias), p(lg_in), p(valid), T, d, E, k,
                           int(case["norm_topk_prob"]), topk_idx.data_ptr(), topk_w.data_ptr(), logits.data_ptr(),
                           sel.data_ptr(), counts.data_ptr(), stats.data_ptr(), ws.data_ptr(), ws_bytes,
                           torch.cuda.current_stream().cuda_stream)
    pkg._lib.check(st, "route")
    torch.cuda.synchronize()
    return {n: t.cpu().numpy() for n, t in dict(topk_idx=topk_idx, topk_w=topk_w, logits=logits, sel=sel,
                                                 counts=counts, stats=stats).items()}


def _active(case):
    return np.arange(case["t"]) if case["valid"] is None else np.nonzero(case["valid"])[0]


@pytest.mark.parametrize("case", routing_cases(), ids=lambda c: c[0])
def test_topk_and_stats_exact_given_reference_logits(moe_pkg, golden, case):
    name, c = case
    g = golden("routing")
    act = _active(c)
    full = np.zeros((c["t"], c["e"]), np.float32)
    full[act] = g[f"{name}__logits"]
    r = _route(moe_pkg, c, logits_in=full)
    np.testing.assert_array_equal(r["topk_idx"][act], g[f"{name}__topk_indices"])
    np.testing.assert_array_equal(r["sel"].astype(np.uint8), g[f"{name}__sel_mask"])
    np.testing.assert_array_equal(r["stats"][3:], g[f"{name}__counts"])
    np.testing.assert_allclose(r["stats"][0], g[f"{name}__aux"], rtol=1e-5)
    np.testing.assert_allclose(r["stats"][1], g[f"{name}__z"], rtol=1e-5)
    vals = g[f"{name}__topk_values"]
    ref_w = vals / np.maximum(vals.sum(-1, keepdims=True), 1e-9) if c["norm_topk_prob"] else vals
    np.testing.assert_allclose(r["topk_w"][act], ref_w, rtol=2e-6, atol=1e-7)
    if c["valid"] is not None:
        inactive = np.nonzero(c["valid"] == 0)[0]
        assert np.all(r["topk_idx"][inactive] == -1) and np.all(r["topk_w"][inactive] == 0)
    assert r["counts"].sum() == len(act) * c["k"]


@pytest.mark.parametrize("case", routing_cases(), ids=lambda c: c[0])
def test_router_product_and_selection_vs_reference(moe_pkg, golden, case):
    name, c = case
    g = golden("routing")
    act = _active(c)
    r = _route(moe_pkg, c)
    ref_logits = g[f"{name}__logits"]
    np.testing.assert_allclose(r["logits"][act], ref_logits, rtol=1e-5, atol=2e-6)
    tie = order_tie_tokens(ref_logits, c["k"])
    same = np.all(r["topk_idx"][act] == g[f"{name}__topk_indices"], axis=1)  # slot order included
    assert np.all(same | tie), f"{int((~same & ~tie).sum())} non-tie tokens routed differently"
    np.testing.assert_allclose(r["stats"][0], g[f"{name}__aux"], rtol=1e-4)
    np.testing.assert_allclose(r["stats"][1], g[f"{name}__z"], rtol=1e-4)


@pytest.mark.parametrize("name", ["r_e64k8", "r_zipf"])
def test_tensor_core_router_on_tiled_batch(moe_pkg, golden, name):
    """Batches above the small-batch limit take the tcgen05 router: tile a golden case to
    2048 tokens (identical rows have identical reference logits) and compare."""
    c = dict(routing_cases())[name]
    reps = 2048 // c["t"]
    big = dict(c, t=c["t"] * reps, x_bf16_bits=np.tile(c["x_bf16_bits"].reshape(c["t"], c["d"]), (reps, 1)))
    g = golden("routing")
    r = _route(moe_pkg, big)
    ref_logits = np.tile(g[f"{name}__logits"], (reps, 1))
    np.testing.assert_allclose(r["logits"], ref_logits, rtol=1e-5, atol=2e-6)
    tie = order_tie_tokens(ref_logits, c["k"])
    ref_idx = np.tile(g[f"{name}__topk_indices"], (reps, 1))
    same = np.all(r["topk_idx"] == ref_idx, axis=1)  # slot order included
    assert np.all(same | tie)


def test_small_batch_wide_rows_take_tensor_core_router(moe_pkg):
    """T <= 1024 with d above the CUDA-core GEMV's shared-memory limit (16 d bytes
    <= 200 KiB): the call must still route, through the tensor-core router."""
    T, d, E, k = 8, 12864, 16, 4
    rng = np.random.default_rng(77)
    xb = rng.standard_normal((T, d), dtype=np.float32)
    wr = (rng.standard_normal((E, d), dtype=np.float32) * 0.02).astype(np.float32)
    case = dict(t=T, d=d, e=E, k=k, norm_topk_prob=True, x_bf16_bits=to_bf16_bits(xb), wr=wr, valid=None,
                logit_bias=None)
    r = _route(moe_pkg, case)
    x = nr.bf16_bits_to_f32(case["x_bf16_bits"]).reshape(T, d)
    ref = moe_ref.route(x, wr, k)
    exact = x.astype(np.float64) @ wr.astype(np.float64).T
    # the tensor pipe's fp32 accumulation error grows with the d/16 MMA steps of the
    # reduction (6.5e-5 on logits of magnitude ~4 at d = 12864): bounded here at 1e-8 * d
    tol = 1e-8 * d
    np.testing.assert_allclose(r["logits"], exact, rtol=0, atol=tol)
    tie = order_tie_tokens(ref.logits, k, eps=2 * tol)
    assert np.all(np.all(r["topk_idx"] == ref.selected, axis=1) | tie)
