"""Host-side behaviour of the drop-in module that needs no GPU."""

import pytest
import torch


def _cfg(pkg, **kw):
    base = dict(d_model=256, expert_hidden_dim=256, num_experts=4, top_k=2)
    base.update(kw)
    return pkg.MoEConfig(**base)


def test_parameter_names_match_the_reference_module(moe_pkg):
    # src/mcl4_coe/backbone.py:182-183, :216-220
    moe = moe_pkg.SparseMoE(_cfg(moe_pkg))
    keys = set(moe.state_dict().keys())
    expected = {"router.weight"}
    for i in range(4):
        expected |= {f"experts.{i}.up_proj.weight", f"experts.{i}.down_proj.weight"}
    assert keys == expected
    assert moe.experts[0].up_proj.weight.shape == (512, 256)  # [2F, d], gate rows first
    assert moe.experts[0].down_proj.weight.shape == (256, 256)
    assert moe.router.weight.shape == (4, 256)


def test_config_validation_mirrors_reference():
    from __graft_entry__ import load_package

    pkg = load_package()
    with pytest.raises(ValueError):
        pkg.MoEConfig(num_experts=2, top_k=3)
    with pytest.raises(ValueError):
        pkg.MoEConfig(d_model=0)


def test_no_cpu_fallback(moe_pkg):
    moe = moe_pkg.SparseMoE(_cfg(moe_pkg))
    with torch.no_grad(), pytest.raises(ValueError, match="CUDA"):
        moe(torch.zeros(2, 3, 256))


def test_cache_rejects_cpu_weights(moe_pkg):
    moe = moe_pkg.SparseMoE(_cfg(moe_pkg))
    with pytest.raises(ValueError, match="CUDA"):
        moe_pkg.get_or_build_grouped_cache(moe.experts, "up_proj")


def test_mitotic_pairs_round_trip_through_state_dict(moe_pkg):
    # src/mcl4_coe/backbone.py:579-616
    a = moe_pkg.SparseMoE(_cfg(moe_pkg))
    a.mitotic_pairs = [(0, 3), (1, 2)]
    sd = a.state_dict()
    assert "mitotic_pairs_tensor" in sd
    b = moe_pkg.SparseMoE(_cfg(moe_pkg))
    b.load_state_dict(sd)
    assert b.mitotic_pairs == [(0, 3), (1, 2)]


def test_routing_variant_detection(moe_pkg):
    """Plain top-k takes the one-call path; every reference variant takes the routed path."""
    moe = moe_pkg.SparseMoE(_cfg(moe_pkg))
    assert moe._routing_variant(None, None, None) is None
    prior = torch.zeros(2, moe.num_experts)
    assert moe._routing_variant(prior, None, None) is None  # no penalty configured
    moe.recurrent_coverage_penalty = 0.5
    assert moe._routing_variant(prior, None, None) == "sparse"
    moe.recurrent_coverage_penalty = 0.0
    moe.mitotic_pairs = [(0, 1)]
    assert moe._routing_variant(None, None, None) == "sparse"
    moe.mitotic_pairs = []
    assert moe._routing_variant(None, [0, 1], None) == "dense"
    assert moe._routing_variant(None, None, 2) == "dense"
    moe.sequence_diversity_coef = 0.1
    assert moe._routing_variant(None, None, None) == "sparse"


def test_expert_parallel_chunk_bounds(moe_pkg):
    """Token chunks of the expert-parallel exchange: weighted cuts, equal chunks,
    one chunk for short batches, and every token in exactly one chunk."""
    from types import SimpleNamespace

    cut = moe_pkg.ExpertParallelMoE._chunk_bounds

    def bounds(T, chunks=1, weights=None, min_tokens=1024):
        return cut(SimpleNamespace(chunks=chunks, chunk_weights=weights, min_chunk_tokens=min_tokens), T)

    assert bounds(32768, 2, [0.6, 0.4]) == [(0, 19661), (19661, 32768)]
    assert bounds(32768, 4) == [(0, 8192), (8192, 16384), (16384, 24576), (24576, 32768)]
    assert bounds(1500, 2, [0.6, 0.4]) == [(0, 1500)]
    assert bounds(0, 2) == [(0, 0)]
    assert bounds(3000, 4) == [(0, 1500), (1500, 3000)]
    for T in (1, 2047, 2048, 9999, 65536):
        for ch, wts in ((1, None), (3, None), (2, [0.6, 0.4]), (3, [0.5, 0.3, 0.2])):
            b = bounds(T, ch, wts)
            assert b[0][0] == 0 and b[-1][1] == T
            assert all(lo < hi for lo, hi in b) and all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))


def test_convert_linear_to_nvfp4(moe_pkg):
    """src/mcl4_coe/nvfp4.py:598-695: expert projections only when SwiGLUExpert blocks
    exist; otherwise eligible Linears outside the excluded names."""
    from torch import nn

    moe = moe_pkg.SparseMoE(_cfg(moe_pkg))
    n = moe_pkg.convert_linear_to_nvfp4(moe, sparsity_mode="none")
    assert n == 2 * moe.num_experts
    assert all(isinstance(e.up_proj, moe_pkg.NVFP4Linear) and isinstance(e.down_proj, moe_pkg.NVFP4Linear)
               for e in moe.experts)
    assert type(moe.router) is nn.Linear
    assert moe.experts[0].up_proj.sparsity_mode == "none" and moe.experts[0].up_proj.bias is None
    assert moe_pkg.convert_linear_to_nvfp4(moe) == 0  # nothing left to convert

    tree = nn.Sequential(nn.Linear(64, 64), nn.ReLU(), nn.Linear(64, 16))
    tree.add_module("router_head", nn.Linear(64, 64))
    assert moe_pkg.convert_linear_to_nvfp4(tree) == 1
    assert isinstance(tree[0], moe_pkg.NVFP4Linear) and type(tree[2]) is nn.Linear
    assert type(tree.router_head) is nn.Linear
    assert tree[0].sparsity_mode == "2to4_transposable"
    with pytest.raises(ValueError):
        moe_pkg.NVFP4Linear(64, 64, sparsity_mode="dense")


def test_peer_exchange_plans_route_every_row(moe_pkg):
    """Simulate every rank's row copies and partial-sum copies (row_plan / back_plan) on
    random counts: each receiver's region holds its senders' rows in rank order, and each
    sender gets every partial back at the row it sent it from."""
    import random

    ep = moe_pkg.expert_parallel
    rnd = random.Random(3)
    for G in (1, 2, 3, 8):
        for n_chunks in (1, 2):
            tab = [[[rnd.randint(0, 5) for _ in range(G)] + [0] * G + [0] for _ in range(n_chunks)]
                   for _ in range(G)]
            for c in range(n_chunks):
                # sender s's send buffer: rows grouped by destination, labelled (s, g, i)
                send = {s: [(s, g, i) for g in range(G) for i in range(tab[s][c][g])] for s in range(G)}
                recv = {g: [None] * sum(tab[s][c][g] for s in range(G)) for g in range(G)}
                for s in range(G):
                    for g, src, n, dst in ep.row_plan(tab, c, s):
                        recv[g][dst:dst + n] = send[s][src:src + n]
                for g in range(G):
                    assert recv[g] == [(s, g, i) for s in range(G) for i in range(tab[s][c][g])]
                # the receiver's partial row j answers its received row j
                back = {s: [None] * len(send[s]) for s in range(G)}
                for g in range(G):
                    for s, src, n, dst in ep.back_plan(tab, c, g):
                        back[s][dst:dst + n] = recv[g][src:src + n]
                for s in range(G):
                    assert back[s] == send[s]


def test_expert_parallel_refuses_routing_variants(moe_pkg):
    """Sharding a layer whose routing is not plain top-k must not silently drop the variant."""
    import os
    import socket

    import torch.distributed as dist

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        moe = moe_pkg.SparseMoE(_cfg(moe_pkg))
        moe_pkg.ExpertParallelMoE.from_dense(moe)  # plain top-k: fine
        moe.mitotic_pairs = [(0, 1)]
        with pytest.raises(NotImplementedError, match="mitotic"):
            moe_pkg.ExpertParallelMoE.from_dense(moe)
        moe.mitotic_pairs = []
        moe.dense_subset_k = 2
        with pytest.raises(NotImplementedError, match="dense"):
            moe_pkg.ExpertParallelMoE.from_dense(moe)
    finally:
        dist.destroy_process_group()


def test_weight_cache_owner_check_sees_every_change(moe_pkg):
    """The per-forward check of the grouped NVFP4 cache (owner snapshot instead of one
    nn.Module attribute walk per expert) must still see each change that makes a slot
    stale, as the reference's per-expert version keys do (src/mcl4_coe/nvfp4.py:962-1048):
    an in-place update, a replaced Parameter, a swapped .data, a changed sparsity mode,
    a replaced projection, growth, and an added bias."""
    import sys

    nv = sys.modules[moe_pkg.__name__ + ".nvfp4"]
    moe = moe_pkg.SparseMoE(_cfg(moe_pkg))
    experts = moe.experts
    entry = nv.GroupedNVFP4Cache(len(experts), 2 * moe.experts[0].down_proj.weight.shape[1],
                                 moe.experts[0].down_proj.weight.shape[0], torch.device("cpu"))

    def remember():
        layers = [e.up_proj for e in experts]
        entry.remember_owners(experts, "up_proj", layers, [lay.weight for lay in layers])
        assert entry.still_current(experts, "up_proj")
        assert not entry.still_current(experts, "down_proj")

    remember()
    with torch.no_grad():
        experts[1].up_proj.weight.mul_(2.0)
    assert not entry.still_current(experts, "up_proj")
    remember()
    experts[0].up_proj.weight = torch.nn.Parameter(experts[0].up_proj.weight.detach().clone())
    assert not entry.still_current(experts, "up_proj")
    remember()
    experts[2].up_proj.weight.data = experts[2].up_proj.weight.detach().clone()
    assert not entry.still_current(experts, "up_proj")
    remember()
    experts[3].up_proj.sparsity_mode = "2to4_row"
    assert not entry.still_current(experts, "up_proj")
    del experts[3].up_proj.sparsity_mode
    remember()
    old = experts[1].up_proj
    experts[1].up_proj = torch.nn.Linear(old.in_features, old.out_features, bias=False)
    assert not entry.still_current(experts, "up_proj")
    remember()
    experts.append(type(experts[0])(experts[0].up_proj.in_features, experts[0].down_proj.in_features))
    assert not entry.still_current(experts, "up_proj")
    del experts[len(experts) - 1]
    assert entry.still_current(experts, "up_proj")
    experts[0].up_proj.bias = torch.nn.Parameter(torch.zeros(experts[0].up_proj.out_features))
    assert not entry.still_current(experts, "up_proj")
