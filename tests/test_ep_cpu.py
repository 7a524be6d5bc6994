"""Expert parallelism over a world-size-2 gloo group on CPU.

``ExpertParallelMoE`` (count exchange, split sizes, row dispatch, partial
return, per-token combine) runs unchanged; the device steps are the oracle
restatement in ``ep_oracle_ops``.  Each rank's output must match the
single-device oracle layer on the same tokens (the only difference is the bf16
rounding of the per-rank partial sums), and the routing statistics must be
identical.
"""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dense_layer(pkg, d, E, k, F, seed, norm):
    torch.manual_seed(seed)
    moe = pkg.SparseMoE(pkg.MoEConfig(d_model=d, expert_hidden_dim=F, num_experts=E, top_k=k,
                                      norm_topk_prob=norm))
    r = np.random.default_rng(seed)
    with torch.no_grad():
        moe.router.weight.copy_(torch.from_numpy((r.standard_normal((E, d)) * 0.02).astype(np.float32)))
        for ex in moe.experts:
            ex.up_proj.weight.copy_(torch.from_numpy((r.standard_normal((2 * F, d)) * 0.02).astype(np.float32)))
            ex.down_proj.weight.copy_(torch.from_numpy((r.standard_normal((d, F)) * 0.02).astype(np.float32)))
    return moe


def _worker(rank, world, port, case):
    sys.path[:0] = [str(ROOT), str(HERE)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from __graft_entry__ import load_package
        from ep_oracle_ops import OracleEPOps
        from oracle import moe_ref
        from oracle import nvfp4_ref as nr

        pkg = load_package()
        d, E, k, F, T = case["d"], case["e"], case["k"], case["f"], case["t"]
        dense = _dense_layer(pkg, d, E, k, F, 7, case["norm"])
        bias = None
        if case["zipf"]:
            bias = torch.from_numpy((2.0 * np.log(1.0 / np.arange(1, E + 1))).astype(np.float32))
            dense.router_logit_bias = bias
        ep = pkg.ExpertParallelMoE.from_dense(dense, ops=OracleEPOps(), chunks=case["chunks"])
        ep.min_chunk_tokens = 8  # several chunks even for these small batches
        assert ep.experts_per_rank == E // world and ep.expert_offset == rank * (E // world)

        r = np.random.default_rng(100 + rank)
        x = torch.from_numpy(r.standard_normal((T, d)).astype(np.float32)).to(torch.bfloat16)
        valid = None
        if case["valid"]:
            valid = torch.from_numpy((r.random(T) < 0.8).astype(np.uint8))
        out, aux, z, counts = ep(x, valid)

        w_up = np.stack([e.up_proj.weight.detach().numpy() for e in dense.experts])
        w_dn = np.stack([e.down_proj.weight.detach().numpy() for e in dense.experts])
        ref_out, ref_aux, ref_z, ref_counts, _ = moe_ref.moe_forward(
            x.float().numpy(), dense.router.weight.detach().numpy(), moe_ref.QuantizedExperts(w_up, w_dn), k,
            case["norm"], None if valid is None else valid.numpy(), None if bias is None else bias.numpy())
        got = out.float().numpy()
        err = np.linalg.norm(got - ref_out) / max(np.linalg.norm(ref_out), 1e-30)
        assert err < 5e-3, f"rank {rank}: relative L2 error {err}"
        assert np.abs(got - ref_out).max() < 1e-1
        if valid is not None:
            assert np.all(got[valid.numpy() == 0] == 0)
        assert float(aux) == float(ref_aux) and float(z) == float(ref_z)
        np.testing.assert_array_equal(counts.numpy(), ref_counts)
        ex = ep.last_exchange
        assert len(ex["rows_to"]) == world and len(ex["rows_from"]) == world
        # rows bound for each rank: tokens with at least one expert there
        sel = ep.ops.routing.selected
        for g in range(world):
            n = int(np.sum(np.any(sel // (E // world) == g, axis=1)))
            assert ex["rows_to"][g] == n, (g, ex["rows_to"][g], n)
    finally:
        dist.destroy_process_group()


CASES = [
    dict(name="uniform_k2", t=40, d=256, e=8, k=2, f=256, norm=True, zipf=False, valid=False, chunks=1),
    dict(name="zipf_valid_k3_chunked", t=48, d=256, e=8, k=3, f=256, norm=False, zipf=True, valid=True, chunks=3),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_expert_parallel_matches_single_device_oracle(case):
    mp.spawn(_worker, args=(2, _free_port(), case), nprocs=2, join=True)


def _reshard_worker(rank, world, port):
    """Grow 4 -> 6 experts (one mitosis copy of expert 1, one new expert) and prune back to
    4 (experts 1 and 4 removed) under expert parallelism; after each step every rank's
    output must equal the single-device oracle layer over the full expert set."""
    sys.path[:0] = [str(ROOT), str(HERE)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from __graft_entry__ import load_package
        from ep_oracle_ops import OracleEPOps
        from oracle import moe_ref

        pkg = load_package()
        d, E, k, F, T = 256, 4, 2, 256, 32
        dense = _dense_layer(pkg, d, E, k, F, 9, True)
        ep = pkg.ExpertParallelMoE.from_dense(dense, ops=OracleEPOps())
        r = np.random.default_rng(300 + rank)
        x = torch.from_numpy(r.standard_normal((T, d)).astype(np.float32)).to(torch.bfloat16)

        def check(router_w, w_up, w_dn):
            out, aux, z, counts = ep(x)
            ref, raux, rz, rcounts, _ = moe_ref.moe_forward(x.float().numpy(), router_w, moe_ref.QuantizedExperts(
                w_up, w_dn), k, True)
            got = out.float().numpy()
            err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
            assert err < 5e-3 and np.abs(got - ref).max() < 1e-1, (rank, err)
            np.testing.assert_array_equal(counts.numpy(), rcounts)

        w_up = np.stack([e.up_proj.weight.detach().numpy() for e in dense.experts])
        w_dn = np.stack([e.down_proj.weight.detach().numpy() for e in dense.experts])
        wr = dense.router.weight.detach().numpy()
        check(wr, w_up, w_dn)
        # grow: expert 4 is a copy of expert 1 (router row duplicated), expert 5 is new
        g = np.random.default_rng(11)  # identical on both ranks
        fresh = pkg.SwiGLUExpert(d, F).requires_grad_(False)
        fresh.up_proj.weight.copy_(torch.from_numpy((g.standard_normal((2 * F, d)) * 0.02).astype(np.float32)))
        fresh.down_proj.weight.copy_(torch.from_numpy((g.standard_normal((d, F)) * 0.02).astype(np.float32)))
        wr6 = np.concatenate([wr, wr[1:2], (g.standard_normal((1, d)) * 0.02).astype(np.float32)])
        router6 = torch.nn.Linear(d, 6, bias=False).requires_grad_(False)
        router6.weight.copy_(torch.from_numpy(wr6))
        stats = ep.reshard(router6, [0, 1, 2, 3], parents={4: 1}, new_experts={5: fresh})
        # 2 ranks: old blocks {0,1} {2,3} -> new {0,1,2} {3,4,5}: expert 2 moves 1 -> 0, the copy of 1 moves 0 -> 1
        assert ep.num_experts == 6 and ep.experts_per_rank == 3 and len(ep.experts) == 3
        assert stats["moved_in"] == 1 and stats["new"] == (1 if rank == 1 else 0)
        w_up6 = np.concatenate([w_up, w_up[1:2], fresh.up_proj.weight.detach().numpy()[None]])
        w_dn6 = np.concatenate([w_dn, w_dn[1:2], fresh.down_proj.weight.detach().numpy()[None]])
        check(wr6, w_up6, w_dn6)
        # prune experts 1 and 4: the others keep their order
        keep = [0, 2, 3, 5]
        router4 = torch.nn.Linear(d, 4, bias=False).requires_grad_(False)
        router4.weight.copy_(torch.from_numpy(wr6[keep]))
        ep.reshard(router4, [0, None, 1, 2, None, 3])
        assert ep.num_experts == 4 and len(ep.experts) == 2
        check(wr6[keep], w_up6[keep], w_dn6[keep])
        with pytest.raises(ValueError):
            ep.reshard(router4, [0, 1, 2])  # wrong length: rejected before any exchange
    finally:
        dist.destroy_process_group()


def test_expert_parallel_reshard_grow_and_prune():
    mp.spawn(_reshard_worker, args=(2, _free_port()), nprocs=2, join=True)
