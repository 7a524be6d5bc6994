"""Expert parallelism over NCCL on 2 GPUs (skipped with fewer than 2 devices).

Each rank shards the same layer (experts split in two), runs its own tokens
through ``ExpertParallelMoE`` and compares with the full single-device layer on
the same tokens; then the expert set grows 16 -> 20 (``reshard``) and the
comparison repeats against the grown single-device layer.
"""

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port):
    sys.path[:0] = [str(ROOT), str(HERE), str(HERE / "golden")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from __graft_entry__ import load_package
        from gpu_ref import build_module
        from inputs import moe_case

        pkg = load_package()
        dev = torch.device("cuda", rank)
        c = moe_case(41, 2048, 1024, 16, 4, 512)  # same weights on every rank
        dense = build_module(pkg, c, dev)
        r = np.random.default_rng(500 + rank)
        for transport, h_back in (("peer", True), ("peer", False), ("collective", False)):
            ep = pkg.ExpertParallelMoE.from_dense(dense, transport=transport)
            if not h_back:
                ep.down_experts = None  # partial sums back
            # ranks hold different token counts; the second call is larger (the peer arena regrows)
            for T in (1536 - 512 * rank, 3072 + 256 * rank):
                x = torch.from_numpy(r.standard_normal((T, 1024)).astype(np.float32)).to(dev, torch.bfloat16)
                with torch.no_grad():
                    out, aux, z, counts = ep(x)
                    ref, raux, rz, rcounts = dense(x)
                torch.cuda.synchronize()
                a, b = out.float(), ref.float()
                rel = (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item()
                assert rel < 5e-3, (transport, rank, T, rel)
                assert (a - b).abs().max().item() < 1e-1
                assert torch.equal(counts, rcounts) and float(aux) == float(raux) and float(z) == float(rz)
                if transport == "peer" and h_back:  # the down projection ran at home: bit for bit
                    assert torch.equal(out, ref), (rank, T)
            if ep._peer is not None:
                ep._peer.close()
        # growth 16 -> 20 under expert parallelism (8 -> 10 experts per rank): experts 8 and 9
        # move from rank 1 to rank 0 with their NVFP4 bytes, 16 is a copy of expert 3 (sent by
        # rank 0), 17 a copy of expert 12 (local to rank 1), 18 and 19 are new (quantised)
        ep = pkg.ExpertParallelMoE.from_dense(dense)
        x = torch.from_numpy(r.standard_normal((1024, 1024)).astype(np.float32)).to(dev, torch.bfloat16)
        with torch.no_grad():
            ep(x)
        g = np.random.default_rng(77)
        new_up = (g.standard_normal((2, 1024, 1024)) * 0.02).astype(np.float32)
        new_dn = (g.standard_normal((2, 1024, 512)) * 0.02).astype(np.float32)
        new_wr = (g.standard_normal((2, 1024)) * 0.02).astype(np.float32)
        c20 = dict(c, e=20, wr=np.concatenate([c["wr"], c["wr"][[3, 12]], new_wr]),
                   w_up=np.concatenate([c["w_up"], c["w_up"][[3, 12]], new_up]),
                   w_dn=np.concatenate([c["w_dn"], c["w_dn"][[3, 12]], new_dn]))
        dense20 = build_module(pkg, c20, dev)
        fresh = {18 + i: dense20.experts[18 + i] for i in range(2)}
        before = dict(pkg.nvfp4.CACHE_STATS)
        stats = ep.reshard(dense20.router, list(range(16)), parents={16: 3, 17: 12}, new_experts=fresh)
        assert stats["moved_in"] == (2 if rank == 0 else 1), stats
        with torch.no_grad():
            out, aux, z, counts = ep(x)
            # only the new experts were quantised (up and down), and only where they live
            assert pkg.nvfp4.CACHE_STATS["quantized"] - before["quantized"] == (0 if rank == 0 else 4)
            ref, raux, rz, rcounts = dense20(x)
        torch.cuda.synchronize()
        a, b = out.float(), ref.float()
        assert (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item() < 5e-3
        assert torch.equal(counts, rcounts)
        # the grown layer with h back (every rank holds the 20 experts' down projections)
        ep.down_experts = dense20.experts
        with torch.no_grad():
            out, aux, z, counts = ep(x)
        torch.cuda.synchronize()
        assert torch.equal(out, ref) and torch.equal(counts, rcounts)
        if ep._peer is not None:
            ep._peer.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_expert_parallel_matches_single_device():
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
