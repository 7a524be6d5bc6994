"""Expert-parallel kernels on one GPU: G ranks emulated with a single source.

With one source rank, what destination g receives is exactly the slice of the
send buffer addressed to g, so dispatch -> per-rank experts -> combine can run
in one process without a collective.  The output must match the single-GPU
layer (up to the bf16 rounding of per-rank partial sums), the dispatched rows
must carry the reference quantiser's bytes, and routing is shared bit for bit.
"""

import numpy as np
import pytest
import torch

from gpu_ref import build_module, x_tensor
from inputs import moe_case
from oracle import nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _emulate(pkg, moe, x, G, valid=None):
    ops = pkg.CudaEPOps()
    T, d = x.shape
    E, k = len(moe.experts), moe.top_k
    E_loc = E // G
    wr = moe.router.weight.detach().float().contiguous()
    idx, w, stats = ops.route(x, wr, None, valid, k, moe.norm_topk_prob)
    send, counts, pos = ops.dispatch(x, idx, w, valid, G, E_loc)
    c = counts.cpu().tolist()
    rows, slots = c[:G], c[G:]
    parts, start = [], 0
    for g in range(G):
        recv = send[start:start + rows[g]]
        parts.append(ops.experts(recv, rows[g], slots[g], d, k, moe.experts[g * E_loc:(g + 1) * E_loc]))
        start += rows[g]
    back = torch.cat(parts, dim=0)
    out = ops.combine(back, pos, T, d, G)
    torch.cuda.synchronize()
    return out, dict(idx=idx, w=w, send=send, rows=rows, slots=slots, pos=pos, stats=stats)


@pytest.mark.parametrize("G", [2, 4, 8])
def test_emulated_ranks_match_single_gpu_layer(moe_pkg, G):
    c = moe_case(31, 1024, 512, 16, 4, 512)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    with torch.no_grad():
        ref = moe.forward_details(x)
    out, info = _emulate(moe_pkg, moe, x, G)
    np.testing.assert_array_equal(info["idx"].cpu().numpy(), ref["topk_idx"].cpu().numpy())
    a, b = out.float(), ref["out"].float()
    rel = (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item()
    assert rel < 5e-3, rel
    assert (a - b).abs().max().item() < 1e-1
    # every (token, destination) row exists exactly when the token has an expert there
    idx = info["idx"].cpu().numpy()
    has = np.stack([np.any(idx // (16 // G) == g, axis=1) for g in range(G)], axis=1)
    pos = info["pos"].cpu().numpy()
    assert np.array_equal(pos >= 0, has)
    assert info["rows"] == has.sum(axis=0).tolist()
    assert sum(info["slots"]) == idx.size


def test_dispatched_rows_carry_reference_quantiser_bytes(moe_pkg):
    c = moe_case(32, 256, 512, 8, 2, 512)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    G, d, k = 2, 512, 2
    _, info = _emulate(moe_pkg, moe, x, G)
    packed, scales = nr.quantize_activations(x.float().cpu().numpy())
    send = info["send"].cpu().numpy()
    pos = info["pos"].cpu().numpy()
    idx = info["idx"].cpu().numpy()
    w = info["w"].cpu().numpy()
    for t in range(x.shape[0]):
        for g in range(G):
            p = pos[t, g]
            if p < 0:
                continue
            row = send[p]
            np.testing.assert_array_equal(row[:d // 2], packed[t])
            np.testing.assert_array_equal(row[d // 2:d // 2 + d // 16], scales[t])
            ids = row[d // 2 + d // 16:d // 2 + d // 16 + k].view(np.int8)
            want = np.where(idx[t] // (8 // G) == g, idx[t] - g * (8 // G), -1)
            np.testing.assert_array_equal(ids, want)
            wts = row[d // 2 + d // 16 + 16:d // 2 + d // 16 + 16 + 4 * k].view(np.float32)
            np.testing.assert_array_equal(wts, w[t])


def test_masked_tokens_and_a_rank_without_rows(moe_pkg):
    c = moe_case(33, 512, 512, 8, 2, 512, valid_frac=0.7)
    moe = build_module(moe_pkg, c, DEV)
    # route every token to experts 0..3 (rank 0 of 2): rank 1 receives nothing
    bias = torch.zeros(8, device=DEV)
    bias[4:] = -1e4
    moe.router_logit_bias = bias
    x = x_tensor(c, DEV)
    valid = torch.from_numpy(c["valid"]).to(DEV)
    with torch.no_grad():
        ref = moe.forward_details(x, valid)
    ops = moe_pkg.CudaEPOps()
    wr = moe.router.weight.detach().float().contiguous()
    idx, w, _ = ops.route(x, wr, bias, valid, 2, moe.norm_topk_prob)
    send, counts, pos = ops.dispatch(x, idx, w, valid, 2, 4)
    rows = counts.cpu().tolist()
    assert rows[1] == 0 and rows[3] == 0
    p0 = ops.experts(send[:rows[0]], rows[0], rows[2], 512, 2, moe.experts[:4])
    p1 = ops.experts(send[rows[0]:rows[0]], 0, 0, 512, 2, moe.experts[4:])
    out = ops.combine(torch.cat([p0, p1]), pos, x.shape[0], 512, 2)
    torch.cuda.synchronize()
    a, b = out.float(), ref["out"].float()
    assert (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item() < 5e-3
    assert torch.all(a[valid == 0] == 0)


def test_split_dispatch_matches_one_call(moe_pkg):
    """dispatch_count + dispatch_pack (counts exchanged in between) write the same
    counts, positions and row bytes as the one-call dispatch."""
    c = moe_case(34, 1000, 512, 16, 4, 512, valid_frac=0.8)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    valid = torch.from_numpy(c["valid"]).to(DEV)
    ops = moe_pkg.CudaEPOps()
    wr = moe.router.weight.detach().float().contiguous()
    idx, w, _ = ops.route(x, wr, None, valid, 4, moe.norm_topk_prob)
    for G in (1, 2, 4, 8):
        send, counts, pos = ops.dispatch(x, idx, w, valid, G, 16 // G, slot=0)
        send, counts, pos = send.clone(), counts.clone(), pos.clone()
        out = torch.full((2 * G,), -7, dtype=torch.int32, device=DEV)
        cnt = ops.dispatch_count(idx, valid, G, 16 // G, slot=1, out=out)
        send2, counts2, pos2 = ops.dispatch_pack(x, idx, w, valid, G, 16 // G, cnt, slot=1)
        torch.cuda.synchronize()
        assert torch.equal(counts, counts2) and torch.equal(out, counts)
        assert torch.equal(pos, pos2)
        n = int(counts[:G].sum())
        assert torch.equal(send[:n], send2[:n])


def _emulate_h_back(pkg, moe, xs, G, valids=None):
    """G source ranks emulated on one GPU with the "h back" exchange: every source
    routes and lays out its own tokens, receiver g runs the gate/up GEMM of the rows
    addressed to it (sources in rank order) and stores each slot's h into its source's
    buffers, every source runs the down projection and combine."""
    E, k = len(moe.experts), moe.top_k
    E_loc = E // G
    d = xs[0].shape[1]
    F = moe.experts[0].down_proj.weight.shape[1]
    wr = moe.router.weight.detach().float().contiguous()
    dn_all = pkg.get_or_build_grouped_cache(moe.experts, "down_proj")
    lib = pkg.library()
    ops = [pkg.CudaEPOps() for _ in range(G)]
    st, sends, counts, hq, hs = [], [], [], [], []
    for s in range(G):
        vm = None if valids is None else valids[s]
        state = ops[s].layout(xs[s], wr, None, vm, k, moe.norm_topk_prob, dn_all, F)
        cnt = ops[s].dispatch_count(state["idx"], vm, G, E_loc)
        send, _, _ = ops[s].dispatch_pack_h(xs[s], state["idx"], vm, G, E_loc, s, state["slot_pos"], cnt)
        mcap = lib.mcl4moe_padded_rows(xs[s].shape[0], E, k)
        st.append(state)
        sends.append(send)
        counts.append(cnt.cpu().tolist())
        hq.append(torch.zeros((mcap, F // 2), dtype=torch.uint8, device=DEV))
        hs.append(torch.zeros((mcap * (F // 16),), dtype=torch.uint8, device=DEV))
    for g in range(G):
        parts, slots = [], 0
        for s in range(G):
            start = sum(counts[s][:g])
            parts.append(sends[s][start:start + counts[s][g]])
            slots += counts[s][G + g]
        recv = torch.cat(parts, dim=0).contiguous()
        ops[g].gateup_to_peers(recv, recv.shape[0], slots, d, k, moe.experts[g * E_loc:(g + 1) * E_loc],
                               [t.data_ptr() for t in hq], [t.data_ptr() for t in hs])
    outs = [ops[s].down(st[s], hq[s], hs[s]) for s in range(G)]
    torch.cuda.synchronize()
    return outs, st


@pytest.mark.parametrize("G", [2, 4, 8])
def test_h_back_exchange_is_the_single_gpu_layer_bit_for_bit(moe_pkg, G):
    """With the gate/up GEMMs sharded and the down projection at each token's home rank,
    every source's output, routing and statistics equal the single-GPU layer's on its
    tokens bit for bit (the h bytes are the same whichever rank computes them)."""
    c = moe_case(41, 1024, 512, 16, 4, 512)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    sizes = [1024 // G] * G  # uneven token counts per rank
    sizes[0] += 37
    sizes[-1] -= 37
    xs = list(torch.split(x, sizes, dim=0))
    xs = [t.contiguous() for t in xs]
    outs, st = _emulate_h_back(moe_pkg, moe, xs, G)
    for s in range(G):
        with torch.no_grad():
            ref = moe.forward_details(xs[s])
        torch.cuda.synchronize()
        assert torch.equal(st[s]["idx"], ref["topk_idx"]), s
        assert torch.equal(outs[s], ref["out"]), s
        assert torch.equal(st[s]["stats"][:2], torch.stack([ref["aux_loss"], ref["router_z_loss"]]).float()), s


def test_h_back_exchange_with_masked_tokens(moe_pkg):
    """Masked tokens are neither dispatched nor combined; the rest is the single-GPU
    layer with the same mask, bit for bit."""
    G = 2
    c = moe_case(43, 600, 512, 8, 2, 256)
    moe = build_module(moe_pkg, c, DEV)
    x = x_tensor(c, DEV)
    xs = [t.contiguous() for t in torch.split(x, [350, 250], dim=0)]
    r = np.random.default_rng(9)
    valids = [torch.from_numpy((r.uniform(size=t.shape[0]) < 0.7).astype(np.uint8)).to(DEV) for t in xs]
    outs, st = _emulate_h_back(moe_pkg, moe, xs, G, valids)
    for s in range(G):
        with torch.no_grad():
            ref = moe.forward_details(xs[s], valids[s])
        torch.cuda.synchronize()
        assert torch.equal(st[s]["idx"], ref["topk_idx"]), s
        assert torch.equal(outs[s], ref["out"]), s
