"""CPU restatement of the expert-parallel device steps, for the gloo tests.

Implements the same four steps as ``CudaEPOps`` (route, dispatch, experts,
combine) with the oracle's numpy quantisers and expert math and the same
dispatch-row format (codes [d/2] | row-major E4M3 scales [d/16] | k int8 local
expert ids padded to 16 | k fp32 weights padded to 16), so the exchange logic
of ``ExpertParallelMoE`` (counts, split sizes, row order, reverse exchange) runs
unchanged on CPU tensors over gloo.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_ref
from oracle import nvfp4_ref as nr


def row_layout(d: int, k: int):
    ids = d // 2 + d // 16
    weights = ids + (k + 15) // 16 * 16
    return dict(codes=0, scales=d // 2, ids=ids, weights=weights, bytes=weights + (4 * k + 15) // 16 * 16)


class OracleEPOps:
    def __init__(self):
        self.routing = None

    def route(self, x, wr, bias, valid, k, norm):
        xs = x.float().numpy()
        T = xs.shape[0]
        r = moe_ref.route(xs, wr.numpy(), k, norm, None if valid is None else valid.numpy(),
                          None if bias is None else bias.numpy())
        self.routing = r
        idx = np.full((T, k), -1, np.int32)
        w = np.zeros((T, k), np.float32)
        idx[r.active] = r.selected
        w[r.active] = r.weights
        stats = np.concatenate([[r.aux_loss, r.z_loss, np.float32(r.active.size)], r.counts]).astype(np.float32)
        return torch.from_numpy(idx), torch.from_numpy(w), torch.from_numpy(stats)

    def dispatch(self, x, idx, w, valid, G, E_loc, slot=0):
        xs = x.float().numpy()
        T, d = xs.shape
        k = idx.shape[1]
        L = row_layout(d, k)
        idx_np, w_np = idx.numpy(), w.numpy()
        rows = [[] for _ in range(G)]
        slots = [0] * G
        for t in range(T):
            if valid is not None and valid[t] == 0:
                continue
            dests = sorted({int(e) // E_loc for e in idx_np[t] if e >= 0})
            for g in dests:
                rows[g].append(t)
                slots[g] += int(sum(1 for e in idx_np[t] if e >= 0 and e // E_loc == g))
        send = np.zeros((T * G, L["bytes"]), np.uint8)
        pos = np.full((T, G), -1, np.int32)
        p = 0
        for g in range(G):
            for t in rows[g]:
                packed, scales = nr.quantize_activations(xs[t:t + 1])
                row = send[p]
                row[L["codes"]:L["codes"] + d // 2] = packed[0]
                row[L["scales"]:L["scales"] + d // 16] = scales[0]
                ids = np.full((k + 15) // 16 * 16, -1, np.int8)
                for j in range(k):
                    e = int(idx_np[t, j])
                    ids[j] = e - g * E_loc if e >= 0 and e // E_loc == g else -1
                row[L["ids"]:L["ids"] + ids.size] = ids.view(np.uint8)
                row[L["weights"]:L["weights"] + 4 * k] = w_np[t].astype(np.float32).view(np.uint8)
                pos[t, g] = p
                p += 1
        counts = np.array([len(r) for r in rows] + slots, np.int32)
        return torch.from_numpy(send), torch.from_numpy(counts), torch.from_numpy(pos)

    def experts(self, recv, R, slots, d, k, experts):
        L = row_layout(d, k)
        w_up = np.stack([e.up_proj.weight.detach().float().numpy() for e in experts])
        w_dn = np.stack([e.down_proj.weight.detach().float().numpy() for e in experts])
        q = moe_ref.QuantizedExperts(w_up, w_dn)
        buf = recv.numpy()
        partial = np.zeros((R, d), np.float32)
        n_slots = 0
        for r in range(R):
            row = buf[r]
            xq = nr.dequantize(row[None, L["codes"]:L["codes"] + d // 2], row[None, L["scales"]:L["scales"] + d // 16],
                               np.float32(1.0), 1, d)
            ids = row[L["ids"]:L["ids"] + k].view(np.int8)
            wts = row[L["weights"]:L["weights"] + 4 * k].view(np.float32)
            acc = np.zeros((1, d), np.float32)
            for j in range(k):
                e = int(ids[j])
                if e < 0:
                    continue
                n_slots += 1
                f = q.up[e].shape[0] // 2
                up = nr.round_bf16((xq @ q.up[e].T).astype(np.float32))
                h = nr.round_bf16((moe_ref.silu_bf16(up[:, :f]) * up[:, f:]).astype(np.float32))
                y = nr.round_bf16((nr.fake_quantize_activations(h) @ q.dn[e].T).astype(np.float32))
                acc = (acc + nr.round_bf16((y * nr.round_bf16(np.array([wts[j]], np.float32))).astype(np.float32)))
                acc = acc.astype(np.float32)
            partial[r] = nr.round_bf16(acc)[0]
        assert n_slots == slots, (n_slots, slots)
        return torch.from_numpy(partial).to(torch.bfloat16)

    def combine(self, back, pos, T, d, G, out=None):
        b = back.float().numpy()
        p = pos.numpy()
        res = np.zeros((T, d), np.float32)
        for t in range(T):
            acc = np.zeros(d, np.float32)
            for g in range(G):
                if p[t, g] >= 0:
                    acc = (acc + b[p[t, g]]).astype(np.float32)
            res[t] = nr.round_bf16(acc)
        res = torch.from_numpy(res).to(torch.bfloat16)
        if out is not None:
            out.copy_(res)
            return out
        return res
