"""Expert-parallel SparseMoE: the experts of one layer sharded over a process group.

Rank g of G owns the contiguous experts ``[g*E/G, (g+1)*E/G)``; the router is
replicated and every rank routes its own tokens (weak scaling: the layer's
forward over each rank's batch is exactly the single-device forward over that
batch, up to the summation order of the per-rank partial outputs).  One call:

1. route all E experts for the local tokens (``mcl4moe_route``);
2. dispatch: one NVFP4 row per (token, rank holding any of its experts), with
   the token's local expert ids there and its k routing weights
   (``mcl4moe_ep_dispatch``);
3. exchange row and slot counts, then the rows (all-to-all);
4. the grouped gate/up + SwiGLU and down GEMMs over the received rows, reduced
   to one bf16 partial per row (``mcl4moe_ep_experts``);
5. return the partials (all-to-all, reverse splits) and add them per token in
   rank order (``mcl4moe_ep_combine``).

The reference runs the layer on one device (src/mcl4_coe/backbone.py:618-911);
this module has no counterpart there.  The exchange logic is independent of
where the device steps run: ``ops`` provides them (the CUDA library by default;
the CPU tests plug in an oracle-based implementation over gloo).
"""

from __future__ import annotations

import ctypes
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor, nn

from . import _lib
from .moe import SwiGLUExpert
from .nvfp4 import get_or_build_grouped_cache


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


class CudaEPOps:
    """Device steps through ``libmcl4moe.so``."""

    def __init__(self) -> None:
        self._ws: dict[str, Tensor] = {}

    def _scratch(self, name: str, nbytes: int, device) -> Tensor:
        t = self._ws.get(name)
        if t is None or t.numel() < nbytes or t.device != device:
            t = torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=device)
            self._ws[name] = t
        return t

    def row_bytes(self, d: int, k: int) -> int:
        rb = _lib.load().mcl4moe_ep_row_bytes(d, k)
        if rb == 0:
            raise ValueError(f"unsupported expert-parallel shape d={d} k={k}")
        return rb

    def route(self, x: Tensor, wr: Tensor, bias: Tensor | None, valid: Tensor | None, k: int, norm: bool):
        lib = _lib.load()
        T, d = x.shape
        E = wr.shape[0]
        dev = x.device
        idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        w = torch.empty((T, k), dtype=torch.float32, device=dev)
        counts = torch.empty((E,), dtype=torch.int32, device=dev)
        stats = torch.empty((3 + E,), dtype=torch.float32, device=dev)
        ws = self._scratch("route", lib.mcl4moe_route_workspace_size(T, E, k, d), dev)
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        _lib.check(lib.mcl4moe_route(x.data_ptr(), wr.data_ptr(), p(bias), None, p(valid), T, d, E, k, int(norm),
                                     idx.data_ptr(), w.data_ptr(), None, None, counts.data_ptr(), stats.data_ptr(),
                                     ws.data_ptr(), ws.numel(), _stream_handle()), "mcl4moe_route")
        return idx, w, stats

    def dispatch(self, x: Tensor, idx: Tensor, w: Tensor, valid: Tensor | None, G: int, E_loc: int):
        lib = _lib.load()
        T, d = x.shape
        k = idx.shape[1]
        dev = x.device
        rb = self.row_bytes(d, k)
        send_buf = self._scratch("send", T * G * rb, dev)
        counts = torch.empty((2 * G,), dtype=torch.int32, device=dev)
        pos = torch.empty((T, G), dtype=torch.int32, device=dev)
        ws = self._scratch("dispatch", lib.mcl4moe_ep_dispatch_workspace_size(T, G), dev)
        _lib.check(lib.mcl4moe_ep_dispatch(x.data_ptr(), idx.data_ptr(), w.data_ptr(),
                                           None if valid is None else valid.data_ptr(), T, d, k, G, E_loc,
                                           counts.data_ptr(), pos.data_ptr(), send_buf.data_ptr(), ws.data_ptr(),
                                           ws.numel(), _stream_handle()), "mcl4moe_ep_dispatch")
        return send_buf[: T * G * rb].view(T * G, rb), counts, pos

    def prepare(self, experts: nn.ModuleList) -> None:
        """Validate / refresh the NVFP4 weight caches of this rank's experts.  Called
        before routing, so this host work overlaps the device work instead of
        following the host synchronisation of the exchange."""
        self._caches = (get_or_build_grouped_cache(experts, "up_proj"), get_or_build_grouped_cache(experts, "down_proj"))

    def experts(self, recv: Tensor, R: int, slots: int, d: int, k: int, experts: nn.ModuleList) -> Tensor:
        lib = _lib.load()
        dev = recv.device
        E_loc = len(experts)
        F = experts[0].down_proj.weight.shape[1]
        up, dn = getattr(self, "_caches", None) or (get_or_build_grouped_cache(experts, "up_proj"),
                                                    get_or_build_grouped_cache(experts, "down_proj"))
        self._caches = None
        partial = torch.empty((R, d), dtype=torch.bfloat16, device=dev)
        ws = self._scratch("experts", lib.mcl4moe_ep_experts_workspace_size(R, slots, d, k, E_loc, F), dev)
        _lib.check(lib.mcl4moe_ep_experts(recv.data_ptr(), R, slots, d, k, E_loc, F, up.packed.data_ptr(),
                                          up.scales.data_ptr(), up.g.data_ptr(), dn.packed.data_ptr(),
                                          dn.scales.data_ptr(), dn.g.data_ptr(), partial.data_ptr(), None,
                                          ws.data_ptr(), ws.numel(), _stream_handle()), "mcl4moe_ep_experts")
        return partial

    def combine(self, back: Tensor, pos: Tensor, T: int, d: int, G: int) -> Tensor:
        out = torch.empty((T, d), dtype=torch.bfloat16, device=pos.device)
        _lib.check(_lib.load().mcl4moe_ep_combine(back.data_ptr() if back.numel() else None, pos.data_ptr(), T, d,
                                                  G, out.data_ptr(), _stream_handle()), "mcl4moe_ep_combine")
        return out


class PeerExchange:
    """Exchange between the ranks of one node through peer memory.

    Every rank owns one arena (a receive region for dispatched rows and one for
    returned partial sums) and maps every other rank's arena through CUDA IPC.
    A sender copies its pieces straight into the receiver's arena with
    copy-engine copies (one stream per destination, so several copy engines run
    at once and no SMs are taken from the GEMMs); a one-element all-reduce on
    the group afterwards orders every receiver after every sender's copies.
    Region sizes are decided from numbers all ranks share, so growing the arena
    (a collective) happens on all ranks together.
    """

    ALIGN = 4096

    def __init__(self, group: dist.ProcessGroup | None, device: torch.device) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        self.streams = [torch.cuda.Stream(device=device) for _ in range(self.world)]
        self.token = torch.zeros((1,), dtype=torch.float32, device=device)
        self.arena: Tensor | None = None
        self.regions: dict[str, tuple[int, int]] = {}
        self.peer_base: list[int] = []
        self._imported: list[int] = []

    def reserve(self, sizes: dict[str, int]) -> None:
        """Make every named region at least ``sizes[name]`` bytes (collective when it grows)."""
        if self.arena is not None and all(n in self.regions and self.regions[n][1] >= b for n, b in sizes.items()):
            return
        self.close()
        lib = _lib.load()
        off, regions = 0, {}
        for name in sorted(sizes):
            nbytes = max(int(sizes[name]) * 5 // 4, self.ALIGN)  # headroom: fewer regrowths
            regions[name] = (off, nbytes)
            off += (nbytes + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        arena = torch.empty((off,), dtype=torch.uint8, device=self.device)
        handle = (ctypes.c_uint8 * 64)()
        offset = ctypes.c_uint64()
        _lib.check(lib.mcl4moe_ipc_export(arena.data_ptr(), handle, ctypes.byref(offset)), "mcl4moe_ipc_export")
        gathered: list[Any] = [None] * self.world
        dist.all_gather_object(gathered, (bytes(handle), offset.value), group=self.group)
        bases = []
        for g, (h, o) in enumerate(gathered):
            if g == self.rank:
                bases.append(arena.data_ptr())
                continue
            base = ctypes.c_void_p()
            _lib.check(lib.mcl4moe_ipc_import((ctypes.c_uint8 * 64).from_buffer_copy(h), ctypes.byref(base)),
                       "mcl4moe_ipc_import")
            self._imported.append(base.value)
            bases.append(base.value + o)
        self.arena, self.regions, self.peer_base = arena, regions, bases

    def close(self) -> None:
        """Unmap the peers' arenas (collective: nobody frees an arena a peer still maps)."""
        if self.arena is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _lib.load()
        for b in self._imported:
            lib.mcl4moe_ipc_close(ctypes.c_void_p(b))
        self._imported = []
        dist.barrier(group=self.group)
        self.arena, self.regions, self.peer_base = None, {}, []

    def local(self, name: str, nbytes: int) -> Tensor:
        off, size = self.regions[name]
        assert nbytes <= size
        return self.arena[off:off + nbytes]

    def put(self, name: str, pieces: list[tuple[int, Tensor, int]]) -> None:
        """Copy each ``(dest, src, byte_offset)`` into region ``name`` of ``dest``,
        then wait (on the device) until every rank's copies have landed."""
        lib = _lib.load()
        cur = torch.cuda.current_stream(self.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        off0, size = self.regions[name]
        used = set()
        for dest, src, byte_off in pieces:
            n = src.numel() * src.element_size()
            if n == 0:
                continue
            assert byte_off + n <= size, (name, byte_off, n, size)
            st = self.streams[dest]
            if dest not in used:
                st.wait_event(ready)
                used.add(dest)
            _lib.check(lib.mcl4moe_copy_async(ctypes.c_void_p(self.peer_base[dest] + off0 + byte_off),
                                              ctypes.c_void_p(src.data_ptr()), n, st.cuda_stream),
                       "mcl4moe_copy_async")
            src.record_stream(st)
        for dest in used:
            cur.wait_stream(self.streams[dest])
        dist.all_reduce(self.token, group=self.group)


class ExpertParallelMoE(nn.Module):
    """SparseMoE whose experts are sharded over ``group`` (one process per GPU).

    Parameters: ``router.weight`` [E, d] (replicated) and ``experts`` (the
    ``E / world`` experts of this rank, global ids ``expert_offset + i``).
    ``forward(x, valid=None) -> (out, aux_loss, router_z_loss, counts)`` with
    the statistics of this rank's tokens, as the single-device layer computes
    them for the same batch.
    """

    def __init__(self, config: Any, group: dist.ProcessGroup | None = None, ops: Any = None,
                 transport: str = "auto") -> None:
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        d = int(getattr(config, "d_model"))
        E = int(getattr(config, "num_experts"))
        F = int(getattr(config, "expert_hidden_dim"))
        if E % self.world != 0:
            raise ValueError(f"num_experts={E} must be a multiple of the group size {self.world}")
        self.num_experts = E
        self.experts_per_rank = E // self.world
        self.expert_offset = self.rank * self.experts_per_rank
        self.top_k = int(getattr(config, "top_k"))
        self.norm_topk_prob = bool(getattr(config, "norm_topk_prob", True))
        if not 0 < self.top_k <= E:
            raise ValueError("top_k must be in [1, num_experts]")
        self.router = nn.Linear(d, E, bias=False)
        self.experts = nn.ModuleList([SwiGLUExpert(d, F) for _ in range(self.experts_per_rank)])
        self.router_logit_bias: Tensor | None = None
        self.last_selected_mask: Tensor | None = None
        self.ops = ops if ops is not None else CudaEPOps()
        self.last_exchange: dict[str, list[int]] = {}
        # "peer": copy-engine copies into peer memory (CUDA tensors, one node);
        # "collective": all-to-all through torch.distributed (any backend, e.g. gloo)
        self.transport = transport
        self._peer: PeerExchange | None = None
        # optional 7 CUDA events recorded around the six steps (route, dispatch,
        # row exchange, experts, partial exchange, combine), for stage timing
        self.stage_events: list | None = None

    @classmethod
    def from_dense(cls, moe: nn.Module, group: dist.ProcessGroup | None = None, ops: Any = None,
                   transport: str = "auto") -> "ExpertParallelMoE":
        """Shard a single-device layer (this package's or the reference's SparseMoE):
        the router is shared, this rank keeps its block of experts."""
        E = len(moe.experts)
        cfg = type("Cfg", (), dict(d_model=moe.router.in_features, num_experts=E,
                                   expert_hidden_dim=moe.experts[0].down_proj.in_features, top_k=moe.top_k,
                                   norm_topk_prob=moe.norm_topk_prob))()
        mod = cls(cfg, group, ops, transport)
        mod.router = moe.router
        lo = mod.expert_offset
        mod.experts = nn.ModuleList(list(moe.experts)[lo:lo + mod.experts_per_rank])
        mod.router_logit_bias = getattr(moe, "router_logit_bias", None)
        return mod

    def _all_to_all(self, out: Tensor, inp: Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    @torch.no_grad()
    def forward(self, x: Tensor, valid: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        flat = x.reshape(-1, x.shape[-1])
        T, d = flat.shape
        G, k, E_loc = self.world, self.top_k, self.experts_per_rank
        xb = flat.to(torch.bfloat16).contiguous()
        wr = self.router.weight.detach().to(device=xb.device, dtype=torch.float32).contiguous()
        bias = None
        if self.router_logit_bias is not None:
            bias = self.router_logit_bias.detach().to(device=xb.device, dtype=torch.float32).contiguous()
        vmask = None
        if valid is not None:
            vmask = valid.reshape(-1).to(device=xb.device, dtype=torch.uint8).contiguous()

        ev = self.stage_events
        mark = (lambda i: ev[i].record()) if ev is not None else (lambda i: None)
        mark(0)
        if hasattr(self.ops, "prepare"):
            self.ops.prepare(self.experts)
        idx, w, stats = self.ops.route(xb, wr, bias, vmask, k, self.norm_topk_prob)
        mark(1)
        send, counts, pos = self.ops.dispatch(xb, idx, w, vmask, G, E_loc)
        mark(2)

        use_peer = self.transport == "peer" or (
            self.transport == "auto" and xb.is_cuda and dist.get_backend(self.group) == "nccl")
        if use_peer:
            back = self._exchange_peer(send, counts, T, d, k, mark)
        else:
            back = self._exchange_collective(send, counts, d, k, mark)
        mark(5)
        out = self.ops.combine(back, pos, T, d, G)
        mark(6)
        return out.to(x.dtype).view_as(x), stats[0], stats[1], stats[3:3 + self.num_experts]

    def _exchange_collective(self, send: Tensor, counts: Tensor, d: int, k: int, mark) -> Tensor:
        """Rows out and partial sums back through ``all_to_all_single``."""
        G = self.world
        # row and slot counts: [G, 2] per rank, one entry pair per destination
        send_tab = torch.stack([counts[:G], counts[G:]], dim=1).contiguous()
        recv_tab = torch.empty_like(send_tab)
        self._all_to_all(recv_tab, send_tab, [1] * G, [1] * G)
        tab = torch.cat([send_tab, recv_tab], dim=0).cpu()  # the split sizes are needed on the host
        rows_to = tab[:G, 0].tolist()
        rows_from = tab[G:, 0].tolist()
        slots_here = int(tab[G:, 1].sum())
        R = int(sum(rows_from))
        self.last_exchange = dict(rows_to=rows_to, rows_from=rows_from, slots=[slots_here])
        sent = sum(rows_to)
        recv = torch.empty((R, send.shape[1]), dtype=torch.uint8, device=send.device)
        self._all_to_all(recv, send[:sent], rows_from, rows_to)
        mark(3)
        partial = self.ops.experts(recv, R, slots_here, d, k, self.experts)
        mark(4)
        back = torch.empty((sent, d), dtype=torch.bfloat16, device=partial.device)
        self._all_to_all(back, partial, rows_to, rows_from)
        return back

    def _exchange_peer(self, send: Tensor, counts: Tensor, T: int, d: int, k: int, mark) -> Tensor:
        """Rows out and partial sums back through peer memory (copy engines)."""
        G, me = self.world, self.rank
        if self._peer is None:
            self._peer = PeerExchange(self.group, send.device)
        px = self._peer
        # every rank's per-destination row and slot counts and its token count
        mine = torch.cat([counts, torch.tensor([T], dtype=torch.int32, device=counts.device)])
        allc = torch.empty((G, 2 * G + 1), dtype=torch.int32, device=counts.device)
        dist.all_gather_into_tensor(allc, mine, group=self.group)
        tab = allc.cpu().tolist()
        rows = [r[:G] for r in tab]          # rows[s][g]: rows from s to g
        slots = [r[G:2 * G] for r in tab]
        t_max = max(r[2 * G] for r in tab)
        rb = send.shape[1]
        px.reserve({"rows": G * t_max * rb, "back": G * t_max * d * 2})
        rows_to, rows_from = rows[me], [rows[s][me] for s in range(G)]
        R = sum(rows_from)
        slots_here = sum(slots[s][me] for s in range(G))
        self.last_exchange = dict(rows_to=rows_to, rows_from=rows_from, slots=[slots_here])
        # my rows for g go after the rows of lower ranks in g's receive region
        pieces, start = [], 0
        for g in range(G):
            n = rows[me][g]
            at = sum(rows[s][g] for s in range(me))
            pieces.append((g, send[start:start + n].reshape(-1), at * rb))
            start += n
        px.put("rows", pieces)
        recv = px.local("rows", R * rb).view(R, rb)
        mark(3)
        partial = self.ops.experts(recv, R, slots_here, d, k, self.experts)
        mark(4)
        # partials of the rows from s go where s keeps its segment for me
        pieces, at_here = [], 0
        for s in range(G):
            n = rows[s][me]
            at = sum(rows[s][g] for g in range(me))
            pieces.append((s, partial[at_here:at_here + n].reshape(-1), at * d * 2))
            at_here += n
        px.put("back", pieces)
        sent = sum(rows_to)
        return px.local("back", sent * d * 2).view(torch.bfloat16).view(sent, d)

