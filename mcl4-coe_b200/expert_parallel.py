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
from .nvfp4 import get_or_build_grouped_cache, seed_grouped_cache


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

    def dispatch(self, x: Tensor, idx: Tensor, w: Tensor, valid: Tensor | None, G: int, E_loc: int, slot: int = 0):
        lib = _lib.load()
        T, d = x.shape
        k = idx.shape[1]
        dev = x.device
        rb = self.row_bytes(d, k)
        send_buf = self._scratch(f"send{slot}", T * G * rb, dev)
        counts = torch.empty((2 * G,), dtype=torch.int32, device=dev)
        pos = torch.empty((T, G), dtype=torch.int32, device=dev)
        ws = self._scratch("dispatch", lib.mcl4moe_ep_dispatch_workspace_size(T, G), dev)
        _lib.check(lib.mcl4moe_ep_dispatch(x.data_ptr(), idx.data_ptr(), w.data_ptr(),
                                           None if valid is None else valid.data_ptr(), T, d, k, G, E_loc,
                                           counts.data_ptr(), pos.data_ptr(), send_buf.data_ptr(), ws.data_ptr(),
                                           ws.numel(), _stream_handle()), "mcl4moe_ep_dispatch")
        return send_buf[: T * G * rb].view(T * G, rb), counts, pos

    def dispatch_count(self, idx: Tensor, valid: Tensor | None, G: int, E_loc: int, slot: int = 0,
                       out: Tensor | None = None) -> Tensor:
        """First half of ``dispatch``: the rows and slots bound for each rank (device int32 [2G],
        written to ``out`` when given)."""
        lib = _lib.load()
        T, k = idx.shape
        dev = idx.device
        counts = out if out is not None else torch.empty((2 * G,), dtype=torch.int32, device=dev)
        assert counts.is_contiguous() and counts.numel() == 2 * G and counts.dtype == torch.int32
        ws = self._scratch(f"dispatch{slot}", lib.mcl4moe_ep_dispatch_workspace_size(T, G), dev)
        _lib.check(lib.mcl4moe_ep_dispatch_count(idx.data_ptr(), None if valid is None else valid.data_ptr(), T, k,
                                                 G, E_loc, counts.data_ptr(), ws.data_ptr(), ws.numel(),
                                                 _stream_handle()), "mcl4moe_ep_dispatch_count")
        return counts

    def dispatch_pack(self, x: Tensor, idx: Tensor, w: Tensor, valid: Tensor | None, G: int, E_loc: int,
                      counts: Tensor, slot: int = 0):
        """Second half of ``dispatch`` (after ``dispatch_count`` with the same ``slot``)."""
        lib = _lib.load()
        T, d = x.shape
        k = idx.shape[1]
        dev = x.device
        rb = self.row_bytes(d, k)
        send_buf = self._scratch(f"send{slot}", T * G * rb, dev)
        pos = torch.empty((T, G), dtype=torch.int32, device=dev)
        ws = self._scratch(f"dispatch{slot}", lib.mcl4moe_ep_dispatch_workspace_size(T, G), dev)
        _lib.check(lib.mcl4moe_ep_dispatch_pack(x.data_ptr(), idx.data_ptr(), w.data_ptr(),
                                                None if valid is None else valid.data_ptr(), T, d, k, G, E_loc,
                                                counts.data_ptr(), pos.data_ptr(), send_buf.data_ptr(), ws.data_ptr(),
                                                ws.numel(), _stream_handle()), "mcl4moe_ep_dispatch_pack")
        return send_buf[: T * G * rb].view(T * G, rb), counts, pos

    def prepare(self, experts: nn.ModuleList) -> tuple:
        """Validate / refresh the NVFP4 weight caches of this rank's experts and return
        them for the ``experts`` calls of one forward.  Called before routing, so this
        host work overlaps the device work instead of following the host
        synchronisation of the exchange, and runs once per forward, not per chunk."""
        return get_or_build_grouped_cache(experts, "up_proj"), get_or_build_grouped_cache(experts, "down_proj")

    def experts(self, recv: Tensor, R: int, slots: int, d: int, k: int, experts: nn.ModuleList,
                caches: tuple | None = None) -> Tensor:
        lib = _lib.load()
        dev = recv.device
        E_loc = len(experts)
        F = experts[0].down_proj.weight.shape[1]
        up, dn = caches or self.prepare(experts)
        partial = torch.empty((R, d), dtype=torch.bfloat16, device=dev)
        ws = self._scratch("experts", lib.mcl4moe_ep_experts_workspace_size(R, slots, d, k, E_loc, F), dev)
        _lib.check(lib.mcl4moe_ep_experts(recv.data_ptr(), R, slots, d, k, E_loc, F, up.packed.data_ptr(),
                                          up.scales.data_ptr(), up.g.data_ptr(), dn.packed.data_ptr(),
                                          dn.scales.data_ptr(), dn.g.data_ptr(), partial.data_ptr(), None,
                                          ws.data_ptr(), ws.numel(), _stream_handle()), "mcl4moe_ep_experts")
        return partial

    def experts_to_peers(self, recv: Tensor, R: int, slots: int, d: int, k: int, experts: nn.ModuleList,
                         seg_start: list[int], dst: list[int], caches: tuple | None = None) -> None:
        """The experts step with each partial-sum row stored straight to ``dst[s]``
        (a peer mapping for rows from another rank)."""
        lib = _lib.load()
        dev = recv.device
        E_loc = len(experts)
        F = experts[0].down_proj.weight.shape[1]
        up, dn = caches or self.prepare(experts)
        G = len(dst)
        starts = (ctypes.c_int32 * (G + 1))(*seg_start)
        ptrs = (ctypes.c_void_p * G)(*dst)
        ws = self._scratch("experts", lib.mcl4moe_ep_experts_workspace_size(R, slots, d, k, E_loc, F), dev)
        _lib.check(lib.mcl4moe_ep_experts_to_peers(recv.data_ptr(), R, slots, d, k, E_loc, F, up.packed.data_ptr(),
                                                   up.scales.data_ptr(), up.g.data_ptr(), dn.packed.data_ptr(),
                                                   dn.scales.data_ptr(), dn.g.data_ptr(), G, starts, ptrs, None,
                                                   ws.data_ptr(), ws.numel(), _stream_handle()),
                   "mcl4moe_ep_experts_to_peers")

    # ---- "h back": gate/up sharded, the down projection at the token's home GPU

    def layout(self, x: Tensor, wr: Tensor, bias: Tensor | None, valid: Tensor | None, k: int, norm: bool,
               dn_all, F: int, slot: int = 0) -> dict:
        """Routing and this rank's expert-major layout of its own slots
        (``mcl4moe_moe_forward_layout``); the state that ``down`` continues from."""
        lib = _lib.load()
        T, d = x.shape
        E = wr.shape[0]
        dev = x.device
        st = dict(T=T, d=d, E=E, k=k, F=F)
        st["idx"] = torch.empty((T, k), dtype=torch.int32, device=dev)
        st["w"] = torch.empty((T, k), dtype=torch.float32, device=dev)
        st["stats"] = torch.empty((3 + E,), dtype=torch.float32, device=dev)
        st["out"] = torch.empty((T, d), dtype=torch.bfloat16, device=dev)
        ws = self._scratch(f"moe{slot}", lib.mcl4moe_moe_workspace_size(T, d, E, k, F), dev)
        if T > 0 and ws.numel() < lib.mcl4moe_moe_workspace_size(T, d, E, k, F):
            raise ValueError("unsupported layer shape for the expert-parallel layout")
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        args = _lib.MoeArgs(
            x=x.data_ptr(), router_w=wr.data_ptr(), logit_bias=p(bias), valid=p(valid),
            w_dn=dn_all.packed.data_ptr(), w_dn_scales=dn_all.scales.data_ptr(), w_dn_g=dn_all.g.data_ptr(),
            T=T, d=d, E=E, k=k, F=F, norm_topk_prob=int(norm), out=st["out"].data_ptr(),
            stats=st["stats"].data_ptr(), topk_idx=st["idx"].data_ptr(), topk_w=st["w"].data_ptr(),
            workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        _lib.check(lib.mcl4moe_moe_forward_layout(args, _stream_handle()), "mcl4moe_moe_forward_layout")
        st["args"], st["ws"] = args, ws
        mcap = lib.mcl4moe_padded_rows(T, E, k)
        st["mcap"] = mcap
        st["slot_pos"] = torch.empty((0, k), dtype=torch.int32, device=dev)
        if T > 0:
            base = ws.data_ptr()
            off = lib.mcl4moe_workspace_region(base, 6, T, d, E, k, F) - base
            st["slot_pos"] = ws[off:off + 4 * T * k].view(torch.int32).view(T, k)
        return st

    def dispatch_pack_h(self, x: Tensor, idx: Tensor, valid: Tensor | None, G: int, E_loc: int, rank: int,
                        slot_pos: Tensor, counts: Tensor, slot: int = 0):
        """``dispatch_pack`` whose rows carry the slots' h destinations on this rank."""
        lib = _lib.load()
        T, d = x.shape
        k = idx.shape[1]
        dev = x.device
        rb = self.row_bytes(d, k)
        send_buf = self._scratch(f"send{slot}", T * G * rb, dev)
        pos = torch.empty((T, G), dtype=torch.int32, device=dev)
        ws = self._scratch(f"dispatch{slot}", lib.mcl4moe_ep_dispatch_workspace_size(T, G), dev)
        _lib.check(lib.mcl4moe_ep_dispatch_pack_h(x.data_ptr(), idx.data_ptr(),
                                                  None if valid is None else valid.data_ptr(), T, d, k, G, E_loc,
                                                  rank, slot_pos.data_ptr(), counts.data_ptr(), pos.data_ptr(),
                                                  send_buf.data_ptr(), ws.data_ptr(), ws.numel(), _stream_handle()),
                   "mcl4moe_ep_dispatch_pack_h")
        return send_buf[: T * G * rb].view(T * G, rb), counts, pos

    def gateup_to_peers(self, recv: Tensor, R: int, slots: int, d: int, k: int, experts: nn.ModuleList,
                        hq_dst: list[int], hs_dst: list[int], up_cache=None) -> None:
        """The received slots' gate/up GEMM with each slot's NVFP4 h stored into its
        source's layout (``hq_dst[s]`` / ``hs_dst[s]``, peer mappings for other ranks)."""
        lib = _lib.load()
        dev = recv.device
        E_loc = len(experts)
        F = experts[0].down_proj.weight.shape[1]
        up = up_cache if up_cache is not None else get_or_build_grouped_cache(experts, "up_proj")
        G = len(hq_dst)
        hq = (ctypes.c_void_p * G)(*hq_dst)
        hs = (ctypes.c_void_p * G)(*hs_dst)
        ws = self._scratch("experts", lib.mcl4moe_ep_experts_workspace_size(R, slots, d, k, E_loc, F), dev)
        _lib.check(lib.mcl4moe_ep_gateup_to_peers(recv.data_ptr(), R, slots, d, k, E_loc, F, up.packed.data_ptr(),
                                                  up.scales.data_ptr(), up.g.data_ptr(), G, hq, hs, None,
                                                  ws.data_ptr(), ws.numel(), _stream_handle()),
                   "mcl4moe_ep_gateup_to_peers")

    def down(self, st: dict, hq: Tensor, hs: Tensor) -> Tensor:
        """Down projection and combine of this rank's slots from the h rows in hq / hs."""
        if st["T"] > 0:
            _lib.check(_lib.load().mcl4moe_moe_forward_down(st["args"], hq.data_ptr(), hs.data_ptr(),
                                                            _stream_handle()), "mcl4moe_moe_forward_down")
        return st["out"]

    def combine(self, back: Tensor, pos: Tensor, T: int, d: int, G: int, out: Tensor | None = None) -> Tensor:
        if out is None:
            out = torch.empty((T, d), dtype=torch.bfloat16, device=pos.device)
        _lib.check(_lib.load().mcl4moe_ep_combine(back.data_ptr() if back.numel() else None, pos.data_ptr(), T, d,
                                                  G, out.data_ptr(), _stream_handle()), "mcl4moe_ep_combine")
        return out


def row_plan(tab: list, c: int, me: int) -> list[tuple[int, int, int, int]]:
    """Row copies of rank ``me`` for chunk ``c``: ``(dest, first send row, rows, first row
    in dest's receive region)``.  ``tab[s][c][g]`` = rows rank s sends to rank g; a sender's
    rows are grouped by destination in rank order, and a receiver's region holds its
    senders' rows in rank order, which is the row order its experts step reads."""
    G = len(tab)
    plan, start = [], 0
    for g in range(G):
        n = tab[me][c][g]
        plan.append((g, start, n, sum(tab[s][c][g] for s in range(me))))
        start += n
    return plan


def back_plan(tab: list, c: int, me: int) -> list[tuple[int, int, int, int]]:
    """Partial-sum copies of rank ``me`` for chunk ``c``: ``(source rank, first partial row,
    rows, first row in the source's return region)``.  Partial row i of a receiver belongs
    to its i-th received row; the source keeps its returns in send order, so the combine
    finds each token's partials at the rows it sent them from."""
    G = len(tab)
    plan, at_here = [], 0
    for s in range(G):
        n = tab[s][c][me]
        plan.append((s, at_here, n, sum(tab[s][c][g] for g in range(me))))
        at_here += n
    return plan


class PeerExchange:
    """Exchange between the ranks of one node through peer memory.

    Every rank owns one arena (a receive region for dispatched rows and one for
    returned partial sums) and maps every other rank's arena through CUDA IPC.
    A sender copies its pieces straight into the receiver's arena with
    copy-engine copies (staggered destination order, two streams; no SMs are
    taken from the GEMMs); a one-element all-reduce on
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
        # two copy streams per direction (dispatched rows, returned partial sums), so a
        # chunk's rows never queue behind the previous chunk's partial sums
        self.streams = [torch.cuda.Stream(device=device) for _ in range(4)]
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

    def address(self, rank: int, name: str, byte_offset: int = 0) -> int:
        """Device address (in this process) of region ``name`` of ``rank`` plus an offset."""
        return self.peer_base[rank] + self.regions[name][0] + byte_offset

    def local(self, name: str, nbytes: int) -> Tensor:
        off, size = self.regions[name]
        assert nbytes <= size
        return self.arena[off:off + nbytes]

    def issue(self, name: str, pieces: list[tuple[int, int, int, int]], lane: int = 0) -> list:
        """Start the copies ``(dest, src_address, nbytes, byte_offset)`` into region
        ``name`` of ``dest`` once the current stream has produced their sources;
        returns the events that mark the end of these copies (for ``complete``).
        The caller keeps the source memory alive until ``complete``.

        Schedule: destinations in the staggered order me+1, me+2, ... (the local
        copy last), alternating over two streams.  At any moment every rank then
        targets a different rank; issuing all copies at once, or in the same order
        on every rank, piles the traffic onto the same destinations (measured on
        8 x B200: 200-430 GB/s per GPU against 660 GB/s staggered).  ``lane`` 0 or 1
        picks the stream pair (one per direction of the exchange).  One library call
        issues the whole list."""
        cur = torch.cuda.current_stream(self.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        off0, size = self.regions[name]
        order = sorted((pc for pc in pieces if pc[2] > 0), key=lambda pc: (pc[0] - self.rank - 1) % self.world)
        lanes = self.streams[2 * lane:2 * lane + 2]
        for st in lanes:
            st.wait_event(ready)
        n = len(order)
        if n:
            for dest, _, nbytes, byte_off in order:
                assert byte_off + nbytes <= size, (name, byte_off, nbytes, size)
            dst = (ctypes.c_void_p * n)(*[self.peer_base[dest] + off0 + off for dest, _, _, off in order])
            src = (ctypes.c_void_p * n)(*[a for _, a, _, _ in order])
            nb = (ctypes.c_uint64 * n)(*[b for _, _, b, _ in order])
            sts = (ctypes.c_void_p * len(lanes))(*[st.cuda_stream for st in lanes])
            _lib.check(_lib.load().mcl4moe_copy_list_async(dst, src, nb, n, sts, len(lanes)),
                       "mcl4moe_copy_list_async")
        done = []
        for st in lanes:
            ev = torch.cuda.Event()
            ev.record(st)
            done.append(ev)
        return done

    def complete(self, events: list) -> None:
        """Order the current stream after this rank's copies (``events``) and, with
        a one-element all-reduce, after every other rank's copies issued before
        its matching call."""
        cur = torch.cuda.current_stream(self.device)
        for ev in events:
            cur.wait_event(ev)
        dist.all_reduce(self.token, group=self.group)

    def put(self, name: str, pieces: list[tuple[int, int, int, int]], lane: int = 0) -> None:
        self.complete(self.issue(name, pieces, lane))


class ExpertParallelMoE(nn.Module):
    """SparseMoE whose experts are sharded over ``group`` (one process per GPU).

    Parameters: ``router.weight`` [E, d] (replicated) and ``experts`` (the
    ``E / world`` experts of this rank, global ids ``expert_offset + i``).
    ``forward(x, valid=None) -> (out, aux_loss, router_z_loss, counts)`` with
    the statistics of this rank's tokens, as the single-device layer computes
    them for the same batch.
    """

    def __init__(self, config: Any, group: dist.ProcessGroup | None = None, ops: Any = None,
                 transport: str = "auto", chunks: int = 0) -> None:
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
        # the batch is cut into token chunks; with the peer transport the exchange of one
        # chunk overlaps the experts step of another.  ``chunks`` > 0: that many equal
        # chunks; ``chunk_weights`` (relative sizes) overrides it.  0 = automatic: one
        # chunk up to 2 ranks (the exchange is small and smaller GEMMs cost more than
        # the overlap gains), two equal chunks beyond (measured on 8 x B200: 2.9-3.2 ms
        # against 3.5 ms for 1 chunk, 3.1-3.3 ms for 3, 4 or 6, and 3.0-3.3 ms for
        # uneven splits 0.55:0.45 to 0.65:0.35)
        self.chunks = int(chunks) if chunks > 0 else (1 if self.world <= 2 else 2)
        self.chunk_weights: list[float] | None = None
        self.min_chunk_tokens = 1024
        # optional 8 CUDA events recorded around the seven steps (route, dispatch,
        # count exchange, row exchange, experts, partial exchange, combine), for stage timing
        self.stage_events: list | None = None
        # how partial sums return with the peer transport: "copy" (copy engines after the
        # summing kernel) or "kernel" (stored over NVLink by the summing kernel itself; its
        # stores from all ranks at once contend: slower at 8 GPUs)
        self.partials_via = "copy"
        # "h back" (peer transport): receivers return each slot's NVFP4 h (F/2 + F/16 bytes)
        # instead of bf16 partial sums (2d bytes per row), and every rank runs the down
        # projection of its own tokens with all experts' down weights (``down_experts``,
        # all E experts; set by ``from_dense``): 2.7x fewer bytes back at 8 GPUs for the
        # OLMoE shape, h stored straight into the source by the gate/up GEMM, and the
        # output is the single-device layer's bit for bit.  None: partial sums.
        self.down_experts: nn.ModuleList | None = None

    @classmethod
    def from_dense(cls, moe: nn.Module, group: dist.ProcessGroup | None = None, ops: Any = None,
                   transport: str = "auto", chunks: int = 0) -> "ExpertParallelMoE":
        """Shard a single-device layer (this package's or the reference's SparseMoE):
        the router is shared, this rank keeps its block of experts."""
        variant = [name for name, on in (
            ("mitotic twin routing", bool(getattr(moe, "mitotic_pairs", None))),
            ("lineage family routing", getattr(moe, "lineage_top_families", 0) > 0
             and getattr(moe, "lineage_root_ids", None) is not None),
            ("dense expert subsets", bool(getattr(moe, "dense_expert_indices", ()))
             or getattr(moe, "dense_subset_k", 0) > 0),
            ("the recurrent coverage penalty", getattr(moe, "recurrent_coverage_penalty", 0.0) > 0.0),
            ("sequence-diversity / mitotic-orthogonality losses", getattr(moe, "sequence_diversity_coef", 0.0) > 0.0
             or getattr(moe, "mitotic_ortho_coef", 0.0) > 0.0)) if on]
        if variant:
            raise NotImplementedError(f"the expert-parallel layer routes plain top-k only; this layer uses {variant[0]}")
        E = len(moe.experts)
        cfg = type("Cfg", (), dict(d_model=moe.router.in_features, num_experts=E,
                                   expert_hidden_dim=moe.experts[0].down_proj.in_features, top_k=moe.top_k,
                                   norm_topk_prob=moe.norm_topk_prob))()
        mod = cls(cfg, group, ops, transport, chunks)
        mod.router = moe.router
        lo = mod.expert_offset
        mod.experts = nn.ModuleList(list(moe.experts)[lo:lo + mod.experts_per_rank])
        mod.down_experts = nn.ModuleList(list(moe.experts))
        mod.router_logit_bias = getattr(moe, "router_logit_bias", None)
        return mod

    @torch.no_grad()
    def reshard(self, router: nn.Linear, old_to_new, *, parents: dict | None = None,
                new_experts: dict | None = None, dense_experts: nn.ModuleList | None = None) -> dict:
        """Follow a change of the expert set between calls (ExpertLifecycle's
        ``grow_experts`` / ``prune_experts``, src/mcl4_coe/ornith_rl.py:468-595, and the
        trainer's in-place mitosis, src/mcl4_coe/trainer.py:1624-1712) while the experts
        stay sharded: rank g owns ``[g*E'/G, (g+1)*E'/G)`` of the new count E'.

        Every rank calls it with the same arguments (it is a collective):
        ``router``: the new replicated router (E' rows);
        ``old_to_new[i]``: the new index of old expert i, or None if it was pruned (the
        ``ExpertMorphResult.old_to_new`` of the reference);
        ``parents[j] = p``: new expert j is a copy of old expert p (mitosis);
        ``new_experts[j]``: a module (``up_proj`` / ``down_proj``) for a new expert that
        is neither kept nor copied, given on every rank;
        ``dense_experts``: all E' experts of the changed dense layer, for the "h back"
        exchange (every rank runs the down projection of its own tokens); without it the
        layer returns partial sums.
        Experts whose owner changes travel to their new rank with their weights and, on
        CUDA, their NVFP4 bytes (one all-to-all); a copy takes its parent's bytes; only
        the ``new_experts`` are quantised (by the next forward).  Experts that keep their
        rank keep their modules, and their bytes are carried into the new cache.
        Returns counts of the experts moved, copied and new, and the bytes sent.
        Dense (non-2:4) experts only."""
        G, me = self.world, self.rank
        E_old, loc_old = self.num_experts, self.experts_per_rank
        E_new = int(router.weight.shape[0])
        parents, fresh = dict(parents or {}), dict(new_experts or {})
        if len(old_to_new) != E_old:
            raise ValueError(f"old_to_new must have one entry per current expert ({E_old})")
        if E_new % G != 0 or E_new < self.top_k:
            raise ValueError(f"the new expert count {E_new} must be a multiple of the group size {G} and >= top_k")
        src: list = [None] * E_new  # old index of the expert (or its parent) that new slot j holds; -1: new
        for i, j in enumerate(old_to_new):
            if j is None:
                continue
            if not 0 <= int(j) < E_new or src[int(j)] is not None:
                raise ValueError(f"old_to_new[{i}] = {j} is out of range or taken twice")
            src[int(j)] = i
        for j, par in parents.items():
            if not 0 <= j < E_new or src[j] is not None or not 0 <= par < E_old:
                raise ValueError(f"parents[{j}] = {par} is out of range or collides")
            src[j] = int(par)
        for j in fresh:
            if not 0 <= j < E_new or src[j] is not None:
                raise ValueError(f"new_experts[{j}] is out of range or collides")
            src[j] = -1
        if any(v is None for v in src):
            raise ValueError("every new expert index needs a kept expert, a parent or a new module")
        for ex in self.experts:
            for proj in (ex.up_proj, ex.down_proj):
                if str(getattr(proj, "sparsity_mode", "none")) != "none":
                    raise NotImplementedError("resharding 2:4-sparse experts")
        loc_new = E_new // G
        owner_old = lambda i: i // loc_old  # noqa: E731
        owner_new = lambda j: j // loc_new  # noqa: E731
        ex0 = self.experts[0]
        dev, wdtype = ex0.up_proj.weight.device, ex0.up_proj.weight.dtype
        d, F = ex0.down_proj.weight.shape
        move_bytes = hasattr(self.ops, "prepare")  # the CUDA steps keep NVFP4 caches; bring them along
        caches = self.ops.prepare(self.experts) if move_bytes else None  # refreshed: bytes of current weights

        def payload(li: int) -> list[Tensor]:
            ex = self.experts[li]
            parts = [ex.up_proj.weight.detach(), ex.down_proj.weight.detach()]
            if move_bytes:
                for c in caches:
                    parts += [c.packed[li], c.scales[li], c.g[li:li + 1]]
            return [t.contiguous().view(torch.uint8).reshape(-1) for t in parts]

        sizes = [t.numel() for t in payload(0)]  # the same on every rank (same shapes)
        per = sum(sizes)
        moving = [j for j in range(E_new) if src[j] >= 0 and owner_old(src[j]) != owner_new(j)]
        send_js = [[j for j in moving if owner_old(src[j]) == me and owner_new(j) == r] for r in range(G)]
        recv_js = [[j for j in moving if owner_new(j) == me and owner_old(src[j]) == s_] for s_ in range(G)]
        received: dict[int, list[Tensor]] = {}
        sent = sum(len(js) for js in send_js) * per
        if moving:  # the same decision on every rank: all of them enter the all-to-all
            pieces = [torch.cat(payload(src[j] - me * loc_old)) for r in range(G) for j in send_js[r]]
            send = torch.cat(pieces) if pieces else torch.empty((0,), dtype=torch.uint8, device=dev)
            recv = torch.empty((sum(len(js) for js in recv_js) * per,), dtype=torch.uint8, device=dev)
            dist.all_to_all_single(recv, send, [len(js) * per for js in recv_js], [len(js) * per for js in send_js],
                                   group=self.group)
            off = 0
            for s_ in range(G):
                for j in recv_js[s_]:
                    chunk, parts = recv[off:off + per], []
                    o = 0
                    for n in sizes:
                        parts.append(chunk[o:o + n])
                        o += n
                    received[j] = parts
                    off += per

        def module_from(up_bytes: Tensor, dn_bytes: Tensor) -> nn.Module:
            ex = SwiGLUExpert(d, F).to(device=dev, dtype=wdtype)
            ex.up_proj.weight.copy_(up_bytes.view(wdtype).view(2 * F, d))
            ex.down_proj.weight.copy_(dn_bytes.view(wdtype).view(d, F))
            return ex

        new_list, filled_up, filled_dn = [], {}, {}
        stats = dict(moved_in=0, copied=0, kept=0, new=0, bytes_sent=sent)
        for li in range(loc_new):
            j = me * loc_new + li
            i = src[j]
            if i < 0:
                new_list.append(fresh[j].to(dev))
                stats["new"] += 1
                continue
            if owner_old(i) == me:
                lo = i - me * loc_old
                if old_to_new[i] is not None and int(old_to_new[i]) == j:
                    new_list.append(self.experts[lo])  # same module: its bytes are carried over
                    stats["kept"] += 1
                    continue
                parts = payload(lo)  # a copy of a local parent
                stats["copied"] += 1
            else:
                parts = received[j]
                stats["moved_in"] += 1
            new_list.append(module_from(parts[0], parts[1]))
            if move_bytes:  # (packed, scales, g) as bytes; g back to its fp32 value
                filled_up[li] = (parts[2], parts[3], parts[4].view(torch.float32))
                filled_dn[li] = (parts[5], parts[6], parts[7].view(torch.float32))
        experts = nn.ModuleList(new_list)
        if move_bytes:
            seed_grouped_cache(experts, "up_proj", filled_up)
            seed_grouped_cache(experts, "down_proj", filled_dn)
        self.router = router
        self.experts = experts
        self.num_experts = E_new
        self.experts_per_rank = loc_new
        self.expert_offset = me * loc_new
        self.down_experts = dense_experts
        return stats

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
        use_peer = self.transport == "peer" or (
            self.transport == "auto" and xb.is_cuda and dist.get_backend(self.group) == "nccl")
        if use_peer and self.down_experts is not None and hasattr(self.ops, "gateup_to_peers"):
            return self._forward_h_back(x, xb, wr, bias, vmask, mark)
        caches = self.ops.prepare(self.experts) if hasattr(self.ops, "prepare") else None
        idx, w, stats = self.ops.route(xb, wr, bias, vmask, k, self.norm_topk_prob)
        mark(1)
        bounds = self._chunk_bounds(T)
        out = torch.empty((T, d), dtype=torch.bfloat16, device=xb.device)
        if use_peer:
            disp, backs = self._exchange_peer(xb, idx, w, vmask, bounds, caches, mark)
        else:
            disp = []
            for c, (lo, hi) in enumerate(bounds):
                vm = None if vmask is None else vmask[lo:hi]
                disp.append(self.ops.dispatch(xb[lo:hi], idx[lo:hi], w[lo:hi], vm, G, E_loc, c))
            mark(2)
            backs = self._exchange_collective(disp, d, k, caches, mark)
        mark(6)
        for c, (lo, hi) in enumerate(bounds):
            self.ops.combine(backs[c], disp[c][2], hi - lo, d, G, out[lo:hi])
        mark(7)
        return out.to(x.dtype).view_as(x), stats[0], stats[1], stats[3:3 + self.num_experts]

    def _forward_h_back(self, x: Tensor, xb: Tensor, wr: Tensor, bias: Tensor | None, vmask: Tensor | None,
                        mark) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        """Peer transport, "h back": route and lay out this rank's slots; rows out per
        chunk (the rows of chunk c+1 travel while the receivers' gate/up GEMMs of chunk c
        run and store each slot's NVFP4 h straight into its source's layout); a
        one-element all-reduce orders every rank after every rank's stores; down
        projection and combine of this rank's tokens (the single-device kernels)."""
        T, d = xb.shape
        G, me, k, E = self.world, self.rank, self.top_k, self.num_experts
        E_loc = self.experts_per_rank
        F = self.experts[0].down_proj.weight.shape[1]
        dev = xb.device
        lib = _lib.load()
        up = get_or_build_grouped_cache(self.experts, "up_proj")
        dn_all = get_or_build_grouped_cache(self.down_experts, "down_proj")
        st = self.ops.layout(xb, wr, bias, vmask, k, self.norm_topk_prob, dn_all, F)
        idx, stats = st["idx"], st["stats"]
        mark(1)
        if self._peer is None:
            self._peer = PeerExchange(self.group, dev)
        px = self._peer
        bounds = self._chunk_bounds(T)
        n = len(bounds)
        vm = (lambda lo, hi: None) if vmask is None else (lambda lo, hi: vmask[lo:hi])
        cnts = torch.empty((n, 2 * G + 1), dtype=torch.int32, device=dev)
        for c, (lo, hi) in enumerate(bounds):
            self.ops.dispatch_count(idx[lo:hi], vm(lo, hi), G, E_loc, c, out=cnts[c, :2 * G])
        host, arrived = self._counts_tab(cnts, bounds)
        disp = [self.ops.dispatch_pack_h(xb[lo:hi], idx[lo:hi], vm(lo, hi), G, E_loc, me, st["slot_pos"][lo:hi],
                                         cnts[c, :2 * G], c)
                for c, (lo, hi) in enumerate(bounds)]
        mark(2)
        arrived.synchronize()
        tab = host.view(G, n, 2 * G + 1).tolist()
        mark(3)
        rb = disp[0][0].shape[1]
        t_tot = [sum(tab[s][c][2 * G] for c in range(n)) for s in range(G)]
        mcap_max = max(lib.mcl4moe_padded_rows(t, E, k) for t in t_tot)
        sizes = {"hq": mcap_max * (F // 2), "hs": mcap_max * (F // 16)}
        for c in range(n):
            t_max = max(tab[s][c][2 * G] for s in range(G))
            sizes[f"rows{c}"] = G * t_max * rb
        px.reserve(sizes)
        ex = dict(rows_to=[0] * G, rows_from=[0] * G, slots=[0])
        for c in range(n):
            ex["rows_to"] = [a + tab[me][c][g] for a, g in zip(ex["rows_to"], range(G))]
            ex["rows_from"] = [a + tab[s][c][me] for a, s in zip(ex["rows_from"], range(G))]
            ex["slots"][0] += sum(tab[s][c][G + me] for s in range(G))
        self.last_exchange = ex

        def rows_pieces(c):
            base = disp[c][0].data_ptr()
            return [(g, base + src * rb, cnt * rb, dst * rb) for g, src, cnt, dst in row_plan(tab, c, me)]

        hq_dst = [px.address(s, "hq") for s in range(G)]
        hs_dst = [px.address(s, "hs") for s in range(G)]
        px.complete(px.issue("rows0", rows_pieces(0)))
        mark(4)
        for c in range(n):
            nxt = px.issue(f"rows{c + 1}", rows_pieces(c + 1)) if c + 1 < n else None
            R = sum(tab[s][c][me] for s in range(G))
            slots_here = sum(tab[s][c][G + me] for s in range(G))
            if R > 0:
                recv = px.local(f"rows{c}", R * rb).view(R, rb)
                self.ops.gateup_to_peers(recv, R, slots_here, d, k, self.experts, hq_dst, hs_dst, up)
            if nxt is not None:
                px.complete(nxt)
        mark(5)
        px.complete([])  # every rank's h stores into this rank's layout are done
        mark(6)
        mcap = lib.mcl4moe_padded_rows(T, E, k)
        out = self.ops.down(st, px.local("hq", mcap * (F // 2)), px.local("hs", mcap * (F // 16)))
        mark(7)
        return out.to(x.dtype).view_as(x), stats[0], stats[1], stats[3:3 + E]

    def _chunk_bounds(self, T: int) -> list[tuple[int, int]]:
        """Token ranges of the chunks (``chunk_weights`` or ``chunks`` equal parts); one
        chunk when a chunk would hold fewer than ``min_chunk_tokens`` tokens."""
        weights = self.chunk_weights or [1.0] * max(1, self.chunks)
        if T <= 0 or T < len(weights) * self.min_chunk_tokens:
            if T <= 0 or T < 2 * self.min_chunk_tokens:
                return [(0, max(T, 0))]
            weights = [1.0] * (T // self.min_chunk_tokens)
        total, acc, cuts = float(sum(weights)), 0.0, [0]
        for wgt in weights[:-1]:
            acc += wgt
            cuts.append(int(round(T * acc / total)))
        cuts.append(T)
        return [(lo, hi) for lo, hi in zip(cuts[:-1], cuts[1:])]

    def _experts(self, recv: Tensor, R: int, slots: int, d: int, k: int, caches) -> Tensor:
        if caches is None:
            return self.ops.experts(recv, R, slots, d, k, self.experts)
        return self.ops.experts(recv, R, slots, d, k, self.experts, caches)

    def _exchange_collective(self, disp: list, d: int, k: int, caches, mark) -> list[Tensor]:
        """Rows out and partial sums back through ``all_to_all_single``, chunk after chunk."""
        G = self.world
        backs, ex = [], dict(rows_to=[0] * G, rows_from=[0] * G, slots=[0])
        for send, counts, _ in disp:
            # row and slot counts: [G, 2] per rank, one entry pair per destination
            send_tab = torch.stack([counts[:G], counts[G:]], dim=1).contiguous()
            recv_tab = torch.empty_like(send_tab)
            self._all_to_all(recv_tab, send_tab, [1] * G, [1] * G)
            tab = torch.cat([send_tab, recv_tab], dim=0).cpu()  # the split sizes are needed on the host
            rows_to = tab[:G, 0].tolist()
            rows_from = tab[G:, 0].tolist()
            slots_here = int(tab[G:, 1].sum())
            R = int(sum(rows_from))
            sent = sum(rows_to)
            recv = torch.empty((R, send.shape[1]), dtype=torch.uint8, device=send.device)
            self._all_to_all(recv, send[:sent], rows_from, rows_to)
            partial = self._experts(recv, R, slots_here, d, k, caches)
            back = torch.empty((sent, d), dtype=torch.bfloat16, device=partial.device)
            self._all_to_all(back, partial, rows_to, rows_from)
            backs.append(back)
            ex = dict(rows_to=[a + b for a, b in zip(ex["rows_to"], rows_to)],
                      rows_from=[a + b for a, b in zip(ex["rows_from"], rows_from)], slots=[ex["slots"][0] + slots_here])
        self.last_exchange = ex
        mark(3)
        mark(4)
        mark(5)
        return backs

    def _counts_tab(self, cnts: Tensor, bounds: list) -> tuple[Tensor, Any]:
        """All-gather every rank's per-chunk counts and chunk sizes and start their
        copy to pinned host memory; returns the host buffer and the event that marks
        its arrival, so the rows can be packed while the host waits."""
        G, n = self.world, len(bounds)
        dev = cnts.device
        key = (tuple(bounds), str(dev))
        if getattr(self, "_sizes_key", None) != key:
            self._sizes_dev = torch.tensor([hi - lo for lo, hi in bounds], dtype=torch.int32, device=dev)
            self._sizes_key = key
        cnts[:, 2 * G].copy_(self._sizes_dev)
        allc = torch.empty((G * n * (2 * G + 1),), dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(allc, cnts.view(-1), group=self.group)
        host = getattr(self, "_tab_host", None)
        if host is None or host.numel() < allc.numel():
            host = torch.empty((allc.numel(),), dtype=torch.int32, pin_memory=True)
            self._tab_host = host
        host = host[: allc.numel()]
        host.copy_(allc, non_blocking=True)
        arrived = torch.cuda.Event()
        arrived.record()
        return host, arrived

    def _exchange_peer(self, xb: Tensor, idx: Tensor, w: Tensor, vmask: Tensor | None, bounds: list, caches,
                       mark) -> tuple[list, list[Tensor]]:
        """Dispatch, rows out and partial sums back through peer memory (copy
        engines), the exchange of one chunk overlapping the experts step of another.

        The chunks' row / slot counts are counted first and exchanged; the host
        reads them (it needs the copy sizes) while the rows are packed."""
        G, me, n = self.world, self.rank, len(bounds)
        T, d = xb.shape
        k, E_loc = idx.shape[1], self.experts_per_rank
        dev = xb.device
        if self._peer is None:
            self._peer = PeerExchange(self.group, dev)
        px = self._peer
        vm = (lambda lo, hi: None) if vmask is None else (lambda lo, hi: vmask[lo:hi])
        cnts = torch.empty((n, 2 * G + 1), dtype=torch.int32, device=dev)
        if hasattr(self.ops, "dispatch_count"):
            for c, (lo, hi) in enumerate(bounds):
                self.ops.dispatch_count(idx[lo:hi], vm(lo, hi), G, E_loc, c, out=cnts[c, :2 * G])
            host, arrived = self._counts_tab(cnts, bounds)
            disp = [self.ops.dispatch_pack(xb[lo:hi], idx[lo:hi], w[lo:hi], vm(lo, hi), G, E_loc, cnts[c, :2 * G], c)
                    for c, (lo, hi) in enumerate(bounds)]
        else:
            disp = [self.ops.dispatch(xb[lo:hi], idx[lo:hi], w[lo:hi], vm(lo, hi), G, E_loc, c)
                    for c, (lo, hi) in enumerate(bounds)]
            for c in range(n):
                cnts[c, :2 * G].copy_(disp[c][1])
            host, arrived = self._counts_tab(cnts, bounds)
        mark(2)
        arrived.synchronize()
        tab = host.view(G, n, 2 * G + 1).tolist()
        mark(3)
        rb = disp[0][0].shape[1]
        sizes = {}
        for c in range(n):
            t_max = max(tab[s][c][2 * G] for s in range(G))
            sizes[f"rows{c}"] = G * t_max * rb
            sizes[f"back{c}"] = G * t_max * d * 2
        px.reserve(sizes)
        ex = dict(rows_to=[0] * G, rows_from=[0] * G, slots=[0])
        for c in range(n):
            ex["rows_to"] = [a + tab[me][c][g] for a, g in zip(ex["rows_to"], range(G))]
            ex["rows_from"] = [a + tab[s][c][me] for a, s in zip(ex["rows_from"], range(G))]
            ex["slots"][0] += sum(tab[s][c][G + me] for s in range(G))
        self.last_exchange = ex

        def rows_pieces(c):
            base = disp[c][0].data_ptr()
            return [(g, base + src * rb, n * rb, dst * rb) for g, src, n, dst in row_plan(tab, c, me)]

        def back_pieces(c, partial):
            base = partial.data_ptr()
            return [(s, base + src * d * 2, n * d * 2, dst * d * 2) for s, src, n, dst in back_plan(tab, c, me)]

        px.complete(px.issue("rows0", rows_pieces(0)))
        mark(4)
        back_events, partials = [], []  # the partial tensors stay referenced until their copies are complete
        for c in range(n):
            nxt = px.issue(f"rows{c + 1}", rows_pieces(c + 1)) if c + 1 < n else None
            R = sum(tab[s][c][me] for s in range(G))
            slots_here = sum(tab[s][c][G + me] for s in range(G))
            recv = px.local(f"rows{c}", R * rb).view(R, rb)
            if self.partials_via == "kernel" and hasattr(self.ops, "experts_to_peers"):
                # partial sums stored over NVLink by the kernel that computes them
                seg = [0]
                for s in range(G):
                    seg.append(seg[-1] + tab[s][c][me])
                dst = [px.address(s, f"back{c}", sum(tab[s][c][g] for g in range(me)) * d * 2) for s in range(G)]
                self.ops.experts_to_peers(recv, R, slots_here, d, k, self.experts, seg, dst, caches)
            else:
                partial = self._experts(recv, R, slots_here, d, k, caches)
                partials.append(partial)
                back_events += px.issue(f"back{c}", back_pieces(c, partial), lane=1)
            if nxt is not None:
                px.complete(nxt)
        mark(5)
        px.complete(back_events)
        del partials
        backs = []
        for c in range(n):
            sent = sum(tab[me][c][g] for g in range(G))
            backs.append(px.local(f"back{c}", sent * d * 2).view(torch.bfloat16).view(sent, d))
        return disp, backs
