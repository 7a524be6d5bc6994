"""Drop-in ``SparseMoE`` for the MCL4-CED backbone, running on the B200 kernels.

Keeps the reference module's constructor, parameter names and forward
signature (src/mcl4_coe/backbone.py:190-626):

    SparseMoE(config)                       # reads d_model, num_experts, top_k,
                                            # expert_hidden_dim, norm_topk_prob, ...
    .router                nn.Linear(d_model, E, bias=False)   (fp32 routing)
    .experts[i].up_proj    nn.Linear(d_model, 2F)  gate rows first
    .experts[i].down_proj  nn.Linear(F, d_model)
    .num_experts, .top_k, .norm_topk_prob, .mitotic_pairs, .last_selected_mask
    forward(x, valid=None, *, prior_expert_mask=None, dense_expert_indices=None,
            dense_subset_k=None) -> (out, aux_loss, router_z_loss, counts)

so a checkpoint's ``state_dict`` loads unchanged and ExpertLifecycle
(``grow_experts`` / ``prune_experts``, src/mcl4_coe/ornith_rl.py:468-595, and
the trainer's in-place mitosis, src/mcl4_coe/trainer.py:1624-1712) can
replace ``experts`` / ``router`` and change ``num_experts`` between calls: the
NVFP4 weight cache is keyed by the expert count, shapes and weight versions.

The whole forward is one call into ``libmcl4moe.so``
(``mcl4moe_moe_forward``): router + top-k + statistics, stable expert-major
permutation with NVFP4 activation quantisation, tcgen05 grouped gate/up GEMM
with fused SwiGLU and re-quantisation, tcgen05 grouped down GEMM with the
routing weight, and the k-way combine.  ``valid`` follows the reference's loop
branch (src/mcl4_coe/backbone.py:913-1047): masked tokens are not routed and
get zero output and a zero ``last_selected_mask`` row.

Routing variants (mitotic twins, lineage families, recurrent coverage
penalty, dense subsets with an optional sparse remainder, the sequence-diversity
and mitotic-orthogonality losses) compute the reference's selection on the
library's router logits (``routing_variants.py``) and run the experts through
``mcl4moe_moe_forward_routed``.

Training: under autograd (plain top-k routing) the forward keeps the gate / value
rows, the permuted bf16 inputs, h and the unweighted down-projection rows, and the
backward runs the reference's _NVFP4GroupedLinear.backward path
(src/mcl4_coe/nvfp4.py:1112-1216) on the library: stochastic-rounded NVFP4
gradients into grouped NVFP4 input-gradient GEMMs on the transposed weights, the
SwiGLU and routing derivatives, and bf16-operand weight gradients.  Routing
variants run forward only (``NotImplementedError`` under autograd).
"""

from __future__ import annotations

import ctypes
import random
from dataclasses import dataclass
from typing import Any, Sequence

import torch
from torch import Tensor, nn

from . import _lib
from .nvfp4 import _stream_handle, get_or_build_grouped_cache, invalidate_cache, nvfp4_grouped_linear


@dataclass
class MoEConfig:
    """The MoE fields of the reference's ``MCL4CEDConfig`` (src/mcl4_coe/backbone.py:35-77)."""

    d_model: int = 256
    expert_hidden_dim: int = 512
    num_experts: int = 4
    top_k: int = 2
    norm_topk_prob: bool = True
    aux_loss_coef: float = 0.01
    router_z_loss_coef: float = 0.001
    recurrent_coverage_penalty: float = 0.0
    mitotic_ortho_coef: float = 0.0
    sequence_diversity_coef: float = 0.0
    dense_expert_indices: tuple[int, ...] = ()
    dense_subset_k: int = 0
    combine_dense_and_sparse: bool = False

    def __post_init__(self) -> None:  # src/mcl4_coe/backbone.py:84-108
        for name in ("d_model", "expert_hidden_dim", "num_experts", "top_k"):
            val = getattr(self, name)
            if isinstance(val, bool) or not isinstance(val, int) or val <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if self.top_k > self.num_experts:
            raise ValueError("top_k cannot exceed num_experts")


def _opt_ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class SwiGLUExpert(nn.Module):
    """src/mcl4_coe/backbone.py:179-187 (parameters only; the math runs in the grouped kernels)."""

    def __init__(self, d_model: int, hidden_dim: int) -> None:
        super().__init__()
        self.up_proj = nn.Linear(d_model, 2 * hidden_dim, bias=False)
        self.down_proj = nn.Linear(hidden_dim, d_model, bias=False)


class SparseMoE(nn.Module):
    """Dropless top-k SwiGLU MoE with fp32 routing, NVFP4 experts on B200."""

    def __init__(self, config: Any) -> None:
        super().__init__()
        self.num_experts = int(config.num_experts)
        self.top_k = int(config.top_k)
        self.norm_topk_prob = bool(getattr(config, "norm_topk_prob", True))
        self.recurrent_coverage_penalty = float(getattr(config, "recurrent_coverage_penalty", 0.0))
        self.mitotic_ortho_coef = float(getattr(config, "mitotic_ortho_coef", 0.0))
        self.sequence_diversity_coef = float(getattr(config, "sequence_diversity_coef", 0.0))
        self.dense_expert_indices: tuple[int, ...] = tuple(int(i) for i in getattr(config, "dense_expert_indices", ()))
        self.dense_subset_k = int(getattr(config, "dense_subset_k", 0))
        self.combine_dense_and_sparse = bool(getattr(config, "combine_dense_and_sparse", False))
        d_model = int(config.d_model)
        hidden = int(config.expert_hidden_dim)
        self.router = nn.Linear(d_model, self.num_experts, bias=False)
        self.experts = nn.ModuleList(SwiGLUExpert(d_model, hidden) for _ in range(self.num_experts))
        self.mitotic_pairs: list[tuple[int, int]] = []
        self.last_selected_mask: Tensor | None = None
        self.lineage_num_roots = 0
        self.lineage_top_families = 0
        self.lineage_child_share = 0.25
        self.lineage_root_ids: Tensor | None = None
        self.lineage_logit_prior: Tensor | None = None
        # Optional additive router bias [E] (not in the reference module; the
        # benchmark's skewed configuration injects one in front of the softmax).
        self.router_logit_bias: Tensor | None = None
        self.debug_capture_h = False  # keep the SwiGLU output of the last call (tests)
        # Optional 6 torch.cuda.Event (already recorded once, so their handles
        # exist) recorded at the stage boundaries of the next forward calls.
        self.stage_events: Sequence[torch.cuda.Event] | None = None
        self.last_h: Tensor | None = None
        self._ws: Tensor | None = None
        self._ws_key: tuple | None = None
        self._graphs: dict | None = None  # CUDA-graph replay (enable_cuda_graph)

    @torch.no_grad()
    def configure_lineage_family_routing(self, num_roots: int = 64, *, top_families: int = 8,
                                         child_share: float = 0.25) -> None:
        """Root-anchored expert families for lineage routing (src/mcl4_coe/backbone.py:231-271):
        each expert after the first ``num_roots`` joins the root whose up_proj weight is
        most cosine-similar; a root keeps ``1 - child_share`` of its family's prior mass
        and its descendants share the rest.  Out-of-range arguments switch it off."""
        E = len(self.experts)
        if num_roots <= 0 or top_families <= 0 or num_roots >= E:
            self.lineage_num_roots = self.lineage_top_families = 0
            self.lineage_root_ids = self.lineage_logit_prior = None
            return
        dev = self.router.weight.device
        ups = torch.nn.functional.normalize(
            torch.stack([e.up_proj.weight.detach().float().reshape(-1) for e in self.experts]), p=2.0, dim=-1,
            eps=1e-8)
        parent = (ups[num_roots:] @ ups[:num_roots].T).argmax(dim=-1)
        root_ids = torch.cat([torch.arange(num_roots, dtype=torch.long, device=dev), parent.to(dev)])
        family_size = torch.bincount(root_ids, minlength=num_roots).tolist()
        share = float(max(0.0, min(0.95, child_share)))
        prior = torch.ones(E, dtype=torch.float32, device=dev)
        for e, r in enumerate(root_ids.tolist()):
            if family_size[r] > 1:
                prior[e] = max(1e-6, 1.0 - share) if e < num_roots else max(1e-6, share / float(family_size[r] - 1))
        self.lineage_num_roots = int(num_roots)
        self.lineage_top_families = int(min(top_families, num_roots))
        self.lineage_child_share = share
        self.lineage_root_ids = root_ids
        self.lineage_logit_prior = torch.log(prior)

    def enable_cuda_graph(self, enabled: bool = True) -> None:
        """Serve repeated calls of one shape from a captured CUDA graph.

        The first call per (tokens, mask, bias, device) captures the whole layer
        forward (one library call) with static input and output buffers; later calls
        copy x in, replay the graph and return copies of the outputs, which removes
        the per-call host work (weight-cache checks, argument set-up, kernel launches)
        that dominates small decode batches.  While enabled the weights are not
        re-checked per call: call ``enable_cuda_graph()`` again after changing them
        (or growing / pruning experts) to capture afresh.  Forward only; no
        ``forward_details``.
        """
        self._graphs = {} if enabled else None

    def _graph_forward(self, flat: Tensor, valid: Tensor | None, x_shape, x_dtype):
        T, d = flat.shape
        dev = flat.device
        bias = self.router_logit_bias
        key = (T, d, str(dev), valid is not None, bias is not None)
        ent = self._graphs.get(key)
        if ent is None:
            ent = {"x": torch.empty((T, d), dtype=torch.bfloat16, device=dev),
                   "valid": None if valid is None else torch.empty((T,), dtype=torch.uint8, device=dev)}
            ent["x"].copy_(flat)
            if valid is not None:
                ent["valid"].copy_(valid.reshape(-1))
            # eager call first: builds the weight caches and sizes the workspace
            self._forward_impl(ent["x"], ent["valid"], None, None, None, details=False, static=ent)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._forward_impl(ent["x"], ent["valid"], None, None, None, details=False, static=ent)
            ent["graph"] = g
            self._graphs[key] = ent
        ent["x"].copy_(flat)
        if valid is not None:
            ent["valid"].copy_(valid.reshape(-1).to(torch.uint8))
        ent["graph"].replay()
        E = len(self.experts)
        self.last_selected_mask = ent["sel"].clone().view(*x_shape[:-1], E)
        stats = ent["stats"].clone()
        out = ent["out"].to(x_dtype).view(x_shape) if x_dtype != torch.bfloat16 else ent["out"].clone().view(x_shape)
        return out, stats[0], stats[1], stats[3:3 + E]

    @classmethod
    def from_reference(cls, ref: nn.Module) -> "SparseMoE":
        """Build from a reference ``SparseMoE`` instance, sharing its parameters."""
        cfg = MoEConfig(d_model=ref.router.in_features, expert_hidden_dim=ref.experts[0].down_proj.in_features,
                        num_experts=ref.num_experts, top_k=ref.top_k, norm_topk_prob=ref.norm_topk_prob)
        mod = cls(cfg)
        mod.router = ref.router
        mod.experts = ref.experts
        mod.mitotic_pairs = list(getattr(ref, "mitotic_pairs", []))
        return mod

    # ------------------------------------------------------------------ helpers
    def _routing_variant(self, prior_expert_mask, dense_expert_indices, dense_subset_k) -> str | None:
        """Which routing variant this call needs (None: plain top-k, served by one library call)."""
        if dense_expert_indices is not None and len(dense_expert_indices) > 0:
            return "dense"
        if self.dense_expert_indices or int(self.dense_subset_k if dense_subset_k is None else dense_subset_k) > 0:
            return "dense"
        if (self.mitotic_pairs or (self.lineage_top_families > 0 and self.lineage_root_ids is not None)
                or (prior_expert_mask is not None and self.recurrent_coverage_penalty > 0.0)
                or self.sequence_diversity_coef > 0.0 or self.mitotic_ortho_coef > 0.0):
            return "sparse"
        return None

    def _workspace(self, T: int, d: int, E: int, k: int, F: int, device: torch.device) -> Tensor:
        key = (T, d, E, k, F, str(device))
        if self._ws is None or self._ws_key != key:
            nbytes = _lib.load().mcl4moe_moe_workspace_size(T, d, E, k, F)
            if nbytes == 0 and T > 0:
                raise ValueError(f"unsupported MoE shape T={T} d={d} E={E} k={k} F={F}")
            self._ws = torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=device)
            self._ws_key = key
        return self._ws

    def _run_grouped_experts(self, gx: Tensor, offs: Tensor) -> Tensor:
        """The reference's operator seam (src/mcl4_coe/backbone.py:569-577)."""
        up = nvfp4_grouped_linear(gx.to(torch.bfloat16), self.experts, "up_proj", offs)
        gate, val = up.chunk(2, dim=-1)
        return nvfp4_grouped_linear(torch.nn.functional.silu(gate) * val, self.experts, "down_proj", offs)

    # ------------------------------------------------------------------ forward
    def forward(self, x: Tensor, valid: Tensor | None = None, *, prior_expert_mask: Tensor | None = None,
                dense_expert_indices: Sequence[int] | Tensor | None = None,
                dense_subset_k: int | None = None) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        if (self._graphs is not None and x.is_cuda and not torch.is_grad_enabled()
                and self._routing_variant(prior_expert_mask, dense_expert_indices, dense_subset_k) is None):
            return self._graph_forward(x.reshape(-1, x.shape[-1]).to(torch.bfloat16), valid, x.shape, x.dtype)
        r = self._forward_impl(x, valid, prior_expert_mask, dense_expert_indices, dense_subset_k, details=False)
        return r["out"], r["aux_loss"], r["router_z_loss"], r["counts"]

    @torch.no_grad()
    def forward_details(self, x: Tensor, valid: Tensor | None = None, *,
                        quant_bytes: bool = False) -> dict[str, Tensor]:
        """Forward plus the routing internals: ``topk_idx``/``topk_w`` [T, k]
        (-1 / 0 for masked tokens), ``offs`` [E] (inclusive ends), ``perm``
        [n_routed*k] (flat slot ids t*k+j in stable expert-major order) and,
        when ``debug_capture_h`` is set, ``h`` (bf16 SwiGLU output in padded
        expert-major rows) and ``pad_start`` [E+1].  With ``quant_bytes`` also
        the first GEMM's NVFP4 operand as the permute kernel wrote it:
        ``xq`` [M, d/2] codes and ``xs`` [M, d/16] E4M3 scales (row-major) of
        the M padded expert-major rows, ``slot_pos`` [T, k] (padded row of each
        slot, -1 for masked tokens) and ``pad_start``."""
        return self._forward_impl(x, valid, None, None, None, details="quant" if quant_bytes else True)

    def _forward_impl(self, x, valid, prior_expert_mask, dense_expert_indices, dense_subset_k, details, static=None):
        flat = x.reshape(-1, x.shape[-1])
        if flat.device.type != "cuda":
            raise ValueError("SparseMoE on B200 requires CUDA tensors (there is no CPU fallback)")
        variant = self._routing_variant(prior_expert_mask, dense_expert_indices, dense_subset_k)
        if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())):
            if variant is not None or details or static is not None:
                raise NotImplementedError("training (autograd) runs plain top-k routing through forward() only")
            return self._forward_train(x, valid)
        if variant is not None:
            if details or static is not None:
                raise NotImplementedError("routing variants run through forward() only")
            return self._forward_variant(x, valid, prior_expert_mask, dense_expert_indices, dense_subset_k,
                                         variant)
        E = len(self.experts)
        if self.router.weight.shape[0] != E:
            raise ValueError("router rows must match the number of experts")
        self.num_experts = E
        T, d = flat.shape
        k = self.top_k
        F = self.experts[0].down_proj.weight.shape[1]
        dev = flat.device

        up = get_or_build_grouped_cache(self.experts, "up_proj")
        dn = get_or_build_grouped_cache(self.experts, "down_proj")
        xb = flat.to(torch.bfloat16).contiguous()
        wr = self.router.weight.detach().to(torch.float32).contiguous()
        bias = None
        if self.router_logit_bias is not None:
            bias = self.router_logit_bias.detach().to(device=dev, dtype=torch.float32).contiguous()
            if bias.numel() != E:
                raise ValueError("router_logit_bias must have one entry per expert")
        vmask = None
        if valid is not None:
            vmask = valid.reshape(-1).to(device=dev, dtype=torch.uint8).contiguous()
            if vmask.numel() != T:
                raise ValueError("valid must have one entry per token")

        if static is not None:  # graph capture: fixed output buffers and workspace
            if "out" not in static:
                static["out"] = torch.empty((T, d), dtype=torch.bfloat16, device=dev)
                static["stats"] = torch.empty((3 + E,), dtype=torch.float32, device=dev)
                static["sel"] = torch.empty((T, E), dtype=torch.float32, device=dev)
                static["ws"] = torch.empty((max(_lib.load().mcl4moe_moe_workspace_size(T, d, E, k, F), 256),),
                                           dtype=torch.uint8, device=dev)
            out, stats, sel, ws = static["out"], static["stats"], static["sel"], static["ws"]
        else:
            out = torch.empty((T, d), dtype=torch.bfloat16, device=dev)
            stats = torch.empty((3 + E,), dtype=torch.float32, device=dev)
            sel = torch.empty((T, E), dtype=torch.float32, device=dev)
            ws = self._workspace(T, d, E, k, F, dev)
        extra = {}
        if details:
            extra = dict(topk_idx=torch.empty((T, k), dtype=torch.int32, device=dev),
                         topk_w=torch.empty((T, k), dtype=torch.float32, device=dev),
                         offs=torch.empty((E,), dtype=torch.int32, device=dev),
                         perm=torch.full((max(T * k, 1),), -1, dtype=torch.int32, device=dev))
        h_dbg = None
        if self.debug_capture_h and T > 0:
            h_dbg = torch.zeros((_lib.load().mcl4moe_padded_rows(T, E, k), F), dtype=torch.bfloat16, device=dev)
        args = _lib.MoeArgs(
            x=xb.data_ptr(), router_w=wr.data_ptr(), logit_bias=None if bias is None else bias.data_ptr(),
            valid=None if vmask is None else vmask.data_ptr(),
            w_up=up.packed.data_ptr(), w_up_scales=up.scales.data_ptr(), w_up_g=up.g.data_ptr(),
            w_dn=dn.packed.data_ptr(), w_dn_scales=dn.scales.data_ptr(), w_dn_g=dn.g.data_ptr(),
            T=T, d=d, E=E, k=k, F=F, norm_topk_prob=int(self.norm_topk_prob),
            out=out.data_ptr(), stats=stats.data_ptr(), sel_mask=sel.data_ptr(),
            topk_idx=_opt_ptr(extra.get("topk_idx")), topk_w=_opt_ptr(extra.get("topk_w")),
            offs=_opt_ptr(extra.get("offs")), perm=_opt_ptr(extra.get("perm")),
            h_debug=None if h_dbg is None else h_dbg.data_ptr(), error_word=None,
            workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        if self.stage_events is not None:
            handles = (ctypes.c_void_p * 6)(*[ev.cuda_event for ev in self.stage_events])
            args.stage_events = ctypes.cast(handles, ctypes.POINTER(ctypes.c_void_p))
        _lib.check(_lib.load().mcl4moe_moe_forward(args, _stream_handle()), "mcl4moe_moe_forward")
        self.last_h = h_dbg
        self.last_selected_mask = sel.view(*x.shape[:-1], E)
        res = dict(out=out.to(x.dtype).view_as(x), aux_loss=stats[0], router_z_loss=stats[1],
                   counts=stats[3:3 + E], n_routed=stats[2], sel_mask=sel)
        if details:
            n_routed = int(stats[2].item())
            res.update(extra)
            res["perm"] = extra["perm"][: n_routed * k]
            lib = _lib.load()
            mcap = lib.mcl4moe_padded_rows(T, E, k)

            def region(idx: int, nbytes: int) -> Tensor:
                off = lib.mcl4moe_workspace_region(ws.data_ptr(), idx, T, d, E, k, F) - ws.data_ptr()
                return ws[off:off + nbytes]

            if h_dbg is not None or details == "quant":
                res["pad_start"] = region(5, 4 * (E + 1)).view(torch.int32).clone()
            if h_dbg is not None:
                res["h"] = h_dbg
                res["hq"] = region(2, mcap * F // 2).view(mcap, F // 2).clone()
                res["hs"] = region(3, mcap * F // 16).clone()
            if details == "quant" and T > 0:
                res["xq"] = region(0, mcap * d // 2).view(mcap, d // 2).clone()
                res["xs"] = region(1, mcap * d // 16).view(mcap, d // 16).clone()
                res["slot_pos"] = region(6, 4 * T * k).view(torch.int32).view(T, k).clone()
        return res

    # ------------------------------------------------------------------ training
    def _forward_train(self, x: Tensor, valid: Tensor | None) -> dict:
        """Forward under autograd: the same library forward, which also keeps what the
        backward reads (``_MoETrainFunction``)."""
        E = len(self.experts)
        if self.router.weight.shape[0] != E:
            raise ValueError("router rows must match the number of experts")
        self.num_experts = E
        ups = [e.up_proj.weight for e in self.experts]
        dns = [e.down_proj.weight for e in self.experts]
        out, aux, z, counts = _MoETrainFunction.apply(self, x, valid, self.router.weight, *ups, *dns)
        return dict(out=out, aux_loss=aux, router_z_loss=z, counts=counts)

    # ------------------------------------------------------------------ routing variants
    def _router_logits(self, xb: Tensor, wr: Tensor, bias: Tensor | None) -> Tensor:
        """fp32 router logits [T, E] from the library's router (the same logits its
        top-k uses; the plain top-k it also computes is discarded)."""
        lib = _lib.load()
        T, d = xb.shape
        E, k = wr.shape[0], self.top_k
        dev = xb.device
        logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        idx = torch.empty((max(T, 1), k), dtype=torch.int32, device=dev)
        w = torch.empty((max(T, 1), k), dtype=torch.float32, device=dev)
        counts = torch.empty((E,), dtype=torch.int32, device=dev)
        stats = torch.empty((3 + E,), dtype=torch.float32, device=dev)
        ws = torch.empty((max(lib.mcl4moe_route_workspace_size(T, E, k, d), 256),), dtype=torch.uint8, device=dev)
        _lib.check(lib.mcl4moe_route(xb.data_ptr(), wr.data_ptr(), _opt_ptr(bias), None, None, T, d, E, k,
                                     int(self.norm_topk_prob), idx.data_ptr(), w.data_ptr(), logits.data_ptr(), None,
                                     counts.data_ptr(), stats.data_ptr(), ws.data_ptr(), ws.numel(), _stream_handle()),
                   "mcl4moe_route")
        return logits

    def _forward_routed(self, xb: Tensor, vmask: Tensor | None, idx: Tensor, w: Tensor) -> Tensor:
        """Layer output [T, d] (bf16) for a routing given as expert ids / weights [T, k_eff]
        (``mcl4moe_moe_forward_routed``); rows of masked tokens are zero."""
        T, d = xb.shape
        k_eff = idx.shape[1]
        if not 0 < k_eff <= 32:
            raise NotImplementedError(f"routing with {k_eff} experts per token (the kernels take 1 to 32)")
        E = len(self.experts)
        F = self.experts[0].down_proj.weight.shape[1]
        dev = xb.device
        up = get_or_build_grouped_cache(self.experts, "up_proj")
        dn = get_or_build_grouped_cache(self.experts, "down_proj")
        idx = idx.to(device=dev, dtype=torch.int32).contiguous()
        w = w.to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty((T, d), dtype=torch.bfloat16, device=dev)
        ws = self._workspace(T, d, E, k_eff, F, dev)
        args = _lib.MoeArgs(
            x=xb.data_ptr(), router_w=None, logit_bias=None, valid=_opt_ptr(vmask),
            w_up=up.packed.data_ptr(), w_up_scales=up.scales.data_ptr(), w_up_g=up.g.data_ptr(),
            w_dn=dn.packed.data_ptr(), w_dn_scales=dn.scales.data_ptr(), w_dn_g=dn.g.data_ptr(),
            T=T, d=d, E=E, k=k_eff, F=F, norm_topk_prob=int(self.norm_topk_prob),
            out=out.data_ptr(), stats=None, sel_mask=None, topk_idx=idx.data_ptr(), topk_w=w.data_ptr(),
            offs=None, perm=None, h_debug=None, error_word=None, workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        _lib.check(_lib.load().mcl4moe_moe_forward_routed(args, _stream_handle()), "mcl4moe_moe_forward_routed")
        return out

    def _forward_variant(self, x, valid, prior_expert_mask, dense_expert_indices, dense_subset_k, variant):
        """Routing variants (mitotic twins, lineage families, coverage penalty, dense
        subsets, extra auxiliary losses): the reference's selection on the library's
        router logits, then the native layer on that routing.  Masked tokens are
        dropped before routing, as in the reference's loop branch and dense-subset
        head (src/mcl4_coe/backbone.py:913-1047, :640-785)."""
        from . import routing_variants as rv

        flat = x.reshape(-1, x.shape[-1])
        T, d = flat.shape
        E = len(self.experts)
        if self.router.weight.shape[0] != E:
            raise ValueError("router rows must match the number of experts")
        self.num_experts = E
        dev = flat.device
        flat_valid = (torch.ones(T, dtype=torch.bool, device=dev) if valid is None
                      else valid.reshape(-1).to(device=dev).bool())
        if flat_valid.numel() != T:
            raise ValueError("valid must have one entry per token")
        active = flat_valid.nonzero(as_tuple=False).squeeze(-1)
        n_act = active.numel()
        if n_act == 0:
            zero = torch.zeros((), dtype=torch.float32, device=dev)
            self.last_selected_mask = torch.zeros((*x.shape[:-1], E), dtype=torch.float32, device=dev)
            return dict(out=torch.zeros_like(x), aux_loss=zero, router_z_loss=zero,
                        counts=torch.zeros(E, dtype=torch.float32, device=dev))
        xb = flat.to(torch.bfloat16).contiguous()
        wr = self.router.weight.detach().to(device=dev, dtype=torch.float32).contiguous()
        bias = None
        if self.router_logit_bias is not None:
            bias = self.router_logit_bias.detach().to(device=dev, dtype=torch.float32).contiguous()
        logits = self._router_logits(xb, wr, bias).index_select(0, active)
        prior = None
        if prior_expert_mask is not None and self.recurrent_coverage_penalty > 0.0:
            prior = prior_expert_mask.reshape(-1, E).to(dev).index_select(0, active)
        vmask = None if valid is None else flat_valid.to(torch.uint8).contiguous()

        def full_rows(t: Tensor, fill) -> Tensor:  # active-token rows -> all T rows
            res = torch.full((T,) + tuple(t.shape[1:]), fill, dtype=t.dtype, device=dev)
            res.index_copy_(0, active, t)
            return res

        with torch.autocast(device_type=dev.type, enabled=False):
            if variant == "dense":
                if dense_expert_indices is not None:
                    dense_idx = ([int(i) for i in dense_expert_indices.detach().cpu().reshape(-1).tolist()]
                                 if isinstance(dense_expert_indices, Tensor) else [int(i) for i in dense_expert_indices])
                else:
                    dense_idx = list(self.dense_expert_indices)
                dense_k = int(self.dense_subset_k if dense_subset_k is None else dense_subset_k)
                sel = rv.dense_selection(self, logits, prior, dense_idx, dense_k)
                mask, aux, z, counts = rv.dense_statistics(self, logits, sel["probs"], sel["chosen"], sel["chosen_t"])
                probs = sel["probs"]
                # experts in ascending id order: the reference sums the subset's outputs in that order
                order = sorted(range(len(sel["chosen"])), key=lambda i: sel["chosen"][i])
                chosen_sorted = torch.tensor([sel["chosen"][i] for i in order], dtype=torch.int32, device=dev)
                w_sorted = sel["weights"][:, order]
                if sel["chosen"]:
                    idx = full_rows(chosen_sorted.unsqueeze(0).expand(n_act, -1).contiguous(), -1)
                    out = self._forward_routed(xb, vmask, idx, full_rows(w_sorted.contiguous(), 0.0))
                else:  # no valid expert id: the subset contributes nothing (src/mcl4_coe/backbone.py:324-325)
                    out = torch.zeros((T, d), dtype=torch.bfloat16, device=dev)
                rem = rv.dense_remainder(self, sel, xb.dtype)
                if rem is not None:
                    sparse = self._forward_routed(xb, vmask, full_rows(rem["selected"].to(torch.int32), -1),
                                                  full_rows(rem["weights"].contiguous(), 0.0))
                    mixed = (rem["alpha_dense"] * out.index_select(0, active)
                             + rem["alpha_rem"] * sparse.index_select(0, active))
                    out = torch.zeros_like(out)
                    out.index_copy_(0, active, mixed)
            else:
                probs, weights, selected = rv.sparse_selection(self, logits, prior)
                aux, z, counts = rv.sparse_statistics(self, logits, probs, selected)
                mask = torch.nn.functional.one_hot(selected, num_classes=E).sum(dim=1).to(torch.float32)
                out = self._forward_routed(xb, vmask, full_rows(selected.to(torch.int32), -1),
                                           full_rows(weights.contiguous(), 0.0))
            aux = rv.add_extra_aux(self, aux, tuple(x.shape), probs, active, T, valid)
        self.last_selected_mask = full_rows(mask, 0.0).view(*x.shape[:-1], E)
        return dict(out=out.to(x.dtype).view_as(x), aux_loss=aux, router_z_loss=z, counts=counts.detach())

    @torch.no_grad()
    def forward_dense_subset(self, x: Tensor, expert_indices: Sequence[int] | Tensor, *,
                             expert_weights: Tensor | None = None, valid: Tensor | None = None) -> Tensor:
        """The listed experts on every token, summed with ``expert_weights`` ([M] shared
        or [.., M] per token; none = weight 1), masked rows zero
        (src/mcl4_coe/backbone.py:307-398, grouped path :352-379).  Runs as a routing
        with the M experts (ascending id, the reference's summation order) in every
        token's slots."""
        if isinstance(expert_indices, Tensor):
            ids = [int(i) for i in expert_indices.detach().cpu().reshape(-1).tolist()]
        else:
            ids = [int(i) for i in expert_indices]
        flat = x.reshape(-1, x.shape[-1])
        if not ids or flat.shape[0] == 0:
            return torch.zeros_like(x)
        if flat.device.type != "cuda":
            raise ValueError("SparseMoE on B200 requires CUDA tensors (there is no CPU fallback)")
        T, m = flat.shape[0], len(ids)
        dev = flat.device
        if expert_weights is None:
            w = torch.ones((T, m), dtype=torch.float32, device=dev)
        elif expert_weights.ndim == 1:
            w = expert_weights.to(device=dev, dtype=torch.float32).view(1, m).expand(T, m)
        else:
            w = expert_weights.to(device=dev, dtype=torch.float32).reshape(-1, m)
        order = sorted(range(m), key=lambda i: ids[i])
        idx = torch.tensor([ids[i] for i in order], dtype=torch.int32, device=dev).view(1, m).expand(T, m)
        w = w[:, order].contiguous()
        vmask = None if valid is None else valid.reshape(-1).to(device=dev, dtype=torch.uint8).contiguous()
        out = self._forward_routed(flat.to(torch.bfloat16).contiguous(), vmask, idx.contiguous(), w)
        return out.to(x.dtype).view_as(x)

    def read_device_error(self) -> int:
        """Synchronise and return the error word of the last forward (0 = every
        device-side wait completed; 1xx/2xx/3xx = TMA producer / MMA issuer /
        epilogue wait of a GEMM gave up after its time limit)."""
        if self._ws is None or self._ws_key is None:
            return 0
        T, d, E, k, F, _ = self._ws_key
        lib = _lib.load()
        off = lib.mcl4moe_workspace_region(self._ws.data_ptr(), 8, T, d, E, k, F) - self._ws.data_ptr()
        return int(self._ws[off:off + 4].view(torch.int32).item())

    # ------------------------------------------------------------------ state dict
    def _save_to_state_dict(self, destination: dict, prefix: str, keep_vars: bool) -> None:
        super()._save_to_state_dict(destination, prefix, keep_vars)
        if self.mitotic_pairs:  # src/mcl4_coe/backbone.py:579-584
            destination[prefix + "mitotic_pairs_tensor"] = torch.tensor(self.mitotic_pairs, dtype=torch.long)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs) -> None:
        invalidate_cache(self.experts)  # src/mcl4_coe/backbone.py:596-598
        mp_key = prefix + "mitotic_pairs_tensor"
        if mp_key in state_dict:
            mp_val = state_dict.pop(mp_key)
            if isinstance(mp_val, torch.Tensor) and mp_val.ndim == 2 and mp_val.shape[1] == 2:
                self.mitotic_pairs = [(int(r[0]), int(r[1])) for r in mp_val.detach().cpu().tolist()]
            else:
                self.mitotic_pairs = []
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)


def _region(ws: Tensor, idx: int, nbytes: int, T: int, d: int, E: int, k: int, F: int) -> Tensor:
    lib = _lib.load()
    off = lib.mcl4moe_workspace_region(ws.data_ptr(), idx, T, d, E, k, F) - ws.data_ptr()
    return ws[off:off + nbytes]


def _weight_grads(d_rows: Tensor, rows: Tensor, pad_start: Tensor, E: int) -> Tensor:
    """Per-expert ``d_rows[seg]^T @ rows[seg]`` in float32 ([E, N, K]) over the padded
    expert segments of ``pad_start`` (``mcl4moe_moe_backward_wgrad``: the reference's
    ``_grouped_wgrad_kernel``, src/mcl4_coe/nvfp4.py:877-920, on tcgen05)."""
    mcap, n = d_rows.shape
    k = rows.shape[1]
    dw = torch.empty((E, n, k), dtype=torch.float32, device=d_rows.device)
    _lib.check(_lib.load().mcl4moe_moe_backward_wgrad(d_rows.data_ptr(), rows.data_ptr(), mcap, n, k,
                                                      pad_start.data_ptr(), E, dw.data_ptr(), None, _stream_handle()),
               "mcl4moe_moe_backward_wgrad")
    return dw


class _MoETrainFunction(torch.autograd.Function):
    """The layer under autograd (src/mcl4_coe/backbone.py:787-911 with
    _NVFP4GroupedLinear, src/mcl4_coe/nvfp4.py:1051-1216).

    Forward: ``mcl4moe_moe_forward`` with the training saves (gate | value rows, the
    permuted bf16 input rows, h, the unweighted down-projection rows, the router
    logits).  Backward: ``mcl4moe_moe_backward_experts`` (routing-weight and
    down-projection output gradients, stochastic-rounded NVFP4 input-gradient GEMMs on
    the transposed weights, SwiGLU derivative), ``mcl4moe_router_backward`` (softmax /
    top-k / renormalisation / aux / z derivative), the router's fp32 matrix products,
    ``mcl4moe_moe_backward_dx`` and the per-expert weight gradients
    (``mcl4moe_moe_backward_wgrad``)."""

    @staticmethod
    def forward(ctx, mod, x, valid, wr_param, *expert_weights):
        lib = _lib.load()
        flat = x.reshape(-1, x.shape[-1])
        T, d = flat.shape
        E = len(mod.experts)
        k = mod.top_k
        F = mod.experts[0].down_proj.weight.shape[1]
        dev = flat.device
        up = get_or_build_grouped_cache(mod.experts, "up_proj", with_bwd=True)
        dn = get_or_build_grouped_cache(mod.experts, "down_proj", with_bwd=True)
        xb = flat.detach().to(torch.bfloat16).contiguous()
        wr = wr_param.detach().to(torch.float32).contiguous()
        bias = None
        if mod.router_logit_bias is not None:
            bias = mod.router_logit_bias.detach().to(device=dev, dtype=torch.float32).contiguous()
        vmask = None if valid is None else valid.reshape(-1).to(device=dev, dtype=torch.uint8).contiguous()
        mcap = lib.mcl4moe_padded_rows(T, E, k)
        bf = dict(dtype=torch.bfloat16, device=dev)
        out = torch.empty((T, d), **bf)
        stats = torch.empty((3 + E,), dtype=torch.float32, device=dev)
        sel = torch.empty((T, E), dtype=torch.float32, device=dev)
        topk_idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        topk_w = torch.empty((T, k), dtype=torch.float32, device=dev)
        logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        up_save = torch.empty((mcap, 2 * F), **bf)
        x_rows = torch.empty((mcap, d), **bf)
        y_save = torch.empty((mcap, d), **bf)
        h_save = torch.empty((mcap, F), **bf)
        ws = mod._workspace(T, d, E, k, F, dev)
        args = _lib.MoeArgs(
            x=xb.data_ptr(), router_w=wr.data_ptr(), logit_bias=_opt_ptr(bias), valid=_opt_ptr(vmask),
            w_up=up.packed.data_ptr(), w_up_scales=up.scales.data_ptr(), w_up_g=up.g.data_ptr(),
            w_dn=dn.packed.data_ptr(), w_dn_scales=dn.scales.data_ptr(), w_dn_g=dn.g.data_ptr(),
            T=T, d=d, E=E, k=k, F=F, norm_topk_prob=int(mod.norm_topk_prob),
            out=out.data_ptr(), stats=stats.data_ptr(), sel_mask=sel.data_ptr(),
            topk_idx=topk_idx.data_ptr(), topk_w=topk_w.data_ptr(), offs=None, perm=None,
            h_debug=h_save.data_ptr() if T > 0 else None, error_word=None, workspace=ws.data_ptr(),
            workspace_bytes=ws.numel(), up_save=up_save.data_ptr() if T > 0 else None,
            x_rows_save=x_rows.data_ptr() if T > 0 else None, y_save=y_save.data_ptr() if T > 0 else None,
            logits_out=logits.data_ptr() if T > 0 else None)
        _lib.check(lib.mcl4moe_moe_forward(args, _stream_handle()), "mcl4moe_moe_forward")
        # the expert layout of this call (the workspace is reused by the next call)
        slot_pos = _region(ws, 6, 4 * T * k, T, d, E, k, F).view(torch.int32).view(T, k).clone()
        pad_start = _region(ws, 5, 4 * (E + 1), T, d, E, k, F).view(torch.int32).clone()
        counts_i = _region(ws, 9, 4 * E, T, d, E, k, F).view(torch.int32).clone()
        offs_start = _region(ws, 10, 4 * E, T, d, E, k, F).view(torch.int32).clone()
        mod.last_selected_mask = sel.view(*x.shape[:-1], E)
        ctx.mod = mod
        ctx.shape = (T, d, E, k, F)
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        ctx.caches = (up, dn)
        ctx.save_for_backward(xb, wr, vmask, topk_idx, topk_w, logits, stats, slot_pos, pad_start, counts_i,
                              offs_start, up_save, x_rows, y_save, h_save)
        aux, z, counts = stats[0].clone(), stats[1].clone(), stats[3:3 + E].clone()
        ctx.mark_non_differentiable(counts)
        return out.to(x.dtype).view(x.shape), aux, z, counts

    @staticmethod
    def backward(ctx, d_out, d_aux, d_z, _d_counts):
        lib = _lib.load()
        (xb, wr, vmask, topk_idx, topk_w, logits, stats, slot_pos, pad_start, counts_i, offs_start, up_save, x_rows,
         y_save, h_save) = ctx.saved_tensors
        mod = ctx.mod
        up, dn = ctx.caches
        T, d, E, k, F = ctx.shape
        dev = xb.device
        mcap = up_save.shape[0]
        n_exp = len(mod.experts)
        if d_out is None:
            d_out = torch.zeros((T, d), dtype=torch.bfloat16, device=dev)
        d_out = d_out.reshape(T, d).to(torch.bfloat16).contiguous()
        f32 = dict(dtype=torch.float32, device=dev)
        d_aux = torch.zeros((), **f32) if d_aux is None else d_aux.detach().to(torch.float32).reshape(()).contiguous()
        d_z = torch.zeros((), **f32) if d_z is None else d_z.detach().to(torch.float32).reshape(()).contiguous()
        bf = dict(dtype=torch.bfloat16, device=dev)
        d_y = torch.empty((mcap, d), **bf)
        d_up = torch.empty((mcap, 2 * F), **bf)
        d_rows = torch.empty((mcap, d), **bf)
        d_w = torch.zeros((T, k), **f32)
        ws = torch.empty((max(lib.mcl4moe_moe_backward_workspace_size(T, d, E, k, F), 256),), dtype=torch.uint8,
                         device=dev)
        args = _lib.MoeBwdArgs(
            T=T, d=d, E=E, k=k, F=F, d_out=d_out.data_ptr(), slot_pos=slot_pos.data_ptr(),
            topk_w=topk_w.data_ptr(), pad_start=pad_start.data_ptr(), counts=counts_i.data_ptr(),
            offs_start=offs_start.data_ptr(), y_save=y_save.data_ptr(), up_save=up_save.data_ptr(),
            w_up_t=up.packed_t.data_ptr(), w_up_t_scales=up.scales_t.data_ptr(), w_up_g=up.g.data_ptr(),
            w_dn_t=dn.packed_t.data_ptr(), w_dn_t_scales=dn.scales_t.data_ptr(), w_dn_g=dn.g.data_ptr(),
            seed_down=random.getrandbits(31), seed_up=random.getrandbits(31),  # src/mcl4_coe/nvfp4.py:1140
            d_y=d_y.data_ptr(), d_up=d_up.data_ptr(), d_rows=d_rows.data_ptr(), d_w=d_w.data_ptr(),
            error_word=None, workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        stream = _stream_handle()
        if T > 0:
            _lib.check(lib.mcl4moe_moe_backward_experts(args, stream), "mcl4moe_moe_backward_experts")
        d_logits = torch.empty((T, E), **f32)
        _lib.check(lib.mcl4moe_router_backward(logits.data_ptr(), topk_idx.data_ptr(), topk_w.data_ptr(),
                                               d_w.data_ptr(), _opt_ptr(vmask), stats.data_ptr(), d_aux.data_ptr(),
                                               d_z.data_ptr(), T, E, k, int(mod.norm_topk_prob),
                                               d_logits.data_ptr(), stream), "mcl4moe_router_backward")
        # the router's fp32 products (F.linear(x.float(), W) at src/mcl4_coe/backbone.py:790)
        d_x_router = (d_logits @ wr).contiguous()
        d_wr = d_logits.t() @ xb.float()
        d_x = torch.empty((T, d), **bf)
        _lib.check(lib.mcl4moe_moe_backward_dx(d_rows.data_ptr(), slot_pos.data_ptr(), d_x_router.data_ptr(), T, k, d,
                                               d_x.data_ptr(), stream), "mcl4moe_moe_backward_dx")
        # expert weight gradients over the padded segments (padding rows are zero in d_y / d_up)
        if T > 0:
            dw_dn = _weight_grads(d_y, h_save, pad_start, E)
            dw_up = _weight_grads(d_up, x_rows, pad_start, E)
        else:
            dw_dn = torch.zeros((E, d, F), **f32)
            dw_up = torch.zeros((E, 2 * F, d), **f32)
        ups = [e.up_proj.weight for e in mod.experts]
        dns = [e.down_proj.weight for e in mod.experts]
        g_up = [dw_up[i].to(ups[i].dtype) if ctx.needs_input_grad[4 + i] else None for i in range(n_exp)]
        g_dn = [dw_dn[i].to(dns[i].dtype) if ctx.needs_input_grad[4 + n_exp + i] else None for i in range(n_exp)]
        g_x = d_x.to(ctx.x_dtype).view(ctx.x_shape) if ctx.needs_input_grad[1] else None
        g_wr = d_wr.to(mod.router.weight.dtype) if ctx.needs_input_grad[3] else None
        return (None, g_x, None, g_wr, *g_up, *g_dn)
