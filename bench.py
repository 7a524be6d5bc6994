#!/usr/bin/env python
"""NVFP4 MoE-layer tokens/s on B200 — the reference's headline metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

One step = one forward of the MoE layer (router top-k, permutation + NVFP4
activation quantisation, grouped gate/up GEMM with fused SwiGLU, grouped down
GEMM, weighted combine) over T tokens of synthetic input resident in HBM.
Default workload: the OLMoE-style headline configuration (configs[2]:
T=32768, d=2048, E=64, top-8, F=1024).  Synthetic data: x ~ N(0,1) bf16,
router and expert weights ~ N(0, 0.02) fp32, quantised to NVFP4 once (the
quantised-weight cache is reused across steps, as in the reference).

Multi-GPU (torchrun, one process per GPU): weak scaling with expert
parallelism.  Every rank routes its own T tokens; the experts are sharded in
contiguous blocks of E/N (``ExpertParallelMoE``), each rank sends its tokens'
NVFP4 rows to the ranks holding their experts (copy-engine copies into
CUDA-IPC-mapped peer buffers, ordered by a one-element NCCL all-reduce); by
default (``--ep-back h``) the receivers' gate/up GEMMs store each slot's NVFP4 h
straight into its source's layout and every rank runs the down projection and
combine of its own tokens (all experts' down weights on every rank), else
(``--ep-back partials``) bf16 partial sums come back.  ``value`` is the tokens
of all ranks over the slowest rank's device time.

CPU baselines (rank 0, 1 GPU): the reference's own ``SparseMoE.forward``
(installed under ``baseline/_ref``) on the host cores with its expert
projections replaced by dequantised-FP4 linears built from the reference's
``_quantize_nvfp4_core`` / ``_dequantize_nvfp4`` (the "dequantised-FP4 CPU
path"); the numpy restatement in ``oracle/`` stands in when ``baseline/_ref``
is missing.  ``cpu_baseline`` runs the full batch once; ``--impl reference``
runs a bounded token sample per step so that the whole run ends in minutes.

``reference_gpu`` (1 GPU): the unmodified reference on the same B200 — its
``SparseMoE.forward`` as dispatched (per-expert ``F.scaled_mm`` loop for the
configurations with E*d >= 65536) and with its grouped branch (Triton
``tl.dot_scaled`` kernels through ``nvfp4_grouped_linear``).

``--fp4-peak`` measures the dense NVFP4 GEMM rate of cuBLAS (``F.scaled_mm``,
16-element E4M3 block scales) at 8192^3, the FP4 counterpart of the bf16 GEMM
peak in MEASURED_PEAKS.json.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "NVFP4 MoE-layer tokens/s"
UNIT = "tokens/s"

CONFIGS = {
    "c0": dict(name="c0_cpu_runnable", seed=0, t=2048, d=256, e=8, k=2, f=512),
    "c1": dict(name="c1_mitotic", seed=1, t=16384, d=1024, e=32, k=4, f=512),
    "c2": dict(name="c2_olmoe_prefill", seed=2, t=32768, d=2048, e=64, k=8, f=1024),
    "c3": dict(name="c3_granite_zipf", seed=3, t=65536, d=1536, e=32, k=8, f=512, zipf=True),
    "c4": dict(name="c4_decode", seed=4, t=64, d=2048, e=64, k=8, f=1024),
}
def kernels_per_forward(T: int, ep: bool = False, h_back: bool = False, chunks: int = 1) -> int:
    """This library's kernel launches per layer forward.
    1 GPU: routing (router-weight split, router, route-scan; one fused kernel for a single
    128-token chunk), permute + quantise, gate/up GEMM, down GEMM, combine.
    Expert parallel, per chunk: dispatch count / scan / pack (3) and on the receiver the
    count / scan / pad / scatter of the received rows (4) with, for partial sums, both GEMMs and
    the partial-sum kernel (3) and the combine (1), or for h back the gate/up GEMM (1); once:
    routing (3), and for h back the layout permute (1), the down GEMM and the combine (2)."""
    if not ep:
        return (1 if T <= 128 else 3) + 4
    if h_back:
        return 3 + 1 + 8 * chunks + 2
    return 3 + 11 * chunks
EP_STAGES = ("route", "dispatch", "counts", "exchange_rows", "experts", "exchange_partials", "combine")
EP_STAGES_H = ("route_layout", "dispatch", "counts", "exchange_rows", "gateup_h_to_home", "h_arrival", "down_combine")


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=float(d["hbm_gbs"]), bf16=float(d["bf16_tflops"]),
                    bf16_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), source="measured")
    return dict(hbm_gbs=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons of one GPU while the timed region runs."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.tmp = None

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        rows = [ln.split(", ") for ln in Path(self.tmp.name).read_text().splitlines() if ln.strip()]
        os.unlink(self.tmp.name)
        mine = [r for r in rows if len(r) >= 9 and self.uuid and self.uuid in r[0]]
        if not mine:
            return None
        def num(v):
            try:
                return float(v)
            except ValueError:
                return float("nan")
        loaded = [r for r in mine if num(r[4]) >= 50.0] or mine
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in loaded for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(num(r[1]) for r in loaded), "sm_max_mhz": num(loaded[0][2]),
                "power_w_max": max(num(r[3]) for r in loaded), "samples_under_load": len(loaded),
                "reasons": reasons}


# ---------------------------------------------------------------------------- our arm
def build_layer(pkg, cfg, device, rank):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(cfg["seed"])
    moe = pkg.SparseMoE(pkg.MoEConfig(d_model=cfg["d"], expert_hidden_dim=cfg["f"], num_experts=cfg["e"],
                                      top_k=cfg["k"])).to(device)
    with torch.no_grad():
        moe.router.weight.copy_(torch.randn(moe.router.weight.shape, generator=g, device=device) * 0.02)
        for ex in moe.experts:
            ex.up_proj.weight.copy_(torch.randn(ex.up_proj.weight.shape, generator=g, device=device) * 0.02)
            ex.down_proj.weight.copy_(torch.randn(ex.down_proj.weight.shape, generator=g, device=device) * 0.02)
    if cfg.get("zipf"):
        moe.router_logit_bias = (2.0 * torch.log(1.0 / torch.arange(1, cfg["e"] + 1, device=device,
                                                                      dtype=torch.float32)))
    gx = torch.Generator(device=device)
    gx.manual_seed(cfg["seed"] * 1000 + 17 + rank)
    x = torch.randn((cfg["t"], cfg["d"]), generator=gx, device=device).to(torch.bfloat16)
    moe.requires_grad_(False)
    return moe, x


def _reference_modules():
    """The reference package installed under baseline/_ref (``mcl4_coe.backbone``,
    ``mcl4_coe.nvfp4``), or None when it is not installed."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "mcl4_coe" / "backbone.py").exists():
        return None
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    import mcl4_coe.backbone as bb
    import mcl4_coe.nvfp4 as nv

    return bb, nv


def _host_threads() -> dict:
    import torch

    try:
        from threadpoolctl import threadpool_info

        blas = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:
        blas = None
    return {"os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(), "blas_threads": blas}


def reference_cpu_layer(cfg, wr, w_up, w_dn, bias):
    """The reference SparseMoE (loop branch on the CPU) with dequantised-FP4 expert
    projections: every projection input is quantised to NVFP4 (1x16 blocks, g = 1)
    and dequantised, the weights are the 16x16-tile NVFP4 weights dequantised, fp32
    product rounded to bf16.  ``wr`` / ``w_up`` / ``w_dn`` are fp32 CPU tensors
    ([E, d], [E, 2F, d], [E, d, F]); ``bias`` an optional [E] router logit bias,
    added to the router output as the benchmark's skewed configuration defines it."""
    import torch
    from torch import nn
    from torch.nn import functional as Fn

    bb, nv = _reference_modules()

    class DequantFP4Linear(nn.Module):
        def __init__(self, weight):
            super().__init__()
            packed, scales, g = nv._quantize_nvfp4_core(weight, True, False, False)
            self.register_buffer("w_deq", nv._dequantize_nvfp4(packed, nv._swizzle_scales(scales), g,
                                                               weight.shape[0], weight.shape[1]))

        def forward(self, x):
            xf = x.float()
            packed, scales, g = nv._quantize_nvfp4_core(xf, False, False, True)
            xd = nv._dequantize_nvfp4(packed, nv._swizzle_scales(scales), g, xf.shape[0], xf.shape[1])
            return Fn.linear(xd, self.w_deq).to(x.dtype)

    E = wr.shape[0]
    conf = bb.MCL4CEDConfig(d_model=cfg["d"], n_heads=4, expert_hidden_dim=cfg["f"], num_experts=E,
                            top_k=cfg["k"], norm_topk_prob=True)
    moe = bb.SparseMoE(conf).eval()
    with torch.no_grad():
        moe.router.weight.copy_(wr)
        for i, ex in enumerate(moe.experts):
            ex.up_proj = DequantFP4Linear(w_up[i])
            ex.down_proj = DequantFP4Linear(w_dn[i])
    if bias is not None:
        _add_router_bias(bb, moe.router.weight, bias)
    return moe


def _add_router_bias(bb, router_weight, bias) -> None:
    """The skewed configuration's additive router logit bias on the reference layer,
    which computes its logits with ``F.linear(x.float(), router.weight.float())``
    (src/mcl4_coe/backbone.py:929): wrap ``F.linear`` so that calls with this router
    weight (``.float()`` of an fp32 tensor is the tensor itself) get the bias added."""
    linear = bb.F.linear

    def biased_linear(inp, weight, b=None):
        out = linear(inp, weight, b)
        return out + bias.to(out.device) if weight is router_weight else out

    bb.F.linear = biased_linear


def cpu_baseline_ours(moe, x, cfg) -> dict:
    """The reference CPU path on this host's cores, over the full batch of the bench's
    own inputs and weights (one forward after a short warm-up)."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    T = x.shape[0]
    wr = moe.router.weight.detach().float().cpu()
    bias = None if moe.router_logit_bias is None else moe.router_logit_bias.detach().float().cpu()
    xs = x.cpu()
    if _reference_modules() is not None:
        w_up = torch.stack([e.up_proj.weight.detach().float().cpu() for e in moe.experts])
        w_dn = torch.stack([e.down_proj.weight.detach().float().cpu() for e in moe.experts])
        ref = reference_cpu_layer(cfg, wr, w_up, w_dn, bias)
        del w_up, w_dn
        with torch.no_grad():
            ref(xs[: min(T, 256)].unsqueeze(0))  # warm-up
            t0 = time.perf_counter()
            ref(xs.unsqueeze(0))
            t = time.perf_counter() - t0
        kind, what = "reference", ("reference SparseMoE.forward (baseline/_ref, loop branch) with dequantised-FP4 "
                                   "expert projections from the reference's own quantiser, torch on all host threads")
    else:
        sys.path.insert(0, str(ROOT))
        from oracle import moe_ref, nvfp4_ref as nr

        pkg = sys.modules["mcl4coe_b200"]
        experts = moe_ref.QuantizedExperts.__new__(moe_ref.QuantizedExperts)
        deq = {}
        for proj in ("up_proj", "down_proj"):
            r = pkg.export_reference_cache(moe.experts, proj)
            b = r["B_fwd"].cpu().numpy()
            sc = r["Bs_fwd"].view(torch.uint8).cpu().numpy()
            gsc = r["Bg"].cpu().numpy()
            deq[proj] = [nr.dequantize_grouped_weight(b, sc, gsc, e) for e in range(cfg["e"])]
        experts.up, experts.dn = deq["up_proj"], deq["down_proj"]
        xn = xs.float().numpy()
        bn = None if bias is None else bias.numpy()
        moe_ref.moe_forward(xn[:8], wr.numpy(), experts, cfg["k"], True, None, bn)
        t0 = time.perf_counter()
        moe_ref.moe_forward(xn, wr.numpy(), experts, cfg["k"], True, None, bn)
        t = time.perf_counter() - t0
        kind, what = "port", "numpy restatement of the reference path (oracle/), numpy/BLAS on all host threads"
    thr = _host_threads()
    return {"value": T / t, "unit": UNIT, "cores": thr["torch_threads"] if kind == "reference" else thr["blas_threads"],
            "kind": kind, "seconds": t, **thr,
            "sample": f"all {T} tokens of {cfg['name']} (one forward, unsampled): {what}"}


def reference_gpu_leg(moe, x, cfg, steps: int) -> dict:
    """The unmodified reference on this GPU: ``SparseMoE.forward`` as dispatched and with
    its grouped branch, NVFP4Linear experts (sparsity "none", weights of our layer)."""
    import torch

    mods = _reference_modules()
    if mods is None:
        return {"unavailable": "reference not installed under baseline/_ref"}
    bb, nv = mods
    dev = x.device
    T, d, E, k = x.shape[0], cfg["d"], cfg["e"], cfg["k"]
    res = {}
    try:
        conf = bb.MCL4CEDConfig(d_model=d, n_heads=4, expert_hidden_dim=cfg["f"], num_experts=E, top_k=k,
                                norm_topk_prob=True)
        ref = bb.SparseMoE(conf).to(dev).eval()
        with torch.no_grad():
            ref.router.weight.copy_(moe.router.weight.detach().float())
            for re_, ex in zip(ref.experts, moe.experts):
                re_.up_proj.weight.copy_(ex.up_proj.weight.detach())
                re_.down_proj.weight.copy_(ex.down_proj.weight.detach())
        nv.convert_linear_to_nvfp4(ref, sparsity_mode="none")
        ref.requires_grad_(False)
        if moe.router_logit_bias is not None:
            _add_router_bias(bb, ref.router.weight, moe.router_logit_bias.detach().float())
        res["nvfp4_native"] = bool(nv.has_native_nvfp4(dev))
        res["triton_grouped"] = bool(nv.has_triton_nvfp4_grouped(dev))
        xin = x.unsqueeze(0)

        def timed(fn, n):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(n):
                fn()
            b.record()
            torch.cuda.synchronize()
            return a.elapsed_time(b) / n

        with torch.no_grad():
            branch = "grouped" if ref._can_use_grouped_dispatch(x) else "loop (per-expert F.scaled_mm)"
            ms = timed(lambda: ref(xin), steps)
            res["as_dispatched"] = {"branch": branch, "ms_per_step": ms, "value": T / (ms / 1e3), "unit": UNIT}
            if res["triton_grouped"]:
                ref._can_use_grouped_dispatch = lambda flat: bool(flat.is_cuda and flat.shape[0] > 0)
                ms = timed(lambda: ref(xin), steps)
                res["grouped_branch"] = {"ms_per_step": ms, "value": T / (ms / 1e3), "unit": UNIT,
                                         "note": "SparseMoE.forward with _can_use_grouped_dispatch forced true: "
                                                 "router, argsort permute, nvfp4_grouped_linear (Triton "
                                                 "tl.dot_scaled) for up and down, bf16 SwiGLU, combine"}
    except Exception as exc:  # the reference's GPU path failing is reported, not fatal
        res["error"] = f"{type(exc).__name__}: {exc}"[:300]
    finally:
        torch.cuda.synchronize()
    return res


def train_step_timing(moe, x, steps: int) -> dict:
    """One training step of the layer: forward with the backward's saves, then the
    backward (stochastic-rounded NVFP4 input-gradient GEMMs, the SwiGLU / routing /
    router derivatives, bf16-operand weight gradients) for an upstream gradient of the
    output plus the auxiliary and z losses; CUDA events around the steps."""
    import torch

    moe.requires_grad_(True)
    xg = x.detach().clone().requires_grad_(True)
    g = torch.Generator(device=x.device).manual_seed(123)
    gout = torch.randn(x.shape, generator=g, device=x.device).to(torch.bfloat16)
    one = torch.ones((), device=x.device)

    def step():
        out, aux, z, _ = moe(xg)
        torch.autograd.backward([out, aux, z], [gout, one * 0.01, one * 0.001])
        moe.zero_grad(set_to_none=True)
        xg.grad = None

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize()
    moe.requires_grad_(False)
    ms = a.elapsed_time(b) / steps
    return {"ms_per_step": ms, "value": x.shape[0] / (ms / 1e3), "unit": UNIT, "steps": steps,
            "what": "forward + backward (input, router and expert weight gradients) of the layer"}


def cublas_fp4_tflops(pkg, device, n: int = 8192, reps: int = 10) -> float:
    """Best-of-``reps`` dense NVFP4 GEMM rate of cuBLAS (``F.scaled_mm`` with the reference's
    recipe: 1x16 E4M3 block scales + fp32 tensor scale) at n^3, in TFLOP/s."""
    import torch
    from torch.nn import functional as Fn

    g = torch.Generator(device=device).manual_seed(0)
    qa, sa, ga = pkg.quantize_nvfp4(torch.randn((n, n), generator=g, device=device).to(torch.bfloat16))
    qb, sb, gb = pkg.quantize_nvfp4(torch.randn((n, n), generator=g, device=device).to(torch.bfloat16))
    recipe = [Fn.ScalingType.BlockWise1x16, Fn.ScalingType.TensorWise]
    swz = [Fn.SwizzleType.SWIZZLE_32_4_4, Fn.SwizzleType.NO_SWIZZLE]

    def mm():
        return Fn.scaled_mm(qa, qb.t(), scale_a=[sa, ga], scale_recipe_a=recipe, scale_b=[sb, gb],
                            scale_recipe_b=recipe, swizzle_a=swz, swizzle_b=swz, output_dtype=torch.bfloat16)

    for _ in range(3):
        mm()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        mm()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b))
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


def fp4_peak(args) -> None:
    """cuBLAS dense NVFP4 GEMM (F.scaled_mm with 1x16 E4M3 block scales + fp32 tensor
    scales, the recipe of the reference's nvfp4_mm) at M = N = K = 8192: best of 10
    (burst) and back to back for 4 s (sustained), with the clocks sampled meanwhile."""
    import torch
    from torch.nn import functional as Fn

    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package

    pkg = load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = 8192
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn((n, n), generator=g, device=dev).to(torch.bfloat16)
    b = torch.randn((n, n), generator=g, device=dev).to(torch.bfloat16)
    qa, sa, ga = pkg.quantize_nvfp4(a)
    qb, sb, gb = pkg.quantize_nvfp4(b)
    recipe = [Fn.ScalingType.BlockWise1x16, Fn.ScalingType.TensorWise]
    swz = [Fn.SwizzleType.SWIZZLE_32_4_4, Fn.SwizzleType.NO_SWIZZLE]

    def mm():
        return Fn.scaled_mm(qa, qb.t(), scale_a=[sa, ga], scale_recipe_a=recipe, scale_b=[sb, gb],
                            scale_recipe_b=recipe, swizzle_a=swz, swizzle_b=swz, output_dtype=torch.bfloat16)

    for _ in range(3):
        mm()
    torch.cuda.synchronize()
    flops = 2.0 * n ** 3
    best = float("inf")
    for _ in range(10):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        mm()
        s1.record()
        torch.cuda.synchronize()
        best = min(best, s0.elapsed_time(s1))
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid)).start()
    time.sleep(0.3)
    iters, t_end = 0, time.time() + 4.0
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    while time.time() < t_end:
        for _ in range(20):
            mm()
        iters += 20
        torch.cuda.synchronize()
    s1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    sust = s0.elapsed_time(s1) / iters
    peaks = load_peaks()
    print(json.dumps({"what": "dense NVFP4 GEMM, F.scaled_mm (cuBLASLt), 1x16 e4m3 block + fp32 tensor scales",
                      "m_n_k": n, "burst_tflops": flops / (best / 1e3) / 1e12,
                      "sustained_tflops": flops / (sust / 1e3) / 1e12, "burst_ms": best, "sustained_ms": sust,
                      "bf16_tflops_measured": peaks["bf16"], "bf16_tflops_sustained_measured": peaks["bf16_sustained"],
                      "clocks": clocks}), flush=True)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package

    pkg = load_package()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun for N > 1")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = CONFIGS[args.config]
    T, d, E, k, F = cfg["t"], cfg["d"], cfg["e"], cfg["k"], cfg["f"]
    moe, x = build_layer(pkg, cfg, dev, rank)
    ep = world > 1
    n_stages = 7 if ep else 5
    if ep:
        # expert parallel: the same layer on every rank, each keeps its E / N experts
        moe = pkg.ExpertParallelMoE.from_dense(moe, chunks=args.ep_chunks)
        moe.partials_via = args.ep_partials
        if args.ep_back == "partials":
            moe.down_experts = None

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    K, W = args.steps, args.warmup
    graph = args.cuda_graph and not ep
    with torch.inference_mode():
        if graph:
            moe.enable_cuda_graph()
        for _ in range(W):
            moe(x)
        torch.cuda.synchronize()
        # stage events: 6 per step, recorded once beforehand so their handles exist
        stage_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(n_stages + 1)] for _ in range(K)]
        for evs in stage_ev:
            for ev in evs:
                ev.record()
        torch.cuda.synchronize()
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        sampler = ClockSampler(uuid).start()
        time.sleep(0.3)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        start.record()
        for i in range(K):
            moe(x)
        end.record()
        torch.cuda.synchronize()
        barrier()
        clocks = sampler.stop()
        elapsed_ms = max_over_ranks(start.elapsed_time(end))
        # stage breakdown in a separate pass: events between the kernels would keep the
        # timed forwards from overlapping one kernel's start with the previous one's end
        if graph:
            moe.enable_cuda_graph(False)
        for i in range(K):
            moe.stage_events = stage_ev[i]
            moe(x)
        torch.cuda.synchronize()
        moe.stage_events = None
        stage_ms = [statistics.mean(evs[j].elapsed_time(evs[j + 1]) for evs in stage_ev) for j in range(n_stages)]
        stage_spread = None
        if ep:  # every rank's stage times: min / max over ranks show imbalance and waiting
            allst = [None] * world
            dist.all_gather_object(allst, stage_ms)
            stage_spread = {name: [round(min(r[i] for r in allst), 4), round(max(r[i] for r in allst), 4)]
                            for i, name in enumerate(EP_STAGES if moe.down_experts is None else EP_STAGES_H)}

        # end to end through the public API with host buffers: every step copies its x from
        # pinned host memory and its output (plus aux / z) back; uploads, layer and downloads
        # run on three streams, double-buffered, the way a serving loop overlaps them
        x_host = x.cpu().pin_memory()
        out_host = [torch.empty((T, d), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        stats_host = [torch.empty((2,), dtype=torch.float32).pin_memory() for _ in range(2)]
        x_dev = [torch.empty_like(x) for _ in range(2)]
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        comp = torch.cuda.current_stream(dev)

        def e2e_steps(n, start_event=None):
            if start_event is not None:
                h2d.wait_event(start_event)  # no upload starts before the timed region
            up_done = [torch.cuda.Event() for _ in range(n)]
            used = [torch.cuda.Event() for _ in range(n)]

            def upload(i):  # issued one step ahead, so the host never waits to start a copy
                with torch.cuda.stream(h2d):
                    if i >= 2:
                        h2d.wait_event(used[i - 2])  # the layer of step i-2 has read x_dev[i % 2]
                    x_dev[i % 2].copy_(x_host, non_blocking=True)
                    up_done[i].record(h2d)

            upload(0)
            for i in range(n):
                if i + 1 < n:
                    upload(i + 1)
                b = i % 2
                comp.wait_event(up_done[i])
                o, aux, z, _ = moe(x_dev[b])
                st = torch.stack([aux.reshape(()), z.reshape(())])
                used[i].record(comp)
                d2h.wait_event(used[i])
                with torch.cuda.stream(d2h):
                    o.record_stream(d2h)
                    st.record_stream(d2h)
                    out_host[b].copy_(o, non_blocking=True)
                    stats_host[b].copy_(st, non_blocking=True)
            comp.wait_stream(d2h)

        e2e_steps(max(2, W))
        torch.cuda.synchronize()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e_start.record()
        e2e_steps(K, e_start)
        e_end.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e_start.elapsed_time(e_end))

    ms_per_step = elapsed_ms / K
    value = T * world / (ms_per_step / 1e3)
    peaks = load_peaks()
    fp4_peak = 4.0 * peaks["bf16"]  # dense FP4 = 4x dense BF16 on Blackwell (9 vs 2.25 PFLOP/s nominal)
    if ep:
        # the rank's experts step (receive layout, both grouped GEMMs, partial sums) on its own slots
        slots_here = moe.last_exchange["slots"][0]
        roof_flops, roof_ms = 6.0 * slots_here * d * F, stage_ms[4]
        roof_kernel = "grouped_gemm_fp4 gate/up + down (expert-parallel experts step of rank 0, incl. row layout)"
    else:
        roof_flops, roof_ms = 4.0 * T * k * d * F, stage_ms[2]
        roof_kernel = "grouped_gemm_fp4 (gate/up, SwiGLU+requant epilogue)"
    achieved = roof_flops / (roof_ms / 1e3) / 1e12
    decode = cfg["name"].startswith("c4")
    if decode and not ep:
        # decode: weight streaming; algorithmic bytes = NVFP4 bytes of every expert that received a
        # token (codes + 16-element scales + global scales) + x and out in bf16 + the fp32 router
        with torch.inference_mode():
            touched = int((moe.forward_details(x)["offs"].diff(prepend=torch.zeros(1, dtype=torch.int32,
                                                                                     device=dev)) > 0).sum())
        dec_bytes = touched * (3 * d * F * (0.5 + 1 / 16) + 8) + 4 * T * d + 4 * E * d
    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        traffic = json.loads(tp.read_text()).get(args.config, {}).get("gateup_gemm_bytes")
    layer_tflops = 6.0 * T * k * d * F / (ms_per_step / 1e3) / 1e12
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "nvfp4 (e2m1 + e4m3/16) x nvfp4 -> fp32 accumulate, bf16 I/O, fp32 router",
        "data": "synthetic (x~N(0,1) bf16, weights~N(0,0.02) fp32 quantised to NVFP4, seeded torch RNG on device)",
        "config": {"workload": cfg["name"], "tokens_per_gpu": T, "d_model": d, "num_experts": E, "top_k": k,
                   "expert_ffn": F, "parallelism": f"ep{world}" if ep else "single",
                   **({"ep_chunks": len(moe._chunk_bounds(T)), "ep_chunk_weights": moe.chunk_weights,
                      "ep_back": "h" if moe.down_experts is not None else "partials",
                      **({"ep_partials": moe.partials_via} if moe.down_experts is None else {})} if ep else {}),
                   **({"cuda_graph": True} if graph else {}),
                   "l2": "no flush: x (%.0f MB) and NVFP4 weights (%.0f MB) exceed the 126 MB L2" % (
                       T * d * 2 / 1e6, E * 3 * d * F * (0.5 + 1 / 16) / 1e6)},
        "stages_ms": dict(zip((EP_STAGES if moe.down_experts is None else EP_STAGES_H) if ep
                              else ("route", "permute_quant", "gateup_gemm", "down_gemm", "combine"),
                              [round(s, 4) for s in stage_ms])),
        **({"stages_ms_over_ranks": stage_spread} if ep else {}),
        "layer_fp4_tflops": layer_tflops,
        "roofline": ({"bound": "hbm", "kernel": "whole layer forward (decode: grouped GEMMs stream the touched experts)",
                      "achieved": dec_bytes / (ms_per_step / 1e3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                      "frac": dec_bytes / (ms_per_step / 1e3) / 1e9 / peaks["hbm_gbs"], "traffic": traffic,
                      "experts_touched": touched, "algorithmic_bytes": dec_bytes,
                      "peak_source": f"{peaks['source']} copy bandwidth (MEASURED_PEAKS.json)"}
                     if decode and not ep else
                     {"bound": "tensor", "kernel": roof_kernel,
                      "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s", "frac": achieved / fp4_peak,
                      "traffic": traffic,
                      "peak_source": f"4 x {peaks['source']} dense bf16 {peaks['bf16']} TFLOP/s "
                                     "(MEASURED_PEAKS.json; FP4 dense = 4x BF16 dense)"}),
        "e2e": {"value": T * world / (e2e_ms / K / 1e3), "unit": UNIT, "h2d_bytes_per_step": T * d * 2,
                "d2h_bytes_per_step": T * d * 2 + 8},
        "gpu_launches": (kernels_per_forward(T, True, moe.down_experts is not None, len(moe._chunk_bounds(T))) if ep
                         else kernels_per_forward(T)) * K,
        "clocks": clocks,
    }
    if world == 1 and not ep and not decode:
        # the FP4 counterpart of MEASURED_PEAKS.json's cuBLAS bf16 figure, measured here on this GPU
        try:
            with torch.no_grad():
                cub = cublas_fp4_tflops(pkg, dev)
            result["roofline"]["cublas_nvfp4_tflops"] = cub
            result["roofline"]["frac_of_cublas_nvfp4"] = result["roofline"]["achieved"] / cub
        except Exception as exc:  # a library without the NVFP4 recipe: report, do not fail the bench
            result["roofline"]["cublas_nvfp4_tflops"] = f"unavailable: {type(exc).__name__}: {exc}"[:200]
    if world == 1 and not ep and not args.no_train:
        result["train"] = train_step_timing(moe, x, max(3, min(K, 10)))
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        # not under inference_mode: the reference keys its weight cache on ``Tensor._version``
        with torch.no_grad():
            result["reference_gpu"] = reference_gpu_leg(moe, x, cfg, max(3, min(K, 10)))
        rg = result["reference_gpu"]
        best = [v["value"] for key, v in rg.items() if isinstance(v, dict) and "value" in v]
        if best:
            rg["speedup_vs_best_reference_gpu"] = value / max(best)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline_ours(moe, x, cfg)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- reference arm
def run_reference(args) -> None:
    """The reference path's CPU implementation on this host's cores, rank 0 only: the
    reference's own SparseMoE.forward with dequantised-FP4 expert projections
    (baseline/_ref), or the numpy restatement in oracle/ when it is not installed.
    Each step is one forward over a bounded token sample of the configuration."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch

    sys.path.insert(0, str(ROOT))
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = CONFIGS[args.config]
    T, d, E, k, F = cfg["t"], cfg["d"], cfg["e"], cfg["k"], cfg["f"]
    r = np.random.Generator(np.random.PCG64(cfg["seed"]))
    wr = (r.standard_normal((E, d), dtype=np.float32) * 0.02).astype(np.float32)
    w_up = (r.standard_normal((E, 2 * F, d), dtype=np.float32) * 0.02).astype(np.float32)
    w_dn = (r.standard_normal((E, d, F), dtype=np.float32) * 0.02).astype(np.float32)
    bias = (2.0 * np.log(1.0 / np.arange(1, E + 1))).astype(np.float32) if cfg.get("zipf") else None
    sample = min(T, args.cpu_sample)
    x = r.standard_normal((T, d), dtype=np.float32)
    if _reference_modules() is not None:
        # weight quantisation happens here, once: cached, not timed (as in the reference)
        layer = reference_cpu_layer(cfg, torch.from_numpy(wr), torch.from_numpy(w_up), torch.from_numpy(w_dn),
                                    None if bias is None else torch.from_numpy(bias))
        xt = torch.from_numpy(x).to(torch.bfloat16)

        def fwd(lo):
            with torch.no_grad():
                layer(xt[lo:lo + sample].unsqueeze(0))

        kind = "reference"
        what = ("reference SparseMoE.forward (baseline/_ref, loop branch) with dequantised-FP4 expert projections "
                "from the reference's own quantiser, torch on all host threads")
    else:
        from oracle import moe_ref

        experts = moe_ref.QuantizedExperts(w_up, w_dn)

        def fwd(lo):
            moe_ref.moe_forward(x[lo:lo + sample], wr, experts, k, True, None, bias)

        kind, what = "port", "numpy restatement of the reference SparseMoE forward on dequantised NVFP4 (oracle/)"
    del w_up, w_dn
    times = []
    for i in range(args.warmup + args.steps):
        lo = (i * sample) % max(1, T - sample + 1)
        t0 = time.perf_counter()
        fwd(lo)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    step = statistics.mean(times)
    value = sample / step
    thr = _host_threads()
    res = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 math on NVFP4-dequantised operands, bf16 I/O",
        "data": "synthetic (numpy PCG64, same shapes and distributions)",
        "config": {"workload": cfg["name"], "tokens_per_gpu": T, "d_model": d, "num_experts": E, "top_k": k,
                   "expert_ffn": F, "parallelism": "host cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": thr["torch_threads"] if kind == "reference"
                         else thr["blas_threads"], "kind": kind, **thr,
                         "sample": f"{sample} tokens of {cfg['name']} per step: {what}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--tokens", type=int, default=0, help="override the configuration's token count (profiling)")
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--cpu-sample", type=int, default=4096,
                    help="--impl reference: tokens per step (a bounded sample of the configuration)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU path on this device")
    ap.add_argument("--fp4-peak", action="store_true", help="measure the cuBLAS dense NVFP4 GEMM rate and exit")
    ap.add_argument("--no-train", action="store_true", help="skip timing a training step (forward + backward)")
    ap.add_argument("--cuda-graph", action="store_true",
                    help="1 GPU: serve the timed forwards from a captured CUDA graph (SparseMoE.enable_cuda_graph)")
    ap.add_argument("--ep-partials", default="copy", choices=("kernel", "copy"),
                    help="expert parallel: partial sums stored to their sources by the summing kernel or copied")
    ap.add_argument("--ep-back", default="h", choices=("h", "partials"),
                    help="expert parallel: NVFP4 h stored to the tokens' home ranks (down projection there), "
                         "or bf16 partial sums returned")
    ap.add_argument("--ep-chunks", type=int, default=0,
                    help="expert parallel (N > 1): token chunks whose exchange overlaps another chunk's experts")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.tokens > 0:
        CONFIGS[args.config] = dict(CONFIGS[args.config], t=args.tokens,
                                    name=f"{CONFIGS[args.config]['name']}_t{args.tokens}")
    if args.fp4_peak:
        fp4_peak(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
