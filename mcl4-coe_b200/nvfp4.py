"""NVFP4 operators of the MoE hot path on the B200 kernels.

Mirrors the reference's operator seam (src/mcl4_coe/nvfp4.py):

* :func:`get_or_build_grouped_cache` — the quantised-weight cache of
  ``_get_or_build_grouped_nvfp4_cache`` (:962-1048): keyed by
  ``(E, N, K, device)``, only experts whose ``(weight._version,
  weight.data_ptr())`` changed are re-quantised, so expert growth / pruning
  (a new ModuleList, or a changed expert count) rebuilds it naturally.
* :func:`nvfp4_grouped_linear` — same signature and result as the reference's
  ``nvfp4_grouped_linear(inputs, experts, proj_name, offs)`` (:1219-1227).
* :func:`quantize_nvfp4` — activation quantisation (``_quantize_nvfp4_core`` in
  the causal-row mode, :197-225), returning packed codes, e4m3 scales, g = 1.
* :func:`export_reference_cache` — the same weight bytes in the reference's
  cache layout (``B_fwd``, ``Bs_fwd``, ``Bg``, ``B_bwd``, ``Bs_bwd``).
* :func:`compute_2to4_mask` — the 2:4 sparsity masks (:70-110); experts whose
  projection carries ``sparsity_mode`` "2to4_row" / "2to4_transposable" (the
  reference's ``NVFP4Linear``) are masked before quantisation, as the
  reference's cache does (:1017-1024), and run on the same dense GEMMs.

Everything runs on CUDA through ``libmcl4moe.so``; CPU tensors are rejected
with ``ValueError`` like the reference's ``quantize_nvfp4`` (:245-246).
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor, nn

from . import _lib

CACHE_ATTR = "_mcl4_b200_nvfp4_cache"


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(t: Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{what} requires a CUDA tensor (the B200 path has no CPU fallback)")


SPARSITY_MODES = ("none", "2to4_row", "2to4_transposable")  # src/mcl4_coe/nvfp4.py:31
_MASK_MODE = {"2to4_row": 1, "2to4_transposable": 2}


def _sparsity_mode(layer: nn.Module) -> str:
    mode = str(getattr(layer, "sparsity_mode", "none"))
    if mode not in SPARSITY_MODES:
        raise ValueError(f"sparsity mode must be one of {SPARSITY_MODES}, got {mode!r}")
    return mode


def _mask_2to4(weight: Tensor, mode: str) -> tuple[Tensor, Tensor]:
    """(w * mask fp32 [N, K], mask uint8 [N, K]) on the device (``mcl4moe_mask_2to4``)."""
    _require_cuda(weight, "the 2:4 sparsity mask")
    w = weight.detach().to(torch.float32).contiguous()
    n, k = w.shape
    if k % 4:
        raise ValueError("the B200 2:4 mask needs in_features divisible by 4")
    masked = torch.empty_like(w)
    mask = torch.empty((n, k), dtype=torch.uint8, device=w.device)
    _lib.check(_lib.load().mcl4moe_mask_2to4(w.data_ptr(), n, k, _MASK_MODE[mode], masked.data_ptr(),
                                             mask.data_ptr(), _stream_handle()), "mcl4moe_mask_2to4")
    return masked, mask


@torch.no_grad()
def compute_2to4_mask(weight: Tensor, mode: str = "2to4_transposable") -> Tensor:
    """Boolean 2:4 mask of a weight ``[out_features, in_features]``
    (src/mcl4_coe/nvfp4.py:70-110): ``"2to4_row"`` keeps the two largest |w| of every
    4 consecutive inputs; ``"2to4_transposable"`` keeps, per 4x4 tile, the doubly
    2:4 pattern of largest kept L1, so W and W.T are both 2:4; ``"none"`` keeps all."""
    if mode not in SPARSITY_MODES:
        raise ValueError(f"sparsity mode must be one of {SPARSITY_MODES}, got {mode!r}")
    if mode == "none":
        return torch.ones_like(weight, dtype=torch.bool)
    if weight.ndim != 2:
        raise ValueError("compute_2to4_mask expects a 2D weight matrix")
    return _mask_2to4(weight, mode)[1].bool()


class GroupedNVFP4Cache:
    """Kernel-layout NVFP4 copy of one projection of every expert.

    ``packed``  uint8 ``[E, N, K/2]`` (K-major E2M1 codes, even K in the low nibble)
    ``scales``  uint8 ``[E, N*K/16]`` e4m3 tile scales in 128x4 swizzled atoms
    ``g``       float32 ``[E]`` per-expert global scale ``amax/2688``
    """

    def __init__(self, e_count: int, n: int, k: int, device: torch.device):
        self.shape_key = (e_count, n, k, str(device))
        self.versions: list = [None] * e_count
        self.packed = torch.empty((e_count, n, k // 2), dtype=torch.uint8, device=device)
        n_pad = (n + 127) // 128 * 128
        self.scales = torch.zeros((e_count, n_pad * k // 16), dtype=torch.uint8, device=device)
        self.g = torch.empty((e_count,), dtype=torch.float32, device=device)
        self.amax = torch.empty((e_count,), dtype=torch.float32, device=device)
        self.masks: list[Tensor | None] = [None] * e_count  # bool [N, K] of 2:4-sparse experts
        self.n, self.k = n, k


def quantize_weight_slots(weights: list[Tensor], slots: list[int], cache: GroupedNVFP4Cache,
                          ref_out: dict | None = None) -> None:
    """Quantise ``weights[i]`` (fp32 ``[N, K]``) into ``cache`` slot ``slots[i]``."""
    lib = _lib.load()
    if not weights:
        return
    staged = [w.detach().to(torch.float32).contiguous() for w in weights]
    for w in staged:
        _require_cuda(w, "NVFP4 weight quantisation")
        if tuple(w.shape) != (cache.n, cache.k):
            raise ValueError("all expert weights of a projection must share one shape")
    n_w = len(staged)
    ptrs = (ctypes.c_void_p * n_w)(*[w.data_ptr() for w in staged])
    slot_arr = (ctypes.c_int32 * n_w)(*slots)
    ref = ref_out or {}
    st = lib.mcl4moe_quantize_weights(ptrs, slot_arr, n_w, cache.n, cache.k, cache.packed.data_ptr(),
                                      cache.scales.data_ptr(), cache.g.data_ptr(), _ptr(ref.get("B_fwd")),
                                      _ptr(ref.get("Bs_fwd")), _ptr(ref.get("B_bwd")), _ptr(ref.get("Bs_bwd")),
                                      cache.amax.data_ptr(), _stream_handle())
    _lib.check(st, "mcl4moe_quantize_weights")
    # ``staged`` copies are released to torch's stream-ordered caching allocator,
    # so their memory is only reused by work queued after the kernel.


@torch.no_grad()
def get_or_build_grouped_cache(experts: nn.ModuleList, proj_name: str) -> GroupedNVFP4Cache:
    """src/mcl4_coe/nvfp4.py:962-1048 on the B200 kernels (see module docstring)."""
    layers = [getattr(e, proj_name) for e in experts]
    weights = [layer.weight for layer in layers]
    if not weights:
        raise ValueError("experts must be non-empty")
    for layer in layers:
        if getattr(layer, "bias", None) is not None:
            raise ValueError("grouped NVFP4 experts must be bias-free (src/mcl4_coe/backbone.py:543-544)")
    e_count = len(weights)
    n, k = weights[0].shape
    device = weights[0].device
    _require_cuda(weights[0], "the NVFP4 weight cache")
    modes = [_sparsity_mode(layer) for layer in layers]
    cur = [(w._version, w.data_ptr(), tuple(w.shape), m) for w, m in zip(weights, modes)]
    store = getattr(experts, CACHE_ATTR, None)
    if store is None:
        store = {}
        try:
            setattr(experts, CACHE_ATTR, store)
        except Exception:  # pragma: no cover - ModuleList always accepts attributes
            pass
    entry = store.get(proj_name)
    if entry is None or entry.shape_key != (e_count, n, k, str(device)):
        entry = GroupedNVFP4Cache(e_count, n, k, device)
        store[proj_name] = entry
    if entry.versions == cur:
        return entry
    dirty = [i for i, (old, new) in enumerate(zip(entry.versions, cur)) if old != new]
    staged = []
    for i in dirty:  # 2:4-sparse experts are masked before quantisation (src/mcl4_coe/nvfp4.py:1017-1024)
        if modes[i] == "none":
            entry.masks[i] = None
            staged.append(weights[i])
        else:
            masked, mask = _mask_2to4(weights[i], modes[i])
            entry.masks[i] = mask.bool()
            staged.append(masked)
    quantize_weight_slots(staged, dirty, entry)
    entry.versions = cur
    return entry


def invalidate_cache(experts: nn.ModuleList) -> None:
    try:
        setattr(experts, CACHE_ATTR, None)
    except Exception:  # pragma: no cover
        pass


@torch.no_grad()
def export_reference_cache(experts: nn.ModuleList, proj_name: str) -> dict[str, Tensor]:
    """Quantise every expert of ``proj_name`` into the reference's cache layout
    (``_get_or_build_grouped_nvfp4_cache`` entries, src/mcl4_coe/nvfp4.py:994-998)."""
    layers = [getattr(e, proj_name) for e in experts]
    weights = [layer.weight if _sparsity_mode(layer) == "none" else _mask_2to4(layer.weight, _sparsity_mode(layer))[0]
               for layer in layers]
    e_count = len(weights)
    n, k = weights[0].shape
    dev = weights[0].device
    cache = GroupedNVFP4Cache(e_count, n, k, dev)
    ref = {
        "B_fwd": torch.empty((e_count, k // 2, n), dtype=torch.uint8, device=dev),
        "Bs_fwd": torch.empty((e_count, n, k // 16), dtype=torch.uint8, device=dev),
        "B_bwd": torch.empty((e_count, n // 2, k), dtype=torch.uint8, device=dev),
        "Bs_bwd": torch.empty((e_count, k, n // 16), dtype=torch.uint8, device=dev),
    }
    quantize_weight_slots(weights, list(range(e_count)), cache, ref)
    ref["Bg"] = cache.g
    ref["Bs_fwd"] = ref["Bs_fwd"].view(torch.float8_e4m3fn)
    ref["Bs_bwd"] = ref["Bs_bwd"].view(torch.float8_e4m3fn)
    return ref


@torch.no_grad()
def quantize_nvfp4(matrix: Tensor, *, swizzled: bool = False) -> tuple[Tensor, Tensor, Tensor]:
    """Activation quantisation with 1x16 row scales and global scale 1.

    src/mcl4_coe/nvfp4.py:235-259 with ``causal_row_scale=True`` (no global
    amax, so later rows never influence earlier rows' bytes).  Returns
    ``(packed uint8 [R, C/2], scales e4m3 [R, C/16] (or swizzled atoms),
    g float32 [1] = 1)``.  The input must be bfloat16 (the MoE path's dtype).
    """
    if matrix.ndim != 2 or not matrix.is_floating_point() or matrix.numel() == 0:
        raise ValueError("NVFP4 quantization requires a nonempty floating-point matrix")
    _require_cuda(matrix, "NVFP4 quantization")
    rows, cols = matrix.shape
    if cols % 16:
        raise ValueError("NVFP4 blocks require aligned dimensions divisible by 16")
    x = matrix.to(torch.bfloat16).contiguous()
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
    if swizzled:
        rp = (rows + 127) // 128 * 128
        scales = torch.zeros((rp * cols // 16,), dtype=torch.uint8, device=x.device)
    else:
        scales = torch.empty((rows, cols // 16), dtype=torch.uint8, device=x.device)
    st = _lib.load().mcl4moe_quantize_activations(x.data_ptr(), rows, cols, cols, packed.data_ptr(),
                                                  scales.data_ptr(), int(swizzled), _stream_handle())
    _lib.check(st, "mcl4moe_quantize_activations")
    return packed, scales.view(torch.float8_e4m3fn), torch.ones(1, dtype=torch.float32, device=x.device)


_GEMM_COUNTS = {"forward": 0}


def get_gemm_counts() -> dict[str, int]:
    """Grouped NVFP4 GEMM calls, counted like src/mcl4_coe/nvfp4.py:29-42."""
    return dict(_GEMM_COUNTS)


def reset_gemm_counts() -> None:
    for key in _GEMM_COUNTS:
        _GEMM_COUNTS[key] = 0


@torch.no_grad()
def nvfp4_grouped_linear(inputs: Tensor, experts: nn.ModuleList, proj_name: str, offs: Tensor) -> Tensor:
    """``nvfp4_grouped_linear`` (src/mcl4_coe/nvfp4.py:1219-1227) on tcgen05.

    ``inputs`` bf16 ``[M, K]`` grouped by expert, ``offs`` int32 ``[E]``
    inclusive ends; returns bf16 ``[M, N]`` with
    ``out[m] = bf16(quant(x[m]) . W_e^T * g_e)``.
    """
    _require_cuda(inputs, "nvfp4_grouped_linear")
    m_total, k = inputs.shape
    entry = get_or_build_grouped_cache(experts, proj_name)
    e_count = entry.packed.shape[0]
    n = entry.n
    if k != entry.k:
        raise ValueError("inputs must end in in_features")
    out = torch.empty((m_total, n), dtype=torch.bfloat16, device=inputs.device)
    if m_total == 0:
        return out
    x = inputs.to(torch.bfloat16).contiguous()
    offs32 = offs.to(device=inputs.device, dtype=torch.int32).contiguous()
    lib = _lib.load()
    ws_bytes = lib.mcl4moe_grouped_linear_workspace_size(m_total, k, e_count)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=inputs.device)
    st = lib.mcl4moe_grouped_linear(x.data_ptr(), m_total, k, offs32.data_ptr(), e_count, entry.packed.data_ptr(),
                                    entry.scales.data_ptr(), entry.g.data_ptr(), n, out.data_ptr(), None,
                                    ws.data_ptr(), ws_bytes, _stream_handle())
    _lib.check(st, "mcl4moe_grouped_linear")
    _GEMM_COUNTS["forward"] += e_count
    return out
