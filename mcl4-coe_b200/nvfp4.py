"""NVFP4 operators of the MoE hot path on the B200 kernels.

Mirrors the reference's operator seam (src/mcl4_coe/nvfp4.py):

* :func:`get_or_build_grouped_cache` — the quantised-weight cache of
  ``_get_or_build_grouped_nvfp4_cache`` (:962-1048): keyed by
  ``(E, N, K, device)``, only experts whose ``(weight._version,
  weight.data_ptr())`` changed are re-quantised.  When expert growth or
  pruning (a new ModuleList, or a changed expert count) makes a new cache, the
  experts it keeps bring their NVFP4 bytes along by a device-to-device copy, so
  only new or changed experts are quantised (the reference re-quantises every
  expert of a rebuilt cache); ``CACHE_STATS`` counts both.
* :func:`nvfp4_grouped_linear` — same signature and result as the reference's
  ``nvfp4_grouped_linear(inputs, experts, proj_name, offs)`` (:1219-1227).
* :func:`quantize_activations` — the MoE path's activation quantisation
  (``_quantize_nvfp4_core`` in the causal-row mode, :197-225): packed codes,
  e4m3 scales (row-major or swizzled), g = 1.
* :func:`quantize_nvfp4`, :func:`nvfp4_mm`, :class:`NVFP4Linear`,
  :func:`convert_linear_to_nvfp4` — the single-matrix operators with the
  reference's signatures (:235-259, :285-334, :398-542, :634-695): quantisation
  in every mode but stochastic rounding, the NVFP4 GEMM with fp32 output on the
  tcgen05 grouped kernel (one segment), the projection module with its cached
  (optionally 2:4-masked) weight, forward only.
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
import operator

import torch
from torch import Tensor, nn

from . import _lib

CACHE_ATTR = "_mcl4_b200_nvfp4_cache"
# Each projection module remembers the cache entry and slot that hold its NVFP4 bytes,
# so a cache built for a new expert set copies them instead of re-quantising.
SLOT_ATTR = "_mcl4_b200_nvfp4_slot"
# Expert matrices quantised and carried over (copied from a previous cache) so far.
CACHE_STATS = {"quantized": 0, "carried": 0}


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
    mode = layer.__dict__.get("sparsity_mode")  # instance attribute: no nn.Module.__getattr__ walk
    if mode is None:
        mode = getattr(layer, "sparsity_mode", "none")
    mode = str(mode)
    if mode not in SPARSITY_MODES:
        raise ValueError(f"sparsity mode must be one of {SPARSITY_MODES}, got {mode!r}")
    return mode


def _submodule(module: nn.Module, name: str) -> nn.Module:
    """``getattr(module, name)`` for a registered submodule through the module's own dict
    (nn.Module.__getattr__ costs ~0.5 us a call, and the weight caches are checked for
    every expert on every forward)."""
    sub = module.__dict__.get("_modules", {}).get(name)
    return sub if sub is not None else getattr(module, name)


def _weight(layer: nn.Module):
    w = layer.__dict__.get("_parameters", {}).get("weight")
    return w if w is not None else layer.weight


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
        # W^T in the kernel layout (the backward's input-gradient operand), made on demand
        self.packed_t: Tensor | None = None
        self.scales_t: Tensor | None = None
        self._owners: tuple | None = None  # what ``versions`` was read from (see still_current)

    def remember_owners(self, experts: nn.ModuleList, proj_name: str, layers: list, weights: list) -> None:
        """Record the module dicts, Parameters, versions and storages ``versions`` was read
        from, so that the next forward can confirm them without a walk through
        nn.Module.__getattr__ per expert (which cost ~150 us per projection at 64 experts)."""
        self._owners = None
        try:
            mods = list(experts.__dict__["_modules"].values())
            subdicts = [m.__dict__["_modules"] for m in mods]
            pdicts = [layer.__dict__["_parameters"] for layer in layers]
        except (KeyError, AttributeError):
            return
        ldicts = [layer.__dict__ for layer in layers]
        if not (all(map(operator.is_, [sd.get(proj_name) for sd in subdicts], layers))
                and all(map(operator.is_, [pd.get("weight") for pd in pdicts], weights))):
            return
        self._owners = (proj_name, mods, subdicts, list(layers), pdicts, ldicts, list(weights),
                        [w._version for w in weights], [w.data_ptr() for w in weights],
                        [ld.get("sparsity_mode") for ld in ldicts])

    def still_current(self, experts: nn.ModuleList, proj_name: str) -> bool:
        """True when the same expert modules hold the same projection modules, whose
        ``weight`` Parameters are the recorded objects at the recorded ``_version`` and
        storage, with the recorded sparsity modes and no bias: ``versions`` is then exact
        for every expert and no slot needs quantising."""
        own = self._owners
        if own is None or own[0] != proj_name:
            return False
        _, mods, subdicts, layers, pdicts, ldicts, weights, versions, ptrs, modes = own
        md = experts.__dict__.get("_modules")
        if md is None or len(md) != len(mods) or not all(map(operator.is_, md.values(), mods)):
            return False
        if not all(map(operator.is_, [sd.get(proj_name) for sd in subdicts], layers)):
            return False
        if not all(map(operator.is_, [pd.get("weight") for pd in pdicts], weights)):
            return False
        if not all(pd.get("bias") is None for pd in pdicts):
            return False
        return ([w._version for w in weights] == versions and [w.data_ptr() for w in weights] == ptrs
                and [ld.get("sparsity_mode") for ld in ldicts] == modes)

    def enable_transposed(self) -> None:
        """Allocate the transposed copy (packed [E, K, N/2], swizzled scales [E, K*N/16]);
        every slot must then be quantised again."""
        if self.packed_t is not None:
            return
        e_count, dev = self.packed.shape[0], self.packed.device
        self.packed_t = torch.empty((e_count, self.k, self.n // 2), dtype=torch.uint8, device=dev)
        self.scales_t = torch.zeros((e_count, (self.k + 127) // 128 * 128 * (self.n // 16)), dtype=torch.uint8,
                                    device=dev)
        self.versions = [None] * e_count
        self._owners = None


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
    if cache.packed_t is not None and ref_out is None:
        st = lib.mcl4moe_quantize_weights_t(ptrs, slot_arr, n_w, cache.n, cache.k, cache.packed.data_ptr(),
                                            cache.scales.data_ptr(), cache.g.data_ptr(), cache.packed_t.data_ptr(),
                                            cache.scales_t.data_ptr(), cache.amax.data_ptr(), _stream_handle())
        _lib.check(st, "mcl4moe_quantize_weights_t")
        return
    st = lib.mcl4moe_quantize_weights(ptrs, slot_arr, n_w, cache.n, cache.k, cache.packed.data_ptr(),
                                      cache.scales.data_ptr(), cache.g.data_ptr(), _ptr(ref.get("B_fwd")),
                                      _ptr(ref.get("Bs_fwd")), _ptr(ref.get("B_bwd")), _ptr(ref.get("Bs_bwd")),
                                      cache.amax.data_ptr(), _stream_handle())
    _lib.check(st, "mcl4moe_quantize_weights")
    # ``staged`` copies are released to torch's stream-ordered caching allocator,
    # so their memory is only reused by work queued after the kernel.


@torch.no_grad()
def get_or_build_grouped_cache(experts: nn.ModuleList, proj_name: str, with_bwd: bool = False) -> GroupedNVFP4Cache:
    """src/mcl4_coe/nvfp4.py:962-1048 on the B200 kernels (see module docstring)."""
    store = experts.__dict__.get(CACHE_ATTR)
    if store:
        entry = store.get(proj_name)
        if (entry is not None and (not with_bwd or entry.packed_t is not None)
                and entry.still_current(experts, proj_name)):
            return entry
    layers = [_submodule(e, proj_name) for e in experts]
    weights = [_weight(layer) for layer in layers]
    if not weights:
        raise ValueError("experts must be non-empty")
    for layer in layers:
        params = layer.__dict__.get("_parameters")
        if (params.get("bias") if params is not None else getattr(layer, "bias", None)) is not None:
            raise ValueError("grouped NVFP4 experts must be bias-free (src/mcl4_coe/backbone.py:543-544)")
    e_count = len(weights)
    n, k = weights[0].shape
    device = weights[0].device
    _require_cuda(weights[0], "the NVFP4 weight cache")
    cur = _current_versions(layers, weights)
    modes = [v[3] for v in cur]
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
        if with_bwd:
            entry.enable_transposed()
        store[proj_name] = entry
        _carry_over(layers, cur, entry)
    elif with_bwd and entry.packed_t is None:
        entry.enable_transposed()  # training starts: every expert also needs its transposed copy
    if entry.versions == cur:
        entry.remember_owners(experts, proj_name, layers, weights)
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
    CACHE_STATS["quantized"] += len(dirty)
    entry.versions = cur
    for i in dirty:
        setattr(layers[i], SLOT_ATTR, (entry, i))
    entry.remember_owners(experts, proj_name, layers, weights)
    return entry


def _carry_over(layers: list, cur: list, entry: GroupedNVFP4Cache) -> None:
    """Copy into the new ``entry`` the NVFP4 bytes of every expert whose weight is
    unchanged since a previous cache quantised it (expert growth / pruning keeps the
    surviving experts' modules): same version, storage, shape and sparsity mode."""
    src_slots: dict[int, list[tuple[int, int]]] = {}
    owners: dict[int, GroupedNVFP4Cache] = {}
    for i, layer in enumerate(layers):
        prev = getattr(layer, SLOT_ATTR, None)
        if prev is None:
            continue
        old, j = prev
        if (old is entry or old.n != entry.n or old.k != entry.k or old.packed.device != entry.packed.device
                or j >= len(old.versions) or old.versions[j] != cur[i]
                or (entry.packed_t is not None and old.packed_t is None)):
            continue
        owners[id(old)] = old
        src_slots.setdefault(id(old), []).append((j, i))
    for key, pairs in src_slots.items():
        old = owners[key]
        src = torch.tensor([j for j, _ in pairs], dtype=torch.long, device=entry.packed.device)
        dst = torch.tensor([i for _, i in pairs], dtype=torch.long, device=entry.packed.device)
        entry.packed.index_copy_(0, dst, old.packed.index_select(0, src))
        entry.scales.index_copy_(0, dst, old.scales.index_select(0, src))
        entry.g.index_copy_(0, dst, old.g.index_select(0, src))
        if entry.packed_t is not None:
            entry.packed_t.index_copy_(0, dst, old.packed_t.index_select(0, src))
            entry.scales_t.index_copy_(0, dst, old.scales_t.index_select(0, src))
        for j, i in pairs:
            entry.masks[i] = old.masks[j]
            entry.versions[i] = cur[i]
            setattr(layers[i], SLOT_ATTR, (entry, i))
        CACHE_STATS["carried"] += len(pairs)


def _current_versions(layers: list, weights: list | None = None) -> list:
    if weights is None:
        weights = [_weight(layer) for layer in layers]
    return [(w._version, w.data_ptr(), tuple(w.shape), _sparsity_mode(layer)) for layer, w in zip(layers, weights)]


@torch.no_grad()
def seed_grouped_cache(experts: nn.ModuleList, proj_name: str, filled: dict) -> GroupedNVFP4Cache:
    """Make the cache of ``experts`` (carrying over the bytes of experts a previous
    cache holds) and install NVFP4 bytes quantised elsewhere: ``filled[i] = (packed
    [N, K/2], scales [N_pad*K/16], g [1])`` for slot i, taken as the quantisation of
    expert i's current weight (expert parallelism moves experts with their bytes)."""
    layers = [getattr(e, proj_name) for e in experts]
    n, k = layers[0].weight.shape
    device = layers[0].weight.device
    cur = _current_versions(layers)
    store = getattr(experts, CACHE_ATTR, None)
    if store is None:
        store = {}
        setattr(experts, CACHE_ATTR, store)
    entry = store.get(proj_name)
    if entry is None or entry.shape_key != (len(layers), n, k, str(device)):
        entry = GroupedNVFP4Cache(len(layers), n, k, device)
        store[proj_name] = entry
        _carry_over(layers, cur, entry)
    entry._owners = None  # versions change below
    for i, (packed, scales, g) in filled.items():
        entry.packed[i].copy_(packed.view(entry.packed[i].shape))
        entry.scales[i].copy_(scales.view(entry.scales[i].shape))
        entry.g[i:i + 1].copy_(g.view(1))
        entry.masks[i] = None
        entry.versions[i] = cur[i]
        setattr(layers[i], SLOT_ATTR, (entry, i))
    CACHE_STATS["carried"] += len(filled)
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
def quantize_activations(matrix: Tensor, *, swizzled: bool = False) -> tuple[Tensor, Tensor, Tensor]:
    """The MoE path's activation quantisation: 1x16 row scales and global scale 1.

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


# ---------------------------------------------------------------------------- single-matrix operators

def _round_up(value: int, multiple: int) -> int:
    return (value + multiple - 1) // multiple * multiple


_FP4_DTYPE = getattr(torch, "float4_e2m1fn_x2", torch.uint8)


def _noise_seed() -> int:
    """31-bit stochastic-rounding seed from torch's default CPU generator, so
    ``torch.manual_seed`` makes the rounding noise reproducible as it does for the
    reference's ``torch.rand_like`` draws."""
    return int(torch.randint(0, 2 ** 31 - 1, (1,)).item())


@torch.no_grad()
def quantize_nvfp4(matrix: Tensor, *, two_dimensional: bool = False, stochastic: bool = False,
                   causal_row_scale: bool = False) -> tuple[Tensor, Tensor, Tensor]:
    """Packed FP4 (``float4_e2m1fn_x2`` [R, C/2]), swizzled E4M3 scales ([R rounded to 128,
    C/16 rounded to 4], the 128x4-atom layout) and fp32 global scale [1]
    (src/mcl4_coe/nvfp4.py:235-259): one-dimensional 1x16 blocks with g = amax/2688, or
    g = 1 when ``causal_row_scale``; ``two_dimensional``: 16x16 tiles with g = amax/2688.
    ``stochastic`` (one-dimensional): codes min(trunc(u + U), 7) with U uniform in [0, 1)
    from Philox4x32-10 under a seed drawn from torch's default generator (the reference
    draws U with ``torch.rand_like``); two-dimensional stochastic rounding, which no
    reference caller uses, raises NotImplementedError."""
    if matrix.ndim != 2 or not matrix.is_floating_point() or matrix.numel() == 0:
        raise ValueError("NVFP4 quantization requires a nonempty floating-point matrix")
    _require_cuda(matrix, "NVFP4 quantization")
    rows, cols = matrix.shape
    if cols % 16 or (two_dimensional and rows % 16):
        raise ValueError("NVFP4 blocks require aligned dimensions divisible by 16")
    if stochastic and two_dimensional:
        raise NotImplementedError("two-dimensional stochastic NVFP4 rounding is not served by the B200 path")
    dev = matrix.device
    cp = _round_up(cols, 64)  # scale columns padded to whole 4-column atoms, as _swizzle_scales pads them
    if two_dimensional:
        w = matrix.detach().to(torch.float32)
        if cp != cols:
            w = torch.nn.functional.pad(w, (0, cp - cols))
        cache = GroupedNVFP4Cache(1, rows, cp, dev)
        quantize_weight_slots([w], [0], cache)
        packed = cache.packed[0][:, : cols // 2].contiguous()
        scales = cache.scales[0].view(_round_up(rows, 128), cp // 16)
        return packed.view(_FP4_DTYPE), scales.view(torch.float8_e4m3fn), cache.g.clone()
    x = matrix.detach()
    dtype = 0 if x.dtype == torch.bfloat16 else 1
    x = x.contiguous() if dtype == 0 else x.to(torch.float32).contiguous()
    if cp != cols:
        x = torch.nn.functional.pad(x, (0, cp - cols))
    rp = _round_up(rows, 128)
    packed = torch.empty((rows, cp // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty((rp, cp // 16), dtype=torch.uint8, device=dev)
    g = torch.empty((1,), dtype=torch.float32, device=dev)
    amax = torch.empty((1,), dtype=torch.float32, device=dev)
    lib = _lib.load()
    if stochastic:
        _lib.check(lib.mcl4moe_quantize_rows_stochastic(x.data_ptr(), dtype, rows, cp, cp, int(bool(causal_row_scale)),
                                                        _noise_seed(), packed.data_ptr(), scales.data_ptr(), rp,
                                                        g.data_ptr(), amax.data_ptr(), _stream_handle()),
                   "mcl4moe_quantize_rows_stochastic")
    else:
        _lib.check(lib.mcl4moe_quantize_rows(x.data_ptr(), dtype, rows, cp, cp, int(bool(causal_row_scale)),
                                             packed.data_ptr(), scales.data_ptr(), rp, g.data_ptr(), amax.data_ptr(),
                                             _stream_handle()), "mcl4moe_quantize_rows")
    return packed[:, : cols // 2].contiguous().view(_FP4_DTYPE), scales.view(torch.float8_e4m3fn), g


def _relayout_operand(packed: Tensor, scales: Tensor, rows: int, cols: int, rows_to: int, cols_to: int):
    """A quantised operand (packed [>=rows, >=cols/2], swizzled scales for its padded shape)
    zero-padded to [rows_to, cols_to] in the kernel layout (K a multiple of 256 so every
    stage reads whole tiles; the swizzled order depends on the padded column count)."""
    dev = packed.device
    pk = torch.zeros((rows_to, cols_to // 2), dtype=torch.uint8, device=dev)
    pk[:rows, : cols // 2] = packed.view(torch.uint8)[:rows, : cols // 2]
    sc = scales.view(torch.uint8)
    rp, cpb = sc.shape
    plain = sc.view(rp // 128, cpb // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(rp, cpb)[:rows, : cols // 16]
    full = torch.zeros((_round_up(rows_to, 128), cols_to // 16), dtype=torch.uint8, device=dev)
    full[:rows, : cols // 16] = plain
    r2, c2 = full.shape
    sw = full.view(r2 // 128, 4, 32, c2 // 4, 4).permute(0, 3, 2, 1, 4).contiguous().view(-1)
    return pk, sw


def _mm_prepared(a: Tensor, b_packed: Tensor, b_scales: Tensor, b_g: Tensor, n_pad: int, k_pad: int,
                 causal_a: bool, bias: Tensor | None, stochastic_a: bool = False) -> Tensor:
    """fp32 [M, n_pad] = deq(A) deq(B)^T g_a g_b (+ bias) on the kernels; B already in the
    kernel layout for [n_pad, k_pad]; A rounded stochastically with ``stochastic_a``."""
    m, k = a.shape
    dtype = 0 if a.dtype == torch.bfloat16 else 1
    x = a.detach().contiguous() if dtype == 0 else a.detach().to(torch.float32).contiguous()
    if k_pad != k:
        x = torch.nn.functional.pad(x, (0, k_pad - k))
    lib = _lib.load()
    out = torch.empty((m, n_pad), dtype=torch.float32, device=a.device)
    ws = torch.empty((max(lib.mcl4moe_nvfp4_mm_workspace_size(m, k_pad), 256),), dtype=torch.uint8, device=a.device)
    if stochastic_a:
        _lib.check(lib.mcl4moe_nvfp4_mm_sr(x.data_ptr(), dtype, m, k_pad, int(bool(causal_a)), _noise_seed(),
                                           b_packed.data_ptr(), b_scales.data_ptr(), b_g.data_ptr(), n_pad, _ptr(bias),
                                           out.data_ptr(), None, None, ws.data_ptr(), ws.numel(), _stream_handle()),
                   "mcl4moe_nvfp4_mm_sr")
    else:
        _lib.check(lib.mcl4moe_nvfp4_mm(x.data_ptr(), dtype, m, k_pad, int(bool(causal_a)), b_packed.data_ptr(),
                                        b_scales.data_ptr(), b_g.data_ptr(), n_pad, _ptr(bias), out.data_ptr(), None,
                                        None, ws.data_ptr(), ws.numel(), _stream_handle()), "mcl4moe_nvfp4_mm")
    return out


@torch.no_grad()
def nvfp4_mm(a: Tensor, b: Tensor, *, weight_b: bool = False, stochastic_a: bool = False, stochastic_b: bool = False,
             causal_a: bool = False, prequantized_b: tuple[Tensor, Tensor, Tensor] | None = None,
             _phase: str = "other") -> Tensor:
    """``a @ b.T`` in NVFP4, fp32 result [M, N] (src/mcl4_coe/nvfp4.py:285-334): A quantised
    one-dimensionally (g = 1 with ``causal_a``), B two-dimensionally with ``weight_b`` (else
    one-dimensionally), or ``prequantized_b`` = (packed, swizzled scales, g) as
    :func:`quantize_nvfp4` returns them for ``b`` padded to multiples of 32.
    ``stochastic_a`` / ``stochastic_b``: stochastic rounding of that operand (one-dimensional
    only for B).  Runs on the tcgen05 block-scaled GEMM with K and N padded to 256."""
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("NVFP4 matmul expects a[M,K] and b[N,K]")
    if a.device != b.device or a.device.type != "cuda":
        raise ValueError("NVFP4 matmul requires both operands on the same CUDA device")
    m, k = a.shape
    n = b.shape[0]
    if min(m, n, k) == 0:
        raise ValueError("NVFP4 matmul requires nonempty operands")
    if stochastic_b and weight_b and prequantized_b is None:
        raise NotImplementedError("two-dimensional stochastic NVFP4 rounding is not served by the B200 path")
    kp, np_ = _round_up(k, 256), _round_up(n, 256)
    if prequantized_b is not None:
        qb, sb, gb = prequantized_b
        rows_b = sb.shape[0] if sb.ndim == 2 else _round_up(n, 32)
        pk, sw = _relayout_operand(qb, sb.view(torch.uint8).view(rows_b, -1), _round_up(n, 32), _round_up(k, 32),
                                   np_, kp)
    else:
        bp = b.detach()
        if kp != k or np_ != n:
            bp = torch.nn.functional.pad(bp.to(torch.float32 if weight_b else bp.dtype), (0, kp - k, 0, np_ - n))
        qb, sb, gb = quantize_nvfp4(bp, two_dimensional=weight_b, stochastic=stochastic_b)
        pk, sw = qb.view(torch.uint8), sb.view(torch.uint8).reshape(-1)
    _GEMM_COUNTS[_phase] = _GEMM_COUNTS.get(_phase, 0) + 1
    return _mm_prepared(a, pk, sw, gb.to(torch.float32).reshape(1), np_, kp, causal_a, None,
                        stochastic_a=stochastic_a)[:, :n]


def _linear_weight_grad(gradient: Tensor, inputs: Tensor, with_bias: bool) -> tuple[Tensor, Tensor | None]:
    """fp32 [N, K] ``nvfp4_mm(_hadamard16(gradient.t()), _hadamard16(inputs.t()),
    stochastic_a=True)`` and, with ``with_bias``, the fp32 column sums of ``gradient``
    (src/mcl4_coe/nvfp4.py:454-459, :468-469), on mcl4moe_nvfp4_linear_wgrad."""
    m, n = gradient.shape
    k = inputs.shape[1]
    dev = gradient.device

    def operand(t: Tensor) -> tuple[Tensor, int]:
        if t.dtype == torch.bfloat16:
            return t.contiguous(), 0
        return t.to(torch.float32).contiguous(), 1

    g, gdt = operand(gradient.detach())
    x, xdt = operand(inputs.detach())
    kp = _round_up(k, 256)
    lib = _lib.load()
    dw = torch.empty((n, kp), dtype=torch.float32, device=dev)
    db = torch.empty((n,), dtype=torch.float32, device=dev) if with_bias else None
    ws = torch.empty((max(lib.mcl4moe_nvfp4_linear_wgrad_workspace_size(m, n, k), 256),), dtype=torch.uint8,
                     device=dev)
    _lib.check(lib.mcl4moe_nvfp4_linear_wgrad(g.data_ptr(), gdt, x.data_ptr(), xdt, m, n, k, _noise_seed(),
                                              dw.data_ptr(), _ptr(db), None, ws.data_ptr(), ws.numel(),
                                              _stream_handle()), "mcl4moe_nvfp4_linear_wgrad")
    _GEMM_COUNTS["wgrad"] = _GEMM_COUNTS.get("wgrad", 0) + 1
    return dw[:, :k], db


class _NVFP4LinearFunction(torch.autograd.Function):
    """_NVFP4Linear (src/mcl4_coe/nvfp4.py:391-472) on the kernels.  Forward: the
    layer's NVFP4 GEMM.  Backward: input gradient = stochastic-rounded gradient x the
    weight's transposed 16x16-tile quantisation (mcl4moe_nvfp4_mm_sr); weight gradient =
    the Hadamard16-transformed NVFP4 product (mcl4moe_nvfp4_linear_wgrad) plus the SR-STE
    decay of masked-out weights; bias gradient = fp32 column sums of the gradient."""

    @staticmethod
    def forward(ctx, flat, weight, bias, layer):
        ctx.layer = layer
        ctx.bias_dtype = None if bias is None else bias.dtype
        ctx.save_for_backward(flat, weight)
        with torch.no_grad():
            return layer._forward_flat(flat)

    @staticmethod
    def backward(ctx, grad_output):
        flat, weight = ctx.saved_tensors
        layer = ctx.layer
        n, k = weight.shape
        gradient = grad_output.reshape(-1, n)
        grad_inputs = grad_weight = grad_bias = None
        need_bias = ctx.bias_dtype is not None and ctx.needs_input_grad[2]
        with torch.no_grad():
            if ctx.needs_input_grad[0]:
                pk_t, sw_t, g, _ = layer._quantised_weight(transposed=True)
                np_, kp = _round_up(n, 256), _round_up(k, 256)
                _GEMM_COUNTS["dgrad"] = _GEMM_COUNTS.get("dgrad", 0) + 1
                grad_inputs = _mm_prepared(gradient, pk_t, sw_t, g, kp, np_, False, None,
                                           stochastic_a=True)[:, :k].to(flat.dtype)
            db = None
            if ctx.needs_input_grad[1]:
                dw, db = _linear_weight_grad(gradient, flat, need_bias)
                grad_weight = dw.to(weight.dtype)
                mask = layer._quantised_weight()[3]
                if mask is not None and layer.sr_ste_decay > 0.0:
                    # SR-STE (src/mcl4_coe/nvfp4.py:460-466): decay of the masked-out weights
                    grad_weight = grad_weight + layer.sr_ste_decay * (~mask).to(weight.dtype) * weight
            if need_bias:
                if db is None:
                    db = gradient.float().sum(dim=0)
                grad_bias = db.to(ctx.bias_dtype)
        return grad_inputs, grad_weight, grad_bias, None


class NVFP4Linear(nn.Linear):
    """Projection on native NVFP4 GEMMs with optional 2:4 weight sparsity
    (src/mcl4_coe/nvfp4.py:474-542).  Forward: 1x16 activation blocks (g = 1 with
    ``causal_activation_scale``), the cached 16x16-tile weight (2:4-masked first when
    ``sparsity_mode`` is not "none"), fp32 accumulation, ``+ bias`` in fp32, cast to the
    input dtype.  Under autograd it trains like the reference (_NVFP4Linear.backward,
    :431-472): stochastic-rounded NVFP4 input and weight gradients, the weight gradient
    through the Hadamard16 transform.  CUDA only (no CPU fallback)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None, dtype=None, *,
                 sparsity_mode: str = "2to4_transposable", sr_ste_decay: float = 1e-4,
                 causal_activation_scale: bool = True) -> None:
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=dtype)
        if sparsity_mode not in SPARSITY_MODES:
            raise ValueError(f"sparsity_mode must be one of {SPARSITY_MODES}")
        self.sparsity_mode = sparsity_mode
        self.sr_ste_decay = float(sr_ste_decay)
        self.causal_activation_scale = bool(causal_activation_scale)
        self._b200_weight_cache: list | None = None

    @classmethod
    def from_linear(cls, layer: nn.Linear, *, sparsity_mode: str = "2to4_transposable", sr_ste_decay: float = 1e-4,
                    causal_activation_scale: bool = True) -> "NVFP4Linear":
        converted = cls(layer.in_features, layer.out_features, bias=layer.bias is not None,
                        device=layer.weight.device, dtype=layer.weight.dtype, sparsity_mode=sparsity_mode,
                        sr_ste_decay=sr_ste_decay, causal_activation_scale=causal_activation_scale)
        converted.load_state_dict(layer.state_dict())
        converted.weight.requires_grad_(layer.weight.requires_grad)
        if converted.bias is not None:
            converted.bias.requires_grad_(layer.bias.requires_grad)
        converted.train(layer.training)
        return converted

    @torch.no_grad()
    def active_2to4_mask(self) -> Tensor:
        """The current 2:4 boolean weight mask [out_features, in_features]."""
        return compute_2to4_mask(self.weight, mode=self.sparsity_mode)

    def _quantised_weight(self, transposed: bool = False) -> tuple:
        """(packed, swizzled scales, g, mask) of the weight padded to multiples of 256, cached
        on (weight._version, data_ptr, shape, device, sparsity_mode) like
        _get_or_build_weight_nvfp4_cache (src/mcl4_coe/nvfp4.py:358-389); ``transposed``:
        the 16x16-tile quantisation of the masked weight's transpose [K, N] (the
        backward's ``bwd_q``, built on first use and cached with the same key)."""
        w = self.weight
        key = (w._version, w.data_ptr(), tuple(w.shape), str(w.device), self.sparsity_mode)
        c = self._b200_weight_cache
        if c is None or c[0] != key:
            n, k = w.shape
            mask = None
            w_eff = w.detach().to(torch.float32)
            if self.sparsity_mode != "none":
                w_eff, m8 = _mask_2to4(w_eff, self.sparsity_mode)
                mask = m8.bool()
            np_, kp = _round_up(n, 256), _round_up(k, 256)
            if (np_, kp) != (n, k):
                w_eff = torch.nn.functional.pad(w_eff, (0, kp - k, 0, np_ - n))
            qb, sb, gb = quantize_nvfp4(w_eff, two_dimensional=True)
            c = self._b200_weight_cache = [key, qb.view(torch.uint8), sb.view(torch.uint8).reshape(-1), gb, mask,
                                           None]
        if not transposed:
            return tuple(c[1:5])
        if c[5] is None:
            n, k = w.shape
            w_eff = w.detach().to(torch.float32)
            if c[4] is not None:
                w_eff = w_eff * c[4].to(torch.float32)
            np_, kp = _round_up(n, 256), _round_up(k, 256)
            wt = torch.zeros((kp, np_), dtype=torch.float32, device=w_eff.device)
            wt[:k, :n] = w_eff.t()
            qt, st, gt = quantize_nvfp4(wt, two_dimensional=True)
            c[5] = (qt.view(torch.uint8), st.view(torch.uint8).reshape(-1), gt)
        return (*c[5], c[4])

    def _forward_flat(self, flat: Tensor) -> Tensor:
        """[M, in_features] -> [M, out_features] in flat.dtype (no autograd)."""
        pk, sw, g, _ = self._quantised_weight()
        n, k = self.weight.shape
        np_, kp = _round_up(n, 256), _round_up(k, 256)
        bias = None
        if self.bias is not None:  # fp32, zero-padded to the GEMM's N; rebuilt when the bias changes
            b = self.bias
            bkey = (b._version, b.data_ptr(), str(flat.device))
            cached = getattr(self, "_b200_bias_cache", None)
            if cached is None or cached[0] != bkey:
                padded = torch.zeros((np_,), dtype=torch.float32, device=flat.device)
                padded[:n] = b.detach().to(device=flat.device, dtype=torch.float32)
                self._b200_bias_cache = cached = (bkey, padded)
            bias = cached[1]
        _GEMM_COUNTS["forward"] = _GEMM_COUNTS.get("forward", 0) + 1
        return _mm_prepared(flat, pk, sw, g, np_, kp, self.causal_activation_scale, bias)[:, :n].to(flat.dtype)

    def forward(self, inputs: Tensor) -> Tensor:
        if inputs.ndim < 1 or inputs.shape[-1] != self.in_features:
            raise ValueError("NVFP4Linear input must end in in_features")
        _require_cuda(inputs, "NVFP4Linear")
        flat = inputs.reshape(-1, self.in_features)
        if flat.shape[0] == 0:
            return inputs.new_empty(*inputs.shape[:-1], self.out_features)
        if torch.is_grad_enabled() and (inputs.requires_grad or self.weight.requires_grad
                                        or (self.bias is not None and self.bias.requires_grad)):
            out = _NVFP4LinearFunction.apply(flat, self.weight, self.bias, self)
        else:
            with torch.no_grad():
                out = self._forward_flat(flat)
        return out.reshape(*inputs.shape[:-1], self.out_features)


def convert_linear_to_nvfp4(module: nn.Module, *, min_features: int = 32, experts_only: bool = True,
                            sparsity_mode: str = "2to4_transposable", sr_ste_decay: float = 1e-4,
                            causal_activation_scale: bool = True,
                            exclude_names: tuple[str, ...] = ("router", "token_scorer", "ple", "route_",
                                                              "start_query")) -> int:
    """Replace eligible ``nn.Linear`` submodules by :class:`NVFP4Linear`
    (src/mcl4_coe/nvfp4.py:598-695): with ``experts_only`` and any ``SwiGLUExpert`` present,
    only the experts' ``up_proj`` / ``down_proj``; otherwise every Linear with both sides
    >= ``min_features`` whose child name contains none of ``exclude_names``.  Returns the
    number converted."""
    kw = dict(sparsity_mode=sparsity_mode, sr_ste_decay=sr_ste_decay, causal_activation_scale=causal_activation_scale)

    def eligible(layer) -> bool:
        return (isinstance(layer, nn.Linear) and not isinstance(layer, NVFP4Linear)
                and layer.in_features >= min_features and layer.out_features >= min_features)

    if experts_only:
        count = 0
        for child in module.modules():
            if child.__class__.__name__ == "SwiGLUExpert":
                for attr in ("up_proj", "down_proj"):
                    layer = getattr(child, attr, None)
                    if eligible(layer):
                        setattr(child, attr, NVFP4Linear.from_linear(layer, **kw))
                        count += 1
        if count > 0:
            return count
    count = 0
    for name, child in list(module.named_children()):
        if any(ex in name for ex in exclude_names):
            continue
        if eligible(child):
            setattr(module, name, NVFP4Linear.from_linear(child, **kw))
            count += 1
        else:
            count += convert_linear_to_nvfp4(child, min_features=min_features, experts_only=False,
                                             exclude_names=exclude_names, **kw)
    return count

