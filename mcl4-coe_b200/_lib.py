"""ctypes binding of ``libmcl4moe.so`` (the C ABI declared in include/mcl4moe.h).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.  Status codes map to the reference's exception types:
invalid arguments -> ValueError (src/mcl4_coe/nvfp4.py:243-249), everything
else -> RuntimeError.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint8, c_uint16, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmcl4moe.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_WORKSPACE = range(6)

# Every symbol include/mcl4moe.h declares (checked by tests/test_abi.py).
EXPORTS = (
    "mcl4moe_status_string",
    "mcl4moe_version",
    "mcl4moe_device_supported",
    "mcl4moe_read_error",
    "mcl4moe_quantize_weights",
    "mcl4moe_mask_2to4",
    "mcl4moe_quantize_rows",
    "mcl4moe_nvfp4_mm_workspace_size",
    "mcl4moe_nvfp4_mm",
    "mcl4moe_quantize_activations",
    "mcl4moe_route_workspace_size",
    "mcl4moe_route",
    "mcl4moe_route_noalloc_scratch_bytes",
    "mcl4moe_route_noalloc",
    "mcl4moe_moe_workspace_size",
    "mcl4moe_moe_forward",
    "mcl4moe_moe_forward_routed",
    "mcl4moe_padded_rows",
    "mcl4moe_set_expert_tiling",
    "mcl4moe_moe_forward_layout",
    "mcl4moe_moe_forward_down",
    "mcl4moe_ep_dispatch_pack_h",
    "mcl4moe_ep_gateup_to_peers",
    "mcl4moe_workspace_region",
    "mcl4moe_grouped_linear_workspace_size",
    "mcl4moe_grouped_linear",
    "mcl4moe_ep_row_bytes",
    "mcl4moe_ep_dispatch_workspace_size",
    "mcl4moe_ep_dispatch",
    "mcl4moe_ep_dispatch_count",
    "mcl4moe_ep_dispatch_pack",
    "mcl4moe_ep_experts_workspace_size",
    "mcl4moe_ep_experts",
    "mcl4moe_ep_combine",
    "mcl4moe_ep_experts_to_peers",
    "mcl4moe_ipc_export",
    "mcl4moe_ipc_import",
    "mcl4moe_ipc_close",
    "mcl4moe_copy_async",
    "mcl4moe_copy_list_async",
    "mcl4moe_quantize_weights_t",
    "mcl4moe_quantize_rows_sr",
    "mcl4moe_moe_backward_workspace_size",
    "mcl4moe_moe_backward_experts",
    "mcl4moe_router_backward",
    "mcl4moe_moe_backward_dx",
    "mcl4moe_moe_backward_wgrad",
    "mcl4moe_quantize_rows_stochastic",
    "mcl4moe_nvfp4_mm_sr",
    "mcl4moe_quantize_hadamard_t",
    "mcl4moe_nvfp4_linear_wgrad_workspace_size",
    "mcl4moe_nvfp4_linear_wgrad",
)


class MoeArgs(ctypes.Structure):
    """Mirror of ``mcl4moe_moe_args``."""

    _fields_ = [
        ("x", c_void_p),
        ("router_w", c_void_p),
        ("logit_bias", c_void_p),
        ("valid", c_void_p),
        ("w_up", c_void_p),
        ("w_up_scales", c_void_p),
        ("w_up_g", c_void_p),
        ("w_dn", c_void_p),
        ("w_dn_scales", c_void_p),
        ("w_dn_g", c_void_p),
        ("T", c_int),
        ("d", c_int),
        ("E", c_int),
        ("k", c_int),
        ("F", c_int),
        ("norm_topk_prob", c_int),
        ("out", c_void_p),
        ("stats", c_void_p),
        ("sel_mask", c_void_p),
        ("topk_idx", c_void_p),
        ("topk_w", c_void_p),
        ("offs", c_void_p),
        ("perm", c_void_p),
        ("h_debug", c_void_p),
        ("error_word", c_void_p),
        ("workspace", c_void_p),
        ("workspace_bytes", c_size_t),
        ("stage_events", POINTER(c_void_p)),
        ("up_save", c_void_p),
        ("x_rows_save", c_void_p),
        ("y_save", c_void_p),
        ("logits_out", c_void_p),
    ]


class MoeBwdArgs(ctypes.Structure):
    """Mirror of ``mcl4moe_moe_bwd_args``."""

    _fields_ = [
        ("T", c_int), ("d", c_int), ("E", c_int), ("k", c_int), ("F", c_int),
        ("d_out", c_void_p), ("slot_pos", c_void_p), ("topk_w", c_void_p), ("pad_start", c_void_p),
        ("counts", c_void_p), ("offs_start", c_void_p), ("y_save", c_void_p), ("up_save", c_void_p),
        ("w_up_t", c_void_p), ("w_up_t_scales", c_void_p), ("w_up_g", c_void_p),
        ("w_dn_t", c_void_p), ("w_dn_t_scales", c_void_p), ("w_dn_g", c_void_p),
        ("seed_down", ctypes.c_uint64), ("seed_up", ctypes.c_uint64),
        ("d_y", c_void_p), ("d_up", c_void_p), ("d_rows", c_void_p), ("d_w", c_void_p),
        ("error_word", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


_lib = None


class ExtensionMissing(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the library once; raise ``ExtensionMissing`` if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ExtensionMissing(
            f"{LIB_PATH} is missing: build it with `python mcl4-coe_b200/build.py` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.mcl4moe_status_string.restype = c_char_p
    lib.mcl4moe_status_string.argtypes = [c_int]
    lib.mcl4moe_version.restype = c_int
    lib.mcl4moe_device_supported.restype = c_int
    lib.mcl4moe_read_error.restype = c_int
    lib.mcl4moe_read_error.argtypes = [c_void_p, POINTER(c_int32), c_void_p]
    lib.mcl4moe_quantize_rows.restype = c_int
    lib.mcl4moe_quantize_rows.argtypes = [c_void_p, c_int, c_int64, c_int, c_int64, c_int, c_void_p, c_void_p, c_int64,
                                          c_void_p, c_void_p, c_void_p]
    lib.mcl4moe_nvfp4_mm_workspace_size.restype = c_size_t
    lib.mcl4moe_nvfp4_mm_workspace_size.argtypes = [c_int64, c_int]
    lib.mcl4moe_nvfp4_mm.restype = c_int
    lib.mcl4moe_nvfp4_mm.argtypes = [c_void_p, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int,
                                     c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_mask_2to4.restype = c_int
    lib.mcl4moe_mask_2to4.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]
    lib.mcl4moe_quantize_weights.restype = c_int
    lib.mcl4moe_quantize_weights.argtypes = [POINTER(c_void_p), POINTER(c_int32), c_int, c_int, c_int,
                                             c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                             c_void_p, c_void_p, c_void_p]
    lib.mcl4moe_quantize_activations.restype = c_int
    lib.mcl4moe_quantize_activations.argtypes = [c_void_p, c_int64, c_int, c_int64, c_void_p, c_void_p, c_int,
                                                 c_void_p]
    lib.mcl4moe_route_workspace_size.restype = c_size_t
    lib.mcl4moe_route_workspace_size.argtypes = [c_int, c_int, c_int, c_int]
    lib.mcl4moe_route.restype = c_int
    lib.mcl4moe_route.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                  c_void_p]
    lib.mcl4moe_route_noalloc_scratch_bytes.restype = c_size_t
    lib.mcl4moe_route_noalloc_scratch_bytes.argtypes = []
    lib.mcl4moe_route_noalloc.restype = c_int
    lib.mcl4moe_route_noalloc.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                          c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p]
    lib.mcl4moe_moe_workspace_size.restype = c_size_t
    lib.mcl4moe_moe_workspace_size.argtypes = [c_int, c_int, c_int, c_int, c_int]
    lib.mcl4moe_moe_forward.restype = c_int
    lib.mcl4moe_moe_forward.argtypes = [POINTER(MoeArgs), c_void_p]
    lib.mcl4moe_moe_forward_routed.restype = c_int
    lib.mcl4moe_moe_forward_routed.argtypes = [POINTER(MoeArgs), c_void_p]
    lib.mcl4moe_padded_rows.restype = c_int64
    lib.mcl4moe_padded_rows.argtypes = [c_int, c_int, c_int]
    lib.mcl4moe_workspace_region.restype = c_void_p
    lib.mcl4moe_workspace_region.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int]
    lib.mcl4moe_grouped_linear_workspace_size.restype = c_size_t
    lib.mcl4moe_grouped_linear_workspace_size.argtypes = [c_int64, c_int, c_int]
    lib.mcl4moe_grouped_linear.restype = c_int
    lib.mcl4moe_grouped_linear.argtypes = [c_void_p, c_int64, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                           c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_ep_row_bytes.restype = c_int
    lib.mcl4moe_ep_row_bytes.argtypes = [c_int, c_int]
    lib.mcl4moe_ep_dispatch_workspace_size.restype = c_size_t
    lib.mcl4moe_ep_dispatch_workspace_size.argtypes = [c_int, c_int]
    lib.mcl4moe_ep_dispatch.restype = c_int
    lib.mcl4moe_ep_dispatch.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                        c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_ep_dispatch_count.restype = c_int
    lib.mcl4moe_ep_dispatch_count.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                              c_size_t, c_void_p]
    lib.mcl4moe_ep_dispatch_pack.restype = c_int
    lib.mcl4moe_ep_dispatch_pack.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                             c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_ep_experts_workspace_size.restype = c_size_t
    lib.mcl4moe_ep_experts_workspace_size.argtypes = [c_int, c_int, c_int, c_int, c_int, c_int]
    lib.mcl4moe_ep_experts.restype = c_int
    lib.mcl4moe_ep_experts.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_size_t, c_void_p]
    lib.mcl4moe_ep_experts_to_peers.restype = c_int
    lib.mcl4moe_ep_experts_to_peers.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                                c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p,
                                                c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_ep_combine.restype = c_int
    lib.mcl4moe_ep_combine.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]
    lib.mcl4moe_ipc_export.restype = c_int
    lib.mcl4moe_ipc_export.argtypes = [c_void_p, c_void_p, POINTER(ctypes.c_uint64)]
    lib.mcl4moe_ipc_import.restype = c_int
    lib.mcl4moe_ipc_import.argtypes = [c_void_p, POINTER(c_void_p)]
    lib.mcl4moe_ipc_close.restype = c_int
    lib.mcl4moe_ipc_close.argtypes = [c_void_p]
    lib.mcl4moe_copy_async.restype = c_int
    lib.mcl4moe_copy_async.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_copy_list_async.restype = c_int
    lib.mcl4moe_copy_list_async.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int]
    lib.mcl4moe_quantize_weights_t.restype = c_int
    lib.mcl4moe_quantize_weights_t.argtypes = [POINTER(c_void_p), POINTER(c_int32), c_int, c_int, c_int, c_void_p,
                                               c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
    lib.mcl4moe_quantize_rows_sr.restype = c_int
    lib.mcl4moe_quantize_rows_sr.argtypes = [c_void_p, c_int64, c_int, ctypes.c_uint64, c_void_p, c_void_p, c_void_p,
                                             c_void_p, c_void_p]
    lib.mcl4moe_moe_backward_workspace_size.restype = c_size_t
    lib.mcl4moe_moe_backward_workspace_size.argtypes = [c_int, c_int, c_int, c_int, c_int]
    lib.mcl4moe_moe_backward_experts.restype = c_int
    lib.mcl4moe_moe_backward_experts.argtypes = [POINTER(MoeBwdArgs), c_void_p]
    lib.mcl4moe_router_backward.restype = c_int
    lib.mcl4moe_router_backward.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]
    lib.mcl4moe_moe_backward_wgrad.restype = c_int
    lib.mcl4moe_moe_backward_wgrad.argtypes = [c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_int, c_void_p,
                                               c_void_p, c_void_p]
    lib.mcl4moe_quantize_rows_stochastic.restype = c_int
    lib.mcl4moe_quantize_rows_stochastic.argtypes = [c_void_p, c_int, c_int64, c_int, c_int64, c_int, ctypes.c_uint64,
                                                     c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]
    lib.mcl4moe_nvfp4_mm_sr.restype = c_int
    lib.mcl4moe_nvfp4_mm_sr.argtypes = [c_void_p, c_int, c_int64, c_int, c_int, ctypes.c_uint64, c_void_p, c_void_p,
                                        c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                        c_void_p]
    lib.mcl4moe_quantize_hadamard_t.restype = c_int
    lib.mcl4moe_quantize_hadamard_t.argtypes = [c_void_p, c_int, c_int64, c_int, c_int64, c_int, c_int, ctypes.c_uint64,
                                                c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]
    lib.mcl4moe_nvfp4_linear_wgrad_workspace_size.restype = c_size_t
    lib.mcl4moe_nvfp4_linear_wgrad_workspace_size.argtypes = [c_int64, c_int, c_int]
    lib.mcl4moe_nvfp4_linear_wgrad.restype = c_int
    lib.mcl4moe_nvfp4_linear_wgrad.argtypes = [c_void_p, c_int, c_void_p, c_int, c_int64, c_int, c_int,
                                               ctypes.c_uint64, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                               c_void_p]
    lib.mcl4moe_moe_forward_layout.restype = c_int
    lib.mcl4moe_moe_forward_layout.argtypes = [POINTER(MoeArgs), c_void_p]
    lib.mcl4moe_moe_forward_down.restype = c_int
    lib.mcl4moe_moe_forward_down.argtypes = [POINTER(MoeArgs), c_void_p, c_void_p, c_void_p]
    lib.mcl4moe_ep_dispatch_pack_h.restype = c_int
    lib.mcl4moe_ep_dispatch_pack_h.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                               c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_ep_gateup_to_peers.restype = c_int
    lib.mcl4moe_ep_gateup_to_peers.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                               c_void_p, c_int, POINTER(c_void_p), POINTER(c_void_p), c_void_p,
                                               c_void_p, c_size_t, c_void_p]
    lib.mcl4moe_set_expert_tiling.restype = c_int
    lib.mcl4moe_set_expert_tiling.argtypes = [c_int]
    lib.mcl4moe_moe_backward_dx.restype = c_int
    lib.mcl4moe_moe_backward_dx.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().mcl4moe_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status == OK:
        return
    msg = f"{what}: {status_string(status)} (status {status})"
    if status == ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


__all__ = ["load", "check", "MoeArgs", "MoeBwdArgs", "EXPORTS", "LIB_PATH", "ExtensionMissing",
           "c_float", "c_uint8", "c_uint16"]
