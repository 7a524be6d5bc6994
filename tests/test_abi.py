"""C-ABI checks that need no GPU: the library loads, exports every symbol the
public header declares, and rejects bad arguments on the host."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "mcl4moe.h").read_text()
    return sorted(set(re.findall(r"\b(mcl4moe_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(moe_pkg):
    lib = moe_pkg.library()
    declared = header_symbols()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/mcl4moe.h but not exported"
    assert sorted(moe_pkg._lib.EXPORTS) == declared


def test_status_strings_and_version(moe_pkg):
    lib = moe_pkg.library()
    assert lib.mcl4moe_version() >= 100
    assert moe_pkg._lib.status_string(0) == "ok"
    assert "invalid" in moe_pkg._lib.status_string(1)


def test_workspace_sizes_are_host_only(moe_pkg):
    lib = moe_pkg.library()
    T, d, E, k, F = 32768, 2048, 64, 8, 1024
    ws = lib.mcl4moe_moe_workspace_size(T, d, E, k, F)
    mcap = lib.mcl4moe_padded_rows(T, E, k)
    assert mcap % 128 == 0 and mcap >= T * k + 127 * E
    # y (bf16) dominates: mcap * d * 2 bytes
    assert ws >= mcap * d * 2 + mcap * (d // 2 + d // 16 + F // 2 + F // 16)
    assert lib.mcl4moe_moe_workspace_size(T, 2000, E, k, F) == 0  # d % 256 != 0 -> unsupported
    assert lib.mcl4moe_route_workspace_size(T, E, k, d) > 0


def test_forward_rejects_bad_arguments_without_touching_the_device(moe_pkg):
    lib = moe_pkg.library()
    L = moe_pkg._lib
    assert lib.mcl4moe_moe_forward(None, None) == L.ERR_INVALID
    args = L.MoeArgs(T=16, d=256, E=4, k=8, F=256)  # k > E
    assert lib.mcl4moe_moe_forward(ctypes.byref(args), None) == L.ERR_INVALID
    args = L.MoeArgs(T=16, d=200, E=4, k=2, F=256)  # d % 256
    assert lib.mcl4moe_moe_forward(ctypes.byref(args), None) == L.ERR_UNSUPPORTED
    args = L.MoeArgs(T=16, d=256, E=4, k=2, F=256)  # null pointers
    assert lib.mcl4moe_moe_forward(ctypes.byref(args), None) == L.ERR_INVALID
    assert lib.mcl4moe_quantize_activations(None, 4, 64, 64, None, None, 0, None) == L.ERR_INVALID
    assert lib.mcl4moe_route(None, None, None, None, None, 8, 64, 4, 5, 1, None, None, None, None, None, None,
                             None, 0, None) == L.ERR_INVALID


def test_check_maps_status_to_reference_exception_types(moe_pkg):
    L = moe_pkg._lib
    L.check(L.OK, "x")
    with pytest.raises(ValueError):
        L.check(L.ERR_INVALID, "x")
    with pytest.raises(RuntimeError):
        L.check(L.ERR_CUDA, "x")
