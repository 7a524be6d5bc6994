"""mcl4moe_route_noalloc (scratch in a fixed device array of the library) against
mcl4moe_route (caller workspace): identical outputs on two calls in a row, no
device memory taken after the first call, and oversized shapes rejected on the
host.  Kept last in collection order so it also runs after every other test has
used the library in the same process."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_ref import x_tensor
from inputs import routing_cases

DEV = "cuda"
OUT_NAMES = ("topk_idx", "topk_w", "logits", "sel", "counts", "stats")


def test_scratch_limit_and_oversize_rejected_on_host(moe_pkg):
    lib = moe_pkg.library()
    L = moe_pkg._lib
    cap = lib.mcl4moe_route_noalloc_scratch_bytes()
    assert cap == 8 << 20
    assert lib.mcl4moe_route_workspace_size(131072, 64, 8, 2048) <= cap
    big_t = 1 << 20
    assert lib.mcl4moe_route_workspace_size(big_t, 64, 8, 2048) > cap
    # Stand-in pointers: the size check returns before any pointer is used or
    # the device is touched.
    fake = ctypes.c_void_p(4096)
    st = lib.mcl4moe_route_noalloc(fake, fake, None, None, None, big_t, 2048, 64, 8, 1, fake, fake, None, None,
                                   fake, fake, None)
    assert st == L.ERR_WORKSPACE
    with pytest.raises(RuntimeError, match="workspace"):
        L.check(st, "route_noalloc")
    assert lib.mcl4moe_route_noalloc(None, None, None, None, None, 8, 64, 4, 5, 1, None, None, None, None, None,
                                     None, None) == L.ERR_INVALID


def _buffers(T, E, k):
    # at least one row: an empty batch still passes real (non-null) output pointers
    R = max(T, 1)
    return dict(topk_idx=torch.full((R, k), -7, dtype=torch.int32, device=DEV),
                topk_w=torch.full((R, k), float("nan"), dtype=torch.float32, device=DEV),
                logits=torch.full((R, E), float("nan"), dtype=torch.float32, device=DEV),
                sel=torch.full((R, E), float("nan"), dtype=torch.float32, device=DEV),
                counts=torch.full((E,), -7, dtype=torch.int32, device=DEV),
                stats=torch.full((3 + E,), float("nan"), dtype=torch.float32, device=DEV))


def _call(pkg, inp, out, workspace=None):
    lib = pkg.library()
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    common = (p(inp["x"]), p(inp["wr"]), p(inp["bias"]), p(inp["logits_in"]), p(inp["valid"]), inp["T"], inp["d"],
              inp["E"], inp["k"], inp["norm"], out["topk_idx"].data_ptr(), out["topk_w"].data_ptr(),
              out["logits"].data_ptr(), out["sel"].data_ptr(), out["counts"].data_ptr(), out["stats"].data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    if workspace is None:
        st = lib.mcl4moe_route_noalloc(*common, stream)
    else:
        st = lib.mcl4moe_route(*common, workspace.data_ptr(), workspace.numel(), stream)
    pkg._lib.check(st, "route_noalloc" if workspace is None else "route")


def _case_inputs(c, with_logits_in=False):
    inp = dict(T=c["t"], d=c["d"], E=c["e"], k=c["k"], norm=int(c["norm_topk_prob"]), x=x_tensor(c, DEV),
               wr=torch.from_numpy(c["wr"]).to(DEV), logits_in=None,
               bias=None if c["logit_bias"] is None else torch.from_numpy(c["logit_bias"]).to(DEV),
               valid=None if c["valid"] is None else torch.from_numpy(c["valid"]).to(DEV))
    if with_logits_in:
        inp["logits_in"] = (inp["x"].float() @ inp["wr"].t()).contiguous()
    return inp


def _random_inputs(seed, T, d, E, k):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn((max(T, 1), d), generator=g, device=DEV).to(torch.bfloat16)
    wr = torch.randn((E, d), generator=g, device=DEV) * 0.02
    return dict(T=T, d=d, E=E, k=k, norm=1, x=x, wr=wr, bias=None, logits_in=None, valid=None)


def _pairs():
    cases = dict(routing_cases())
    return [
        ("golden_pair", _case_inputs(cases["r_c0"]), _case_inputs(cases["r_valid"])),
        ("zipf_then_logits_in", _case_inputs(cases["r_zipf"]), _case_inputs(cases["r_e64k8"], with_logits_in=True)),
        ("olmoe_full_size", _random_inputs(20, 32768, 2048, 64, 8), _random_inputs(21, 32768, 2048, 64, 8)),
        # the empty batch (launch_route's own counter reset) and the largest batch the
        # 8 MiB scratch holds at E = 64, k = 8, d = 2048
        ("empty_then_near_cap", _random_inputs(22, 0, 2048, 64, 8), _random_inputs(23, 131072, 2048, 64, 8)),
    ]


@pytest.mark.gpu
def test_noalloc_matches_reference_golden_routing(moe_pkg, golden):
    """The scratch-array entry point against the reference's own recorded routing
    (golden case r_c0: logits, top-k ids in order, weights, statistics)."""
    from gpu_ref import order_tie_tokens

    c = dict(routing_cases())["r_c0"]
    g = golden("routing")
    inp = _case_inputs(c)
    out = _buffers(inp["T"], inp["E"], inp["k"])
    for _ in range(2):
        _call(moe_pkg, inp, out)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out["logits"].cpu().numpy(), g["r_c0__logits"], rtol=1e-5, atol=2e-6)
    tie = order_tie_tokens(g["r_c0__logits"], c["k"])
    same = np.all(out["topk_idx"].cpu().numpy() == g["r_c0__topk_indices"], axis=1)
    assert np.all(same | tie)
    np.testing.assert_allclose(out["stats"].cpu().numpy()[0], g["r_c0__aux"], rtol=1e-4)
    np.testing.assert_allclose(out["stats"].cpu().numpy()[1], g["r_c0__z"], rtol=1e-4)
    if not tie.any():
        np.testing.assert_array_equal(out["stats"].cpu().numpy()[3:], g["r_c0__counts"])


@pytest.mark.gpu
def test_noalloc_matches_workspace_route_on_two_calls_in_a_row(moe_pkg):
    lib = moe_pkg.library()
    for name, a, b in _pairs():
        # reference results through the workspace entry point
        refs = []
        for inp in (a, b):
            ws = torch.empty((lib.mcl4moe_route_workspace_size(inp["T"], inp["E"], inp["k"], inp["d"]),),
                             dtype=torch.uint8, device=DEV)
            out = _buffers(inp["T"], inp["E"], inp["k"])
            _call(moe_pkg, inp, out, workspace=ws)
            torch.cuda.synchronize()
            refs.append({n: t.cpu().numpy() for n, t in out.items()})
            del ws
        outs = [_buffers(a["T"], a["E"], a["k"]), _buffers(b["T"], b["E"], b["k"])]
        _call(moe_pkg, a, outs[0])  # first call on the device performs the set-up
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        # two calls back to back on one stream, no host synchronisation between them
        _call(moe_pkg, a, outs[0])
        _call(moe_pkg, b, outs[1])
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before, f"{name}: device memory was allocated"
        for inp, ref, out in zip((a, b), refs, outs):
            for n in OUT_NAMES:
                got = out[n].cpu().numpy()
                assert np.array_equal(got, ref[n], equal_nan=True), f"{name}: {n} differs"
            if inp["T"] > 0:
                assert np.all(ref["topk_idx"] != -7)
            assert not np.isnan(ref["stats"]).any()
