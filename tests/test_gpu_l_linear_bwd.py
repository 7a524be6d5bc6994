"""Backward of the single-matrix NVFP4 projection on B200 (_NVFP4Linear.backward,
src/mcl4_coe/nvfp4.py:431-472), against the oracle.

* ``mcl4moe_quantize_hadamard_t`` (the weight-gradient operands,
  ``quantize_nvfp4(_hadamard16(y.t()))``): bytes and global scale bit-exact against the
  oracle, which is pinned to the reference's ``_hadamard16`` / quantiser by
  ``hadamard.npz``; to nearest and stochastic, bf16 and fp32 input, ragged token counts,
  row-major and swizzled scales.
* Stochastic rounding of the single-matrix operators (``quantize_nvfp4(stochastic=True)``,
  ``nvfp4_mm(stochastic_a=True)``): codes bit-exact against the oracle for the same seed,
  scales equal to the round-to-nearest ones, results against the dequantised operands.
* ``mcl4moe_nvfp4_linear_wgrad``: the fp32 weight gradient against the product of the
  oracle's dequantised operands; the bias gradient against float64 column sums.
* ``NVFP4Linear`` under autograd: gradients within the stochastic-rounding noise of an fp32
  reference, unbiased over seeds, reproducible under ``torch.manual_seed``, the SR-STE term,
  and the same error magnitude as the reference's own ``_NVFP4Linear`` when its installed
  copy is importable.
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch
from torch import nn

from inputs import hadamard_cases
from oracle import nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _hadamard_t(moe_pkg, y: torch.Tensor, kt: int, rows_out: int, stochastic: bool, seed: int, swizzled: bool):
    lib = moe_pkg.library()
    m, c = y.shape
    packed = torch.empty((rows_out, kt // 2), dtype=torch.uint8, device=DEV)
    scales = torch.empty((rows_out * (kt // 16),), dtype=torch.uint8, device=DEV)
    g = torch.empty((1,), dtype=torch.float32, device=DEV)
    amax = torch.empty((1,), dtype=torch.float32, device=DEV)
    dtype = 0 if y.dtype == torch.bfloat16 else 1
    moe_pkg._lib.check(lib.mcl4moe_quantize_hadamard_t(y.data_ptr(), dtype, m, c, kt, rows_out, int(stochastic), seed,
                                                       packed.data_ptr(), scales.data_ptr(), int(swizzled),
                                                       g.data_ptr(), amax.data_ptr(), _stream()),
                       "mcl4moe_quantize_hadamard_t")
    torch.cuda.synchronize()
    return packed.cpu().numpy(), scales.cpu().numpy(), g.cpu().numpy()


def _cases():
    out = [(name, y) for name, y in hadamard_cases()]
    r = np.random.default_rng(31)
    big = (r.standard_normal((1000, 96)) * np.exp(r.standard_normal((1, 96)))).astype(np.float32)
    out.append(("wide_1000x96", big))
    return out


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
@pytest.mark.parametrize("stochastic", [False, True])
@pytest.mark.parametrize("as_bf16", [False, True])
def test_hadamard_operand_bytes(moe_pkg, case, stochastic, as_bf16):
    name, y = case
    if as_bf16:
        y = nr.round_bf16(y)
    m, c = y.shape
    kt = nr.round_up(m, 128)
    seed = 0x1234_5678_9A if stochastic else 0
    yt = torch.from_numpy(y).to(DEV, torch.bfloat16 if as_bf16 else torch.float32)
    for swizzled in (False, True):
        rows_out = nr.round_up(c, 128 if swizzled else 32)
        packed, scales, g = _hadamard_t(moe_pkg, yt, kt, rows_out, stochastic, seed, swizzled)
        ref_p, ref_s, ref_g = nr.linear_wgrad_operand(y, kt, rows_out, stochastic, seed)
        assert g.view(np.uint32)[0] == ref_g.view(np.uint32)[0]
        np.testing.assert_array_equal(packed, ref_p)
        exp_s = nr.swizzle_scales(ref_s).reshape(-1) if swizzled else ref_s.reshape(-1)
        np.testing.assert_array_equal(scales, exp_s)


def test_quantize_rows_stochastic_bytes(moe_pkg):
    lib = moe_pkg.library()
    r = np.random.default_rng(9)
    for rows, cols, dt in ((40, 256, torch.bfloat16), (130, 320, torch.float32)):
        x = (r.standard_normal((rows, cols)) * 1e-3).astype(np.float32)
        x[3] = 0.0
        x[5, :16] = -0.0
        if dt == torch.bfloat16:
            x = nr.round_bf16(x)
        xt = torch.from_numpy(x).to(DEV, dt)
        rp = nr.round_up(rows, 128)
        for causal in (0, 1):
            packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=DEV)
            scales = torch.empty((rp * cols // 16,), dtype=torch.uint8, device=DEV)
            g = torch.empty((1,), dtype=torch.float32, device=DEV)
            amax = torch.empty((1,), dtype=torch.float32, device=DEV)
            seed = 987654321
            moe_pkg._lib.check(lib.mcl4moe_quantize_rows_stochastic(
                xt.data_ptr(), 0 if dt == torch.bfloat16 else 1, rows, cols, cols, causal, seed, packed.data_ptr(),
                scales.data_ptr(), rp, g.data_ptr(), amax.data_ptr(), _stream()), "stochastic rows")
            torch.cuda.synchronize()
            ref_p, ref_s, ref_g = nr.quantize_nvfp4_sr(x, seed, causal_row_scale=bool(causal))
            assert g.cpu().numpy().view(np.uint32)[0] == ref_g.view(np.uint32)[0]
            np.testing.assert_array_equal(packed.cpu().numpy(), ref_p)
            np.testing.assert_array_equal(scales.cpu().numpy(), nr.swizzle_scales(np.pad(ref_s, ((0, rp - rows),
                                                                                                 (0, 0)))).reshape(-1))


def test_quantize_nvfp4_stochastic_api(moe_pkg):
    """The reference's ``quantize_nvfp4(..., stochastic=True)``: the round-to-nearest
    scales, codes that bracket the value, reproducible under torch.manual_seed, fresh
    noise otherwise."""
    r = np.random.default_rng(10)
    x = torch.from_numpy((r.standard_normal((64, 512)) * 0.02).astype(np.float32)).to(DEV)
    p_rn, s_rn, g_rn = moe_pkg.quantize_nvfp4(x)
    torch.manual_seed(3)
    p1, s1, g1 = moe_pkg.quantize_nvfp4(x, stochastic=True)
    torch.manual_seed(3)
    p2, _, _ = moe_pkg.quantize_nvfp4(x, stochastic=True)
    p3, _, _ = moe_pkg.quantize_nvfp4(x, stochastic=True)
    torch.cuda.synchronize()
    assert torch.equal(s1.view(torch.uint8), s_rn.view(torch.uint8)) and torch.equal(g1, g_rn)
    assert torch.equal(p1.view(torch.uint8), p2.view(torch.uint8))
    assert not torch.equal(p1.view(torch.uint8), p3.view(torch.uint8))
    with pytest.raises(NotImplementedError):
        moe_pkg.quantize_nvfp4(x, stochastic=True, two_dimensional=True)


def _dequant_rows(packed: np.ndarray, scales_rowmajor: np.ndarray, g: float) -> np.ndarray:
    rows, half = packed.shape
    return nr.dequantize(packed, scales_rowmajor, np.float32(g), rows, 2 * half).astype(np.float64)


def test_nvfp4_mm_stochastic_a(moe_pkg):
    """dgrad's GEMM: stochastic A (the gradient) times a prequantised 16x16-tile B."""
    lib = moe_pkg.library()
    r = np.random.default_rng(12)
    m, k, n = 200, 512, 256
    a = nr.round_bf16((r.standard_normal((m, k)) * 1e-2).astype(np.float32))
    b = (r.standard_normal((n, k)) * 0.05).astype(np.float32)
    qb, sb, gb = moe_pkg.quantize_nvfp4(torch.from_numpy(b).to(DEV), two_dimensional=True)
    at = torch.from_numpy(a).to(DEV, torch.bfloat16)
    out = torch.empty((m, n), dtype=torch.float32, device=DEV)
    ws = torch.empty((lib.mcl4moe_nvfp4_mm_workspace_size(m, k),), dtype=torch.uint8, device=DEV)
    ga = torch.empty((1,), dtype=torch.float32, device=DEV)
    seed = 4242
    moe_pkg._lib.check(lib.mcl4moe_nvfp4_mm_sr(at.data_ptr(), 0, m, k, 0, seed, qb.view(torch.uint8).data_ptr(),
                                               sb.view(torch.uint8).data_ptr(), gb.data_ptr(), n, None,
                                               out.data_ptr(), ga.data_ptr(), None, ws.data_ptr(), ws.numel(),
                                               _stream()), "nvfp4_mm_sr")
    torch.cuda.synchronize()
    pa, sa, g_a = nr.quantize_nvfp4_sr(a, seed)
    assert float(ga) == float(g_a[0])
    pb, sb_rm, g_b = nr.quantize_nvfp4_core(b, True, False)
    ref = _dequant_rows(pa, sa, g_a[0]) @ _dequant_rows(pb, sb_rm, g_b[0]).T
    err = np.linalg.norm(out.cpu().numpy() - ref) / np.linalg.norm(ref)
    assert err < 1e-5, err


@pytest.mark.parametrize("m,n,k,g_bf16,x_bf16", [(300, 256, 384, True, True), (1000, 96, 130, False, True),
                                                 (37, 64, 48, True, False)])
def test_linear_wgrad_matches_dequantised_operands(moe_pkg, m, n, k, g_bf16, x_bf16):
    lib = moe_pkg.library()
    r = np.random.default_rng(m + n + k)
    g = (r.standard_normal((m, n)) * 1e-3).astype(np.float32)
    x = r.standard_normal((m, k)).astype(np.float32)
    if g_bf16:
        g = nr.round_bf16(g)
    if x_bf16:
        x = nr.round_bf16(x)
    gt = torch.from_numpy(g).to(DEV, torch.bfloat16 if g_bf16 else torch.float32)
    xt = torch.from_numpy(x).to(DEV, torch.bfloat16 if x_bf16 else torch.float32)
    kp = nr.round_up(k, 256)
    dw = torch.empty((n, kp), dtype=torch.float32, device=DEV)
    db = torch.empty((n,), dtype=torch.float32, device=DEV)
    ws = torch.empty((lib.mcl4moe_nvfp4_linear_wgrad_workspace_size(m, n, k),), dtype=torch.uint8, device=DEV)
    seed = 777
    moe_pkg._lib.check(lib.mcl4moe_nvfp4_linear_wgrad(gt.data_ptr(), 0 if g_bf16 else 1, xt.data_ptr(),
                                                      0 if x_bf16 else 1, m, n, k, seed, dw.data_ptr(),
                                                      db.data_ptr(), None, ws.data_ptr(), ws.numel(), _stream()),
                       "linear_wgrad")
    torch.cuda.synchronize()
    kt = nr.round_up(m, 256)
    pa, sa, g_a = nr.linear_wgrad_operand(g, kt, nr.round_up(n, 256), True, seed)
    pb, sb, g_b = nr.linear_wgrad_operand(x, kt, kp, False)
    ref = _dequant_rows(pa, sa, g_a[0])[:n] @ _dequant_rows(pb, sb, g_b[0]).T
    got = dw.cpu().numpy()
    assert np.all(got[:, k:] == 0.0)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < 1e-5, err
    ref_b = g.astype(np.float64).sum(axis=0)
    np.testing.assert_allclose(db.cpu().numpy(), ref_b, rtol=1e-4, atol=1e-6 * np.abs(g).sum(axis=0).max())
    # the transform is orthonormal over tokens: the product estimates G^T X
    exact = g.astype(np.float64).T @ x.astype(np.float64)
    assert np.linalg.norm(got[:, :k] - exact) / np.linalg.norm(exact) < 0.3


def _linear_pair(moe_pkg, n_out=384, k_in=512, bias=True, sparsity="none", decay=0.0, seed=0):
    r = np.random.default_rng(seed)
    lin = nn.Linear(k_in, n_out, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy((r.standard_normal((n_out, k_in)) * 0.03).astype(np.float32)))
        if bias:
            lin.bias.copy_(torch.from_numpy(r.standard_normal(n_out).astype(np.float32) * 0.1))
    mod = moe_pkg.NVFP4Linear.from_linear(lin, sparsity_mode=sparsity, sr_ste_decay=decay).to(DEV)
    return lin.to(DEV), mod


def _grads(mod, x, gout):
    mod.zero_grad(set_to_none=True)
    xi = x.detach().clone().requires_grad_(True)
    y = mod(xi)
    y.backward(gout)
    return (xi.grad.float().clone(), mod.weight.grad.float().clone(),
            None if mod.bias is None else mod.bias.grad.float().clone(), y.detach())


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def test_nvfp4_linear_backward_against_fp32(moe_pkg):
    """Gradients through the NVFP4 forward and the stochastic-rounded NVFP4 backward
    against fp32 autograd of the same layer (the reference's backward carries the same
    quantisation noise), and the bias gradient exactly the column sums."""
    lin, mod = _linear_pair(moe_pkg)
    r = np.random.default_rng(1)
    x = torch.from_numpy(r.standard_normal((2, 600, 512)).astype(np.float32)).to(DEV, torch.bfloat16)
    gout = torch.from_numpy((r.standard_normal((2, 600, 384)) * 1e-2).astype(np.float32)).to(DEV, torch.bfloat16)
    torch.manual_seed(0)
    dx, dw, db, y = _grads(mod, x, gout)
    assert dx.shape == x.shape and dw.shape == (384, 512) and db.shape == (384,)
    xf = x.float().detach().requires_grad_(True)
    ref = torch.nn.functional.linear(xf, lin.weight.float(), lin.bias.float())
    ref.backward(gout.float())
    assert _rel(dx, xf.grad) < 0.25, _rel(dx, xf.grad)
    assert _rel(dw, lin.weight.grad) < 0.25, _rel(dw, lin.weight.grad)
    torch.testing.assert_close(db, gout.float().reshape(-1, 384).sum(0), rtol=1e-4, atol=1e-4)
    # the forward is unchanged by autograd
    with torch.no_grad():
        assert torch.equal(mod(x), y)
    # same torch seed: the same noise, bit for bit
    torch.manual_seed(0)
    dx2, dw2, _, _ = _grads(mod, x, gout)
    assert torch.equal(dx, dx2) and torch.equal(dw, dw2)
    print(f"[linear bwd] rel err dx {_rel(dx, xf.grad):.3e} dW {_rel(dw, lin.weight.grad):.3e}")


def test_nvfp4_linear_backward_is_unbiased(moe_pkg):
    """Averaging the stochastic-rounded gradients over seeds approaches the products of the
    deterministic operands (the quantised weight for dx; the exact transformed gradient
    times the quantised transformed input for dW): the rounding noise has mean zero."""
    lin, mod = _linear_pair(moe_pkg, bias=False, seed=4)
    r = np.random.default_rng(2)
    m = 512
    x = torch.from_numpy(r.standard_normal((m, 512)).astype(np.float32)).to(DEV, torch.bfloat16)
    gout = torch.from_numpy((r.standard_normal((m, 384)) * 1e-2).astype(np.float32)).to(DEV, torch.bfloat16)
    g_np = gout.float().cpu().numpy()
    x_np = x.float().cpu().numpy()
    w_np = lin.weight.detach().cpu().numpy()
    pw, sw, gw = nr.quantize_nvfp4_core(w_np, True, False)
    ref_x = torch.from_numpy(g_np.astype(np.float64) @ nr.dequantize(pw, sw, gw[0], 384, 512).astype(np.float64))
    kt = nr.round_up(m, 256)
    a_exact = nr.hadamard16(np.pad(g_np.T, ((0, 0), (0, kt - m)))).astype(np.float64)
    pb, sb, gb = nr.linear_wgrad_operand(x_np, kt, 512, False)
    ref_w = torch.from_numpy(a_exact @ _dequant_rows(pb, sb, gb[0]).T)
    n = 24
    acc_x = torch.zeros(ref_x.shape, dtype=torch.float64)
    acc_w = torch.zeros(ref_w.shape, dtype=torch.float64)
    one_x = one_w = None
    for i in range(n):
        dx, dw, _, _ = _grads(mod, x, gout)
        dx, dw = dx.double().cpu(), dw.double().cpu()
        acc_x += dx
        acc_w += dw
        if i == 0:
            one_x, one_w = _rel(dx, ref_x), _rel(dw, ref_w)
    mean_x, mean_w = _rel(acc_x / n, ref_x), _rel(acc_w / n, ref_w)
    print(f"[linear bwd] noise: one draw dx {one_x:.3e} dW {one_w:.3e}; mean of {n} dx {mean_x:.3e} dW {mean_w:.3e}")
    assert mean_x < 0.5 * one_x and mean_w < 0.5 * one_w


def test_nvfp4_linear_sr_ste_term(moe_pkg):
    """With 2:4 sparsity and sr_ste_decay > 0 the weight gradient adds decay * w on the
    masked-out weights (src/mcl4_coe/nvfp4.py:460-466); same noise under the same seed."""
    _, m0 = _linear_pair(moe_pkg, sparsity="2to4_transposable", decay=0.0, seed=7)
    _, m1 = _linear_pair(moe_pkg, sparsity="2to4_transposable", decay=0.05, seed=7)
    r = np.random.default_rng(3)
    x = torch.from_numpy(r.standard_normal((256, 512)).astype(np.float32)).to(DEV, torch.bfloat16)
    gout = torch.from_numpy((r.standard_normal((256, 384)) * 1e-2).astype(np.float32)).to(DEV, torch.bfloat16)
    torch.manual_seed(11)
    dx0, dw0, _, _ = _grads(m0, x, gout)
    torch.manual_seed(11)
    dx1, dw1, _, _ = _grads(m1, x, gout)
    assert torch.equal(dx0, dx1)
    mask = m1.active_2to4_mask()
    term = 0.05 * (~mask).float() * m1.weight.detach().float()
    torch.testing.assert_close(dw1, dw0 + term, rtol=1e-6, atol=1e-7)


def test_nvfp4_linear_backward_matches_reference_error(moe_pkg):
    """Against the reference's own _NVFP4Linear (its installed copy, cuBLAS F.scaled_mm and
    torch.rand_like noise): the same forward output and gradients whose distance to the
    fp32 gradients is of the same size."""
    ref_dir = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
    if not (ref_dir / "mcl4_coe" / "nvfp4.py").exists():
        pytest.skip("the reference package is not installed under baseline/_ref")
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    import mcl4_coe.nvfp4 as ref_mod
    lin, mod = _linear_pair(moe_pkg, sparsity="none", seed=8)
    ref_lin = ref_mod.NVFP4Linear.from_linear(lin, sparsity_mode="none").to(DEV)
    r = np.random.default_rng(5)
    x = torch.from_numpy(r.standard_normal((1024, 512)).astype(np.float32)).to(DEV, torch.bfloat16)
    gout = torch.from_numpy((r.standard_normal((1024, 384)) * 1e-2).astype(np.float32)).to(DEV, torch.bfloat16)
    xf = x.float().detach().requires_grad_(True)
    torch.nn.functional.linear(xf, lin.weight.float(), lin.bias.float()).backward(gout.float())
    dx, dw, db, y = _grads(mod, x, gout)
    rx, rw, rb, ry = _grads(ref_lin, x, gout)
    # same quantised operands; the two GEMMs sum in different orders before the bf16 rounding
    assert float((y.float() - ry.float()).abs().max()) <= 2 ** -7 * float(ry.float().abs().max())
    torch.testing.assert_close(db, rb, rtol=1e-4, atol=1e-4)
    ours = (_rel(dx, xf.grad), _rel(dw, lin.weight.grad))
    theirs = (_rel(rx, xf.grad), _rel(rw, lin.weight.grad))
    print(f"[linear bwd] vs fp32: ours dx {ours[0]:.3e} dW {ours[1]:.3e}; reference dx {theirs[0]:.3e} "
          f"dW {theirs[1]:.3e}")
    for a, b in zip(ours, theirs):
        assert 0.7 * b < a < 1.4 * b
