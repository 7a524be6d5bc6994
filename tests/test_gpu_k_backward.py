"""Backward of the MoE layer on B200 (training), against the reference's arithmetic.

* The stochastic-rounding gradient quantiser (``mcl4moe_quantize_rows_sr``) gives
  the bytes of the oracle restatement of the reference's Triton kernel
  (``_nvfp4_quantize_1d_kernel`` with STOCHASTIC=True), which is itself pinned to the
  reference kernel run on Triton's CPU interpreter.
* The transposed weight copy (``mcl4moe_quantize_weights_t``) holds the bytes of the
  reference's ``B_bwd`` / ``Bs_bwd``.
* ``mcl4moe_moe_backward_experts`` step by step: d_y and the routing-weight gradient
  from their definitions; the stochastic codes of d_up bit-exact against the oracle
  at the reference's row numbering; the input-gradient GEMM against the dequantised
  operands (fp32, 5e-3 rel-L2); the SwiGLU derivative against torch's.
* The router derivative against torch autograd of the reference's formulas.
* End to end through ``SparseMoE`` under autograd: the inference outputs unchanged,
  weight gradients against an fp32 reference on the same saved operands, and the
  input gradient within the stochastic-rounding noise of an fp32 reference (the
  reference's own backward quantises the same way).
"""

import ctypes

import numpy as np
import pytest
import torch

from gpu_ref import build_module, dequant_reference_layout, x_tensor
from inputs import moe_case, sr_quant_cases
from oracle import nvfp4_ref as nr

pytestmark = pytest.mark.gpu
DEV = "cuda"
E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def _p(t):
    return None if t is None else t.data_ptr()


def _dequant_rows(packed: torch.Tensor, scales_u8: torch.Tensor, g: float) -> torch.Tensor:
    """NVFP4 rows (packed [R, K/2], row-major E4M3 scales [R, K/16]) -> fp32 [R, K]."""
    r, kh = packed.shape
    codes = torch.stack(((packed & 0xF), (packed >> 4)), dim=-1).reshape(r, 2 * kh).long()
    vals = E2M1.to(packed.device)[codes]
    sc = scales_u8.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=-1)
    return vals * sc * g


def test_sr_quantiser_bytes(moe_pkg, golden):
    lib = moe_pkg.library()
    g = golden("sr_quant")
    for name, bits, seed in sr_quant_cases():
        m, k = bits.shape
        x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(DEV)
        packed = torch.empty((m, k // 2), dtype=torch.uint8, device=DEV)
        scales = torch.empty((m, k // 16), dtype=torch.uint8, device=DEV)
        gs = torch.empty((1,), dtype=torch.float32, device=DEV)
        amax = torch.empty((1,), dtype=torch.float32, device=DEV)
        moe_pkg._lib.check(lib.mcl4moe_quantize_rows_sr(x.data_ptr(), m, k, seed, packed.data_ptr(),
                                                        scales.data_ptr(), gs.data_ptr(), amax.data_ptr(),
                                                        torch.cuda.current_stream().cuda_stream), "sr")
        torch.cuda.synchronize()
        assert float(gs) == float(g[f"{name}__g"][0])
        ref_p, ref_s = nr.quantize_sr(nr.bf16_bits_to_f32(bits), g[f"{name}__g"][0], seed)
        np.testing.assert_array_equal(scales.cpu().numpy(), ref_s)
        np.testing.assert_array_equal(packed.cpu().numpy(), ref_p)
        # and the reference kernel's own bytes wherever its interpreter run rounds scales like the GPU
        same = g[f"{name}__scales"] == g[f"{name}__rn_scales"]
        np.testing.assert_array_equal(packed.cpu().numpy()[np.repeat(same, 8, axis=1)],
                                      g[f"{name}__packed"][np.repeat(same, 8, axis=1)])


def test_transposed_weight_copy_is_reference_b_bwd(moe_pkg):
    lib = moe_pkg.library()
    r = np.random.default_rng(5)
    E, N, K = 3, 512, 256
    w = (r.standard_normal((E, N, K)) * 0.02).astype(np.float32)
    wt = [torch.from_numpy(w[i]).to(DEV) for i in range(E)]
    ptrs = (ctypes.c_void_p * E)(*[t.data_ptr() for t in wt])
    slots = (ctypes.c_int32 * E)(*range(E))
    packed = torch.empty((E, N, K // 2), dtype=torch.uint8, device=DEV)
    scales = torch.zeros((E, N * K // 16), dtype=torch.uint8, device=DEV)
    gsc = torch.empty((E,), dtype=torch.float32, device=DEV)
    pt = torch.empty((E, K, N // 2), dtype=torch.uint8, device=DEV)
    st = torch.zeros((E, K * N // 16), dtype=torch.uint8, device=DEV)
    amax = torch.empty((E,), dtype=torch.float32, device=DEV)
    moe_pkg._lib.check(lib.mcl4moe_quantize_weights_t(ptrs, slots, E, N, K, packed.data_ptr(), scales.data_ptr(),
                                                      gsc.data_ptr(), pt.data_ptr(), st.data_ptr(),
                                                      amax.data_ptr(), torch.cuda.current_stream().cuda_stream),
                       "quantize_weights_t")
    torch.cuda.synchronize()
    b_fwd, bs_fwd, bg, b_bwd, bs_bwd = nr.quantize_grouped_weights(w, with_bwd=True)
    np.testing.assert_array_equal(gsc.cpu().numpy(), bg)
    np.testing.assert_array_equal(pt.cpu().numpy(), np.ascontiguousarray(b_bwd.transpose(0, 2, 1)))
    for e in range(E):
        np.testing.assert_array_equal(st[e].cpu().numpy(), nr.swizzle_scales(bs_bwd[e]).reshape(-1))


def _train_case(pkg, seed=61, t=384, d=512, e=8, k=2, f=256):
    c = moe_case(seed, t, d, e, k, f)
    moe = build_module(pkg, c, DEV)
    return c, moe


def test_backward_steps_against_reference_arithmetic(moe_pkg):
    """The library backward's intermediate results, each from its definition."""
    lib = moe_pkg.library()
    L = moe_pkg._lib
    c, moe = _train_case(moe_pkg)
    T, d, E, k, F = c["t"], c["d"], c["e"], c["k"], c["f"]
    x = x_tensor(c, DEV)
    up = moe_pkg.nvfp4.get_or_build_grouped_cache(moe.experts, "up_proj", with_bwd=True)
    dn = moe_pkg.nvfp4.get_or_build_grouped_cache(moe.experts, "down_proj", with_bwd=True)
    mcap = lib.mcl4moe_padded_rows(T, E, k)
    bf = dict(dtype=torch.bfloat16, device=DEV)
    f32 = dict(dtype=torch.float32, device=DEV)
    out = torch.empty((T, d), **bf)
    stats = torch.empty((3 + E,), **f32)
    topk_idx = torch.empty((T, k), dtype=torch.int32, device=DEV)
    topk_w = torch.empty((T, k), **f32)
    logits = torch.empty((T, E), **f32)
    up_save, x_rows, y_save, h_save = (torch.empty((mcap, n), **bf) for n in (2 * F, d, d, F))
    ws = torch.empty((lib.mcl4moe_moe_workspace_size(T, d, E, k, F),), dtype=torch.uint8, device=DEV)
    wr = moe.router.weight.detach().float().contiguous()
    s = torch.cuda.current_stream().cuda_stream
    args = L.MoeArgs(x=x.data_ptr(), router_w=wr.data_ptr(), w_up=up.packed.data_ptr(),
                     w_up_scales=up.scales.data_ptr(), w_up_g=up.g.data_ptr(), w_dn=dn.packed.data_ptr(),
                     w_dn_scales=dn.scales.data_ptr(), w_dn_g=dn.g.data_ptr(), T=T, d=d, E=E, k=k, F=F,
                     norm_topk_prob=1, out=out.data_ptr(), stats=stats.data_ptr(), topk_idx=topk_idx.data_ptr(),
                     topk_w=topk_w.data_ptr(), h_debug=h_save.data_ptr(), workspace=ws.data_ptr(),
                     workspace_bytes=ws.numel(), up_save=up_save.data_ptr(), x_rows_save=x_rows.data_ptr(),
                     y_save=y_save.data_ptr(), logits_out=logits.data_ptr())
    L.check(lib.mcl4moe_moe_forward(args, s), "forward")
    with torch.no_grad():
        ref_out = moe(x)[0]
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out), "training forward differs from the inference forward"

    def region(i, n):
        off = lib.mcl4moe_workspace_region(ws.data_ptr(), i, T, d, E, k, F) - ws.data_ptr()
        return ws[off:off + n]

    slot_pos = region(6, 4 * T * k).view(torch.int32).view(T, k).clone()
    pad_start = region(5, 4 * (E + 1)).view(torch.int32).clone()
    counts = region(9, 4 * E).view(torch.int32).clone()
    offs_start = region(10, 4 * E).view(torch.int32).clone()
    g = torch.Generator(device=DEV).manual_seed(3)
    d_out = (torch.randn((T, d), generator=g, device=DEV) * 1e-3).to(torch.bfloat16)
    d_y, d_rows = torch.empty((mcap, d), **bf), torch.empty((mcap, d), **bf)
    d_up = torch.empty((mcap, 2 * F), **bf)
    d_w = torch.empty((T, k), **f32)
    bws = torch.empty((lib.mcl4moe_moe_backward_workspace_size(T, d, E, k, F),), dtype=torch.uint8, device=DEV)
    seed_dn, seed_up = 1234, 98765
    bargs = L.MoeBwdArgs(T=T, d=d, E=E, k=k, F=F, d_out=d_out.data_ptr(), slot_pos=slot_pos.data_ptr(),
                         topk_w=topk_w.data_ptr(), pad_start=pad_start.data_ptr(), counts=counts.data_ptr(),
                         offs_start=offs_start.data_ptr(), y_save=y_save.data_ptr(), up_save=up_save.data_ptr(),
                         w_up_t=up.packed_t.data_ptr(), w_up_t_scales=up.scales_t.data_ptr(), w_up_g=up.g.data_ptr(),
                         w_dn_t=dn.packed_t.data_ptr(), w_dn_t_scales=dn.scales_t.data_ptr(), w_dn_g=dn.g.data_ptr(),
                         seed_down=seed_dn, seed_up=seed_up, d_y=d_y.data_ptr(), d_up=d_up.data_ptr(),
                         d_rows=d_rows.data_ptr(), d_w=d_w.data_ptr(), workspace=bws.data_ptr(),
                         workspace_bytes=bws.numel())
    L.check(lib.mcl4moe_moe_backward_experts(bargs, s), "backward_experts")
    torch.cuda.synchronize()
    # layout of the backward workspace: SR codes [mcap, kmax/2], scales [mcap, kmax/16], d_h [mcap, F]
    kmax = max(d, 2 * F)
    a256 = lambda n: (n + 255) // 256 * 256  # noqa: E731
    qa = bws[:mcap * kmax // 2]
    sa = bws[a256(mcap * kmax // 2):a256(mcap * kmax // 2) + mcap * kmax // 16]
    dh_off = a256(mcap * kmax // 2) + a256(mcap * kmax // 16)
    d_h = bws[dh_off:dh_off + 2 * mcap * F].view(torch.bfloat16).view(mcap, F)

    sp = slot_pos.long()
    live = sp.reshape(-1) >= 0
    rows = sp.reshape(-1)[live]
    tok = torch.arange(T, device=DEV).repeat_interleave(k)[live]
    wb = topk_w.reshape(-1)[live].to(torch.bfloat16).float()
    # d_y = bf16(d_out[t] * bf16(w)); padding rows zero
    exp_dy = (d_out[tok].float() * wb[:, None]).to(torch.bfloat16)
    assert torch.equal(d_y[rows], exp_dy)
    P = int(pad_start[E])
    used = torch.zeros(P, dtype=torch.bool, device=DEV)
    used[rows] = True
    assert torch.all(d_y[:P][~used] == 0)
    # routing-weight gradient bf16(sum_c bf16(d_out * y)) (summation order differs: 1 bf16 ulp)
    prod = (d_out[tok].float() * y_save[rows].float()).to(torch.bfloat16).float().sum(dim=1)
    got_dw = d_w.reshape(-1)[live]
    torch.testing.assert_close(got_dw, prod.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-6)
    # SwiGLU derivative from the same d_h (torch's bf16 silu and silu_backward)
    gate, val = up_save[:P, :F], up_save[:P, F:]
    dh = d_h[:P]
    silu = torch.nn.functional.silu(gate)
    d_val = (dh.float() * silu.float()).to(torch.bfloat16)
    d_s = (dh.float() * val.float()).to(torch.bfloat16)
    d_gate = torch.ops.aten.silu_backward(d_s, gate)
    torch.testing.assert_close(d_up[:P, F:], d_val, rtol=8e-3, atol=1e-9)
    torch.testing.assert_close(d_up[:P, :F], d_gate, rtol=8e-3, atol=1e-9)
    # the stochastic codes of d_up, bit-exact against the oracle at the reference's row numbering
    ref_row = torch.full((P,), -1, dtype=torch.long, device=DEV)
    for e in range(E):
        a, n = int(pad_start[e]), int(counts[e])
        ref_row[a:a + n] = torch.arange(int(offs_start[e]), int(offs_start[e]) + n, device=DEV)
    lv = (ref_row >= 0).cpu().numpy()
    dup_np = d_up[:P].float().cpu().numpy()
    g_up = nr.sr_global_scale(dup_np[lv])
    op, os_ = nr.quantize_sr(dup_np[lv], g_up, seed_up, row_index=ref_row.cpu().numpy()[lv])
    kq = 2 * F
    got_q = qa[:P * kq // 2].view(P, kq // 2).cpu().numpy()
    got_s = sa[:P * kq // 16].view(P, kq // 16).cpu().numpy()
    np.testing.assert_array_equal(got_q[lv], op)
    np.testing.assert_array_equal(got_s[lv], os_)
    assert np.all(got_s[~lv] == 0)
    # the input-gradient GEMM on those bytes: d_rows = deq(SR(d_up)) @ deq(W_up) per expert
    deq = _dequant_rows(qa[:P * kq // 2].view(P, kq // 2), sa[:P * kq // 16].view(P, kq // 16), float(g_up))
    ref_cache = moe_pkg.export_reference_cache(moe.experts, "up_proj")
    w_up = dequant_reference_layout(ref_cache["B_fwd"], ref_cache["Bs_fwd"].view(torch.uint8), ref_cache["Bg"])
    exp_rows = torch.zeros((P, d), **f32)
    for e in range(E):
        a, b = int(pad_start[e]), int(pad_start[e + 1])
        exp_rows[a:b] = deq[a:b] @ w_up[e]
    got = d_rows[:P].float()
    rel = (torch.linalg.norm(got - exp_rows) / torch.linalg.norm(exp_rows)).item()
    assert rel < 5e-3, rel


def test_router_backward_matches_autograd(moe_pkg):
    lib = moe_pkg.library()
    T, E, k = 300, 40, 6
    g = torch.Generator(device=DEV).manual_seed(8)
    logits = torch.randn((T, E), generator=g, device=DEV)
    valid = (torch.rand((T,), generator=g, device=DEV) < 0.85)
    probs = torch.softmax(logits, dim=-1)
    vals, idx = probs.topk(k, dim=-1)
    w = vals / vals.sum(-1, keepdim=True).clamp_min(1e-9)
    n = int(valid.sum())
    sel = torch.zeros((T, E), device=DEV).scatter_add_(1, idx, torch.ones_like(vals))
    counts = (sel * valid[:, None].float()).sum(0) / (n * k)
    stats = torch.cat([torch.zeros(2, device=DEV), torch.tensor([float(n)], device=DEV), counts]).contiguous()
    d_w = torch.randn((T, k), generator=g, device=DEV) * valid[:, None].float()
    d_aux, d_z = torch.tensor(0.37, device=DEV), torch.tensor(-1.3, device=DEV)
    out = torch.empty((T, E), device=DEV)
    moe_pkg._lib.check(lib.mcl4moe_router_backward(
        logits.data_ptr(), idx.int().contiguous().data_ptr(), w.contiguous().data_ptr(), d_w.contiguous().data_ptr(),
        valid.to(torch.uint8).contiguous().data_ptr(), stats.data_ptr(), d_aux.data_ptr(), d_z.data_ptr(), T, E, k, 1,
        out.data_ptr(), torch.cuda.current_stream().cuda_stream), "router_backward")
    # torch autograd of src/mcl4_coe/backbone.py:799-879 (valid branch) with the same selection
    lg = logits.clone().requires_grad_(True)
    pr = torch.softmax(lg, dim=-1)
    v = pr.gather(1, idx)
    ww = v / v.sum(-1, keepdim=True).clamp_min(1e-9) * valid[:, None].float()
    mean_probs = (pr * valid[:, None].float()).sum(0) / n
    aux = E * (counts * mean_probs).sum()
    z = ((torch.logsumexp(lg, dim=-1).square() * valid.float()).sum() / n)
    ((ww * d_w).sum() + d_aux * aux + d_z * z).backward()
    torch.testing.assert_close(out, lg.grad, rtol=1e-4, atol=1e-6)


def test_training_end_to_end(moe_pkg):
    """SparseMoE under autograd: outputs equal the inference forward; weight gradients
    against fp32 products of the same operands; the input gradient against an fp32
    reference within the stochastic-rounding noise."""
    c, moe = _train_case(moe_pkg, seed=62, t=512, d=512, e=8, k=2, f=512)
    T, d, E, k, F = c["t"], c["d"], c["e"], c["k"], c["f"]
    x = x_tensor(c, DEV).requires_grad_(True)
    with torch.no_grad():
        ref_out, ref_aux, ref_z, ref_counts = moe(x.detach())
    out, aux, z, counts = moe(x)
    assert torch.equal(out.detach(), ref_out) and torch.equal(counts, ref_counts)
    assert float(aux.detach()) == float(ref_aux) and float(z.detach()) == float(ref_z)
    g = torch.Generator(device=DEV).manual_seed(4)
    gout = torch.randn((T, d), generator=g, device=DEV)
    loss = (out.float() * gout).sum() + 0.01 * aux + 0.001 * z
    loss.backward()
    torch.cuda.synchronize()
    assert x.grad is not None and torch.isfinite(x.grad.float()).all()
    assert moe.router.weight.grad is not None and torch.isfinite(moe.router.weight.grad).all()
    for ex in moe.experts:
        assert ex.up_proj.weight.grad is not None and torch.isfinite(ex.up_proj.weight.grad).all()
        assert ex.down_proj.weight.grad is not None and torch.isfinite(ex.down_proj.weight.grad).all()
    # fp32 reference: dequantised weights, fake-quantised activations with straight-through gradients
    # (the reference's quantisers pass gradients unchanged; its backward adds stochastic-rounding noise)
    caches = {p: moe_pkg.export_reference_cache(moe.experts, p) for p in ("up_proj", "down_proj")}
    w_up = dequant_reference_layout(caches["up_proj"]["B_fwd"], caches["up_proj"]["Bs_fwd"].view(torch.uint8),
                                    caches["up_proj"]["Bg"]).requires_grad_(True)
    w_dn = dequant_reference_layout(caches["down_proj"]["B_fwd"], caches["down_proj"]["Bs_fwd"].view(torch.uint8),
                                    caches["down_proj"]["Bg"]).requires_grad_(True)
    wr = moe.router.weight.detach().clone().requires_grad_(True)
    xr = x.detach().float().clone().requires_grad_(True)

    class QLinear(torch.autograd.Function):
        """fq(a) @ w^T in the forward; the backward of the reference's NVFP4 projection
        without its stochastic rounding: input gradient g @ w, weight gradient g^T @ a
        with the UNQUANTISED input (src/mcl4_coe/nvfp4.py:1172-1216)."""

        @staticmethod
        def forward(ctx, a, w):
            ctx.save_for_backward(a, w)
            q = torch.from_numpy(nr.fake_quantize_activations(a.detach().float().cpu().numpy())).to(DEV)
            return q @ w.t()

        @staticmethod
        def backward(ctx, gr):
            a, w = ctx.saved_tensors
            return gr @ w, gr.t() @ a

    logits = xr @ wr.t()
    probs = torch.softmax(logits, dim=-1)
    vals, idx = probs.topk(k, dim=-1)
    wts = vals / vals.sum(-1, keepdim=True)
    out_ref = torch.zeros((T, d), device=DEV)
    for e in range(E):
        tt, jj = (idx == e).nonzero(as_tuple=True)
        if tt.numel() == 0:
            continue
        upv = QLinear.apply(xr[tt], w_up[e])
        hv = torch.nn.functional.silu(upv[:, :F]) * upv[:, F:]
        y = QLinear.apply(hv, w_dn[e])
        out_ref = out_ref.index_add(0, tt, y * wts[tt, jj][:, None])
    n = T
    cnt = torch.zeros(E, device=DEV).scatter_add_(0, idx.reshape(-1), torch.ones(T * k, device=DEV)) / (T * k)
    aux_r = E * (cnt * probs.mean(0)).sum()
    z_r = torch.logsumexp(logits, dim=-1).square().sum() / n
    ((out_ref * gout).sum() + 0.01 * aux_r + 0.001 * z_r).backward()

    def rel(a, b):
        return (torch.linalg.norm(a.float() - b.float()) / torch.linalg.norm(b.float())).item()

    def cos(a, b):
        return torch.nn.functional.cosine_similarity(a.float().reshape(-1), b.float().reshape(-1), dim=0).item()

    g_dn = torch.stack([ex.down_proj.weight.grad for ex in moe.experts])
    g_up = torch.stack([ex.up_proj.weight.grad for ex in moe.experts])
    print(f"\n[train] rel err: dW_down {rel(g_dn, w_dn.grad):.2e} dW_router {rel(moe.router.weight.grad, wr.grad):.2e} "
          f"dW_up {rel(g_up, w_up.grad):.2e} dx {rel(x.grad, xr.grad):.2e}")
    # the down projection's weight gradient sees exact bf16 operands: close to fp32
    assert rel(g_dn, w_dn.grad) < 1.5e-2, rel(g_dn, w_dn.grad)
    assert rel(moe.router.weight.grad, wr.grad) < 5e-2, rel(moe.router.weight.grad, wr.grad)
    # behind one (up) or two (x) stochastic-rounded NVFP4 gradients: agreement within their noise
    assert cos(g_up, w_up.grad) > 0.95 and rel(g_up, w_up.grad) < 0.35, (cos(g_up, w_up.grad), rel(g_up, w_up.grad))
    assert cos(x.grad, xr.grad) > 0.95 and rel(x.grad, xr.grad) < 0.35, (cos(x.grad, xr.grad), rel(x.grad, xr.grad))


def test_stochastic_rounding_is_unbiased_end_to_end(moe_pkg):
    """Averaging the input gradient over independent backward passes (fresh noise seeds,
    as the reference draws per call) shrinks its distance to the mean: the stochastic
    rounding adds zero-mean noise, not a bias."""
    c, moe = _train_case(moe_pkg, seed=63, t=256, d=512, e=8, k=2, f=512)
    x = x_tensor(c, DEV).requires_grad_(True)
    out = moe(x)[0]
    g = torch.Generator(device=DEV).manual_seed(9)
    gout = torch.randn(out.shape, generator=g, device=DEV)
    loss = (out.float() * gout).sum()
    grads = [torch.autograd.grad(loss, x, retain_graph=True)[0].float() for _ in range(16)]
    mean = torch.stack(grads).mean(0)
    single = torch.stack([torch.linalg.norm(gr - mean) for gr in grads]).mean().item()
    avg4 = torch.stack([torch.linalg.norm(torch.stack(grads[i:i + 4]).mean(0) - mean)
                        for i in range(0, 16, 4)]).mean().item()
    # independent zero-mean noise: averaging 4 passes halves the spread (1/sqrt(4))
    assert avg4 < 0.65 * single, (avg4, single)
    assert not torch.equal(grads[0], grads[1])  # a new seed per backward call


@pytest.mark.parametrize("N,K", [(512, 256), (256, 1024)])
def test_wgrad_gemm_per_expert_products(moe_pkg, N, K):
    """mcl4moe_moe_backward_wgrad (tcgen05, MN-major operands) against fp32 products per
    expert segment, with an empty expert (zeros) and segments of 256 to 1024 rows."""
    lib = moe_pkg.library()
    seg = [512, 0, 256, 1024, 256]
    E = len(seg)
    pad = torch.tensor([0] + list(np.cumsum(seg)), dtype=torch.int32, device=DEV)
    rows = int(pad[-1]) + 256  # capacity beyond the last segment is not read
    g = torch.Generator(device=DEV).manual_seed(21)
    G = torch.randn((rows, N), generator=g, device=DEV).to(torch.bfloat16)
    X = torch.randn((rows, K), generator=g, device=DEV).to(torch.bfloat16)
    dw = torch.full((E, N, K), float("nan"), device=DEV)
    moe_pkg._lib.check(lib.mcl4moe_moe_backward_wgrad(G.data_ptr(), X.data_ptr(), rows, N, K, pad.data_ptr(), E,
                                                      dw.data_ptr(), None, torch.cuda.current_stream().cuda_stream),
                       "wgrad")
    torch.cuda.synchronize()
    for e in range(E):
        a, b = int(pad[e]), int(pad[e + 1])
        ref = G[a:b].float().t() @ X[a:b].float() if b > a else torch.zeros((N, K), device=DEV)
        torch.testing.assert_close(dw[e], ref, rtol=1e-4, atol=1e-3)
