"""2:4 sparsity on the GPU: ``mcl4moe_mask_2to4``, the masked weight cache and
the layer with 2:4-sparse experts, against the reference's fixtures.

The mask kernel breaks ties to the lower index (row mode) and takes the first
best pattern (transposable mode, scores summed in row-major tile order); it
must equal the oracle everywhere except transposable tiles whose best scores
tie within fp32 rounding, and the reference everywhere outside its own tie
groups.  Cache bytes and layer outputs follow the reference's masks.
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch
from torch import nn

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

from gpu_ref import build_module, rel_l2, x_tensor  # noqa: E402
from inputs import sparse_cases, sparse_layer_cases  # noqa: E402
from oracle import nvfp4_ref as nr  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = np.load(HERE / "golden" / "sparse.npz")
MODES = ("2to4_row", "2to4_transposable")


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", [n for n, _ in sparse_cases()])
def test_mask_kernel_matches_oracle_and_reference(moe_pkg, name, mode):
    w = dict(sparse_cases())[name]
    gold = GOLD[f"{name}__{mode}__mask"].astype(bool)
    for i in range(len(w)):
        got = moe_pkg.compute_2to4_mask(torch.from_numpy(w[i]).to(DEV), mode).cpu().numpy()
        ties = nr.mask_tie_groups(w[i], mode)
        ora = nr.mask_2to4(w[i], mode)
        if mode == "2to4_row":
            np.testing.assert_array_equal(got, ora)  # same tie rule
        else:
            np.testing.assert_array_equal(got[~ties], ora[~ties])
        np.testing.assert_array_equal(got[~ties], gold[i][~ties])


class _Proj(nn.Module):
    def __init__(self, w: np.ndarray, mode: str):
        super().__init__()
        self.proj = nn.Linear(w.shape[1], w.shape[0], bias=False)
        with torch.no_grad():
            self.proj.weight.copy_(torch.from_numpy(w))
        self.proj.sparsity_mode = mode


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", [n for n, w in sparse_cases() if w.shape[1] % 16 == 0 and w.shape[2] % 64 == 0])
def test_masked_cache_bytes_match_reference(moe_pkg, name, mode):
    """Experts whose projection has ``sparsity_mode`` set are masked before
    quantisation (src/mcl4_coe/nvfp4.py:1017-1024): reference bytes wherever the
    kernel's masks equal the reference's (a stack with tie-broken groups of unequal
    signs may legitimately differ)."""
    w = dict(sparse_cases())[name]
    experts = nn.ModuleList([_Proj(w[i], mode) for i in range(len(w))]).to(DEV)
    masks = np.stack([moe_pkg.compute_2to4_mask(experts[i].proj.weight, mode).cpu().numpy() for i in range(len(w))])
    gold_mask = GOLD[f"{name}__{mode}__mask"].astype(bool)
    ref = moe_pkg.export_reference_cache(experts, "proj")
    cache = moe_pkg.get_or_build_grouped_cache(experts, "proj")
    torch.cuda.synchronize()
    for i in range(len(w)):
        assert torch.equal(cache.masks[i].cpu(), torch.from_numpy(masks[i]))
    same = [i for i in range(len(w)) if np.array_equal(masks[i], gold_mask[i])]
    assert same or name in ("w_mixed", "w_edges", "w_ties")
    b = ref["B_fwd"].cpu().numpy()
    s = ref["Bs_fwd"].view(torch.uint8).cpu().numpy()
    g = ref["Bg"].cpu().numpy()
    for i in same:
        np.testing.assert_array_equal(b[i], GOLD[f"{name}__{mode}__b_fwd"][i])
        np.testing.assert_array_equal(s[i], GOLD[f"{name}__{mode}__bs_fwd"][i])
        assert g[i] == GOLD[f"{name}__{mode}__bg"][i]


def test_mask_follows_weight_updates(moe_pkg):
    """A changed weight (new ``_version``) gets a new mask and new bytes; switching
    an expert's mode re-quantises it too."""
    w = dict(sparse_cases())["w_randn"]
    experts = nn.ModuleList([_Proj(w[i], "2to4_transposable") for i in range(len(w))]).to(DEV)
    c0 = moe_pkg.get_or_build_grouped_cache(experts, "proj")
    m0 = c0.masks[1].clone()
    p0 = c0.packed[1].clone()
    with torch.no_grad():
        experts[1].proj.weight.mul_(-1.0).add_(0.001)
    c1 = moe_pkg.get_or_build_grouped_cache(experts, "proj")
    assert not torch.equal(c1.packed[1], p0)
    experts[2].proj.sparsity_mode = "none"
    c2 = moe_pkg.get_or_build_grouped_cache(experts, "proj")
    torch.cuda.synchronize()
    assert c2.masks[2] is None and c2.masks[0] is not None and m0.dtype == torch.bool


@pytest.mark.parametrize("name", [n for n, _, _ in sparse_layer_cases()])
def test_layer_with_sparse_experts_matches_reference(moe_pkg, name):
    case, mode = {n: (c, m) for n, c, m in sparse_layer_cases()}[name]
    moe = build_module(moe_pkg, case, DEV)
    for ex in moe.experts:
        ex.up_proj.sparsity_mode = mode
        ex.down_proj.sparsity_mode = mode
    x = x_tensor(case, DEV)
    valid = None if case["valid"] is None else torch.from_numpy(case["valid"]).to(DEV)
    with torch.no_grad():
        out, aux, z, counts = moe(x, valid)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    ref = nr.bf16_bits_to_f32(GOLD[f"{name}__out_bf16"]).reshape(got.shape)
    assert rel_l2(got, ref) < 5e-3 and np.abs(got - ref).max() < 1e-1
    np.testing.assert_array_equal(counts.cpu().numpy(), GOLD[f"{name}__counts"])
