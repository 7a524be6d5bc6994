"""Seeded inputs shared by ``make_golden.py`` and the tests.

All data come from numpy's PCG64 generator, so the same arrays are rebuilt on
any machine; the golden files store SHA-256 digests of the large ones.
"""

from __future__ import annotations

import zlib

import numpy as np


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_values(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(to_bf16_bits(x))


def _edge_rows(cols: int) -> np.ndarray:
    """Rows of 16-element blocks that hit every E2M1 rounding tie, signed
    zeros, all-zero blocks, e4m3 subnormal scales and the 448 clamp."""
    ties = np.array([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0,
                     -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -0.0], dtype=np.float32)
    blocks = [
        ties,                                   # scale exactly 1: exact ties
        ties * 2.0,                             # scale exactly 2
        ties * 0.5,                             # scale 0.5
        ties * (7.0 / 6.0),                     # inexact scale
        np.zeros(16, np.float32),               # all zero
        np.full(16, -0.0, np.float32),          # all negative zero
        np.linspace(-1e-3, 1e-3, 16, dtype=np.float32),   # e4m3 subnormal scale
        np.linspace(-1e6, 1e6, 16, dtype=np.float32),     # scale clamped at 448
        np.full(16, 1e-40, np.float32),         # float32 denormals
        np.array([3.0] + [2.5000002] * 15, np.float32),    # just above a tie
        np.array([3.0] + [2.4999998] * 15, np.float32),    # just below a tie
        np.array([6.0, 5.9999995, 4.0000005, 3.9999998] * 4, np.float32),
    ]
    flat = np.concatenate(blocks)
    reps = -(-cols * 4 // flat.size)
    data = np.tile(flat, reps)[: cols * 4]
    return data.reshape(4, cols)


def act_quant_cases():
    """(name, float32 matrix, mode) triples for the quantiser goldens."""
    cases = []
    r = rng(100)
    x = bf16_values(r.standard_normal((256, 512), dtype=np.float32))
    cases.append(("act_randn_bf16", x, "act"))
    mags = np.power(10.0, r.uniform(-40, 37, size=(64, 1))).astype(np.float32)
    cases.append(("act_wide_range", (r.standard_normal((64, 256), dtype=np.float32) * mags).astype(np.float32), "act"))
    cases.append(("act_fp32", (r.standard_normal((128, 256), dtype=np.float32) * 3.0).astype(np.float32), "act"))
    cases.append(("act_edges", _edge_rows(256), "act"))
    cases.append(("act_edges_bf16", bf16_values(_edge_rows(256) * 1.5), "act"))
    cases.append(("tensor1d_randn", (r.standard_normal((128, 256), dtype=np.float32) * 0.7).astype(np.float32), "tensor1d"))
    cases.append(("tile2d_randn", (r.standard_normal((64, 128), dtype=np.float32) * 0.02).astype(np.float32), "tile2d"))
    cases.append(("tile2d_edges", np.concatenate([_edge_rows(128)] * 4, axis=0), "tile2d"))
    return cases


def weight_quant_cases():
    """(name, float32 [D, N, K]) stacks for the grouped weight quantiser."""
    r = rng(200)
    randn = (r.standard_normal((3, 64, 128), dtype=np.float32) * 0.02).astype(np.float32)
    mixed = np.empty((4, 32, 64), dtype=np.float32)
    mixed[0] = 0.0                                                    # all-zero expert
    tile_mag = np.power(10.0, r.uniform(-6, 0, size=(2, 1, 4, 1))).astype(np.float32)
    mixed[1] = (r.standard_normal((2, 16, 4, 16), dtype=np.float32) * tile_mag).reshape(32, 64)
    mixed[2] = (r.standard_normal((32, 64), dtype=np.float32) * 1e-37).astype(np.float32)
    mixed[3] = np.float32(1e-40)                                      # denormal decoding scales
    mixed[3, 0, 0] = np.float32(1e-36)
    edges = np.stack([_edge_rows(64).reshape(4, 64).repeat(4, axis=0)[:16].reshape(16, 64)] * 2)
    edges = np.concatenate([edges, edges * np.float32(0.02)], axis=0).reshape(4, 16, 64)
    return [("w_randn", randn), ("w_mixed", mixed), ("w_edges", edges.astype(np.float32))]


def moe_case(seed: int, t: int, d: int, e: int, k: int, f: int, norm_topk_prob: bool = True,
             valid_frac: float | None = None, zipf_bias: bool = False, dead_experts: int = 0):
    """One MoE layer instance with the benchmark's initialisation:
    ``x ~ N(0,1)`` in bf16, router and expert weights ``~ N(0, 0.02)`` fp32."""
    r = rng(seed)
    x_bits = to_bf16_bits(r.standard_normal((t, d), dtype=np.float32))
    wr = (r.standard_normal((e, d), dtype=np.float32) * 0.02).astype(np.float32)
    w_up = (r.standard_normal((e, 2 * f, d), dtype=np.float32) * 0.02).astype(np.float32)
    w_dn = (r.standard_normal((e, d, f), dtype=np.float32) * 0.02).astype(np.float32)
    valid = None
    if valid_frac is not None:
        valid = (r.uniform(size=t) < valid_frac).astype(np.uint8)
    bias = None
    if zipf_bias:
        bias = (2.0 * np.log(1.0 / np.arange(1, e + 1, dtype=np.float64))).astype(np.float32)
    if dead_experts:
        bias = np.zeros(e, np.float32) if bias is None else bias
        bias[-dead_experts:] -= np.float32(1e4)
    return dict(t=t, d=d, e=e, k=k, f=f, norm_topk_prob=norm_topk_prob, x_bf16_bits=x_bits, wr=wr,
                w_up=w_up, w_dn=w_dn, valid=valid, logit_bias=bias)


def routing_cases():
    return [
        ("r_c0", moe_case(300, 1024, 256, 8, 2, 64)),
        ("r_c0_nonorm", moe_case(301, 1024, 256, 8, 2, 64, norm_topk_prob=False)),
        ("r_valid", moe_case(302, 512, 256, 8, 2, 64, valid_frac=0.8)),
        ("r_zipf", moe_case(303, 512, 256, 32, 8, 32, zipf_bias=True)),
        ("r_e64k8", moe_case(304, 512, 512, 64, 8, 32)),
        ("r_dead", moe_case(305, 256, 256, 16, 3, 32, dead_experts=5)),
    ]


def layer_case():
    return ("layer_c0", moe_case(400, 256, 256, 8, 2, 512))


def variant_cases():
    """Routing variants of SparseMoE (src/mcl4_coe/backbone.py:274-398, :640-1047):
    (name, moe_case, options).  ``shape`` reshapes x to [B, S, d] (the
    sequence-diversity loss needs a sequence axis); ``prior_frac`` draws a 0/1
    prior_expert_mask; ``lineage`` = (num_roots, top_families, child_share)."""
    def opt(**kw):
        base = dict(pairs=(), lineage=None, coverage=0.0, prior_frac=None, dense_idx=None, dense_k=0,
                    combine=False, seq_div=0.0, ortho=0.0, shape=None)
        base.update(kw)
        return base

    return [
        ("v_twins_norm", moe_case(500, 96, 256, 8, 2, 256, valid_frac=0.8), opt(pairs=((0, 4), (2, 6)))),
        ("v_twins_nonorm", moe_case(501, 96, 256, 8, 2, 256, norm_topk_prob=False), opt(pairs=((1, 5), (3, 7)))),
        ("v_lineage", moe_case(502, 96, 256, 12, 2, 256), opt(lineage=(4, 2, 0.25))),
        ("v_coverage", moe_case(503, 96, 256, 8, 3, 256, valid_frac=0.9), opt(coverage=0.6, prior_frac=0.4)),
        ("v_dense_idx", moe_case(504, 96, 256, 8, 2, 256, valid_frac=0.75), opt(dense_idx=(5, 1, 3))),
        ("v_dense_k_mixed", moe_case(505, 96, 256, 8, 2, 256), opt(dense_k=2, combine=True, coverage=0.5,
                                                                  prior_frac=0.3)),
        ("v_aux_terms", moe_case(506, 96, 256, 8, 2, 256, valid_frac=0.85),
         opt(pairs=((0, 1),), seq_div=0.1, ortho=0.05, shape=(4, 24))),
    ]


# The five benchmark configurations (seeds 0-4); shapes only — tensors are built
# on the device by the tests / bench from these seeds.
BENCH_CONFIGS = [
    dict(name="c0_cpu", seed=0, t=2048, d=256, e=8, k=2, f=512),
    dict(name="c1_mitotic", seed=1, t=16384, d=1024, e=32, k=4, f=512),
    dict(name="c2_olmoe", seed=2, t=32768, d=2048, e=64, k=8, f=1024),
    dict(name="c3_granite_zipf", seed=3, t=65536, d=1536, e=32, k=8, f=512, e_grow=40, zipf_bias=True),
    dict(name="c4_decode", seed=4, t=64, d=2048, e=64, k=8, f=1024),
]


def variant_prior(name: str, t: int, e: int, frac: float | None) -> np.ndarray | None:
    """0/1 prior_expert_mask [t, e] of the variant case ``name`` (None when it has none)."""
    if frac is None:
        return None
    return (rng(zlib.crc32(name.encode())).uniform(size=(t, e)) < frac).astype(np.float32)


def sparse_cases():
    """(name, float32 [D, N, K]) stacks for the 2:4 masks (src/mcl4_coe/nvfp4.py:70-110):
    the weight-quantiser stacks, a 256 x 256 random stack, and tiles with exact ties
    (repeated magnitudes, zeros, sign-only differences)."""
    r = rng(210)
    big = (r.standard_normal((2, 256, 256), dtype=np.float32) * 0.02).astype(np.float32)
    ties = np.tile(np.array([0.5, -0.5, 0.25, 0.0], np.float32), (1, 32, 16)).reshape(1, 32, 64)
    ties = np.concatenate([ties, np.abs(ties), -ties], axis=0)
    ties[1, 4:8, 8:12] = np.float32(0.75)
    return weight_quant_cases() + [("w_big", big), ("w_ties", ties)]


def sparse_layer_cases():
    """(name, moe_case, sparsity mode of the experts' projections)."""
    return [
        ("s_transposable", moe_case(600, 128, 256, 8, 2, 256), "2to4_transposable"),
        ("s_row", moe_case(601, 128, 256, 8, 2, 256, valid_frac=0.8), "2to4_row"),
    ]



def sr_quant_cases():
    """(name, bf16 bits [M, K], seed) for the stochastic-rounding gradient quantiser
    (the reference's _nvfp4_quantize_1d_kernel with STOCHASTIC=True): gradient-like
    magnitudes, an all-zero row block, signed zeros and the E2M1 edge rows scaled down."""
    cases = []
    r = rng(700)
    g = (r.standard_normal((40, 256), dtype=np.float32) * 0.01).astype(np.float32)
    cases.append(("sr_grad_40x256", to_bf16_bits(g), 12345))
    r = rng(701)
    g = (r.standard_normal((64, 1024), dtype=np.float32) * 1e-4).astype(np.float32)
    g[5] = 0.0
    g[9, :512] = -0.0
    g[17:21] = _edge_rows(1024) * np.float32(1e-3)
    g[30] = np.float32(3e-2) * np.sign(g[30])
    cases.append(("sr_mixed_64x1024", to_bf16_bits(g), 7))
    r = rng(702)
    g = (r.standard_normal((33, 512), dtype=np.float32) * np.float32(2.0)).astype(np.float32)
    cases.append(("sr_ragged_33x512", to_bf16_bits(g), 2 ** 31 - 1))
    return cases


def hadamard_cases():
    """(name, float32 [M, C]) matrices for the single-matrix weight gradient's
    Hadamard16 transform and quantisation (src/mcl4_coe/nvfp4.py:337-355, :454-459):
    inputs-like and gradient-like values, token counts that are not multiples of 16,
    an outlier column, an all-zero column and bf16-representable values."""
    cases = []
    r = rng(800)
    x = bf16_values(r.standard_normal((40, 48), dtype=np.float32))
    x[:, 7] *= np.float32(50.0)
    x[:, 11] = 0.0
    cases.append(("ht_inputs_40x48", x))
    r = rng(801)
    g = bf16_values((r.standard_normal((37, 32), dtype=np.float32) * np.float32(1e-3)).astype(np.float32))
    g[3] = -0.0
    cases.append(("ht_grad_37x32", g))
    r = rng(802)
    y = r.standard_normal((150, 64), dtype=np.float32)
    cases.append(("ht_f32_150x64", y))
    return cases
