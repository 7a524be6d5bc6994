"""numpy restatement of the reference NVFP4 quantisers (test infrastructure only).

Every function cites the reference lines it restates (paths relative to the
reference project root).  All arithmetic is float32 with IEEE round-to-nearest
(numpy's float32 ``/``, ``*``, ``+`` and ``np.rint`` are correctly rounded,
exactly like the reference's eager torch CPU ops), so outputs are bit-exact.
"""

from __future__ import annotations

import numpy as np

FLT_MAX = np.float32(3.402823466e38)
FLT_MIN_NORMAL = np.float32(1.17549435e-38)

# src/mcl4_coe/nvfp4.py:160-165 — magnitudes of the 8 E2M1 codes.
E2M1_LEVELS = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def round_up(value: int, multiple: int) -> int:
    """src/mcl4_coe/nvfp4.py:45-46."""
    return (value + multiple - 1) // multiple * multiple


# --------------------------------------------------------------------------
# float8 e4m3fn and bfloat16 conversions (the torch CPU semantics the
# reference relies on through ``.to(torch.float8_e4m3fn)`` / ``.to(bf16)``).
# --------------------------------------------------------------------------

def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn bit patterns, round-to-nearest-even.

    Restates PyTorch's c10 ``fp8e4m3fn_from_fp32_value`` (used by
    ``.to(torch.float8_e4m3fn)`` at src/mcl4_coe/nvfp4.py:215 and :931):
    magnitudes >= 480 become NaN (0x7F); magnitudes below 2**-6 round to a
    multiple of 2**-9 (subnormal codes 0..8); the rest round the fp32
    mantissa to 3 bits with ties to even.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    sign = ((bits >> np.uint32(24)) & np.uint32(0x80)).astype(np.uint8)
    mag_bits = bits & np.uint32(0x7FFFFFFF)
    mag = mag_bits.view(np.float32)
    out = np.zeros(x.shape, dtype=np.uint8)
    nan_or_big = mag_bits >= np.uint32(1087 << 20)  # >= 480.0 or NaN
    small = mag_bits < np.uint32(121 << 23)  # < 2**-6
    normal = ~(nan_or_big | small)
    out[nan_or_big] = 0x7F
    out[small] = np.rint(mag[small] * np.float32(512.0)).astype(np.uint8)
    nb = mag_bits[normal]
    odd = (nb >> np.uint32(20)) & np.uint32(1)
    r = (nb + np.uint32(0x7FFFF) + odd) >> np.uint32(20)
    out[normal] = (r - np.uint32((127 - 7) << 3)).astype(np.uint8)
    return out | sign


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    """float8_e4m3fn bit patterns -> float32 (exact)."""
    c = np.asarray(codes, dtype=np.uint8)
    sign = np.where((c & 0x80) != 0, np.float32(-1.0), np.float32(1.0))
    e = ((c >> 3) & 0x0F).astype(np.int32)
    m = (c & 0x07).astype(np.float32)
    val = np.where(e == 0, m * np.float32(2.0 ** -9),
                   (np.float32(1.0) + m / np.float32(8.0)) * np.exp2(e - 7).astype(np.float32))
    val = np.where((c & 0x7F) == 0x7F, np.float32(np.nan), val)
    return (sign * val).astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns with round-to-nearest-even (torch ``.to(bf16)``)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    rounded = ((b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((b[nan] >> np.uint64(16)) | np.uint64(0x40)).astype(np.uint16)
    return rounded


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# --------------------------------------------------------------------------
# E2M1 code rounding and the quantisers.
# --------------------------------------------------------------------------

def e2m1_codes(values: np.ndarray) -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:186-194 (deterministic branch).

    ``m = min(|v|, 6)``; ``u = 2m`` (m <= 2), ``m + 2`` (m <= 4) else
    ``0.5 m + 4``, each step rounded to float32; ``code = rint(u)`` (ties to
    even) or'ed with ``signbit(v) << 3`` (so ``-0.0`` maps to code 8).
    """
    v = np.asarray(values, dtype=np.float32)
    m = np.minimum(np.abs(v), np.float32(6.0))
    u = np.where(m <= np.float32(2.0), m * np.float32(2.0),
                 np.where(m <= np.float32(4.0), m + np.float32(2.0),
                          m * np.float32(0.5) + np.float32(4.0)))
    code = np.rint(u).astype(np.uint8)
    return code | (np.signbit(v).astype(np.uint8) << np.uint8(3))


def _pack_codes(codes: np.ndarray) -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:224 — even column in the low nibble."""
    return (codes[..., 0::2] | (codes[..., 1::2] << np.uint8(4))).astype(np.uint8)


def _inverse_decoding(decoding: np.ndarray) -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:217-221: ``1/dec`` clamped to FLT_MAX, 0 where dec <= 0."""
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        inv = np.minimum(np.float32(1.0) / decoding, FLT_MAX)
    return np.where(decoding > 0, inv, np.float32(0.0)).astype(np.float32)


def quantize_nvfp4_core(values: np.ndarray, two_dimensional: bool, causal_row_scale: bool):
    """src/mcl4_coe/nvfp4.py:197-225 (``stochastic=False``).

    Returns ``(packed uint8 [R, C/2], block_scales e4m3 bits [R, C/16],
    global_scale float32 [1])``.  With ``two_dimensional`` the scale is shared
    by each 16x16 tile and repeated over its 16 rows (:210-212); with
    ``causal_row_scale`` (and 1-D blocks) the global scale is 1 (:204-205).
    """
    values = np.ascontiguousarray(values, dtype=np.float32)
    rows, cols = values.shape
    if causal_row_scale and not two_dimensional:
        g = np.ones(1, dtype=np.float32)
    else:
        amax = np.abs(values).max() if values.size else np.float32(0.0)
        g = np.where(amax > 0, np.float32(amax) / np.float32(2688.0), np.float32(1.0))
        g = np.maximum(g, FLT_MIN_NORMAL).astype(np.float32).reshape(1)
    absv = np.abs(values)
    if two_dimensional:
        tile = absv.reshape(rows // 16, 16, cols // 16, 16).max(axis=(1, 3))
        block_amax = np.repeat(tile, 16, axis=0)
    else:
        block_amax = absv.reshape(rows, cols // 16, 16).max(axis=-1)
    denom = np.float32(6.0) * g[0]
    scales = f32_to_e4m3(np.minimum(block_amax / denom, np.float32(448.0)))
    decoding = e4m3_to_f32(scales) * g[0]
    inv = _inverse_decoding(decoding)
    normalized = (values.reshape(rows, cols // 16, 16) * inv[..., None]).reshape(rows, cols)
    codes = e2m1_codes(normalized)
    return _pack_codes(codes), scales, g


def quantize_activations(x: np.ndarray):
    """Activation mode used by the MoE path: 1x16 row blocks, global scale 1.

    src/mcl4_coe/nvfp4.py:197-225 with ``two_dimensional=False,
    causal_row_scale=True`` — the math of the Triton kernel launched at
    src/mcl4_coe/nvfp4.py:1074-1086 (whose only divergence, ``-0.0`` getting
    code 0 instead of 8 at :731, is not followed: the torch core is the oracle).
    """
    packed, scales, _ = quantize_nvfp4_core(x, False, True)
    return packed, scales


def quantize_grouped_weights(w_batch: np.ndarray, with_bwd: bool = True):
    """src/mcl4_coe/nvfp4.py:923-952 (``_quantize_grouped_weights_core``).

    ``w_batch`` float32 ``[D, N, K]``.  Returns ``(b_fwd [D, K/2, N],
    bs_fwd [D, N, K/16], bg [D], b_bwd [D, N/2, K], bs_bwd [D, K, N/16])`` with
    the e4m3 scales as uint8 bit patterns (the transposed copies are ``None``
    when ``with_bwd`` is false).  One float32 scale per expert
    (``amax/2688``, :928-929); one e4m3 scale per 16x16 tile (:930-931).
    """
    w = np.ascontiguousarray(w_batch, dtype=np.float32)
    d, n, k = w.shape
    w_abs = np.abs(w)
    amax = w_abs.reshape(d, -1).max(axis=1)
    bg = np.where(amax > 0, amax / np.float32(2688.0), np.float32(1.0))
    bg = np.maximum(bg, FLT_MIN_NORMAL).astype(np.float32)
    block_amax = w_abs.reshape(d, n // 16, 16, k // 16, 16).max(axis=(2, 4))
    denom = (np.float32(6.0) * bg).reshape(d, 1, 1)
    bs_tiles = f32_to_e4m3(np.minimum(block_amax / denom, np.float32(448.0)))

    bs_fwd = np.repeat(bs_tiles, 16, axis=1)  # [d, n, k/16]
    inv_fwd = _inverse_decoding(e4m3_to_f32(bs_fwd) * bg.reshape(d, 1, 1))
    norm_fwd = (w.reshape(d, n, k // 16, 16) * inv_fwd[..., None]).reshape(d, n, k)
    b_fwd = np.ascontiguousarray(_pack_codes(e2m1_codes(norm_fwd)).transpose(0, 2, 1))
    if not with_bwd:
        return b_fwd, np.ascontiguousarray(bs_fwd), bg, None, None

    w_t = np.ascontiguousarray(w.transpose(0, 2, 1))
    bs_bwd = np.repeat(bs_tiles.transpose(0, 2, 1), 16, axis=1)  # [d, k, n/16]
    inv_bwd = _inverse_decoding(e4m3_to_f32(bs_bwd) * bg.reshape(d, 1, 1))
    norm_bwd = (w_t.reshape(d, k, n // 16, 16) * inv_bwd[..., None]).reshape(d, k, n)
    b_bwd = np.ascontiguousarray(_pack_codes(e2m1_codes(norm_bwd)).transpose(0, 2, 1))
    return b_fwd, np.ascontiguousarray(bs_fwd), bg, b_bwd, np.ascontiguousarray(bs_bwd)


# --------------------------------------------------------------------------
# Scale swizzle (cuBLASLt / tcgen05 block-scale atom) and dequantisation.
# --------------------------------------------------------------------------

def swizzle_scales(scales: np.ndarray) -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:131-144: 128-row x 4-scale atoms, inner 32x4x4.

    Element ``(r, c)`` lands at byte
    ``((r//128) * Cp/4 + c//4) * 512 + (r%32) * 16 + ((r%128)//32) * 4 + c%4``.
    """
    s = np.asarray(scales, dtype=np.uint8)
    rows, cols = s.shape
    rp, cp = round_up(rows, 128), round_up(cols, 4)
    padded = np.zeros((rp, cp), dtype=np.uint8)
    padded[:rows, :cols] = s
    return np.ascontiguousarray(
        padded.reshape(rp // 128, 4, 32, cp // 4, 4).transpose(0, 3, 2, 1, 4).reshape(rp, cp))


def unswizzle_scales(swizzled: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:147-156 (bit patterns instead of float32)."""
    s = np.asarray(swizzled, dtype=np.uint8)
    rp, cp = s.shape
    return np.ascontiguousarray(
        s.reshape(rp // 128, cp // 4, 32, 4, 4).transpose(0, 3, 2, 1, 4).reshape(rp, cp)[:rows, :cols])


def decode_codes(packed: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Unpack E2M1 nibbles to float32 values (src/mcl4_coe/nvfp4.py:271-278)."""
    raw = np.asarray(packed, dtype=np.uint8)
    c0 = raw & 0x0F
    c1 = (raw >> 4) & 0x0F
    codes = np.stack((c0, c1), axis=-1).reshape(rows, cols)
    sign = np.where((codes & 0x08) != 0, np.float32(-1.0), np.float32(1.0))
    return (sign * E2M1_LEVELS[codes & 0x07]).astype(np.float32)


def dequantize(packed: np.ndarray, scales_rowmajor: np.ndarray, g, rows: int, cols: int) -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:263-281 with row-major (unswizzled) scales."""
    vals = decode_codes(packed, rows, cols)
    dec = e4m3_to_f32(scales_rowmajor) * np.float32(np.asarray(g, dtype=np.float32).reshape(-1)[0])
    return (vals.reshape(rows, cols // 16, 16) * dec[..., None]).reshape(rows, cols).astype(np.float32)


def fake_quantize_activations(x: np.ndarray) -> np.ndarray:
    """Quantise-then-dequantise rows of ``x`` (1x16 blocks, g = 1)."""
    rows, cols = x.shape
    packed, scales = quantize_activations(x)
    return dequantize(packed, scales, np.float32(1.0), rows, cols)


def dequantize_grouped_weight(b_fwd: np.ndarray, bs_fwd: np.ndarray, bg: np.ndarray, e: int) -> np.ndarray:
    """Dense float32 ``[N, K]`` weight of expert ``e`` from the reference cache layout."""
    kh, n = b_fwd.shape[1], b_fwd.shape[2]
    packed_nk = np.ascontiguousarray(b_fwd[e].T)  # [N, K/2]
    return dequantize(packed_nk, bs_fwd[e], bg[e], n, 2 * kh)


# --------------------------------------------------------------------------
# The kernel-side ("MMA") layout of the same bytes.
# --------------------------------------------------------------------------

def weights_to_mma_layout(b_fwd: np.ndarray, bs_fwd: np.ndarray):
    """Reference cache layout -> the layout the tcgen05 kernels read.

    Packed codes become K-major ``[E, N, K/2]`` (``b_fwd.transpose``); the
    per-16 scales of each expert are swizzled into 128x4 atoms
    (:func:`swizzle_scales`), giving ``[E, N/128 * K/64 * 512]`` bytes.  The
    bytes themselves are unchanged.
    """
    e, kh, n = b_fwd.shape
    packed = np.ascontiguousarray(b_fwd.transpose(0, 2, 1))
    sw = np.stack([swizzle_scales(bs_fwd[i]).reshape(-1) for i in range(e)])
    return packed, sw


# --------------------------------------------------------------------------
# 2:4 structured sparsity masks (applied before weight quantisation).
# --------------------------------------------------------------------------

def catalog_2to4() -> np.ndarray:
    """The 90 4x4 0/1 tiles with two ones in every row and column, float32 [90, 16]
    row-major, in the order of src/mcl4_coe/nvfp4.py:50-67 (four nested loops over
    the six 2-of-4 row patterns, first row outermost)."""
    rows = [(1, 1, 0, 0), (1, 0, 1, 0), (1, 0, 0, 1), (0, 1, 1, 0), (0, 1, 0, 1), (0, 0, 1, 1)]
    tiles = [a + b + c + d for a in rows for b in rows for c in rows for d in rows
             if all(a[j] + b[j] + c[j] + d[j] == 2 for j in range(4))]
    return np.array(tiles, dtype=np.float32)


def mask_2to4(w: np.ndarray, mode: str) -> np.ndarray:
    """Boolean mask of ``compute_2to4_mask`` (src/mcl4_coe/nvfp4.py:70-110).

    ``"2to4_row"`` (or a side not divisible by 4): the two largest |w| of every 4
    consecutive elements of a row (zero-padded), ties to the lower index (the
    reference's ``topk`` leaves tie order to the backend).  ``"2to4_transposable"``:
    per 4x4 tile the catalog pattern with the largest float32 sum of kept |w|, first
    maximum on ties (``argmax``)."""
    rows, cols = w.shape
    a = np.abs(w.astype(np.float32))
    if mode == "2to4_row" or rows % 4 or cols % 4:
        pad = round_up(cols, 4) - cols
        g = np.pad(a, ((0, 0), (0, pad))).reshape(rows, -1, 4)
        order = np.argsort(-g, axis=-1, kind="stable")[..., :2]
        m = np.zeros(g.shape, dtype=bool)
        np.put_along_axis(m, order, True, axis=-1)
        return m.reshape(rows, -1)[:, :cols]
    cat = catalog_2to4()
    tiles = a.reshape(rows // 4, 4, cols // 4, 4).transpose(0, 2, 1, 3).reshape(-1, 16)
    best = np.argmax(tiles @ cat.T, axis=-1)
    chosen = cat[best].astype(bool)
    return chosen.reshape(rows // 4, cols // 4, 4, 4).transpose(0, 2, 1, 3).reshape(rows, cols)


def mask_tie_groups(w: np.ndarray, mode: str) -> np.ndarray:
    """Boolean [N, K]: elements whose mask the reference leaves to tie order or to
    float32 summation order — row mode: the 4-groups whose 2nd and 3rd largest |w|
    are equal; transposable mode: the 4x4 tiles whose two best pattern scores are
    within 2e-6 relative (the sums' rounding depends on the BLAS kernel's order)."""
    rows, cols = w.shape
    a = np.abs(w.astype(np.float32))
    if mode == "2to4_row" or rows % 4 or cols % 4:
        pad = round_up(cols, 4) - cols
        g = np.sort(np.pad(a, ((0, 0), (0, pad))).reshape(rows, -1, 4), axis=-1)
        tie = g[..., 1] == g[..., 2]
        return np.repeat(tie, 4, axis=-1)[:, :cols]
    tiles = a.reshape(rows // 4, 4, cols // 4, 4).transpose(0, 2, 1, 3).reshape(-1, 16).astype(np.float64)
    s = np.sort(tiles @ catalog_2to4().astype(np.float64).T, axis=-1)
    near = (s[:, -1] - s[:, -2]) <= 2e-6 * np.maximum(s[:, -1], 1e-30)
    return np.repeat(near[:, None], 16, axis=1).reshape(rows // 4, cols // 4, 4, 4).transpose(0, 2, 1, 3).reshape(
        rows, cols)


# --------------------------------------------------------------------------
# Stochastic rounding of gradients (backward of the grouped NVFP4 projection).
# --------------------------------------------------------------------------

_PHILOX_ROUND_A = np.uint64(0xD2511F53)
_PHILOX_ROUND_B = np.uint64(0xCD9E8D57)
_PHILOX_KEY_A = np.uint64(0x9E3779B9)
_PHILOX_KEY_B = np.uint64(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)


def philox_first_word(counter: np.ndarray, seed: int) -> np.ndarray:
    """Word 0 of Philox4x32-10 (Salmon, Moraes, Dror and Shaw, SC'11) for the counter
    ``(counter, 0, 0, 0)`` and key ``(seed mod 2^32, seed >> 32)``: the draw of Triton's
    ``tl.rand(seed, offset)`` for a 32-bit offset, which the reference's gradient
    quantiser uses as its rounding noise (src/mcl4_coe/nvfp4.py:771-773)."""
    c0 = np.asarray(counter).astype(np.uint64) & _MASK32
    c1 = np.zeros_like(c0)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = np.uint64(seed & 0xFFFFFFFF)
    k1 = np.uint64((seed >> 32) & 0xFFFFFFFF)
    for _ in range(10):
        p0, p2 = c0, c2
        hi_b = (_PHILOX_ROUND_B * p2) >> np.uint64(32)
        hi_a = (_PHILOX_ROUND_A * p0) >> np.uint64(32)
        c0 = hi_b ^ c1 ^ k0
        c2 = hi_a ^ c3 ^ k1
        c1 = (_PHILOX_ROUND_B * p2) & _MASK32
        c3 = (_PHILOX_ROUND_A * p0) & _MASK32
        k0 = (k0 + _PHILOX_KEY_A) & _MASK32
        k1 = (k1 + _PHILOX_KEY_B) & _MASK32
    return c0.astype(np.uint32)


def uniform_from_word(w: np.ndarray) -> np.ndarray:
    """Triton's ``uint_to_uniform_float`` for 32-bit words: the word as int32 x,
    ``x < 0 ? -x - 1 : x``, times 4.6566127342e-10 in float32 (in [0, 1))."""
    x = np.asarray(w, dtype=np.uint32).view(np.int32).astype(np.int64)
    x = np.where(x < 0, -x - 1, x)
    return (x.astype(np.float32) * np.float32(4.6566127342e-10)).astype(np.float32)


def sr_global_scale(x: np.ndarray) -> np.float32:
    """Tensor-wise global scale of a gradient (src/mcl4_coe/nvfp4.py:1129-1134):
    ``max(amax/2688 if amax > 0 else 1, FLT_MIN)``."""
    amax = np.float32(np.abs(np.asarray(x, np.float32)).max()) if np.size(x) else np.float32(0.0)
    g = np.float32(amax / np.float32(2688.0)) if amax > 0 else np.float32(1.0)
    return np.float32(max(g, FLT_MIN_NORMAL))


def quantize_sr(x: np.ndarray, g: float, seed: int, row_index: np.ndarray | None = None):
    """The stochastic branch of the reference's ``_nvfp4_quantize_1d_kernel``
    (src/mcl4_coe/nvfp4.py:735-790 with ``STOCHASTIC=True``, codes :716-732):
    per 16-element row block ``s = e4m3(min(amax / (6 g), 448))``, ``inv = 1/(s g)``
    (0 when ``s g`` is 0), ``u = 2m | m+2 | m/2+4`` of ``m = min(|x inv|, 6)``,
    ``code = min(trunc(u + U), 7)`` with ``U`` the Philox draw of element offset
    ``row * K + col`` (32-bit wrap), sign 8 when ``x inv < 0``.

    ``x``: float32 values of bf16 [M, K]; ``row_index``: the row number each row
    has in the reference's matrix (default 0..M-1).  Returns ``(packed uint8 [M, K/2],
    scales e4m3 bits [M, K/16])``."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    g = np.float32(g)
    blocks = x.reshape(rows, cols // 16, 16)
    amax = np.abs(blocks).max(axis=-1)
    scales = f32_to_e4m3(np.minimum(amax / (np.float32(6.0) * g), np.float32(448.0)))
    dec = (e4m3_to_f32(scales) * g).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(dec > 0, np.float32(1.0) / dec, np.float32(0.0)).astype(np.float32)
    v = (blocks * inv[..., None]).reshape(rows, cols).astype(np.float32)
    m = np.minimum(np.abs(v), np.float32(6.0))
    u = np.where(m <= np.float32(2.0), m * np.float32(2.0),
                 np.where(m <= np.float32(4.0), m + np.float32(2.0), m * np.float32(0.5) + np.float32(4.0)))
    r = np.arange(rows, dtype=np.uint64) if row_index is None else np.asarray(row_index, np.uint64)
    offsets = (r[:, None] * np.uint64(cols) + np.arange(cols, dtype=np.uint64)[None, :]) & _MASK32
    noise = uniform_from_word(philox_first_word(offsets, int(seed)))
    with np.errstate(invalid="ignore"):
        code = np.minimum(np.floor((u + noise).astype(np.float32)), 7).astype(np.uint8)
    code = code | ((v < 0).astype(np.uint8) << np.uint8(3))
    return _pack_codes(code), scales


# --------------------------------------------------------------------------
# Backward of the single-matrix projection (_NVFP4Linear.backward).
# --------------------------------------------------------------------------

# src/mcl4_coe/nvfp4.py:172-178 — signs of the 16 Hadamard rows.
HADAMARD16_SIGNS = np.array([1, 1, 1, -1, 1, -1, -1, -1, -1, -1, -1, 1, -1, 1, -1, -1], dtype=np.float32)


def hadamard16_matrix() -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:337-346: ``eye(16) * signs`` (row i scaled by sign i), four
    butterfly stages over each row's entries (pairs ``(i, i + w)`` inside blocks of ``2w``
    become ``(a + b, a - b)``, w = 1, 2, 4, 8), times 0.25: ``h16[i, j] = signs[i] *
    (-1)^popcount(i & j) / 4``, orthonormal."""
    v = np.eye(16, dtype=np.float32) * HADAMARD16_SIGNS[:, None]
    for w in (1, 2, 4, 8):
        p = v.reshape(16, 16 // (2 * w), 2, w)
        left, right = p[:, :, 0, :].copy(), p[:, :, 1, :].copy()
        v = np.stack((left + right, left - right), axis=2).reshape(16, 16)
    return (v * np.float32(0.25)).astype(np.float32)


def hadamard16(matrix: np.ndarray) -> np.ndarray:
    """src/mcl4_coe/nvfp4.py:349-355: columns zero-padded to a multiple of 16, every
    16-column group times ``h16`` — evaluated in float32 as sign flips, the four
    butterfly stages (pairs ``(i, i + w)`` inside blocks of ``2w``, w = 1, 2, 4, 8) and the
    exact scale 1/4, the operation order of the CUDA kernel.  The reference's fp32
    matmul sums the same 16 signed terms in its own order, so the two agree to float32
    rounding (pinned against the reference's function by a golden fixture)."""
    x = np.asarray(matrix, dtype=np.float32)
    rows, cols = x.shape
    cp = round_up(cols, 16)
    if cp != cols:
        x = np.pad(x, ((0, 0), (0, cp - cols)))
    v = (x.reshape(-1, 16) * HADAMARD16_SIGNS[None, :]).astype(np.float32)
    for w in (1, 2, 4, 8):
        p = v.reshape(-1, 16 // (2 * w), 2, w)
        a, b = p[:, :, 0, :].copy(), p[:, :, 1, :].copy()
        v = np.stack((a + b, a - b), axis=2).reshape(-1, 16).astype(np.float32)
    return (v * np.float32(0.25)).reshape(rows, cp).astype(np.float32)


def quantize_nvfp4_sr(values: np.ndarray, seed: int, causal_row_scale: bool = False):
    """``quantize_nvfp4(stochastic=True)`` in the one-dimensional mode
    (src/mcl4_coe/nvfp4.py:197-225 with the stochastic branch of ``_e2m1_codes``,
    :186-194): scales and global scale as :func:`quantize_nvfp4_core`, codes
    ``min(trunc(u + U), 7) | signbit << 3``.  The reference draws ``U`` with
    ``torch.rand_like``; this build draws it from Philox4x32-10 (:func:`philox_first_word`)
    at offset ``row * cols + col`` (32-bit wrap) under ``seed`` — the same uniform
    distribution, so the codes are the reference's in law, and bit-exact against the
    CUDA kernels for the same seed.  Returns ``(packed [R, C/2], scales [R, C/16], g [1])``."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    rows, cols = values.shape
    _, scales, g = quantize_nvfp4_core(values, False, causal_row_scale)
    dec = (e4m3_to_f32(scales) * g[0]).astype(np.float32)
    inv = _inverse_decoding(dec)
    v = (values.reshape(rows, cols // 16, 16) * inv[..., None]).reshape(rows, cols).astype(np.float32)
    m = np.minimum(np.abs(v), np.float32(6.0))
    u = np.where(m <= np.float32(2.0), m * np.float32(2.0),
                 np.where(m <= np.float32(4.0), m + np.float32(2.0), m * np.float32(0.5) + np.float32(4.0)))
    offsets = (np.arange(rows, dtype=np.uint64)[:, None] * np.uint64(cols)
               + np.arange(cols, dtype=np.uint64)[None, :]) & _MASK32
    noise = uniform_from_word(philox_first_word(offsets, int(seed)))
    code = np.minimum(np.floor((u + noise).astype(np.float32)), 7).astype(np.uint8)
    code = code | (np.signbit(v).astype(np.uint8) << np.uint8(3))
    return _pack_codes(code), scales, g


def linear_wgrad_operand(y: np.ndarray, kt: int, rows_out: int, stochastic: bool, seed: int = 0):
    """One operand of the weight gradient of ``_NVFP4Linear.backward``
    (src/mcl4_coe/nvfp4.py:454-459): ``quantize_nvfp4(_hadamard16(y.T))`` for ``y``
    [M, C] (the gradient, stochastic, or the input, to nearest), the token dimension
    zero-padded to ``kt`` and the rows to ``rows_out`` (as nvfp4_mm pads before its
    GEMM; zero rows and columns quantise to zero codes and scales and leave the global
    scale alone).  Returns ``(packed [rows_out, kt/2], scales [rows_out, kt/16], g [1])``."""
    y = np.asarray(y, dtype=np.float32)
    m, c = y.shape
    t = np.zeros((rows_out, kt), dtype=np.float32)
    t[:c, :m] = y.T
    h = hadamard16(t)
    if stochastic:
        return quantize_nvfp4_sr(h, seed)
    return quantize_nvfp4_core(h, False, False)
