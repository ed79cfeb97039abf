"""Block formats of the decode path, restated in numpy (oracle, test-only).

Formats (GGUF type ids as the reference's loader uses them,
``qw35-server/src/loader/tensors.rs:123-172``):

* GF4  (type 100): one little-endian uint32 per 8 consecutive input columns.
  bits 0..7   e5m2 scale byte (top byte of the fp16 of the signed group max,
              rounded half-up on the bit pattern),
  bits 8+3i.. 3-bit prepared code ``q_prep_i = q_raw_i ^ 4``.
  weight = (4 - q_raw) * 0.25 * scale.
  Reference: ``tools/qw35_cook_common.py:48-119``.
* Q8_0 (type 8): 34-byte blocks ``{f16 d; int8 qs[32]}``, weight = d * q.
  Reference: ``qw35-server/src/metal/qw35_types.metal:24-27``,
  ``qw35_matvec.metal:630-654``; gguf-py ``Q8_0.dequantize_blocks``.
* Q4_K (type 12): 144-byte blocks ``{f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}``
  over 256 weights; eight 32-weight sub-blocks with 6-bit scale/min;
  weight = d*sc_j*q - dmin*m_j.
  Reference: ``qw35_types.metal:2-7``, ``:70-83``, ``qw35_matvec.metal:2-12``;
  gguf-py ``Q4_K.dequantize_blocks``.
* Q5_K (type 13): 176-byte blocks ``{f16 d; f16 dmin; u8 scales[12]; u8 qh[32];
  u8 qs[128]}``; Q4_K's sub-blocks with a fifth code bit (bit j of qh[l] for
  sub-block j), weight = d*sc_j*(q + 16 h) - dmin*m_j.
  Reference: ``qw35_types.metal:9-15``, ``qw35_matvec.metal:41-64``;
  gguf-py ``Q5_K.dequantize_blocks``.
* Q6_K (type 14): 210-byte blocks ``{u8 ql[128]; u8 qh[64]; i8 scales[16];
  f16 d}``; sixteen 16-weight sub-blocks, weight = d*sc_j*(q6 - 32).
  Reference: ``qw35_types.metal:17-22``, ``qw35_matvec.metal:66-98``,
  ``qw35_output.metal:2-139`` (the fused argmax head); gguf-py
  ``Q6_K.dequantize_blocks``.

All dequantisers return float32 and are bit-exact with the reference's
arithmetic (every product involved is exact in fp32; the single rounding is
the final subtraction in Q4_K / Q5_K, done in the same order as gguf-py).
"""
from __future__ import annotations

import numpy as np

GF4_TYPE = 100
Q8_0_TYPE = 8
Q4_K_TYPE = 12
Q5_K_TYPE = 13
Q6_K_TYPE = 14
F32_TYPE = 0

BLOCK = {GF4_TYPE: (8, 4), Q8_0_TYPE: (32, 34), Q4_K_TYPE: (256, 144), Q5_K_TYPE: (256, 176),
         Q6_K_TYPE: (256, 210)}


def row_bytes(type_id: int, k: int) -> int:
    elems, nbytes = BLOCK[type_id]
    if k % elems:
        raise ValueError(f"K={k} not a multiple of {elems} for type {type_id}")
    return k // elems * nbytes


# --------------------------------------------------------------------------
# e5m2 scale byte (tools/qw35_cook_common.py:48-56)
# --------------------------------------------------------------------------
def f32_to_e5m2_byte(values: np.ndarray) -> np.ndarray:
    """Top byte of the fp16 bit pattern after adding 0x80 (round half up on bits)."""
    bits = np.asarray(values, dtype=np.float32).astype(np.float16).view(np.uint16).astype(np.uint32)
    return (((bits + 0x80) >> 8) & 0xFF).astype(np.uint8)


def e5m2_byte_to_f32(b: np.ndarray) -> np.ndarray:
    """e5m2 byte -> fp16 (byte << 8) -> fp32, exact."""
    return (np.asarray(b, dtype=np.uint16) << 8).astype(np.uint16).view(np.float16).astype(np.float32)


# --------------------------------------------------------------------------
# GF4 (tools/qw35_cook_common.py:67-119; qw35_gf4.metal:8-20)
# --------------------------------------------------------------------------
def gf4_pack(rows: np.ndarray) -> np.ndarray:
    """Pack float rows [R, K] into GF4 words [R, K/8] (no scale search).

    Restates ``pack_gf4_prepared(rows, scale_search=False)``: the group scale is
    the signed element of largest magnitude (first on ties), rounded to e5m2;
    codes ``q_raw = clip(rint(x/s * -4 + 4), 0, 7)`` (0 where s == 0).
    """
    rows = np.asarray(rows, dtype=np.float32)
    r, k = rows.shape
    if k % 8:
        raise ValueError("GF4 needs K % 8 == 0")
    g = rows.reshape(r, k // 8, 8)
    idx = np.abs(g).argmax(axis=2)
    gmax = np.take_along_axis(g, idx[..., None], axis=2)[..., 0]
    sbyte = f32_to_e5m2_byte(gmax)
    s = e5m2_byte_to_f32(sbyte)
    norm = np.zeros_like(g)
    np.divide(g, s[..., None], out=norm, where=s[..., None] != 0.0)
    q_raw = np.clip(np.rint(norm * np.float32(-4.0) + np.float32(4.0)), 0.0, 7.0).astype(np.uint32)
    words = sbyte.astype(np.uint32)
    for i in range(8):
        words |= (q_raw[:, :, i] ^ np.uint32(4)) << np.uint32(8 + 3 * i)
    return words.astype("<u4")


def _gf4_fields(words: np.ndarray):
    w = np.asarray(words, dtype=np.uint32)
    s = e5m2_byte_to_f32((w & 0xFF).astype(np.uint8))
    prep = np.stack([(w >> np.uint32(8 + 3 * i)) & np.uint32(7) for i in range(8)], axis=-1)
    return w, s, prep


def gf4_dequant_exact(words: np.ndarray) -> np.ndarray:
    """The cooker's reconstruction ``(4 - q_raw) * 0.25 * s`` -> float32 [R, K]."""
    w, s, prep = _gf4_fields(words)
    q_raw = (prep ^ np.uint32(4)).astype(np.float32)
    out = (np.float32(4.0) - q_raw) * np.float32(0.25) * s[..., None]
    return out.reshape(w.shape[0], -1).astype(np.float32)


def gf4_metal_element4_junk(words: np.ndarray) -> np.ndarray:
    """Junk the Metal decode adds to element 4 of every word, in units of 2^-13.

    ``qw35_gf4_dot8_vec_f32`` builds ``packed`` with codes 0..3 at bits 4..15 and
    codes 4..7 at bits 20..31, then for i == 0 shifts ``packed << 9`` without
    the ``0xe000e000`` mask, so the high int16 keeps packed bits 7..15 (codes
    1..3, 9 bits) below code 4: junk = (w >> 11) & 0x1ff.
    """
    w = np.asarray(words, dtype=np.uint32)
    return ((w >> np.uint32(11)) & np.uint32(0x1FF)).astype(np.uint32)


def gf4_dequant_metal(words: np.ndarray) -> np.ndarray:
    """Bit-exact weights as the reference decode kernel sees them -> float32 [R, K].

    Element j of a word is ``int16_j * scale'`` with ``scale' = s * -0.25 * 2^-13``;
    ``int16_j = signed3(prep_j) * 8192`` except element 4, which carries the
    junk bits described in :func:`gf4_metal_element4_junk`.  Every product is
    exact in fp32.
    """
    w, s, prep = _gf4_fields(words)
    signed = (prep.astype(np.int32) ^ 4) - 4  # sign-extend the 3-bit prepared code
    ints = signed * 8192
    ints[..., 4] += gf4_metal_element4_junk(w).astype(np.int32)
    scale = s * np.float32(-0.25) * np.float32(0.0001220703125)
    out = ints.astype(np.float32) * scale[..., None]
    return out.reshape(w.shape[0], -1).astype(np.float32)


def gf4_dequant_metal_half(words: np.ndarray) -> np.ndarray:
    """The reference's multi-token (tiled) dequant, qw35_dequantize_gf4
    (qw35_gf4.metal:42-58): the Metal decode values rounded to half (only
    element 4 of a word is not already exact in half)."""
    return gf4_dequant_metal(words).astype(np.float16).astype(np.float32)


def gf4_dequant_batched(words: np.ndarray) -> np.ndarray:
    """Metal-mode weights as the batched (tensor-core, 3+ rows) path of this
    build uses them: the reference decode values exactly (levels and the
    element-4 junk), except in a 16-byte piece (4 words) holding a scale with
    |s| > 252 (e5m2 byte & 0x7f > 0x5B), where element 4 takes the tiled
    path's half rounding (``gf4_dequant_metal_half``)."""
    w = np.asarray(words, dtype=np.uint32)
    exact = gf4_dequant_metal(w)
    rows = w.shape[0]
    big = ((w & np.uint32(0x7F)) > np.uint32(0x5B)).reshape(rows, -1, 4).any(axis=-1)  # [rows, quads]
    if not big.any():
        return exact
    half = gf4_dequant_metal_half(w).reshape(rows, -1, 32)
    out = exact.reshape(rows, -1, 32).copy()
    out[big] = half[big]
    return out.reshape(exact.shape)


def gf4_dequant(words: np.ndarray, exact: bool = False, half: bool = False, batched: bool = False) -> np.ndarray:
    if exact:
        return gf4_dequant_exact(words)
    if batched:
        return gf4_dequant_batched(words)
    return gf4_dequant_metal_half(words) if half else gf4_dequant_metal(words)


# --------------------------------------------------------------------------
# Q8_0 (qw35_types.metal:24-27; qw35_matvec.metal:630-654)
# --------------------------------------------------------------------------
def q8_0_dequant(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    b = np.asarray(raw, dtype=np.uint8).reshape(rows * (k // 32), 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].copy().view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, k)


# --------------------------------------------------------------------------
# Q4_K (qw35_types.metal:2-7, :70-83; qw35_matvec.metal:2-12)
# --------------------------------------------------------------------------
def q4_k_scale_min(scales: np.ndarray):
    """6-bit sub-block scale/min unpack (qw35_get_scale_min_k4), [n,12] -> ([n,8],[n,8])."""
    q = np.asarray(scales, dtype=np.uint8)
    sc = np.empty(q.shape[:-1] + (8,), dtype=np.uint8)
    mn = np.empty_like(sc)
    for j in range(8):
        if j < 4:
            sc[..., j] = q[..., j] & 63
            mn[..., j] = q[..., j + 4] & 63
        else:
            sc[..., j] = (q[..., j + 4] & 0x0F) | ((q[..., j - 4] >> 6) << 4)
            mn[..., j] = (q[..., j + 4] >> 4) | ((q[..., j] >> 6) << 4)
    return sc, mn


def q4_k_dequant(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    b = np.asarray(raw, dtype=np.uint8).reshape(rows * (k // 256), 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    sc, mn = q4_k_scale_min(b[:, 4:16])
    qs = b[:, 16:144]
    out = np.empty((b.shape[0], 256), dtype=np.float32)
    for j in range(8):
        grp = qs[:, (j // 2) * 32:(j // 2) * 32 + 32]
        q = (grp & 0x0F) if (j % 2 == 0) else (grp >> 4)
        dl = d * sc[:, j:j + 1].astype(np.float32)
        ml = dmin * mn[:, j:j + 1].astype(np.float32)
        out[:, j * 32:(j + 1) * 32] = dl * q.astype(np.float32) - ml
    return out.reshape(rows, k)


# --------------------------------------------------------------------------
# Q5_K (qw35_types.metal:9-15; qw35_matvec.metal:41-64)
# --------------------------------------------------------------------------
def q5_k_codes(b: np.ndarray) -> np.ndarray:
    """[n,176] blocks -> [n,256] 5-bit codes: element 32j+l = nibble (j even: low,
    j odd: high) of qs[32(j//2)+l] plus 16 * bit j of qh[l]."""
    qh, qs = b[:, 16:48], b[:, 48:176]
    out = np.empty((b.shape[0], 256), dtype=np.uint8)
    for j in range(8):
        grp = qs[:, (j // 2) * 32:(j // 2) * 32 + 32]
        lo = (grp & 0x0F) if (j % 2 == 0) else (grp >> 4)
        out[:, j * 32:(j + 1) * 32] = lo | (((qh >> j) & 1) << 4)
    return out


def q5_k_dequant(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    b = np.asarray(raw, dtype=np.uint8).reshape(rows * (k // 256), 176)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    sc, mn = q4_k_scale_min(b[:, 4:16])
    q = q5_k_codes(b).astype(np.float32).reshape(-1, 8, 32)
    dl = (d * sc.astype(np.float32))[:, :, None]
    ml = (dmin * mn.astype(np.float32))[:, :, None]
    return (dl * q - ml).reshape(rows, k)


# --------------------------------------------------------------------------
# Q6_K (qw35_types.metal:17-22; qw35_matvec.metal:66-98, :458-542)
# --------------------------------------------------------------------------
def q6_k_codes(b: np.ndarray) -> np.ndarray:
    """[n,210] blocks -> [n,256] unsigned 6-bit codes (weight uses code - 32).
    In each 128-element half h, element 128h+32m+l takes the low (m < 2) or
    high (m >= 2) nibble of ql[64h + 32(m&1) + l] and bits 2m..2m+1 of
    qh[32h + l]."""
    ql, qh = b[:, 0:128], b[:, 128:192]
    out = np.empty((b.shape[0], 256), dtype=np.uint8)
    for h in range(2):
        for m in range(4):
            src = ql[:, 64 * h + 32 * (m & 1):64 * h + 32 * (m & 1) + 32]
            lo = (src & 0x0F) if m < 2 else (src >> 4)
            hi = (qh[:, 32 * h:32 * h + 32] >> (2 * m)) & 3
            out[:, 128 * h + 32 * m:128 * h + 32 * m + 32] = lo | (hi << 4)
    return out


def q6_k_dequant(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    b = np.asarray(raw, dtype=np.uint8).reshape(rows * (k // 256), 210)
    sc = b[:, 192:208].copy().view(np.int8).astype(np.float32)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)
    dl = (d * sc)[:, :, None]                                     # exact in fp32
    q = (q6_k_codes(b).astype(np.float32) - 32.0).reshape(-1, 16, 16)
    return (dl * q).reshape(rows, k)


def dequant(type_id: int, raw: np.ndarray, rows: int, k: int, gf4_exact: bool = False,
            gf4_half: bool = False, tiled: bool = False) -> np.ndarray:
    """Dequantised weights [rows, k] float32.

    ``tiled=True`` gives the weights of this build's batched (tensor-core)
    path: GF4 exactly the decode values (``gf4_dequant_batched``; element 4
    rounded to half only in pieces with a scale past 252, as the reference's
    tiled path ``qw35_tiled_mm.metal:197-255`` rounds it everywhere), and the
    K-quants' fp32 values rounded to half as the reference's tiled path
    computes them (Q4_K ``dl*q - ml``,
    ``qw35_matvec.metal:20-38``; Q5_K the same with the fifth bit, :40-64;
    Q6_K ``d*sc*(q - 32)``, exact in fp32, :66-98).
    """
    if type_id == GF4_TYPE:
        return gf4_dequant(np.asarray(raw).view(np.uint32).reshape(rows, k // 8), exact=gf4_exact,
                           half=gf4_half, batched=tiled and not gf4_exact)
    if type_id == Q8_0_TYPE:
        return q8_0_dequant(raw, rows, k)
    if type_id == Q4_K_TYPE:
        w = q4_k_dequant(raw, rows, k)
        return w.astype(np.float16).astype(np.float32) if tiled else w
    if type_id in (Q5_K_TYPE, Q6_K_TYPE):
        w = (q5_k_dequant if type_id == Q5_K_TYPE else q6_k_dequant)(raw, rows, k)
        return w.astype(np.float16).astype(np.float32) if tiled else w
    if type_id == F32_TYPE:
        return np.asarray(raw).view(np.float32).reshape(rows, k)
    raise ValueError(f"unsupported type {type_id}")


# --------------------------------------------------------------------------
# Synthetic generators (benchmark configs 1, 2 and 5)
# --------------------------------------------------------------------------
def gen_gf4(rng: np.random.Generator, rows: int, k: int) -> np.ndarray:
    """GF4 words: 8 uniform 3-bit codes + e5m2 scale of |N(0, 0.02)| per word."""
    words = rng.integers(0, 1 << 32, size=(rows, k // 8), dtype=np.uint64).astype(np.uint32)
    sbyte = f32_to_e5m2_byte(np.abs(rng.normal(0.0, 0.02, size=(rows, k // 8))).astype(np.float32))
    return ((words & np.uint32(0xFFFFFF00)) | sbyte.astype(np.uint32)).astype("<u4")


def gen_q8_0(rng: np.random.Generator, rows: int, k: int, d_div: float = 1.0) -> np.ndarray:
    """Q8_0 blocks: int8 codes uniform in [-127, 127], d = fp16(|N(0,0.02)| / d_div)."""
    nb = rows * (k // 32)
    out = np.empty((nb, 34), dtype=np.uint8)
    d = (np.abs(rng.normal(0.0, 0.02, size=nb)) / d_div).astype(np.float16)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    return out.reshape(-1)


def gen_q4_k(rng: np.random.Generator, rows: int, k: int, d_div: float = 1.0) -> np.ndarray:
    """Q4_K blocks: fp16 d, dmin = |N(0,0.02)|/d_div; 6-bit scales/mins and 4-bit codes uniform."""
    nb = rows * (k // 256)
    out = rng.integers(0, 256, size=(nb, 144), dtype=np.uint16).astype(np.uint8)
    d = (np.abs(rng.normal(0.0, 0.02, size=nb)) / d_div).astype(np.float16)
    dmin = (np.abs(rng.normal(0.0, 0.02, size=nb)) / d_div).astype(np.float16)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def gen_q5_k(rng: np.random.Generator, rows: int, k: int, d_div: float = 1.0) -> np.ndarray:
    """Q5_K blocks: fp16 d, dmin = |N(0,0.02)|/d_div / 2; scales, mins, qh and qs uniform."""
    nb = rows * (k // 256)
    out = rng.integers(0, 256, size=(nb, 176), dtype=np.uint16).astype(np.uint8)
    out[:, 0:2] = (np.abs(rng.normal(0.0, 0.01, size=nb)) / d_div).astype(np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = (np.abs(rng.normal(0.0, 0.01, size=nb)) / d_div).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def gen_q6_k(rng: np.random.Generator, rows: int, k: int, d_div: float = 1.0) -> np.ndarray:
    """Q6_K blocks: ql/qh uniform, int8 scales uniform in [-64, 63], d = fp16(|N(0,0.001)|/d_div)."""
    nb = rows * (k // 256)
    out = rng.integers(0, 256, size=(nb, 210), dtype=np.uint16).astype(np.uint8)
    out[:, 192:208] = rng.integers(-64, 64, size=(nb, 16)).astype(np.int8).view(np.uint8)
    out[:, 208:210] = (np.abs(rng.normal(0.0, 0.001, size=nb)) / d_div).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def gen_weight(rng: np.random.Generator, type_id: int, rows: int, k: int, d_div: float = 1.0) -> np.ndarray:
    """Raw GGUF-layout bytes (uint8) of a synthetic weight."""
    if type_id == GF4_TYPE:
        return gen_gf4(rng, rows, k).view(np.uint8).reshape(-1)
    if type_id == Q8_0_TYPE:
        return gen_q8_0(rng, rows, k, d_div)
    if type_id == Q4_K_TYPE:
        return gen_q4_k(rng, rows, k, d_div)
    if type_id == Q5_K_TYPE:
        return gen_q5_k(rng, rows, k, d_div)
    if type_id == Q6_K_TYPE:
        return gen_q6_k(rng, rows, k, d_div)
    raise ValueError(type_id)
