"""The oracle's block formats against the reference's golden vectors.

The fixtures under tests/golden/ were produced by the reference's own GF4
cooker (tools/qw35_cook_common.py) and by gguf-py 0.19.0, see make_golden.py.
"""
import os

import numpy as np
import pytest

from oracle import quants as Q

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_gf4_pack_matches_reference_cooker():
    g = load("gf4.npz")
    with np.errstate(over="ignore", invalid="ignore"):
        words = Q.gf4_pack(g["rows"])
    np.testing.assert_array_equal(words, g["words"])


def test_gf4_exact_dequant_matches_cooker_reconstruction():
    g = load("gf4.npz")
    with np.errstate(over="ignore", invalid="ignore"):
        deq = Q.gf4_dequant_exact(g["words"])
    ref = g["x_hat"]
    assert deq.dtype == np.float32
    np.testing.assert_array_equal(deq.view(np.uint32)[np.isfinite(ref)],
                                  ref.astype(np.float32).view(np.uint32)[np.isfinite(ref)])
    assert np.array_equal(np.isnan(deq), np.isnan(ref))


def test_e5m2_round_trip_matches_reference():
    g = load("gf4.npz")
    np.testing.assert_array_equal(
        Q.e5m2_byte_to_f32(np.arange(256, dtype=np.uint8)).view(np.uint32),
        g["e5m2_table"].view(np.uint32))


def test_gf4_metal_equals_exact_except_element4():
    g = load("gf4.npz")
    words = g["words"][:48]  # finite rows only
    ex = Q.gf4_dequant_exact(words).reshape(48, -1, 8)
    me = Q.gf4_dequant_metal(words).reshape(48, -1, 8)
    keep = [0, 1, 2, 3, 5, 6, 7]
    np.testing.assert_array_equal(ex[..., keep], me[..., keep])
    junk = Q.gf4_metal_element4_junk(words)
    s = Q.e5m2_byte_to_f32((words & 0xFF).astype(np.uint8))
    # element 4 = exact - 0.25 * s * junk / 8192, exactly
    np.testing.assert_array_equal(me[..., 4], ex[..., 4] - np.float32(0.25) * s * junk.astype(np.float32) / np.float32(8192))
    assert (junk != 0).mean() > 0.9


def test_gf4_metal_known_answer_words():
    # Hand-derived from qw35_gf4.metal:8-20.  Word with scale byte 0x3c (fp16 0x3c00 = 1.0),
    # all prepared codes 0 except code1 = 5: q_raw = [4,1,4,4,4,4,4,4].
    w = np.array([[0x3C | (5 << 11)]], dtype=np.uint32)
    ex = Q.gf4_dequant_exact(w)[0]
    me = Q.gf4_dequant_metal(w)[0]
    assert list(ex) == [0.0, 0.75, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0]
    # element 4 junk = (w >> 11) & 0x1ff = 5 -> -0.25 * 5 / 8192
    assert me[4] == np.float32(-0.25 * 5 / 8192)
    assert list(me[[0, 1, 2, 3, 5, 6, 7]]) == [0.0, 0.75, 0.0, 0.0, 0.0, 0.0, 0.0]
    # negative scale byte 0xbc (-1.0), all prepared codes 4 -> q_raw 0 -> weight = s = -1
    w2 = np.array([[0xBC | sum(4 << (8 + 3 * i) for i in range(8))]], dtype=np.uint32)
    assert list(Q.gf4_dequant_exact(w2)[0]) == [-1.0] * 8
    me2 = Q.gf4_dequant_metal(w2)[0]
    junk = (int(w2[0, 0]) >> 11) & 0x1FF
    assert me2[4] == np.float32(-1.0 + 0.25 * junk / 8192)


def test_q8_0_dequant_matches_gguf():
    g = load("q8_0.npz")
    np.testing.assert_array_equal(Q.q8_0_dequant(g["raw"], 32, 256).view(np.uint32), g["deq"].view(np.uint32))
    np.testing.assert_array_equal(Q.q8_0_dequant(g["raw_rand"], 16, 256).view(np.uint32),
                                  g["deq_rand"].view(np.uint32))


def test_q4_k_dequant_matches_gguf():
    g = load("q4_k.npz")
    np.testing.assert_array_equal(Q.q4_k_dequant(g["raw"], 16, 1024).view(np.uint32), g["deq"].view(np.uint32))


@pytest.mark.parametrize("name,fn", [("q5_k.npz", Q.q5_k_dequant), ("q6_k.npz", Q.q6_k_dequant)])
def test_q5_k_q6_k_dequant_matches_gguf(name, fn):
    g = load(name)
    np.testing.assert_array_equal(fn(g["raw"], 16, 1024).view(np.uint32), g["deq"].view(np.uint32))


def test_q6_k_code_order_follows_the_block_layout():
    # one block whose ql/qh encode code = element index % 64 in GGUF order
    blk = np.zeros(210, dtype=np.uint8)
    want = np.arange(256) % 64
    for h in range(2):
        for m in range(4):
            for l in range(32):
                e = 128 * h + 32 * m + l
                qi = 64 * h + 32 * (m & 1) + l
                blk[qi] |= (want[e] & 15) << (0 if m < 2 else 4)
                blk[128 + 32 * h + l] |= (want[e] >> 4) << (2 * m)
    np.testing.assert_array_equal(Q.q6_k_codes(blk[None]), want[None])


def test_q5_k_code_order_follows_the_block_layout():
    # code of element 32j + l: nibble of qs[32(j//2) + l] (high for odd j) + 16 * bit j of qh[l]
    blk = np.zeros(176, dtype=np.uint8)
    want = (np.arange(256) * 7) % 32
    for e in range(256):
        j, l = divmod(e, 32)
        blk[48 + 32 * (j // 2) + l] |= (want[e] & 15) << (4 * (j % 2))
        blk[16 + l] |= (want[e] >> 4) << j
    np.testing.assert_array_equal(Q.q5_k_codes(blk[None]), want[None])


@pytest.mark.parametrize("t", [Q.Q4_K_TYPE, Q.Q5_K_TYPE, Q.Q6_K_TYPE])
def test_tiled_semantics_round_k_quants_to_half(t):
    rng = np.random.default_rng(4)
    raw = Q.gen_weight(rng, t, 4, 512)
    w, wt = Q.dequant(t, raw, 4, 512), Q.dequant(t, raw, 4, 512, tiled=True)
    np.testing.assert_array_equal(wt, w.astype(np.float16).astype(np.float32))
    assert np.any(wt != w)  # the fp32 values are not all halves


def test_q8_0_tiled_semantics_keep_fp32():
    rng = np.random.default_rng(5)
    raw = Q.gen_weight(rng, Q.Q8_0_TYPE, 4, 256)
    np.testing.assert_array_equal(Q.dequant(Q.Q8_0_TYPE, raw, 4, 256, tiled=True), Q.dequant(Q.Q8_0_TYPE, raw, 4, 256))


@pytest.mark.parametrize("t", [Q.GF4_TYPE, Q.Q8_0_TYPE, Q.Q4_K_TYPE, Q.Q5_K_TYPE, Q.Q6_K_TYPE])
def test_generators_row_bytes(t):
    rng = np.random.default_rng(1)
    raw = Q.gen_weight(rng, t, 8, 512)
    assert raw.dtype == np.uint8 and raw.size == 8 * Q.row_bytes(t, 512)
    assert np.isfinite(Q.dequant(t, raw, 8, 512)).all()


def test_gf4_metal_half_rounds_only_element4():
    g = load("gf4.npz")
    words = g["words"][:48]
    me = Q.gf4_dequant_metal(words).reshape(48, -1, 8)
    mh = Q.gf4_dequant_metal_half(words).reshape(48, -1, 8)
    keep = [0, 1, 2, 3, 5, 6, 7]
    np.testing.assert_array_equal(me[..., keep], mh[..., keep])
    assert np.max(np.abs(mh[..., 4] - me[..., 4]) / (np.abs(me[..., 4]) + 1e-30)) <= 2.0 ** -11
