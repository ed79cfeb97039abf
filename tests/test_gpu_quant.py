"""GPU parity of the dequant and fused dequant-matvec kernels against the oracle.

Bit-exact: repack + dequantised weights (all codecs, both GF4 modes) and
argmax token ids.  Matvec family: max relative error 1e-3 (north-star
tolerance) measured as max|y - y_ref| / max|y_ref|, fp64 reference.
"""
import numpy as np
from parity import normerr, relerr
import pytest
import torch

from oracle import ops as O
from oracle import quants as Q
from qwowl35_b200 import ops

pytestmark = pytest.mark.gpu
TOL = 1e-3
CODECS = [Q.GF4_TYPE, Q.Q8_0_TYPE, Q.Q4_K_TYPE, Q.Q5_K_TYPE, Q.Q6_K_TYPE]




def make(t, rows, k, seed=0):
    rng = np.random.default_rng(seed)
    raw = Q.gen_weight(rng, t, rows, k)
    return raw, ops.upload(t, raw, rows, k)


@pytest.mark.parametrize("t", CODECS)
@pytest.mark.parametrize("exact", [False, True])
def test_dequant_bit_exact(t, exact):
    if exact and t != Q.GF4_TYPE:
        pytest.skip("mode only affects GF4")
    rows, k = 64, 4096
    raw, w = make(t, rows, k, 1)
    got = ops.dequant(t, w, rows, k, exact=exact).cpu().numpy()
    ref = Q.dequant(t, raw, rows, k, gf4_exact=exact)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_gf4_dequant_of_reference_cooker_words():
    g = np.load("tests/golden/gf4.npz")
    words = g["words"][:48]
    raw = words.astype("<u4").view(np.uint8).reshape(-1)
    w = ops.upload(Q.GF4_TYPE, raw, 48, 512)
    got = ops.dequant(Q.GF4_TYPE, w, 48, 512, exact=True).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), g["x_hat"][:48].astype(np.float32).view(np.uint32))


def test_q8_0_and_q4_k_dequant_of_gguf_golden():
    g = np.load("tests/golden/q8_0.npz")
    w = ops.upload(Q.Q8_0_TYPE, g["raw"], 32, 256)
    np.testing.assert_array_equal(ops.dequant(Q.Q8_0_TYPE, w, 32, 256).cpu().numpy().view(np.uint32),
                                  g["deq"].view(np.uint32))
    g = np.load("tests/golden/q4_k.npz")
    w = ops.upload(Q.Q4_K_TYPE, g["raw"], 16, 1024)
    np.testing.assert_array_equal(ops.dequant(Q.Q4_K_TYPE, w, 16, 1024).cpu().numpy().view(np.uint32),
                                  g["deq"].view(np.uint32))


@pytest.mark.parametrize("t,name", [(Q.Q5_K_TYPE, "q5_k"), (Q.Q6_K_TYPE, "q6_k")])
def test_q5_k_q6_k_dequant_of_gguf_golden(t, name):
    g = np.load(f"tests/golden/{name}.npz")
    w = ops.upload(t, g["raw"], 16, 1024)
    np.testing.assert_array_equal(ops.dequant(t, w, 16, 1024).cpu().numpy().view(np.uint32),
                                  g["deq"].view(np.uint32))


@pytest.mark.parametrize("t", CODECS)
@pytest.mark.parametrize("shape", [(12288, 4096), (4096, 12288), (1024, 4096), (80, 256), (333, 1280)])
@pytest.mark.parametrize("b", [1, 2, 3])
def test_matvec_parity(t, shape, b):
    rows, k = shape
    raw, w = make(t, rows, k, 2)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((b, k)).astype(np.float32)
    y = ops.matvec(t, w, torch.from_numpy(x).cuda(), rows, k).cpu().numpy()
    # 3+ rows run the tensor-core path: its weight semantics (Q.dequant tiled=True)
    ref = O.matvec(Q.dequant(t, raw, rows, k, tiled=b >= 3), x)
    assert relerr(y, ref) < TOL


@pytest.mark.parametrize("t", CODECS)
def test_matvec_f16_input_and_accumulate(t):
    rows, k = 4096, 4096
    raw, w = make(t, rows, k, 4)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, k)).astype(np.float16)
    base = rng.standard_normal((2, rows)).astype(np.float32)
    y = torch.from_numpy(base.copy()).cuda()
    ops.matvec(t, w, torch.from_numpy(x).cuda(), rows, k, y=y, accumulate=True)
    ref = base + O.matvec(Q.dequant(t, raw, rows, k), x.astype(np.float32))
    assert relerr(y.cpu().numpy(), ref) < TOL


def test_gf4_exact_mode_matvec():
    rows, k = 2048, 4096
    raw, w = make(Q.GF4_TYPE, rows, k, 6)
    x = np.random.default_rng(7).standard_normal((1, k)).astype(np.float32)
    y = ops.matvec(Q.GF4_TYPE, w, torch.from_numpy(x).cuda(), rows, k, exact=True).cpu().numpy()
    assert relerr(y, O.matvec(Q.dequant(Q.GF4_TYPE, raw, rows, k, gf4_exact=True), x)) < TOL


@pytest.mark.parametrize("t", CODECS)
@pytest.mark.parametrize("b", [1, 2, 5])
def test_gate_up_swiglu(t, b):
    rows, k = 12288, 4096
    rawg, wg = make(t, rows, k, 8)
    rawu, wu = make(t, rows, k, 9)
    x = np.random.default_rng(10).standard_normal((b, k)).astype(np.float32)
    h = ops.gate_up_swiglu(t, wg, wu, torch.from_numpy(x).cuda(), rows, k).cpu().numpy()
    ref = O.gate_up_swiglu(Q.dequant(t, rawg, rows, k, tiled=b >= 3), Q.dequant(t, rawu, rows, k, tiled=b >= 3), x)
    assert relerr(h, ref) < TOL


@pytest.mark.parametrize("t", [Q.Q8_0_TYPE, Q.GF4_TYPE, Q.Q6_K_TYPE])
@pytest.mark.parametrize("b", [1, 3])
def test_argmax_head_matches_logits_bit_exact(t, b):
    rows, k = 50000, 4096
    raw, w = make(t, rows, k, 11)
    x = np.random.default_rng(12).standard_normal((b, k)).astype(np.float32)
    tok, val, logits = ops.argmax_head(t, w, torch.from_numpy(x).cuda(), rows, k, want_logits=True)
    logits = logits.cpu().numpy()
    for i in range(b):
        ref_id, ref_v = O.argmax_lowest(logits[i])
        assert int(tok[i]) == ref_id and float(val[i]) == ref_v
    ref = O.matvec(Q.dequant(t, raw, rows, k, tiled=b >= 3), x)
    assert relerr(logits, ref) < TOL
    for i in range(b):
        top2 = np.sort(ref[i])[-2:]
        if top2[1] - top2[0] > 1e-3 * np.abs(ref[i]).max():
            assert int(tok[i]) == int(np.argmax(ref[i]))


def test_argmax_ties_resolve_to_lowest_id():
    # rows identical -> identical logits everywhere: the lowest id must win
    rows, k = 4096, 256
    rng = np.random.default_rng(13)
    one = Q.gen_weight(rng, Q.Q8_0_TYPE, 1, k)
    raw = np.tile(one, rows)
    w = ops.upload(Q.Q8_0_TYPE, raw, rows, k)
    x = torch.from_numpy(rng.standard_normal((2, k)).astype(np.float32)).cuda()
    tok, _, _ = ops.argmax_head(Q.Q8_0_TYPE, w, x, rows, k)
    assert tok.tolist() == [0, 0]
    # a duplicated maximum late in the vocabulary: lowest of the two ids
    raw2 = Q.gen_weight(rng, Q.Q8_0_TYPE, rows, k)
    blk = Q.row_bytes(Q.Q8_0_TYPE, k)
    raw2[3000 * blk:3001 * blk] = raw2[1234 * blk:1235 * blk]
    w2 = ops.upload(Q.Q8_0_TYPE, raw2, rows, k)
    _, _, logits = ops.argmax_head(Q.Q8_0_TYPE, w2, x, rows, k, want_logits=True)
    lg = logits.cpu().numpy()
    # force the duplicated rows to be the maximum by choosing x along row 1234
    deq = Q.dequant(Q.Q8_0_TYPE, raw2, rows, k)
    xs = torch.from_numpy(np.stack([deq[1234], deq[1234]]).astype(np.float32)).cuda()
    tok2, _, lg2 = ops.argmax_head(Q.Q8_0_TYPE, w2, xs, rows, k, want_logits=True)
    lg2 = lg2.cpu().numpy()
    if lg2[0, 1234] == lg2[0].max():
        assert tok2.tolist() == [1234, 1234]
    assert lg.shape == (2, rows)


def test_no_device_wait_timed_out():
    from qwowl35_b200 import lib
    torch.cuda.synchronize()
    assert lib().qw35_cuda_device_error() == 0


# ---- batched (B >= 3) tensor-core path ------------------------------------------
@pytest.mark.parametrize("t", CODECS)
@pytest.mark.parametrize("b", [3, 8, 16, 32, 64, 20])
@pytest.mark.parametrize("shape", [(12288, 4096), (4096, 12288), (333, 1280)])
def test_batched_matvec_parity(t, b, shape):
    rows, k = shape
    raw, w = make(t, rows, k, 20)
    x = np.random.default_rng(21).standard_normal((b, k)).astype(np.float32)
    y = ops.matvec(t, w, torch.from_numpy(x).cuda(), rows, k).cpu().numpy()
    ref = O.matvec(Q.dequant(t, raw, rows, k, tiled=True), x)
    assert relerr(y, ref) < TOL
    if t == Q.GF4_TYPE:  # exact mode too
        ye = ops.matvec(t, w, torch.from_numpy(x).cuda(), rows, k, exact=True).cpu().numpy()
        assert relerr(ye, O.matvec(Q.dequant(t, raw, rows, k, gf4_exact=True), x)) < TOL


@pytest.mark.parametrize("t", CODECS)
def test_batched_accumulate_swiglu_and_head(t):
    rows, k, b = 4096, 4096, 32
    raw, w = make(t, rows, k, 22)
    rng = np.random.default_rng(23)
    x = rng.standard_normal((b, k)).astype(np.float32)
    base = rng.standard_normal((b, rows)).astype(np.float32)
    y = torch.from_numpy(base.copy()).cuda()
    ops.matvec(t, w, torch.from_numpy(x).cuda(), rows, k, y=y, accumulate=True)
    deq = Q.dequant(t, raw, rows, k, tiled=True)
    assert relerr(y.cpu().numpy(), base + O.matvec(deq, x)) < TOL
    raw2, w2 = make(t, rows, k, 24)
    h = ops.gate_up_swiglu(t, w, w2, torch.from_numpy(x).cuda(), rows, k).cpu().numpy()
    assert relerr(h, O.gate_up_swiglu(deq, Q.dequant(t, raw2, rows, k, tiled=True), x)) < TOL
    tok, val, logits = ops.argmax_head(t, w, torch.from_numpy(x).cuda(), rows, k, want_logits=True)
    lg = logits.cpu().numpy()
    assert relerr(lg, O.matvec(deq, x)) < TOL
    for i in range(b):
        rid, rv = O.argmax_lowest(lg[i])
        assert int(tok[i]) == rid and float(val[i]) == rv


def test_batched_and_single_paths_agree():
    rows, k = 4096, 4096
    raw, w = make(Q.Q8_0_TYPE, rows, k, 25)
    x = torch.from_numpy(np.random.default_rng(26).standard_normal((32, k)).astype(np.float32)).cuda()
    yb = ops.matvec(Q.Q8_0_TYPE, w, x, rows, k).cpu().numpy()
    ys = np.concatenate([ops.matvec(Q.Q8_0_TYPE, w, x[i:i + 1], rows, k).cpu().numpy() for i in range(32)])
    assert normerr(yb, ys.astype(np.float64)) < 1e-5
    from qwowl35_b200 import lib
    torch.cuda.synchronize()
    assert lib().qw35_cuda_device_error() == 0


def _random_words_all_scales(rng, rows, k):
    """GF4 words with every finite e5m2 scale byte (both decode paths of the
    tensor-core kernel: |s| <= 252 and larger) and random codes / junk bits."""
    w = rng.integers(0, 2**32, size=(rows, k // 8), dtype=np.uint64).astype(np.uint32)
    sb = rng.integers(0, 256, size=w.shape, dtype=np.uint32)
    sb = np.where((sb & 0x7C) == 0x7C, sb & 0xF3, sb)  # no inf / NaN scales
    return ((w & np.uint32(0xFFFFFF00)) | sb).view(np.uint8).reshape(-1)


@pytest.mark.parametrize("t", CODECS)
@pytest.mark.parametrize("exact", [False, True])
def test_batched_path_weights_bit_exact(t, exact):
    """One-hot activation rows make y[b][r] = W[r][k_b] a single exact product,
    so the tensor-core path's decoded weights are compared bit for bit with the
    oracle: GF4 and Q8_0 exactly the decode values (GF4 element 4 with its
    junk, except in pieces with a scale past 252), the K-quants rounded to half
    as the reference's tiled path does."""
    if t != Q.GF4_TYPE and exact:
        pytest.skip("one mode")
    rows, k, b = 333, 256, 64
    rng = np.random.default_rng(31)
    if t == Q.GF4_TYPE:
        raw = _random_words_all_scales(rng, rows, k)
    elif t in (Q.Q4_K_TYPE, Q.Q5_K_TYPE):  # d, dmin over a wide range, both signs
        raw = Q.gen_weight(rng, t, rows, k)
        blocks = raw.reshape(-1, Q.BLOCK[t][1])
        for off in (0, 2):
            v = (rng.standard_normal(blocks.shape[0]) * 10.0 ** rng.integers(-4, 1, size=blocks.shape[0]))
            blocks[:, off:off + 2] = v.astype(np.float16).view(np.uint8).reshape(-1, 2)
    elif t == Q.Q6_K_TYPE:  # d over a wide range, both signs (scales are signed too)
        raw = Q.gen_weight(rng, t, rows, k)
        blocks = raw.reshape(-1, 210)
        v = rng.standard_normal(blocks.shape[0]) * 10.0 ** rng.integers(-5, 0, size=blocks.shape[0])
        blocks[:, 208:210] = v.astype(np.float16).view(np.uint8).reshape(-1, 2)
    else:
        raw = Q.gen_weight(rng, t, rows, k)
        blocks = raw.reshape(-1, 34)
        d = rng.standard_normal(blocks.shape[0]).astype(np.float16) * np.float16(4)
        blocks[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    w = ops.upload(t, raw, rows, k)
    deq = Q.dequant(t, raw, rows, k, gf4_exact=exact, tiled=True).astype(np.float32)
    for k0 in range(0, k, b):
        x = np.zeros((b, k), dtype=np.float32)
        x[np.arange(b), k0 + np.arange(b)] = 1.0
        y = ops.matvec(t, w, torch.from_numpy(x).cuda(), rows, k, exact=exact).cpu().numpy()
        np.testing.assert_array_equal(y, deq[:, k0:k0 + b].T)


@pytest.mark.parametrize("b", [1, 32])
def test_full_size_q6_k_head_argmax_matches_its_logits(b):
    """The real model's head shape (Q6_K 248320 x 4096): argmax ids are
    bit-exact with the lowest-id argmax of the returned logits, at the batch
    sizes of both matvec paths; a row sample of the logits is checked
    against the oracle."""
    from qwowl35_b200 import synth
    rows, k = 248320, 4096
    g = synth._Gen(41, torch.device("cuda"))
    raw = synth.gen_tensor(g, Q.Q6_K_TYPE, k, rows, "weight")
    w = ops.repack(Q.Q6_K_TYPE, raw, rows, k)
    x = torch.randn(b, k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(42))
    tok, val, logits = ops.argmax_head(Q.Q6_K_TYPE, w, x, rows, k, want_logits=True)
    lg = logits.cpu().numpy()
    for i in range(b):
        ref_id, ref_v = O.argmax_lowest(lg[i])
        assert int(tok[i]) == ref_id and float(val[i]) == ref_v
    sel = np.arange(0, rows, 997)
    raw_h = raw.cpu().numpy().reshape(rows, -1)[sel].reshape(-1)
    ref = O.matvec(Q.dequant(Q.Q6_K_TYPE, raw_h, len(sel), k, tiled=b >= 3), x.cpu().numpy())
    assert relerr(lg[:, sel], ref) < TOL
