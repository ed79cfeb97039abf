"""CPU self-checks of the oracle's op restatements (no GPU)."""
import numpy as np

from oracle import ops as O


def test_deltanet_core_identity_gate_zero_beta():
    rng = np.random.default_rng(0)
    S = rng.normal(0, 0.01, (32, 128, 128))
    q = rng.normal(0, 1, (16, 128)); k = rng.normal(0, 1, (16, 128))
    v = rng.normal(0, 1, (32, 128))
    y, Sn = O.deltanet_core(S, q, k, v, np.zeros(32), np.zeros(32), 1.0)
    np.testing.assert_allclose(Sn, S)              # beta 0, gate 1: state unchanged
    np.testing.assert_allclose(y[0], S[0] @ q[0])   # readout = S q


def test_deltanet_core_delta_rule_stores_value():
    # beta = 1, gate = 1, unit k: after the update S k == v exactly
    S = np.zeros((32, 128, 128)); k = np.zeros((16, 128)); k[:, 0] = 1.0
    v = np.arange(32 * 128, dtype=np.float64).reshape(32, 128)
    _, Sn = O.deltanet_core(S, k, k, v, np.ones(32), np.zeros(32), 1.0)
    for h in range(32):
        np.testing.assert_allclose(Sn[h] @ k[h % 16], v[h])


def test_softplus_threshold():
    assert O.softplus(25.0) == 25.0
    assert abs(O.softplus(0.0) - np.log(2.0)) < 1e-15


def test_gqa_decode_uniform_scores_average_values():
    K = np.zeros((10, 4, 256), np.float16)
    V = np.random.default_rng(1).normal(0, 1, (10, 4, 256)).astype(np.float16)
    out = O.gqa_decode(np.ones((16, 256)), None, K, V)
    np.testing.assert_allclose(out[0], V[:, 0].astype(np.float64).mean(0), rtol=1e-12)
    np.testing.assert_allclose(out[5], V[:, 1].astype(np.float64).mean(0), rtol=1e-12)


def test_attended_positions_window_and_sink():
    assert list(O.attended_positions(10)) == list(range(10))
    assert list(O.attended_positions(10, window=3, sink=2)) == [0, 1, 7, 8, 9]
    assert list(O.attended_positions(10, window=8, sink=2)) == list(range(10))


def test_argmax_lowest_tie():
    assert O.argmax_lowest(np.array([1.0, 3.0, 2.0, 3.0])) == (1, 3.0)


def test_rope_freqs_ladder():
    f = O.rope_freqs(1.0e7)
    assert f.dtype == np.float32 and f[0] == 1.0 and len(f) == 32
    assert np.all(np.diff(f) < 0)


# ---- q8_0 KV cache (qw35_attention.metal:425-793) ------------------------------
def test_q8_0_kv_quantize_known_blocks():
    x = np.zeros((3, 32), dtype=np.float32)
    x[1, :] = np.arange(-16, 16, dtype=np.float32) * 8.0      # amax 128 -> d = 128/127
    x[2, 0], x[2, 1], x[2, 2], x[2, 3] = 127.0, 2.5, -2.5, 0.49999997
    d, qs = O.q8_0_kv_quantize(x)
    assert d[0] == 0 and not qs[0].any()                       # all-zero block
    assert qs[1, 0] == -127 and qs[1, 31] == round(120 * 127 / 128)
    assert d[2] == np.float16(1.0)
    assert list(qs[2, :4]) == [127, 3, -3, 0]                   # half away from zero; 0.49999997 -> 0


def test_q8_0_kv_codes_use_the_fp32_scale_and_store_half():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, size=(64, 32)).astype(np.float32)
    d, qs = O.q8_0_kv_quantize(x)
    d32 = np.max(np.abs(x), axis=1) / np.float32(127.0)
    assert d.shape == (64, 1) and np.any(d[:, 0].astype(np.float32) != d32)  # half(d) differs from the fp32 d
    ref = np.clip(np.round(x.astype(np.float64) / d32[:, None].astype(np.float64)), -127, 127)
    assert np.max(np.abs(qs.astype(np.float64) - ref)) <= 1     # ties / reciprocal rounding only
    deq = O.q8_0_kv_dequant(d, qs)
    assert np.max(np.abs(deq - x) / np.max(np.abs(x), axis=1, keepdims=True)) < 1.0 / 127 + 1e-3


def test_gqa_decode_q8_0_close_to_f16_cache():
    rng = np.random.default_rng(1)
    L = 300
    K = rng.normal(0, 1, size=(L, 4, 256)).astype(np.float32)
    V = rng.normal(0, 1, size=(L, 4, 256)).astype(np.float32)
    q, gate = rng.normal(0, 1, size=(16, 256)), rng.normal(0, 1, size=(16, 256))
    ref = O.gqa_decode(q, gate, K.astype(np.float16), V.astype(np.float16))
    got = O.gqa_decode_q8_0(q, gate, O.q8_0_kv_quantize(K), O.q8_0_kv_quantize(V))
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) < 0.05
    kd, kq = O.q8_0_kv_quantize(K)
    assert kd.shape == (L, 4, 8) and kq.shape == (L, 4, 256) and kq.dtype == np.int8


def test_attn_preprocess_q8_0_matches_f16_twin_up_to_quantisation():
    rng = np.random.default_rng(2)
    qf, k, v = rng.normal(0, 1, (16, 512)), rng.normal(0, 1, (4, 256)), rng.normal(0, 1, (4, 256))
    qn, kn = np.abs(rng.normal(1, 0.1, 256)), np.abs(rng.normal(1, 0.1, 256))
    fr = O.rope_freqs()
    q16, g16, k16, v16 = O.attn_preprocess(qf, k, v, qn, kn, 7, fr)
    q8, g8, (kd, kq), (vd, vq) = O.attn_preprocess_q8_0(qf, k, v, qn, kn, 7, fr)
    np.testing.assert_array_equal(q8, q16)
    np.testing.assert_array_equal(g8, g16)
    kdq = O.q8_0_kv_dequant(kd, kq)
    assert np.max(np.abs(kdq - k16.astype(np.float64))) <= np.max(np.abs(k16.astype(np.float64))) / 127 + 1e-2
    np.testing.assert_array_equal(O.q8_0_kv_quantize(v.astype(np.float32))[1], vq)


def test_parity_measure_catches_small_row_errors():
    """The GPU tests' relerr adds a per-element bound above 1e-3 of the largest
    output, so a 1% error on a small element fails although it is far below the
    norm-wise 1e-3 of the largest one."""
    from parity import elemerr, normerr, relerr
    ref = np.array([1000.0, 2.0, -3.0, 1e-4])
    y = ref.copy()
    y[1] *= 1.01
    assert normerr(y, ref) < 1e-3 and relerr(y, ref) > 1e-3
    y = ref.copy()
    y[3] *= 2.0  # below the significance floor: norm-wise only
    assert elemerr(y, ref) == 0.0 and relerr(y, ref) < 1e-6


def test_deltanet_core_known_answer_two_by_two():
    """The delta rule on a 2-dimensional head, derived by hand from
    qw35_ssm.metal:393-428 (k_dot / q_dot from the OLD state; gate 1/2):
    S = [[1, 0], [0, 2]], k = e0, q = e1, v = (3, 4), beta = 1/2, gate = 1/2:
    k_dot = (1, 0), q_dot = (0, 2), k.q = 0, delta = (3 - 1/2, 4) / 2 = (1.25, 2),
    S' = S / 2 + delta (x) k = [[1.75, 0], [2, 1]], y = (gate * q_dot) * scale = (0, 1)."""
    S = np.array([[[1.0, 0.0], [0.0, 2.0]]])
    k = np.array([[1.0, 0.0]])
    q = np.array([[0.0, 1.0]])
    v = np.array([[3.0, 4.0]])
    y, Sn = O.deltanet_core(S, q, k, v, np.array([0.5]), np.array([np.log(0.5)]), 1.0)
    np.testing.assert_allclose(Sn[0], [[1.75, 0.0], [2.0, 1.0]], rtol=0, atol=1e-15)
    np.testing.assert_allclose(y[0], [0.0, 1.0], rtol=0, atol=1e-15)
