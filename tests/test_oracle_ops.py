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
