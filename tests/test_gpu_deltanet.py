"""Gated DeltaNet decode step: CUDA (thread-block cluster kernel) vs the fp64
oracle restating qw35_ssm.metal:260-451.  Tolerance: max relative error 1e-3."""
import numpy as np
from parity import normerr, relerr
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3




def layer_params(rng):
    return dict(conv_w=rng.normal(0, 0.3, (8192, 4)).astype(np.float32),
                dt=rng.normal(0, 1, 32).astype(np.float32),
                a=(-np.exp(rng.normal(0, 0.5, 32))).astype(np.float32),
                norm_w=np.abs(rng.normal(1, 0.1, 128)).astype(np.float32))


@pytest.mark.parametrize("n,nslots", [(1, 1), (3, 5), (17, 17)])
def test_deltanet_step_matches_oracle(n, nslots):
    rng = np.random.default_rng(n)
    P = layer_params(rng)
    proj = rng.normal(0, 1, (n, 12352)).astype(np.float32)
    conv = rng.normal(0, 1, (nslots, 8192 * 3)).astype(np.float32)
    ssm = rng.normal(0, 0.01, (nslots, 32 * 128 * 128)).astype(np.float32)
    slots = rng.permutation(nslots)[:n].astype(np.int32)
    d = {k: torch.from_numpy(v).cuda() for k, v in P.items()}
    conv_d, ssm_d = torch.from_numpy(conv.copy()).cuda(), torch.from_numpy(ssm.copy()).cuda()
    from qwowl35_b200 import ops
    out = ops.deltanet_step(torch.from_numpy(proj).cuda(), d["conv_w"], d["dt"], d["a"], d["norm_w"], conv_d, ssm_d,
                            slots=torch.from_numpy(slots).cuda()).cpu().numpy()
    conv_new, ssm_new = conv_d.cpu().numpy(), ssm_d.cpu().numpy()
    for i in range(n):
        s = slots[i]
        qkv, z = proj[i, :8192], proj[i, 8192:12288]
        beta, alpha = proj[i, 12288:12320], proj[i, 12320:12352]
        ref_out, ref_cs, ref_S = O.deltanet_step(qkv, P["conv_w"], conv[s].reshape(8192, 3), beta, alpha, P["dt"],
                                                 P["a"], ssm[s].reshape(32, 128, 128), z, P["norm_w"])
        assert relerr(out[i], ref_out) < TOL
        np.testing.assert_array_equal(conv_new[s].reshape(8192, 3), ref_cs.astype(np.float32))
        assert relerr(ssm_new[s], ref_S.reshape(-1)) < TOL
    untouched = sorted(set(range(nslots)) - set(slots.tolist()))
    for s in untouched:
        np.testing.assert_array_equal(conv_new[s], conv[s])
        np.testing.assert_array_equal(ssm_new[s], ssm[s])


def test_deltanet_repeated_steps_stay_in_tolerance():
    rng = np.random.default_rng(42)
    P = layer_params(rng)
    d = {k: torch.from_numpy(v).cuda() for k, v in P.items()}
    conv = np.zeros((1, 8192 * 3), np.float32)
    ssm = np.zeros((1, 32 * 128 * 128), np.float32)
    conv_d, ssm_d = torch.from_numpy(conv.copy()).cuda(), torch.from_numpy(ssm.copy()).cuda()
    from qwowl35_b200 import ops
    cs_ref, S_ref = conv[0].reshape(8192, 3).astype(np.float64), ssm[0].reshape(32, 128, 128).astype(np.float64)
    for step in range(6):
        proj = rng.normal(0, 1, (1, 12352)).astype(np.float32)
        out = ops.deltanet_step(torch.from_numpy(proj).cuda(), d["conv_w"], d["dt"], d["a"], d["norm_w"], conv_d,
                                ssm_d).cpu().numpy()
        ref, cs_ref, S_ref = O.deltanet_step(proj[0, :8192], P["conv_w"], cs_ref, proj[0, 12288:12320],
                                             proj[0, 12320:12352], P["dt"], P["a"], S_ref, proj[0, 8192:12288],
                                             P["norm_w"])
        assert relerr(out[0], ref) < TOL, step


@pytest.mark.parametrize("n", [1, 4, 64])
def test_deltanet_core_config3(n):
    """prepared q/k (L2-normalised f16), v f16, beta, log-decay g."""
    rng = np.random.default_rng(100 + n)
    q = rng.normal(0, 1, (n, 16, 128))
    k = rng.normal(0, 1, (n, 16, 128))
    q = (q / np.linalg.norm(q, axis=-1, keepdims=True)).astype(np.float16)
    k = (k / np.linalg.norm(k, axis=-1, keepdims=True)).astype(np.float16)
    v = rng.normal(0, 1, (n, 32, 128)).astype(np.float16)
    beta = O.sigmoid(rng.normal(0, 1, (n, 32))).astype(np.float32)
    g = (-O.softplus(rng.normal(0, 1, (n, 32)))).astype(np.float32)
    S = rng.normal(0, 0.01, (n, 32, 128, 128)).astype(np.float32)
    from qwowl35_b200 import ops
    Sd = torch.from_numpy(S.copy()).cuda()
    y = ops.deltanet_core(*(torch.from_numpy(a).cuda() for a in (q, k, v, beta, g)), Sd).cpu().numpy()
    Sn = Sd.cpu().numpy()
    for i in range(n):
        yr, Sr = O.deltanet_core(S[i], q[i].astype(np.float64), k[i].astype(np.float64), v[i], beta[i], g[i],
                                 1.0 / np.sqrt(128))
        assert relerr(y[i], yr) < TOL
        assert relerr(Sn[i], Sr) < TOL


def test_deltanet_core_known_answer():
    """Hand-derived values pin the order of the delta rule (qw35_ssm.metal:393-428):
    k_dot and q_dot read the OLD state, delta = (v - gate * k_dot) * beta, the
    state becomes S * gate + delta (x) k, y = (gate * q_dot + delta * (k . q)) * scale.
    Head 0 (qk group 0): S = [[1, 0], [0, 2]], k = e0, q = e1, v = (3, 4), beta 1/2,
    gate 1 (g = 0): k_dot = (1, 0), q_dot = (0, 2), k.q = 0, delta = (1, 2),
    S' = [[2, 0], [2, 2]], y = (0, 2) * scale.  Head 1 (group 1): S = [[1, 0], [0, 2]],
    q = k = e0, v = (3, 4), beta 1, gate 1: k_dot = q_dot = (1, 0), k.q = 1,
    delta = (2, 4), S' = [[3, 0], [4, 2]], y = (1 + 2, 0 + 4) * scale = (3, 4) * scale.
    Every other entry is zero.  All values are exact in fp32: the match is exact."""
    q = np.zeros((1, 16, 128), np.float16)
    k = np.zeros((1, 16, 128), np.float16)
    v = np.zeros((1, 32, 128), np.float16)
    S = np.zeros((1, 32, 128, 128), np.float32)
    beta = np.zeros((1, 32), np.float32)
    g = np.zeros((1, 32), np.float32)
    k[0, 0, 0], q[0, 0, 1] = 1, 1
    k[0, 1, 0], q[0, 1, 0] = 1, 1
    for h in (0, 1):
        S[0, h, 0, 0], S[0, h, 1, 1] = 1, 2
        v[0, h, 0], v[0, h, 1] = 3, 4
    beta[0, 0], beta[0, 1] = 0.5, 1.0
    from qwowl35_b200 import ops
    Sd = torch.from_numpy(S.copy()).cuda()
    y = ops.deltanet_core(*(torch.from_numpy(a).cuda() for a in (q, k, v, beta, g)), Sd).cpu().numpy()
    Sn = Sd.cpu().numpy()
    scale = np.float32(1.0 / np.sqrt(128.0))
    ey = np.zeros((32, 128), np.float32)
    ey[0, 1] = np.float32(2) * scale
    ey[1, 0], ey[1, 1] = np.float32(3) * scale, np.float32(4) * scale
    eS = np.zeros((32, 128, 128), np.float32)
    eS[0, :2, :2] = [[2, 0], [2, 2]]
    eS[1, :2, :2] = [[3, 0], [4, 2]]
    np.testing.assert_array_equal(y[0], ey)
    np.testing.assert_array_equal(Sn[0], eS)
    # the oracle restatement gives the same numbers
    yr, Sr = O.deltanet_core(S[0], q[0].astype(np.float64), k[0].astype(np.float64), v[0], beta[0], g[0],
                             float(scale))
    np.testing.assert_allclose(yr, ey, rtol=0, atol=1e-7)
    np.testing.assert_array_equal(Sr, eS.astype(np.float64))
