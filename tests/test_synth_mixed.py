"""Synthetic models with per-tensor type overrides (the mixed-type layout of
the reference's source GGUFs), on the CPU: the tensor plan, the generated
byte sizes and the fp64 oracle model decoding them."""
import numpy as np

from oracle import quants as Q
from oracle.model import OracleModel
from qwowl35_b200 import synth


def _cfg(**kw):
    return synth.ModelConfig(layers=4, ffn=1024, vocab=1024, proj_type=synth.Q4_K, head_type=synth.Q6_K,
                             embd_type=synth.Q4_K,
                             overrides={"attn_v.weight": synth.Q6_K, "attn_gate.weight": synth.Q5_K,
                                        "ssm_beta.weight": synth.Q8_0, "ssm_alpha.weight": synth.Q8_0,
                                        "ffn_up.weight": synth.Q4_K, "ffn_down.weight": synth.Q6_K}, **kw)


def test_overrides_apply_by_name_suffix():
    plan = {n: t for n, t, _ in synth.tensor_plan(_cfg())}
    assert plan["blk.3.attn_v.weight"] == synth.Q6_K and plan["blk.3.attn_q.weight"] == synth.Q4_K
    assert plan["blk.0.attn_gate.weight"] == synth.Q5_K and plan["blk.0.ssm_alpha.weight"] == synth.Q8_0
    assert plan["blk.1.ffn_gate.weight"] == synth.GF4 and plan["blk.1.ffn_up.weight"] == synth.Q4_K
    assert plan["output.weight"] == synth.Q6_K and plan["blk.2.attn_norm.weight"] == synth.F32
    assert {t for n, t, _ in synth.tensor_plan(synth.ModelConfig(layers=4))} == {synth.F32, synth.GF4, synth.Q8_0}


def test_mixed_model_bytes_and_oracle_decode():
    m = synth.build(_cfg(), seed=2)
    for name, (t, k, r, off, n) in m.offsets.items():
        if t != synth.F32:
            assert n == Q.row_bytes(t, k) * r, name
    orc = OracleModel(m)
    y0 = orc.step(5, 0)
    y1 = orc.step(700, 1)
    assert y0.shape == (1024,) and np.isfinite(y0).all() and np.isfinite(y1).all()
    assert not np.array_equal(y0, y1)
    # the tiled semantics differ only by half rounding of the K-quant / GF4 weights
    orc_t = OracleModel(m, tiled=True)
    yt = orc_t.step(5, 0)
    assert np.max(np.abs(yt - y0)) / np.max(np.abs(y0)) < 1e-2
