"""End-to-end decode through the drop-in C ABI (qw35_metal_* and the batched
extensions) on a small synthetic model, against the fp64 oracle model."""
import numpy as np
from parity import modelerr as relerr  # decode-step logits (see parity.py)
from parity import relerr as elem_relerr
import pytest

from oracle.model import OracleModel
from qwowl35_b200 import synth
from qwowl35_b200.runtime import LogitsMode, Runtime
from qwowl35_b200._lib import Qw35Error

pytestmark = pytest.mark.gpu
TOL = 1e-3




@pytest.fixture(scope="module")
def small():
    cfg = synth.ModelConfig(layers=4, ffn=1024, vocab=4096)
    return synth.build(cfg, seed=3)


TOKENS = [17, 4000, 5, 123, 77, 2048, 9]


def test_full_logits_match_oracle(small):
    rt = Runtime(small, ctx=512)
    orc = OracleModel(small)
    for pos, tok in enumerate(TOKENS):
        rt.eval_token(tok, pos, LogitsMode.FULL)
        got = rt.copy_logits()
        ref = orc.step(tok, pos)
        e = relerr(got, ref)
        assert e < TOL, (pos, e)
    rt.close()


def test_argmax_mode_equals_full_logits_argmax(small):
    rt = Runtime(small, ctx=512)
    full = []
    for pos, tok in enumerate(TOKENS):
        rt.eval_token(tok, pos, LogitsMode.FULL)
        full.append(rt.copy_logits())
    rt.reset()
    for pos, tok in enumerate(TOKENS):
        rt.eval_token(tok, pos, LogitsMode.ARGMAX)
        t, v = rt.argmax()
        m = full[pos].max()
        assert t == int(np.flatnonzero(full[pos] == m)[0]) and v == m
    rt.close()


@pytest.mark.parametrize("mode", ["0", "1", "2"])
def test_prefill_chunk_equals_token_steps(small, monkeypatch, mode):
    # QW35_PREFILL=0 runs the chunk as decode steps (bit-identical); 1 and 2 run
    # it as one batched pass, whose tensor-core matvecs use the reference's
    # tiled-path weights and sum in another order (tolerance)
    monkeypatch.setenv("QW35_PREFILL", mode)
    rt = Runtime(small, ctx=512, prefill_chunk=8)
    rt.eval_prefill_chunk(TOKENS, 0, LogitsMode.FULL)
    a = rt.copy_logits()
    rt.reset()
    for pos, tok in enumerate(TOKENS):
        rt.eval_token(tok, pos, LogitsMode.FULL if pos == len(TOKENS) - 1 else LogitsMode.NONE)
    b = rt.copy_logits()
    if mode == "0":
        np.testing.assert_array_equal(a, b)
    else:
        assert relerr(a, b.astype(np.float64)) < TOL
    rt.close()


def _single_logits(small, seqs):
    single = []
    rt1 = Runtime(small, ctx=512)
    for s in seqs:
        rt1.reset()
        for pos, tok in enumerate(s):
            rt1.eval_token(tok, pos, LogitsMode.FULL)
        single.append(rt1.copy_logits())
    rt1.close()
    return single


def _batch_logits(small, seqs):
    rt = Runtime(small, ctx=512, max_seqs=4)
    ids = [0] + [rt.seq_alloc() for _ in range(len(seqs) - 1)]
    for pos in range(len(seqs[0])):
        rt.eval_batch(ids, [s[pos] for s in seqs], [pos] * len(seqs), LogitsMode.FULL)
    out = rt.copy_logits_batch(len(seqs))
    rt.close()
    return out


def test_batch_of_two_equals_single_sequence_bitwise(small):
    # batches of 1-2 run the CUDA-core matvecs, whose per-row arithmetic does not
    # depend on the batch
    seqs = [[3, 9, 27, 81], [100, 200, 300, 400]]
    single, out = _single_logits(small, seqs), _batch_logits(small, seqs)
    for i in range(2):
        np.testing.assert_array_equal(out[i], single[i])


def test_batch_of_three_matches_single_sequences(small):
    # from 3 rows on, the matvecs run on the tensor cores (f16 hi + lo
    # activations): the same results within the 1e-3 bar, not bit for bit
    seqs = [[3, 9, 27, 81], [100, 200, 300, 400], [4095, 0, 1, 2]]
    single, out = _single_logits(small, seqs), _batch_logits(small, seqs)
    for i in range(3):
        assert relerr(out[i], single[i].astype(np.float64)) < TOL


def test_ragged_positions_in_one_batch(small):
    rt = Runtime(small, ctx=2048, max_seqs=2)
    b = rt.seq_alloc()
    orc0, orc1 = OracleModel(small), OracleModel(small)
    # sequence 0 runs ahead alone past a chunk boundary, then both step together
    for pos in range(300):
        rt.eval_token(pos % 4096, pos, LogitsMode.NONE)
        orc0.step(pos % 4096, pos)
    rt.eval_batch([0, b], [11, 12], [300, 0], LogitsMode.FULL)
    got = rt.copy_logits_batch(2)
    assert relerr(got[0], orc0.step(11, 300)) < TOL
    assert relerr(got[1], orc1.step(12, 0)) < TOL
    rt.close()


def test_state_export_import_replays_bitwise(small):
    rt = Runtime(small, ctx=512)
    for pos, tok in enumerate(TOKENS[:3]):
        rt.eval_token(tok, pos, LogitsMode.NONE)
    st = rt.state_export()
    assert len(st) == rt.state_size() == 3 * (8192 * 3 + 32 * 128 * 128) * 4
    rt.eval_token(TOKENS[3], 3, LogitsMode.NONE)
    rt.eval_token(TOKENS[4], 4, LogitsMode.FULL)
    a = rt.copy_logits()
    rt.state_import(st)
    rt.eval_token(TOKENS[3], 3, LogitsMode.NONE)
    rt.eval_token(TOKENS[4], 4, LogitsMode.FULL)
    np.testing.assert_array_equal(a, rt.copy_logits())
    with pytest.raises(Qw35Error, match="size mismatch"):
        rt.state_import(st[:-4])
    rt.close()


def test_host_side_guards(small):
    rt = Runtime(small, ctx=64)
    with pytest.raises(Qw35Error, match="exceeds allocated context"):
        rt.eval_token(1, 64)
    with pytest.raises(Qw35Error, match="outside the Qw35 vocabulary"):
        rt.eval_token(4096, 0)
    rt.eval_token(1, 0, LogitsMode.NONE)
    with pytest.raises(Qw35Error, match="argmax"):
        rt.argmax()
    rt.set_ctx_size(32)          # lower: no-op success
    rt.set_ctx_size(128)
    rt.eval_token(2, 100, LogitsMode.ARGMAX)
    with pytest.raises(Qw35Error, match="exceeds the maximum"):
        rt.set_ctx_size(1 << 20)
    with pytest.raises(Qw35Error):
        rt.seq_alloc()           # only one slot
    rt.close()
    with pytest.raises(Qw35Error, match="invalid kv_cache_type"):
        Runtime(small, ctx=64, kv_cache_type=2)


def test_window_and_sink_match_oracle(small):
    rt = Runtime(small, ctx=1024, window=64, sink=4)
    orc = OracleModel(small, window=64, sink=4)
    for pos in range(80):
        mode = LogitsMode.FULL if pos == 79 else LogitsMode.NONE
        rt.eval_token((pos * 7) % 4096, pos, mode)
        ref = orc.step((pos * 7) % 4096, pos)
    assert relerr(rt.copy_logits(), ref) < TOL
    rt.close()


def test_seq_fork_continues_identically(small):
    # two rows run the CUDA-core matvecs: a fork continues bit for bit
    rt = Runtime(small, ctx=1024, max_seqs=3)
    b, c = rt.seq_alloc(), rt.seq_alloc()
    for pos in range(270):  # crosses a 256-position chunk boundary
        rt.eval_token((pos * 13) % 4096, pos, LogitsMode.NONE)
    rt.seq_fork(0, b)
    rt.eval_batch([0, b], [5, 5], [270, 270], LogitsMode.FULL)
    out = rt.copy_logits_batch(2)
    np.testing.assert_array_equal(out[0], out[1])
    # three rows run on the tensor cores, whose split tiles are added in L2 in
    # an order that may differ per batch column: equal within the 1e-3 bar
    rt.seq_fork(0, c)
    rt.seq_fork(0, b)
    rt.eval_batch([0, b, c], [7, 7, 7], [271, 271, 271], LogitsMode.FULL)
    out = rt.copy_logits_batch(3)
    assert relerr(out[1], out[0].astype(np.float64)) < TOL
    assert relerr(out[2], out[0].astype(np.float64)) < TOL
    rt.close()


# ---- mixed weight types, as in the reference's source GGUFs --------------------
@pytest.fixture(scope="module")
def mixed():
    """Q4_K projections with a Q6_K attn_v, Q5_K attn_gate / ssm_out and Q8_0
    ssm_beta / ssm_alpha (so both projection groups split into runs of one
    type), a GF4 ffn_gate beside a Q4_K ffn_up, Q6_K ffn_down and head, Q4_K
    embedding."""
    cfg = synth.ModelConfig(layers=4, ffn=1024, vocab=4096, proj_type=synth.Q4_K, head_type=synth.Q6_K,
                            embd_type=synth.Q4_K,
                            overrides={"attn_v.weight": synth.Q6_K, "attn_gate.weight": synth.Q5_K,
                                       "ssm_out.weight": synth.Q5_K, "ssm_beta.weight": synth.Q8_0,
                                       "ssm_alpha.weight": synth.Q8_0, "ffn_up.weight": synth.Q4_K,
                                       "ffn_down.weight": synth.Q6_K})
    return synth.build(cfg, seed=5)


def test_mixed_type_model_matches_oracle(mixed):
    rt = Runtime(mixed, ctx=512)
    orc = OracleModel(mixed)
    for pos, tok in enumerate(TOKENS[:5]):
        rt.eval_token(tok, pos, LogitsMode.FULL)
        e = relerr(rt.copy_logits(), orc.step(tok, pos))
        assert e < TOL, (pos, e)
    rt.eval_token(TOKENS[5], 5, LogitsMode.ARGMAX)
    t, _ = rt.argmax()
    ref = orc.step(TOKENS[5], 5)
    top2 = np.sort(ref)[-2:]
    if top2[1] - top2[0] > 1e-3 * np.abs(ref).max():
        assert t == int(np.argmax(ref))
    rt.close()


def test_mixed_type_model_batch_of_three_matches_oracle(mixed):
    seqs = [[3, 9, 27, 81], [100, 200, 300, 400], [4095, 0, 1, 2]]
    out = None
    rt = Runtime(mixed, ctx=512, max_seqs=4)
    ids = [0] + [rt.seq_alloc() for _ in range(2)]
    orcs = [OracleModel(mixed, tiled=True) for _ in seqs]
    for pos in range(4):
        rt.eval_batch(ids, [s[pos] for s in seqs], [pos] * 3, LogitsMode.FULL)
        out = rt.copy_logits_batch(3)
        for i, s in enumerate(seqs):
            assert relerr(out[i], orcs[i].step(s[pos], pos)) < TOL, (pos, i)
    rt.close()


def test_q8_0_kv_cache_matches_oracle(small):
    from qwowl35_b200.runtime import KvCacheType
    rt = Runtime(small, ctx=512, kv_cache_type=KvCacheType.Q8_0)
    orc = OracleModel(small, kv_q8=True)
    for pos, tok in enumerate(TOKENS):
        rt.eval_token(tok, pos, LogitsMode.FULL)
        e = relerr(rt.copy_logits(), orc.step(tok, pos))
        assert e < TOL, (pos, e)
    rt.close()


@pytest.mark.parametrize("mode", ["1", "2"])
def test_batched_prefill_matches_oracle(small, monkeypatch, mode):
    monkeypatch.setenv("QW35_PREFILL", mode)
    # 7 tokens in one pass: batch-7 matvecs (tensor-core path, the reference's
    # tiled-path weight semantics), 7 attention rows over one sequence, the
    # DeltaNet recurrence row by row (QW35_PREFILL=2: one launch per layer with
    # the state on chip); logits of the last token
    rt = Runtime(small, ctx=512, prefill_chunk=8)
    rt.eval_prefill_chunk(TOKENS, 0, LogitsMode.FULL)
    got = rt.copy_logits()
    orc = OracleModel(small, tiled=True)
    for pos, tok in enumerate(TOKENS):
        ref = orc.step(tok, pos)
    assert relerr(got, ref) < TOL
    # decoding continues from the prefilled state and KV
    rt.eval_token(11, len(TOKENS), LogitsMode.FULL)
    single = Runtime(small, ctx=512)
    for pos, tok in enumerate(TOKENS + [11]):
        single.eval_token(tok, pos, LogitsMode.FULL)
    assert relerr(rt.copy_logits(), single.copy_logits().astype(np.float64)) < TOL
    rt.close()
    single.close()


@pytest.mark.parametrize("T", [1, 7, 64])
def test_deltanet_run_kernel_equals_step_launches(small, monkeypatch, T):
    """The batched prefill's DeltaNet recurrence as one run launch per layer
    (the default) against the same pass with one step launch per token
    (QW35_PREFILL=1): conv windows, SSM state and the last token's logits agree
    (the rest of the pass is the same code; its split-tile sums may add in
    another order, hence a tolerance rather than bit equality)."""
    toks = [(7 * i + 3) % small.cfg.vocab for i in range(T)]
    out = {}
    for mode in ("1", "2"):
        monkeypatch.setenv("QW35_PREFILL", mode)
        rt = Runtime(small, ctx=512, prefill_chunk=64)
        rt.eval_prefill_chunk(toks, 0, LogitsMode.FULL)
        out[mode] = (np.frombuffer(rt.state_export(), dtype=np.float32).astype(np.float64), rt.copy_logits())
        rt.close()
    (s1, l1), (s2, l2) = out["1"], out["2"]
    assert elem_relerr(s2, s1) < TOL
    assert relerr(l2, l1.astype(np.float64)) < TOL


def test_runtimes_own_their_tensor_core_scratch(small):
    """Each runtime keeps the scratch its captured graphs point at: creating a
    larger runtime over the same model leaves the first one's address alone,
    and the first runtime then still decodes like the oracle."""
    from qwowl35_b200._lib import lib
    import ctypes as C
    L = lib()
    a = Runtime(small, ctx=512, max_seqs=4)
    nb = C.c_uint64(0)
    addr_a = L.qw35_cuda_runtime_scratch(a.handle, C.byref(nb))
    assert addr_a != 0 and nb.value > 0
    ids = [a.seq_alloc() for _ in range(3)]
    seqs = [TOKENS[:4], TOKENS[1:5], TOKENS[2:6]]
    orcs = [OracleModel(small, tiled=True) for _ in seqs]
    a.eval_batch(ids, [s[0] for s in seqs], [0] * 3, LogitsMode.FULL)  # graphs captured on A's scratch
    a.sync()
    b = Runtime(small, ctx=512, max_seqs=64)
    addr_b = L.qw35_cuda_runtime_scratch(b.handle, None)
    assert L.qw35_cuda_runtime_scratch(a.handle, None) == addr_a
    assert addr_b not in (0, addr_a)
    for i, s in enumerate(seqs):
        assert relerr(a.copy_logits_batch(3)[i], orcs[i].step(s[0], 0)) < TOL
    for pos in range(1, 4):
        a.eval_batch(ids, [s[pos] for s in seqs], [pos] * 3, LogitsMode.FULL)
        out = a.copy_logits_batch(3)
        for i, s in enumerate(seqs):
            assert relerr(out[i], orcs[i].step(s[pos], pos)) < TOL, (pos, i)
    b.close()
    a.close()


def test_runtimes_over_one_model_keep_their_own_window(small):
    """Weights are shared per mapping; the attention window and sink are each
    runtime's own (a runtime created first without a window must not impose
    it on a later one)."""
    first = Runtime(small, ctx=1024)  # window 0, stays alive
    rt = Runtime(small, ctx=1024, window=16, sink=2)
    orc = OracleModel(small, window=16, sink=2)
    for pos in range(24):
        rt.eval_token((pos * 5) % 4096, pos, LogitsMode.FULL if pos == 23 else LogitsMode.NONE)
        ref = orc.step((pos * 5) % 4096, pos)
    assert relerr(rt.copy_logits(), ref) < TOL
    rt.close()
    first.close()
