"""Parity at the headline shapes.

* BASELINE config 5 (the model ``bench.py`` times): 32 layers (24 Gated
  DeltaNet + 8 gated attention), GF4 FFN 12288, Q8_0 projections and head,
  vocab 248320, random-init weights.  Decoded through the drop-in C ABI at
  batch 1 (``qw35_metal_runtime_eval_token``) and batch 32
  (``qw35_cuda_runtime_eval_batch``), 4 tokens each after nothing, against
  the fp64 oracle model.  Every weight value the oracle uses comes from the
  oracle's own dequantisation (``oracle.quants``, numpy); the 9 G fp64
  multiply-adds per token run as torch float64 products on the GPU (a BLAS,
  not the code under test).
* GQA decode over 32 ragged sequences whose lengths are
  log-uniform in 512..131072 (the seeded list below), K/V in shuffled
  256-position chunks, against the oracle per sequence.

Tolerance: logits ``parity.modelerr`` < 1e-3 (norm-wise, and per element above
5% of the largest logit); GQA ``parity.relerr`` < 1e-3 (per element above
1e-3 of the largest output); argmax ids bit-exact against the argmax of the returned logits
and equal to the oracle's wherever its top-2 gap exceeds the tolerance.
"""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from oracle import ops as O
from oracle import quants as Q
from oracle.model import OracleModel
from parity import MODEL_FLOOR, elemerr, modelerr, normerr, relerr
from qwowl35_b200 import ops, synth
from qwowl35_b200.runtime import LogitsMode, Runtime

pytestmark = pytest.mark.gpu
TOL = 1e-3


class GpuBlasOracle(OracleModel):
    """The oracle model with its dequantised weights held on the GPU (float32,
    exact) and each product W @ x computed in float64 by torch."""

    def __init__(self, synth_model, store, **kw):
        super().__init__(synth_model, **kw)
        self.store = store

    def mv(self, name, x):
        w = self.store[name]
        return (w.double() @ torch.from_numpy(np.asarray(x, np.float64)).cuda()).cpu().numpy()


def dequant_store(m, tiled: bool):
    """Every matrix of the model dequantised by the oracle (threads over tensors)."""
    names = [n for n, (t, k, r, off, nb) in m.offsets.items() if t != Q.F32_TYPE and n != "token_embd.weight"]

    def one(name):
        t, k, r, off, nb = m.offsets[name]
        return name, Q.dequant(t, m.buf[off:off + nb], r, k, tiled=tiled)

    store = {}
    with ThreadPoolExecutor(16) as ex:
        for name, w in ex.map(one, names):
            store[name] = torch.from_numpy(w).cuda()
    return store


@pytest.fixture(scope="module")
def full():
    m = synth.build(synth.ModelConfig(), seed=5, device="cuda")
    yield m
    torch.cuda.empty_cache()


def _check_logits(got, ref, where):
    e = modelerr(got, ref)
    assert e < TOL, (where, "norm-wise", normerr(got, ref), "per element", elemerr(got, ref, MODEL_FLOOR))
    top = np.argsort(ref)[-2:]
    if ref[top[1]] - ref[top[0]] > TOL * np.max(np.abs(ref)):
        assert int(np.argmax(got)) == int(top[1]), where


def test_config5_batch1_matches_oracle(full):
    store = dequant_store(full, tiled=False)
    orc = GpuBlasOracle(full, store)
    rt = Runtime(full, ctx=64)
    am = Runtime(full, ctx=64)  # the same tokens through the fused argmax head
    for pos, tok in enumerate([11, 248000, 7, 90001]):
        rt.eval_token(tok, pos, LogitsMode.FULL)
        am.eval_token(tok, pos, LogitsMode.ARGMAX)
        got = rt.copy_logits()
        _check_logits(got, orc.step(tok, pos), ("b1", pos))
        t, v = am.argmax()
        m = got.max()
        assert t == int(np.flatnonzero(got == m)[0]) and v == m, pos  # batch 1 is deterministic
    rt.close()
    am.close()
    del store
    torch.cuda.empty_cache()


def test_config5_batch32_matches_oracle(full):
    # 3 or more rows run the tensor-core dequant-GEMM
    store = dequant_store(full, tiled=True)
    rng = np.random.default_rng(32)
    seqs = rng.integers(0, full.cfg.vocab, size=(32, 4))
    rt = Runtime(full, ctx=64, max_seqs=32)
    am = Runtime(full, ctx=64, max_seqs=32)
    ids = [0] + [rt.seq_alloc() for _ in range(31)]
    ids_am = [0] + [am.seq_alloc() for _ in range(31)]
    orcs = [GpuBlasOracle(full, store, tiled=True) for _ in range(32)]
    for pos in range(4):
        toks = [int(s[pos]) for s in seqs]
        rt.eval_batch(ids, toks, [pos] * 32, LogitsMode.FULL)
        am.eval_batch(ids_am, toks, [pos] * 32, LogitsMode.ARGMAX)
        out = rt.copy_logits_batch(32)
        tok_am, _ = am.argmax_batch(32)
        for i in range(32):
            _check_logits(out[i], orcs[i].step(toks[i], pos), ("b32", pos, i))
            # the tensor-core path's split tiles add in an order L2 chooses, so two
            # runs agree to ~1e-6: ids must match where the top-2 gap is wider
            top = np.sort(out[i])[-2:]
            if top[1] - top[0] > 1e-5 * np.max(np.abs(out[i])):
                assert int(tok_am[i]) == int(np.argmax(out[i])), (pos, i)
    rt.close()
    am.close()
    del store
    torch.cuda.empty_cache()


# ---- ragged GQA decode to 131072 positions --------------------------
# np.random.default_rng(4) log-uniform in [512, 131072], first two pinned to the ends
CONFIG4_LENS = [131072, 512, 114894, 801, 14856, 4129, 43695, 1347, 64324, 10452, 76211, 7217, 5571, 40667,
                120045, 3977, 110329, 88427, 1371, 14980, 25512, 95448, 20527, 1072, 8095, 7907, 8202, 104175,
                3564, 1770, 9259, 17921]
PLANE = 4 * 256 * 256  # f16 elements of one K (or V) plane of a chunk


def test_config4_ragged_gqa_matches_oracle():
    lens = CONFIG4_LENS
    rng = np.random.default_rng(44)
    nch = [(L + 255) // 256 for L in lens]
    total = sum(nch)
    pool = torch.empty(total * 2 * PLANE, dtype=torch.float16, device="cuda")
    pool.normal_(generator=torch.Generator(device="cuda").manual_seed(4))
    perm = rng.permutation(total)
    table = np.zeros((len(lens), max(nch)), dtype=np.int64)
    blocks = np.zeros_like(table)
    i = 0
    for s, c in enumerate(nch):
        for j in range(c):
            blocks[s, j] = perm[i]
            table[s, j] = pool.data_ptr() + int(perm[i]) * 2 * PLANE * 2
            i += 1
    n = len(lens)
    q = rng.normal(0, 1, (n, 16, 256)).astype(np.float32)
    gate = rng.normal(0, 1, (n, 16, 256)).astype(np.float32)
    out = ops.gqa_decode(torch.from_numpy(q).cuda(), torch.from_numpy(gate).cuda(),
                         torch.tensor(lens, dtype=torch.int32, device="cuda"), max(lens),
                         torch.from_numpy(table).cuda(), 0, PLANE * 2).cpu().numpy()
    chunks = pool.view(total, 2, 4, 256, 256)  # [chunk][K|V][kv head][pos][dim]
    for s, L in enumerate(lens):
        idx = torch.from_numpy(blocks[s, :nch[s]]).cuda()
        kv = chunks.index_select(0, idx)                      # [c, 2, 4, 256, 256]
        kv = kv.permute(1, 0, 3, 2, 4).reshape(2, -1, 4, 256)[:, :L].cpu().numpy()
        ref = O.gqa_decode(q[s], gate[s], kv[0], kv[1])
        assert relerr(out[s].reshape(16, 256), ref) < TOL, (s, L)
    del pool
    torch.cuda.empty_cache()
