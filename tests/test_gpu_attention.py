"""GQA decode attention over a non-contiguous 256-position chunk table vs the
oracle (qw35_attention.metal:29-414).  KV-chunk indexing must be exact;
outputs within max relative error 1e-3."""
import numpy as np
from parity import normerr, relerr
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
PLANE = 4 * 256 * 256  # f16 elements of one K (or V) plane in a chunk




def make_pool(rng, lens, layers=1):
    """Chunks hold `layers` x (K plane, V plane); order in the pool is shuffled."""
    nchunks = [(L + 255) // 256 for L in lens]
    total = sum(nchunks)
    per_chunk = layers * 2 * PLANE
    pool = torch.empty(total * per_chunk, dtype=torch.float16, device="cuda")
    pool.normal_()
    perm = rng.permutation(total)
    maxc = max(nchunks)
    table = np.zeros((len(lens), maxc), dtype=np.uint64)
    base = pool.data_ptr()
    i = 0
    for s, c in enumerate(nchunks):
        for j in range(c):
            table[s, j] = base + int(perm[i]) * per_chunk * 2
            i += 1
    return pool, perm, table, per_chunk


def gather_kv(pool, perm, table_rows, L, layer, per_chunk):
    """Host copy of K, V [L, 4, 256] of one sequence through its chunk list."""
    host = pool.view(-1, per_chunk).cpu().numpy()
    K = np.empty((L, 4, 256), np.float16)
    V = np.empty((L, 4, 256), np.float16)
    for t in range(L):
        c = table_rows[t // 256]
        blk = host[c]
        kpl = blk[layer * 2 * PLANE: layer * 2 * PLANE + PLANE].reshape(4, 256, 256)
        vpl = blk[layer * 2 * PLANE + PLANE: (layer + 1) * 2 * PLANE].reshape(4, 256, 256)
        K[t] = kpl[:, t % 256, :]
        V[t] = vpl[:, t % 256, :]
    return K, V


@pytest.mark.parametrize("lens,window,sink", [([1], 0, 0), ([300], 0, 0), ([1025, 7, 5000], 0, 0),
                                              ([4096, 2048], 512, 4), ([3000], 1024, 0), ([700], 2000, 10)])
def test_gqa_decode_matches_oracle(lens, window, sink):
    rng = np.random.default_rng(sum(lens))
    layers, layer = 2, 1
    pool, perm, table, per_chunk = make_pool(rng, lens, layers)
    n = len(lens)
    q = rng.normal(0, 1, (n, 16, 256)).astype(np.float32)
    gate = rng.normal(0, 1, (n, 16, 256)).astype(np.float32)
    from qwowl35_b200 import ops
    k_off = layer * 2 * PLANE * 2
    v_off = k_off + PLANE * 2
    out = ops.gqa_decode(torch.from_numpy(q).cuda(), torch.from_numpy(gate).cuda(),
                         torch.tensor(lens, dtype=torch.int32, device="cuda"), max(lens),
                         torch.from_numpy(table.view(np.int64)).cuda(), k_off, v_off, window, sink).cpu().numpy()
    # chunk index of table entries -> pool block id
    base = pool.data_ptr()
    blocks = ((table.astype(np.int64) - base) // (per_chunk * 2))
    for s, L in enumerate(lens):
        K, V = gather_kv(pool, perm, blocks[s], L, layer, per_chunk)
        ref = O.gqa_decode(q[s], gate[s], K, V, window, sink)
        assert relerr(out[s].reshape(16, 256), ref) < TOL


def test_preprocess_writes_kv_rows_and_rope():
    rng = np.random.default_rng(7)
    lens = [600, 257]
    pool, perm, table, per_chunk = make_pool(rng, lens, 1)
    n = len(lens)
    pos = np.array([599, 256], dtype=np.int32)
    qkv = rng.normal(0, 1, (n, 10240)).astype(np.float32)
    qn = np.abs(rng.normal(1, 0.1, 256)).astype(np.float32)
    kn = np.abs(rng.normal(1, 0.1, 256)).astype(np.float32)
    freq = O.rope_freqs(1.0e7)
    from qwowl35_b200 import ops
    q, gate = ops.attn_preprocess(torch.from_numpy(qkv).cuda(), torch.from_numpy(qn).cuda(),
                                  torch.from_numpy(kn).cuda(), torch.from_numpy(freq).cuda(),
                                  torch.from_numpy(pos).cuda(), torch.from_numpy(table.view(np.int64)).cuda(),
                                  0, PLANE * 2)
    torch.cuda.synchronize()
    base = pool.data_ptr()
    blocks = ((table.astype(np.int64) - base) // (per_chunk * 2))
    for s in range(n):
        rq, rg, rk, rv = O.attn_preprocess(qkv[s, :8192], qkv[s, 8192:9216], qkv[s, 9216:], qn, kn, int(pos[s]), freq)
        assert normerr(q[s].cpu().numpy(), rq) < 1e-5
        np.testing.assert_array_equal(gate[s].cpu().numpy(), rg.astype(np.float32))
        K, V = gather_kv(pool, perm, blocks[s], int(pos[s]) + 1, 0, per_chunk)
        np.testing.assert_array_equal(V[pos[s]], rv)                      # V: exact f16 RNE
        kd = np.abs(K[pos[s]].astype(np.float32).view(np.int32) if False else
                    K[pos[s]].view(np.int16).astype(np.int32) - rk.view(np.int16).astype(np.int32))
        assert kd.max() <= 1                                              # K: within 1 f16 ulp


def test_kv_chunk_address_math():
    table = np.array([7, 3, 9], dtype=np.uint64)
    assert O.kv_address(table, 0) == (7, 0)
    assert O.kv_address(table, 255) == (7, 255)
    assert O.kv_address(table, 256) == (3, 0)
    assert O.kv_address(table, 700) == (9, 188)


# ---- q8_0 KV cache (kv_cache_type 1, qw35_attention.metal:425-793) -----------------
ROWQ8 = 8 * 34
PLANEQ8 = 4 * 256 * ROWQ8  # bytes of one K (or V) q8_0 plane in a chunk


def make_pool_q8(rng, lens, layers=1):
    """Chunks of `layers` x (K plane, V plane) of valid q8_0 rows, shuffled in the pool."""
    nchunks = [(L + 255) // 256 for L in lens]
    total = sum(nchunks)
    per_chunk = layers * 2 * PLANEQ8
    host = rng.integers(-127, 128, size=(total * per_chunk // 34, 34)).astype(np.int8).view(np.uint8)
    host[:, 0:2] = (np.abs(rng.normal(0, 0.02, size=(host.shape[0], 1)))).astype(np.float16).view(np.uint8)
    pool = torch.from_numpy(host.reshape(-1).copy()).cuda()
    perm = rng.permutation(total)
    table = np.zeros((len(lens), max(nchunks)), dtype=np.uint64)
    base, i = pool.data_ptr(), 0
    for s, c in enumerate(nchunks):
        for j in range(c):
            table[s, j] = base + int(perm[i]) * per_chunk
            i += 1
    return pool, table, per_chunk


def gather_kv_q8(host, block_ids, L, layer, per_chunk):
    """(d [L,4,8] f16, qs [L,4,256] int8) for K and V of one sequence."""
    out = []
    for plane in (0, 1):
        d = np.empty((L, 4, 8), np.float16)
        qs = np.empty((L, 4, 256), np.int8)
        for t in range(L):
            c = int(block_ids[t // 256])
            off = c * per_chunk + (layer * 2 + plane) * PLANEQ8
            rows = host[off:off + PLANEQ8].reshape(4, 256, 8, 34)[:, t % 256]
            d[t] = rows[:, :, 0:2].copy().view(np.float16)[..., 0]
            qs[t] = rows[:, :, 2:].copy().view(np.int8).reshape(4, 256)
        out.append((d, qs))
    return out


@pytest.mark.parametrize("lens,window,sink", [([1], 0, 0), ([300], 0, 0), ([1025, 7, 3000], 0, 0),
                                              ([4096, 2048], 512, 4)])
def test_gqa_decode_q8_0_matches_oracle(lens, window, sink):
    rng = np.random.default_rng(sum(lens) + 1)
    layers, layer = 2, 1
    pool, table, per_chunk = make_pool_q8(rng, lens, layers)
    n = len(lens)
    q = rng.normal(0, 1, (n, 16, 256)).astype(np.float32)
    gate = rng.normal(0, 1, (n, 16, 256)).astype(np.float32)
    from qwowl35_b200 import ops
    k_off = layer * 2 * PLANEQ8
    out = ops.gqa_decode(torch.from_numpy(q).cuda(), torch.from_numpy(gate).cuda(),
                         torch.tensor(lens, dtype=torch.int32, device="cuda"), max(lens),
                         torch.from_numpy(table.view(np.int64)).cuda(), k_off, k_off + PLANEQ8, window, sink,
                         kv_q8=True).cpu().numpy()
    host = pool.cpu().numpy()
    blocks = (table.astype(np.int64) - pool.data_ptr()) // per_chunk
    for s, L in enumerate(lens):
        Kq, Vq = gather_kv_q8(host, blocks[s], L, layer, per_chunk)
        ref = O.gqa_decode_q8_0(q[s], gate[s], Kq, Vq, window, sink)
        assert relerr(out[s].reshape(16, 256), ref) < TOL


def test_preprocess_q8_0_quantises_like_the_reference():
    rng = np.random.default_rng(8)
    lens = [600, 257]
    pool, table, per_chunk = make_pool_q8(rng, lens, 1)
    n = len(lens)
    pos = np.array([599, 256], dtype=np.int32)
    qkv = rng.normal(0, 1, (n, 10240)).astype(np.float32)
    qkv[0, 9216:9216 + 32] = 0.0                                       # an all-zero V block
    qn = np.abs(rng.normal(1, 0.1, 256)).astype(np.float32)
    kn = np.abs(rng.normal(1, 0.1, 256)).astype(np.float32)
    freq = O.rope_freqs(1.0e7)
    from qwowl35_b200 import ops
    q, gate = ops.attn_preprocess(torch.from_numpy(qkv).cuda(), torch.from_numpy(qn).cuda(),
                                  torch.from_numpy(kn).cuda(), torch.from_numpy(freq).cuda(),
                                  torch.from_numpy(pos).cuda(), torch.from_numpy(table.view(np.int64)).cuda(),
                                  0, PLANEQ8, kv_q8=True)
    torch.cuda.synchronize()
    host = pool.cpu().numpy()
    blocks = (table.astype(np.int64) - pool.data_ptr()) // per_chunk
    for s in range(n):
        rq, rg, (rkd, rkq), (rvd, rvq) = O.attn_preprocess_q8_0(qkv[s, :8192], qkv[s, 8192:9216], qkv[s, 9216:],
                                                                qn, kn, int(pos[s]), freq)
        assert normerr(q[s].cpu().numpy(), rq) < 1e-5
        (kd, kq), (vd, vq) = gather_kv_q8(host, blocks[s], int(pos[s]) + 1, 0, per_chunk)
        t = int(pos[s])
        np.testing.assert_array_equal(vq[t], rvq)                       # V: the same fp32 input, exact
        np.testing.assert_array_equal(vd[t].view(np.uint16), rvd.view(np.uint16))
        assert np.abs(kq[t].astype(np.int32) - rkq.astype(np.int32)).max() <= 1   # K: fp32 vs f64 norm/RoPE
        assert np.abs(kd[t].view(np.int16).astype(np.int32) - rkd.view(np.int16).astype(np.int32)).max() <= 1
