"""The allocation-free attention entry point against the workspace one.

qw35_cuda_gqa_decode_noalloc exists for callers that cannot allocate device
memory where they decode (their memory belongs to another allocator, or a
cudaMalloc and its implicit synchronisation is not allowed at that point):
it keeps its split partials in a static device array inside the library.
This file is collected last so that a failure here never hides the others.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from qwowl35_b200._lib import lib

pytestmark = pytest.mark.gpu
TOL = 1e-3
PLANE = 4 * 256 * 256  # f16 elements of one K (or V) plane of a chunk


def _kv(lens, seed):
    """A pool of shuffled 256-position chunks (one layer) and its chunk table."""
    rng = np.random.default_rng(seed)
    nch = [(L + 255) // 256 for L in lens]
    pool = torch.randn(sum(nch) * 2 * PLANE, device="cuda").to(torch.float16)
    perm = rng.permutation(sum(nch))
    table = np.zeros((len(lens), max(nch)), dtype=np.int64)
    i = 0
    for s, c in enumerate(nch):
        for j in range(c):
            table[s, j] = pool.data_ptr() + int(perm[i]) * 2 * PLANE * 2
            i += 1
    return pool, torch.from_numpy(table).cuda()


def _call_both(q, gate, lens_d, max_len, table, window, sink):
    L = lib()
    n = q.shape[0]
    err = C.create_string_buffer(512)
    ws = torch.empty(int(L.qw35_cuda_gqa_workspace_bytes(n, max_len)), dtype=torch.uint8, device="cuda")
    ref = torch.empty(n, 4096, device="cuda")
    got = torch.full((n, 4096), float("nan"), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.qw35_cuda_gqa_decode(n, q.data_ptr(), gate.data_ptr(), lens_d.data_ptr(), max_len, table.data_ptr(),
                                  table.shape[1], 0, PLANE * 2, window, sink, ref.data_ptr(), ws.data_ptr(),
                                  ws.numel(), st, err, 512) == 1, err.value
    assert L.qw35_cuda_gqa_decode_noalloc(n, q.data_ptr(), gate.data_ptr(), lens_d.data_ptr(), max_len,
                                          table.data_ptr(), table.shape[1], 0, PLANE * 2, window, sink,
                                          got.data_ptr(), st, err, 512) == 1, err.value
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy()


@pytest.mark.parametrize("lens,window,sink", [([5000, 300, 1], 0, 0), ([4096, 2048], 512, 4)])
def test_noalloc_matches_workspace_entry_on_two_calls(lens, window, sink):
    pool, table = _kv(lens, sum(lens))
    lens_d = torch.tensor(lens, dtype=torch.int32, device="cuda")
    for call in range(2):  # the second call must not see the first call's partials
        q = torch.randn(len(lens), 16, 256, device="cuda") * (1.0 + call)
        gate = torch.randn(len(lens), 16, 256, device="cuda")
        got, ref = _call_both(q, gate, lens_d, max(lens), table, window, sink)
        assert np.isfinite(got).all()
        rel = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
        assert rel < TOL, (call, rel)
    assert lib().qw35_cuda_device_error() == 0
    del pool


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    L = lib()
    limit = int(L.qw35_cuda_gqa_noalloc_max_bytes())
    assert limit == 16 << 20
    n, max_len = 64, 262144  # 64 sequences x 256 splits of partials: far beyond 16 MiB
    assert L.qw35_cuda_gqa_workspace_bytes(n, max_len) > limit
    err = C.create_string_buffer(512)
    dummy = torch.zeros(16, device="cuda")
    ok = L.qw35_cuda_gqa_decode_noalloc(n, dummy.data_ptr(), None, dummy.data_ptr(), max_len, dummy.data_ptr(),
                                        1024, 0, 0, 0, 0, dummy.data_ptr(), None, err, 512)
    assert ok == 0 and b"static scratch" in err.value


def test_noalloc_call_takes_no_device_memory():
    """After one warm-up call, a further call leaves the device's free bytes unchanged."""
    L = lib()
    lens = [3000, 700]
    pool, table = _kv(lens, 7)
    lens_d = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(len(lens), 16, 256, device="cuda")
    gate = torch.randn(len(lens), 16, 256, device="cuda")
    out = torch.empty(len(lens), 4096, device="cuda")
    err = C.create_string_buffer(512)
    st = torch.cuda.current_stream().cuda_stream

    def call():
        assert L.qw35_cuda_gqa_decode_noalloc(len(lens), q.data_ptr(), gate.data_ptr(), lens_d.data_ptr(),
                                              max(lens), table.data_ptr(), table.shape[1], 0, PLANE * 2, 0, 0,
                                              out.data_ptr(), st, err, 512) == 1, err.value
        torch.cuda.synchronize()

    call()
    free0, _ = torch.cuda.mem_get_info()
    call()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert np.isfinite(out.cpu().numpy()).all()
    del pool
