"""Two devices in one process (skipped with fewer than two GPUs).

The kernels that need more than 48 KB of dynamic shared memory opt in per
device and per kernel; a launch on a second device must not rely on the first
device's opt-in.  The same matvecs (batch 1: CUDA cores; batch 32: tensor
cores) and the allocation-free attention entry point run on devices 0 and 1
with the same inputs and must give the same results.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import quants as Q
from qwowl35_b200 import ops
from qwowl35_b200._lib import lib

pytestmark = pytest.mark.gpu
TOL = 1e-3
PLANE = 4 * 256 * 256


def _two_devices():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


@pytest.mark.parametrize("t", [Q.GF4_TYPE, Q.Q8_0_TYPE])
@pytest.mark.parametrize("b", [1, 32])
def test_matvec_on_two_devices(t, b):
    _two_devices()
    rows, k = 2048, 4096
    raw = Q.gen_weight(np.random.default_rng(5), t, rows, k)
    x = np.random.default_rng(6).standard_normal((b, k)).astype(np.float32)
    out = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            d = f"cuda:{dev}"
            w = ops.upload(t, raw, rows, k, device=d)
            y = ops.matvec(t, w, torch.from_numpy(x).to(d), rows, k)
            torch.cuda.synchronize(dev)
            out.append(y.cpu().numpy())
    rel = np.max(np.abs(out[0] - out[1])) / np.max(np.abs(out[0]))
    assert rel < TOL


def test_noalloc_attention_on_two_devices():
    _two_devices()
    L = lib()
    lens = [1500, 300]
    nch = [(n + 255) // 256 for n in lens]
    g = torch.Generator().manual_seed(9)
    pool_h = torch.randn(sum(nch) * 2 * PLANE, generator=g).to(torch.float16)
    q_h = torch.randn(len(lens), 16, 256, generator=g)
    gate_h = torch.randn(len(lens), 16, 256, generator=g)
    err = C.create_string_buffer(512)
    out = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            d = f"cuda:{dev}"
            pool = pool_h.to(d)
            table = torch.tensor([[pool.data_ptr() + (sum(nch[:s]) + j) * 2 * PLANE * 2 for j in range(max(nch))]
                                  for s in range(len(lens))], dtype=torch.int64, device=d)
            lens_d = torch.tensor(lens, dtype=torch.int32, device=d)
            q, gate = q_h.to(d), gate_h.to(d)
            o = torch.empty(len(lens), 4096, device=d)
            st = torch.cuda.current_stream(dev).cuda_stream
            assert L.qw35_cuda_gqa_decode_noalloc(len(lens), q.data_ptr(), gate.data_ptr(), lens_d.data_ptr(),
                                                  max(lens), table.data_ptr(), table.shape[1], 0, PLANE * 2, 0, 0,
                                                  o.data_ptr(), st, err, 512) == 1, err.value
            torch.cuda.synchronize(dev)
            out.append(o.cpu().numpy())
    rel = np.max(np.abs(out[0] - out[1])) / np.max(np.abs(out[0]))
    assert rel < TOL
