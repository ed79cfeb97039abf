"""Per-op entry points over torch device tensors (tests, benchmarks).

Each function is a thin call into the C ABI of libqw35cuda.so
(include/qw35_cuda.h): torch only provides the device memory and the current
stream.  There is no torch or CPU implementation behind any of them.
"""
from __future__ import annotations

import torch

from ._lib import call, lib

GF4, Q8_0, Q4_K, Q5_K, Q6_K = 100, 8, 12, 13, 14
EXACT = 1


def _p(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _dev(t):
    assert t.is_cuda, "device tensor expected"
    assert t.is_contiguous()
    return t


def weight_bytes(type_id: int, rows: int, k: int) -> int:
    """GGUF-layout bytes of a rows x k matrix."""
    return int(lib().qw35_cuda_weight_bytes(type_id, rows, k))


def device_bytes(type_id: int, rows: int, k: int) -> int:
    """Device-layout bytes (Q8_0 adds a per-row exponent plane)."""
    return int(lib().qw35_cuda_device_bytes(type_id, rows, k))


def repack(type_id: int, raw: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """GGUF-layout bytes (device uint8) -> device layout."""
    out = torch.empty(device_bytes(type_id, rows, k), dtype=torch.uint8, device=raw.device)
    call("qw35_cuda_weight_repack", type_id, _p(_dev(raw)), _p(out), rows, k, _stream())
    return out


def upload(type_id: int, raw_host, rows: int, k: int, device="cuda") -> torch.Tensor:
    """numpy GGUF bytes -> repacked device weight."""
    raw = torch.from_numpy(raw_host).to(device)
    return repack(type_id, raw, rows, k)


def dequant(type_id: int, w: torch.Tensor, rows: int, k: int, exact: bool = False) -> torch.Tensor:
    out = torch.empty((rows, k), dtype=torch.float32, device=w.device)
    call("qw35_cuda_dequant", type_id, _p(_dev(w)), _p(out), rows, k, EXACT if exact else 0, _stream())
    return out


def _xdtype(x):
    if x.dtype == torch.float32:
        return 0
    if x.dtype == torch.float16:
        return 1
    raise TypeError("x must be float32 or float16")


def matvec(type_id: int, w, x, rows: int, k: int, y=None, accumulate=False, exact=False):
    b = x.shape[0] if x.dim() == 2 else 1
    if y is None:
        y = torch.zeros((b, rows), dtype=torch.float32, device=x.device)
    call("qw35_cuda_matvec", type_id, _p(_dev(w)), _p(_dev(x)), _xdtype(x), _p(_dev(y)), rows, k, b,
         1 if accumulate else 0, EXACT if exact else 0, _stream())
    return y


def gate_up_swiglu(type_id: int, wg, wu, x, rows: int, k: int, exact=False):
    b = x.shape[0] if x.dim() == 2 else 1
    h = torch.empty((b, rows), dtype=torch.float32, device=x.device)
    call("qw35_cuda_gate_up_swiglu", type_id, _p(_dev(wg)), _p(_dev(wu)), _p(_dev(x)), _xdtype(x), _p(h), rows, k, b,
         EXACT if exact else 0, _stream())
    return h


def argmax_workspace(rows: int, batch: int, device="cuda"):
    n = int(lib().qw35_cuda_argmax_workspace_bytes(rows, batch))
    return torch.empty(n, dtype=torch.uint8, device=device)


def argmax_head(type_id: int, w, x, rows: int, k: int, want_logits=False, exact=False, ws=None):
    b = x.shape[0] if x.dim() == 2 else 1
    tok = torch.empty(b, dtype=torch.int32, device=x.device)
    val = torch.empty(b, dtype=torch.float32, device=x.device)
    logits = torch.empty((b, rows), dtype=torch.float32, device=x.device) if want_logits else None
    if ws is None:
        ws = argmax_workspace(rows, b, x.device)
    call("qw35_cuda_argmax_head", type_id, _p(_dev(w)), _p(_dev(x)), _p(logits), rows, k, b, _p(tok), _p(val),
         _p(ws), ws.numel(), EXACT if exact else 0, _stream())
    return tok, val, logits


def deltanet_step(proj, conv_w, dt, a, norm_w, conv_state, ssm_state, slots=None, eps=1e-6):
    """proj [n, >=12352]; conv_state [slots, 8192*3]; ssm_state [slots, 32*128*128]."""
    n = proj.shape[0]
    out = torch.empty((n, 4096), dtype=torch.float32, device=proj.device)
    call("qw35_cuda_deltanet_step", n, _p(_dev(proj)), proj.shape[1], _p(_dev(conv_w)), _p(_dev(dt)), _p(_dev(a)),
         _p(_dev(norm_w)), _p(_dev(conv_state)), conv_state[0].numel(), _p(_dev(ssm_state)), ssm_state[0].numel(),
         _p(slots), _p(out), float(eps), _stream())
    return out


def deltanet_core(q, k, v, beta, g, state):
    n = q.shape[0]
    y = torch.empty((n, 32, 128), dtype=torch.float32, device=q.device)
    call("qw35_cuda_deltanet_core", n, _p(_dev(q)), _p(_dev(k)), _p(_dev(v)), _p(_dev(beta)), _p(_dev(g)),
         _p(_dev(state)), _p(y), _stream())
    return y


def attn_preprocess(qkv, q_norm_w, k_norm_w, rope_freq, pos, chunk_ptrs, k_off, v_off, eps=1e-6, kv_q8=False):
    """kv_q8: the planes hold q8_0 rows (272 bytes per head-row) instead of f16."""
    n = qkv.shape[0]
    q = torch.empty((n, 16, 256), dtype=torch.float32, device=qkv.device)
    gate = torch.empty_like(q)
    call("qw35_cuda_attn_preprocess_q8_0" if kv_q8 else "qw35_cuda_attn_preprocess", n, _p(_dev(qkv)), qkv.shape[1], _p(_dev(q_norm_w)), _p(_dev(k_norm_w)),
         _p(_dev(rope_freq)), _p(_dev(pos)), _p(_dev(chunk_ptrs)), chunk_ptrs.shape[1], k_off, v_off, _p(q), _p(gate),
         float(eps), _stream())
    return q, gate


def gqa_workspace(n: int, max_len: int, device="cuda"):
    return torch.empty(int(lib().qw35_cuda_gqa_workspace_bytes(n, max_len)), dtype=torch.uint8, device=device)


def gqa_decode(q, gate, seq_len, max_len, chunk_ptrs, k_off, v_off, window=0, sink=0, ws=None, out=None,
               kv_q8=False):
    n = q.shape[0]
    if out is None:
        out = torch.empty((n, 4096), dtype=torch.float32, device=q.device)
    if ws is None:
        ws = gqa_workspace(n, max_len, q.device)
    call("qw35_cuda_gqa_decode_q8_0" if kv_q8 else "qw35_cuda_gqa_decode", n, _p(_dev(q)), _p(gate), _p(_dev(seq_len)), max_len, _p(_dev(chunk_ptrs)),
         chunk_ptrs.shape[1], k_off, v_off, window, sink, _p(out), _p(ws), ws.numel(), _stream())
    return out
