"""Host-side mirror of the reference's MetalRuntime wrapper over the C ABI.

Method names, arguments and error behaviour follow
qw35-server/src/metal/bridge.rs:249-613 (``MetalRuntime::new``,
``eval_token``, ``eval_prefill_chunk``, ``argmax``, ``copy_logits_into``,
``reset``, ``state_export``/``state_import``, ``set_ctx_size``,
``set_attn_sink``, ``sync``): every failure raises with the message the
library wrote into the error buffer.  The batched methods (``seq_alloc``,
``eval_batch``, ``argmax_batch`` ...) wrap the qw35_cuda_runtime_* extensions.
"""
from __future__ import annotations

import ctypes as C
from enum import IntEnum

import numpy as np

from ._lib import Qw35Error, check, err_buf, lib


class LogitsMode(IntEnum):  # bridge.rs:12-17
    NONE = 0
    ARGMAX = 1
    FULL = 2


class KvCacheType(IntEnum):  # bridge.rs:36-75
    F16 = 0
    Q8_0 = 1


def _u32(a):
    a = np.ascontiguousarray(a, dtype=np.uint32)
    return a, a.ctypes.data_as(C.POINTER(C.c_uint32))


class Runtime:
    def __init__(self, model, ctx: int, prefill_chunk: int = 64, kv_cache_type: int = KvCacheType.F16,
                 max_seqs: int | None = None, window: int = 0, sink: int = 0):
        """``model`` is a synth.SynthModel (host mapping + tensor table)."""
        self.model = model
        self.hp = model.cfg.hparams(window, sink)
        self.vocab = model.cfg.vocab
        self._keep = (model.buf, model.descs)
        e = err_buf(4096)
        L = lib()
        args = (model.buf.ctypes.data_as(C.c_void_p), model.buf.nbytes, model.descs, len(model.descs),
                C.byref(self.hp), ctx, self.vocab, prefill_chunk, int(kv_cache_type))
        if max_seqs is None:
            h = L.qw35_metal_runtime_create(*args, None, 0, e, C.sizeof(e))
        else:
            h = L.qw35_cuda_runtime_create(*args, max_seqs, e, C.sizeof(e))
        if not h:
            raise Qw35Error(e.value.decode(errors="replace"))
        self.handle = C.c_void_p(h)

    # -- lifetime ------------------------------------------------------------
    def close(self):
        if getattr(self, "handle", None):
            lib().qw35_metal_runtime_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _call(self, fn, *args):
        e = err_buf(4096)
        check(getattr(lib(), fn)(self.handle, *args, e, C.sizeof(e)), e)

    # -- single-sequence surface (bridge.rs) ---------------------------------
    def state_size(self) -> int:
        return int(lib().qw35_metal_runtime_state_size(self.handle))

    def state_export(self) -> bytes:
        buf = (C.c_uint8 * self.state_size())()
        self._call("qw35_metal_runtime_state_export", C.cast(buf, C.c_void_p), len(buf))
        return bytes(buf)

    def state_import(self, data: bytes):
        buf = (C.c_uint8 * len(data)).from_buffer_copy(data)
        self._call("qw35_metal_runtime_state_import", C.cast(buf, C.c_void_p), len(buf))

    def reset(self):
        self._call("qw35_metal_runtime_reset")

    def set_ctx_size(self, new_ctx: int):
        self._call("qw35_metal_runtime_set_ctx", new_ctx)

    def set_attn_sink(self, sink: int):
        lib().qw35_metal_runtime_set_attn_sink(self.handle, sink)

    def sync(self):
        self._call("qw35_metal_runtime_sync")

    def eval_token(self, token: int, pos: int, logits: LogitsMode = LogitsMode.ARGMAX):
        self._call("qw35_metal_runtime_eval_token", token, pos, int(logits))

    def eval_prefill_chunk(self, tokens, pos0: int, logits: LogitsMode = LogitsMode.ARGMAX):
        arr, p = _u32(tokens)
        self._call("qw35_metal_runtime_eval_tokens", p, len(arr), pos0, int(logits))

    def argmax(self) -> tuple[int, float]:
        t, v = C.c_uint32(), C.c_float()
        self._call("qw35_metal_runtime_argmax", C.byref(t), C.byref(v))
        return t.value, v.value

    def copy_logits(self) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        self._call("qw35_metal_runtime_copy_logits", out.ctypes.data_as(C.c_void_p), out.size)
        return out

    # -- batched extensions --------------------------------------------------
    def seq_alloc(self) -> int:
        s = C.c_uint32()
        self._call("qw35_cuda_runtime_seq_alloc", C.byref(s))
        return s.value

    def seq_free(self, seq: int):
        self._call("qw35_cuda_runtime_seq_free", seq)

    def seq_fork(self, src: int, dst: int):
        self._call("qw35_cuda_runtime_seq_fork", src, dst)

    def seq_fill_synthetic(self, seq: int, positions: int, seed: int = 0):
        """Benchmark contexts: `positions` pseudo-random KV rows without a prefill."""
        self._call("qw35_cuda_runtime_seq_fill_synthetic", seq, positions, seed)

    def seq_reset(self, seq: int):
        self._call("qw35_cuda_runtime_seq_reset", seq)

    def eval_batch(self, seq_ids, tokens, pos, logits: LogitsMode = LogitsMode.ARGMAX):
        s, sp = _u32(seq_ids)
        t, tp = _u32(tokens)
        q, qp = _u32(pos)
        assert len(s) == len(t) == len(q)
        self._call("qw35_cuda_runtime_eval_batch", len(s), sp, tp, qp, int(logits))

    def argmax_batch(self, n: int):
        tok = np.empty(n, dtype=np.uint32)
        val = np.empty(n, dtype=np.float32)
        self._call("qw35_cuda_runtime_argmax_batch", n, tok.ctypes.data_as(C.POINTER(C.c_uint32)),
                   val.ctypes.data_as(C.POINTER(C.c_float)))
        return tok, val

    def copy_logits_batch(self, n: int) -> np.ndarray:
        out = np.empty((n, self.vocab), dtype=np.float32)
        self._call("qw35_cuda_runtime_copy_logits_batch", n, out.ctypes.data_as(C.c_void_p), out.size)
        return out

    def seq_state_export(self, seq: int) -> bytes:
        buf = (C.c_uint8 * self.state_size())()
        self._call("qw35_cuda_runtime_seq_state_export", seq, C.cast(buf, C.c_void_p), len(buf))
        return bytes(buf)

    def seq_state_import(self, seq: int, data: bytes):
        buf = (C.c_uint8 * len(data)).from_buffer_copy(data)
        self._call("qw35_cuda_runtime_seq_state_import", seq, C.cast(buf, C.c_void_p), len(buf))

    def stream(self) -> int:
        return int(lib().qw35_cuda_runtime_stream(self.handle) or 0)

    def last_step_kernels(self) -> int:
        return int(lib().qw35_cuda_runtime_last_step_kernels(self.handle))

    def kv_bytes(self) -> int:
        return int(lib().qw35_cuda_runtime_kv_bytes(self.handle))
