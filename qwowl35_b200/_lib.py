"""ctypes binding of libqw35cuda.so (the C ABI declared in include/*.h).

The library is the product; this module only declares signatures.  Loading
fails loudly when the shared object is missing -- there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB_PATH = PKG / "libqw35cuda.so"
HEADERS = [ROOT / "include" / "qw35_ffi.h", ROOT / "include" / "qw35_cuda.h"]

u8p = C.POINTER(C.c_uint8)
u32p = C.POINTER(C.c_uint32)
f32p = C.POINTER(C.c_float)
vp = C.c_void_p
cp = C.c_char_p
up = C.c_size_t  # uintptr_t


class WarmReport(C.Structure):
    _fields_ = [("bytes", C.c_uint64), ("mapped_bytes", C.c_uint64), ("touches", C.c_uint64),
                ("checksum", C.c_uint64), ("elapsed_ms", C.c_double), ("view_count", C.c_uint32)]


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_void_p), ("name_len", up), ("dims", C.c_uint64 * 4), ("n_dims", C.c_uint32),
                ("type_id", C.c_uint32), ("abs_offset", C.c_uint64), ("bytes", C.c_uint64),
                ("elements", C.c_uint64)]


class Hparams(C.Structure):
    _fields_ = [("transformer_layers", C.c_uint32), ("embedding_length", C.c_uint32),
                ("feed_forward_length", C.c_uint32), ("attention_heads", C.c_uint32),
                ("attention_kv_heads", C.c_uint32), ("attention_key_length", C.c_uint32),
                ("attention_value_length", C.c_uint32), ("rope_dimension_count", C.c_uint32),
                ("rope_sections", C.c_int32 * 4), ("rope_freq_base", C.c_float), ("rms_epsilon", C.c_float),
                ("ssm_conv_kernel", C.c_uint32), ("ssm_state_size", C.c_uint32), ("ssm_group_count", C.c_uint32),
                ("ssm_time_step_rank", C.c_uint32), ("ssm_inner_size", C.c_uint32),
                ("full_attention_interval", C.c_uint32), ("attn_window", C.c_int32), ("attn_sink", C.c_int32),
                ("attn_gate", C.c_uint32), ("n_cls_out", C.c_uint32)]


_SIGS = {
    # qw35_ffi.h
    "qw35_metal_has_device": (C.c_int, []),
    "qw35_metal_warm_model_views": (C.c_int, [vp, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, vp, up,
                                              C.c_uint64, C.POINTER(WarmReport), cp, up]),
    "qw35_metal_runtime_create": (vp, [vp, C.c_uint64, C.POINTER(TensorDesc), up, C.POINTER(Hparams), C.c_uint32,
                                       C.c_uint32, C.c_uint32, C.c_uint32, vp, up, cp, up]),
    "qw35_metal_runtime_destroy": (None, [vp]),
    "qw35_metal_runtime_reset": (C.c_int, [vp, cp, up]),
    "qw35_metal_runtime_state_size": (C.c_uint64, [vp]),
    "qw35_metal_runtime_state_export": (C.c_int, [vp, vp, C.c_uint64, cp, up]),
    "qw35_metal_runtime_state_import": (C.c_int, [vp, vp, C.c_uint64, cp, up]),
    "qw35_metal_runtime_sync": (C.c_int, [vp, cp, up]),
    "qw35_metal_runtime_set_ctx": (C.c_int, [vp, C.c_uint32, cp, up]),
    "qw35_metal_runtime_set_attn_sink": (None, [vp, C.c_int32]),
    "qw35_metal_runtime_eval_token": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_int, cp, up]),
    "qw35_metal_runtime_eval_tokens": (C.c_int, [vp, u32p, up, C.c_uint32, C.c_int, cp, up]),
    "qw35_metal_runtime_argmax": (C.c_int, [vp, u32p, f32p, cp, up]),
    "qw35_metal_runtime_copy_logits": (C.c_int, [vp, vp, up, cp, up]),
    # qw35_cuda.h
    "qw35_cuda_device_count": (C.c_int, []),
    "qw35_cuda_set_device": (C.c_int, [C.c_int, cp, up]),
    "qw35_cuda_build_info": (C.c_char_p, []),
    "qw35_cuda_device_error": (C.c_uint32, []),
    "qw35_cuda_weight_bytes": (C.c_uint64, [C.c_uint32, C.c_uint32, C.c_uint32]),
    "qw35_cuda_device_bytes": (C.c_uint64, [C.c_uint32, C.c_uint32, C.c_uint32]),
    "qw35_cuda_weight_repack": (C.c_int, [C.c_uint32, vp, vp, C.c_uint32, C.c_uint32, vp, cp, up]),
    "qw35_cuda_dequant": (C.c_int, [C.c_uint32, vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, vp, cp, up]),
    "qw35_cuda_matvec": (C.c_int, [C.c_uint32, vp, vp, C.c_uint32, vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int,
                                   C.c_uint32, vp, cp, up]),
    "qw35_cuda_gate_up_swiglu": (C.c_int, [C.c_uint32, vp, vp, vp, C.c_uint32, vp, C.c_uint32, C.c_uint32,
                                           C.c_uint32, C.c_uint32, vp, cp, up]),
    "qw35_cuda_argmax_workspace_bytes": (C.c_uint64, [C.c_uint32, C.c_uint32]),
    "qw35_cuda_argmax_head": (C.c_int, [C.c_uint32, vp, vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, vp, vp, vp,
                                        C.c_uint64, C.c_uint32, vp, cp, up]),
    "qw35_cuda_deltanet_step": (C.c_int, [C.c_uint32, vp, C.c_uint32, vp, vp, vp, vp, vp, C.c_uint64, vp,
                                          C.c_uint64, vp, vp, C.c_float, vp, cp, up]),
    "qw35_cuda_deltanet_core": (C.c_int, [C.c_uint32, vp, vp, vp, vp, vp, vp, vp, vp, cp, up]),
    "qw35_cuda_attn_preprocess": (C.c_int, [C.c_uint32, vp, C.c_uint32, vp, vp, vp, vp, vp, C.c_uint32,
                                            C.c_uint64, C.c_uint64, vp, vp, C.c_float, vp, cp, up]),
    "qw35_cuda_attn_preprocess_q8_0": (C.c_int, [C.c_uint32, vp, C.c_uint32, vp, vp, vp, vp, vp, C.c_uint32,
                                                 C.c_uint64, C.c_uint64, vp, vp, C.c_float, vp, cp, up]),
    "qw35_cuda_gqa_workspace_bytes": (C.c_uint64, [C.c_uint32, C.c_uint32]),
    "qw35_cuda_gqa_decode": (C.c_int, [C.c_uint32, vp, vp, vp, C.c_uint32, vp, C.c_uint32, C.c_uint64,
                                       C.c_uint64, C.c_int32, C.c_int32, vp, vp, C.c_uint64, vp, cp, up]),
    "qw35_cuda_gqa_decode_q8_0": (C.c_int, [C.c_uint32, vp, vp, vp, C.c_uint32, vp, C.c_uint32, C.c_uint64,
                                            C.c_uint64, C.c_int32, C.c_int32, vp, vp, C.c_uint64, vp, cp, up]),
    "qw35_cuda_gqa_noalloc_max_bytes": (C.c_uint64, []),
    "qw35_cuda_gqa_decode_noalloc": (C.c_int, [C.c_uint32, vp, vp, vp, C.c_uint32, vp, C.c_uint32, C.c_uint64,
                                               C.c_uint64, C.c_int32, C.c_int32, vp, vp, cp, up]),
    "qw35_cuda_runtime_create": (vp, [vp, C.c_uint64, C.POINTER(TensorDesc), up, C.POINTER(Hparams), C.c_uint32,
                                      C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, cp, up]),
    "qw35_cuda_runtime_seq_alloc": (C.c_int, [vp, u32p, cp, up]),
    "qw35_cuda_runtime_seq_free": (C.c_int, [vp, C.c_uint32, cp, up]),
    "qw35_cuda_runtime_seq_reset": (C.c_int, [vp, C.c_uint32, cp, up]),
    "qw35_cuda_runtime_max_seqs": (C.c_uint32, [vp]),
    "qw35_cuda_runtime_seq_fork": (C.c_int, [vp, C.c_uint32, C.c_uint32, cp, up]),
    "qw35_cuda_runtime_seq_fill_synthetic": (C.c_int, [vp, C.c_uint32, C.c_uint32, C.c_uint64, cp, up]),
    "qw35_cuda_runtime_eval_batch": (C.c_int, [vp, C.c_uint32, u32p, u32p, u32p, C.c_int, cp, up]),
    "qw35_cuda_runtime_argmax_batch": (C.c_int, [vp, C.c_uint32, u32p, f32p, cp, up]),
    "qw35_cuda_runtime_copy_logits_batch": (C.c_int, [vp, C.c_uint32, vp, up, cp, up]),
    "qw35_cuda_runtime_seq_state_export": (C.c_int, [vp, C.c_uint32, vp, C.c_uint64, cp, up]),
    "qw35_cuda_runtime_seq_state_import": (C.c_int, [vp, C.c_uint32, vp, C.c_uint64, cp, up]),
    "qw35_cuda_runtime_stream": (vp, [vp]),
    "qw35_cuda_runtime_last_step_kernels": (C.c_uint32, [vp]),
    "qw35_cuda_runtime_kv_bytes": (C.c_uint64, [vp]),
    "qw35_cuda_runtime_weight_bytes": (C.c_uint64, [vp]),
    "qw35_cuda_runtime_scratch": (C.c_uint64, [vp, C.POINTER(C.c_uint64)]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every function name declared in include/*.h."""
    names: list[str] = []
    for h in HEADERS:
        text = re.sub(r"//[^\n]*", "", h.read_text())
        names += re.findall(r"\b(qw35_(?:metal|cuda)_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def lib() -> C.CDLL:
    """Load libqw35cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m qwowl35_b200.build` (no CPU fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class Qw35Error(RuntimeError):
    pass


def err_buf(n: int = 1024):
    return C.create_string_buffer(n)


def check(ok: int, err) -> None:
    if not ok:
        raise Qw35Error(err.value.decode(errors="replace") or "unknown error")


def call(name: str, *args) -> None:
    """Call an int-returning entry point with trailing (err, err_len); raise on failure."""
    e = err_buf()
    check(getattr(lib(), name)(*args, e, C.sizeof(e)), e)
