"""The C-ABI library: it loads, exports every symbol include/*.h declares, and
its host-side argument checks behave like the reference FFI (0/NULL plus a
NUL-terminated message, Qw35FFI.m:15-18) -- no GPU compute here."""
import ctypes as C
import subprocess

import pytest

from qwowl35_b200 import _lib
from qwowl35_b200._lib import LIB_PATH, header_symbols, lib

REFERENCE_FFI = [  # qw35-server/src/metal/bridge/Qw35FFI.h:18-118
    "qw35_metal_has_device", "qw35_metal_warm_model_views", "qw35_metal_runtime_create",
    "qw35_metal_runtime_destroy", "qw35_metal_runtime_reset", "qw35_metal_runtime_state_size",
    "qw35_metal_runtime_state_export", "qw35_metal_runtime_state_import", "qw35_metal_runtime_sync",
    "qw35_metal_runtime_set_ctx", "qw35_metal_runtime_set_attn_sink", "qw35_metal_runtime_eval_token",
    "qw35_metal_runtime_eval_tokens", "qw35_metal_runtime_argmax", "qw35_metal_runtime_copy_logits",
]


def test_library_built_and_loads():
    assert LIB_PATH.exists()
    lib()


def test_every_header_symbol_is_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    declared = header_symbols()
    assert len(declared) >= 40
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    # nothing else leaks (hidden visibility for internals)
    extra = [s for s in exported if s.startswith("qw35") and s not in declared]
    assert not extra, extra


def test_reference_ffi_surface_is_complete():
    declared = set(header_symbols())
    assert set(REFERENCE_FFI) <= declared
    for name in REFERENCE_FFI:
        assert name in _lib._SIGS


def test_struct_layouts_match_reference_abi():
    # sizes/offsets of the reference structs on LP64 (Qw35MetalTypes.h:9-59)
    assert C.sizeof(_lib.TensorDesc) == 8 + 8 + 32 + 4 + 4 + 8 + 8 + 8
    assert _lib.TensorDesc.abs_offset.offset == 56
    assert C.sizeof(_lib.Hparams) == 4 * 8 + 16 + 4 + 4 + 4 * 6 + 4 * 4
    assert _lib.Hparams.n_cls_out.offset == C.sizeof(_lib.Hparams) - 4
    assert C.sizeof(_lib.WarmReport) == 48


def test_weight_bytes_match_gguf_block_sizes():
    L = lib()
    assert L.qw35_cuda_weight_bytes(100, 12288, 4096) == 25165824
    assert L.qw35_cuda_weight_bytes(8, 12288, 4096) == 53477376
    assert L.qw35_cuda_weight_bytes(12, 12288, 4096) == 28311552
    assert L.qw35_cuda_weight_bytes(100, 248320, 4096) == 508559360
    assert L.qw35_cuda_weight_bytes(8, 248320, 4096) == 1080688640
    assert L.qw35_cuda_weight_bytes(12, 248320, 4096) == 572129280
    assert L.qw35_cuda_weight_bytes(13, 4096, 4096) == 4096 * 16 * 176
    assert L.qw35_cuda_weight_bytes(14, 248320, 4096) == 248320 * 16 * 210
    assert L.qw35_cuda_weight_bytes(99, 1, 256) == 0


def test_device_bytes_add_the_q8_0_row_exponent_plane():
    L = lib()
    assert L.qw35_cuda_device_bytes(100, 12288, 4096) == L.qw35_cuda_weight_bytes(100, 12288, 4096)
    assert L.qw35_cuda_device_bytes(12, 12288, 4096) == L.qw35_cuda_weight_bytes(12, 12288, 4096)
    assert L.qw35_cuda_device_bytes(8, 12288, 4096) == 53477376 + 12288
    assert L.qw35_cuda_device_bytes(8, 333, 1280) == 333 * 40 * 34 + 336
    assert L.qw35_cuda_device_bytes(99, 1, 256) == 0
    # Q5_K: nibble + high-bit planes and 16-byte headers: same size as GGUF
    assert L.qw35_cuda_device_bytes(13, 4096, 4096) == L.qw35_cuda_weight_bytes(13, 4096, 4096)
    # Q6_K: 3k/4 code bytes + (k/16 scales + k/128 d bytes, 16-byte padded) per row
    assert L.qw35_cuda_device_bytes(14, 248320, 4096) == 248320 * (3072 + 288)
    assert L.qw35_cuda_device_bytes(14, 7, 256) == 7 * (192 + 32)


def test_invalid_handles_and_error_buffers():
    L = lib()
    e = C.create_string_buffer(256)
    bogus = C.c_void_p(0x1234)
    assert L.qw35_metal_runtime_sync(bogus, e, 256) == 0
    assert b"invalid qw35 runtime handle" in e.value
    assert L.qw35_metal_runtime_reset(None, e, 256) == 0
    # zero-length and one-byte error buffers are honoured (no write past them)
    tiny = C.create_string_buffer(b"Z", 2)
    assert L.qw35_metal_runtime_sync(bogus, tiny, 0) == 0
    assert tiny.raw[0:1] == b"Z"
    assert L.qw35_metal_runtime_sync(bogus, tiny, 1) == 0
    assert tiny.raw[0:1] == b"\x00"
    assert L.qw35_metal_runtime_state_size(bogus) == 0
    L.qw35_metal_runtime_destroy(None)
    L.qw35_metal_runtime_destroy(bogus)  # unknown handle: ignored
    L.qw35_metal_runtime_set_attn_sink(bogus, 5)
    assert L.qw35_cuda_runtime_max_seqs(bogus) == 0


def test_create_rejects_bad_inputs():
    L = lib()
    e = C.create_string_buffer(256)
    h = L.qw35_metal_runtime_create(None, 0, None, 0, None, 4096, 248320, 64, 0, None, 0, e, 256)
    assert not h and b"invalid runtime creation inputs" in e.value


def test_op_argument_checks_need_no_gpu():
    L = lib()
    e = C.create_string_buffer(256)
    # K not a multiple of 256
    assert L.qw35_cuda_matvec(100, 1, 1, 0, 1, 16, 100, 1, 0, 0, None, e, 256) == 0
    assert b"multiple of 256" in e.value
    assert L.qw35_cuda_matvec(7, 1, 1, 0, 1, 16, 256, 1, 0, 0, None, e, 256) == 0
    assert b"unsupported weight type" in e.value
    assert L.qw35_cuda_matvec(100, 1, 1, 0, 1, 16, 256, 0, 0, 0, None, e, 256) == 0
    assert L.qw35_cuda_argmax_head(100, 1, 1, None, 16, 256, 1, 1, None, 1, 0, 0, None, e, 256) == 0
    assert L.qw35_cuda_gqa_decode(1, 1, None, 1, 0, 1, 1, 0, 0, 0, 0, 1, 1, 10, None, e, 256) == 0


def test_warm_model_views_touches_pages():
    L = lib()
    buf = (C.c_uint8 * 65536)(*([1] * 65536))
    rep = _lib.WarmReport()
    e = C.create_string_buffer(256)
    assert L.qw35_metal_warm_model_views(buf, 65536, 0, 65536, 0, None, 0, 4096, C.byref(rep), e, 256) == 1
    assert rep.touches == 16 and rep.checksum == 16 and rep.bytes == 65536
    assert L.qw35_metal_warm_model_views(buf, 65536, 60000, 10000, 0, None, 0, 4096, C.byref(rep), e, 256) == 0


@pytest.mark.skipif(lib().qw35_metal_has_device() != 0, reason="a GPU is present")
def test_no_device_reported_without_gpu():
    assert lib().qw35_cuda_device_count() == 0


def test_kv_cache_type_out_of_range_is_refused_without_gpu():
    """kv_cache_type is 0 (f16) or 1 (q8_0); anything else is refused before any device work."""
    from qwowl35_b200 import synth
    from qwowl35_b200._lib import Qw35Error
    from qwowl35_b200.runtime import Runtime
    m = synth.build(synth.ModelConfig(layers=4, ffn=512, vocab=512), seed=0)
    with pytest.raises(Qw35Error, match="invalid kv_cache_type"):
        Runtime(m, ctx=64, kv_cache_type=2)


def test_plain_c_consumer_compiles_links_and_runs(tmp_path):
    """The headers are C11 (what the reference's Rust extern block binds);
    struct layouts are checked by static asserts, then the library is linked
    and its GPU-free entry points are called from C."""
    import os
    import shutil
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = tmp_path / "abi_consumer"
    libdir = str(LIB_PATH.parent)
    r = subprocess.run([gcc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(root, "include"),
                        os.path.join(root, "tests", "c", "abi_consumer.c"), "-L", libdir, "-lqw35cuda",
                        f"-Wl,-rpath,{libdir}", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and "abi ok" in run.stdout, run.stderr
