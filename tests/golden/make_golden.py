#!/usr/bin/env python3
"""Generate the golden vectors that pin the oracle's block formats.

Runs only where the reference checkout and gguf-py are importable (the build
container).  Sources of truth:

* GF4: the reference's own cooker, ``tools/qw35_cook_common.py``
  (``pack_gf4_prepared``, ``_gf4_quantize_with_scale``, ``e5m2_byte_to_fp32``).
* Q8_0 / Q4_K / Q5_K / Q6_K: gguf-py 0.19.0 ``gguf.quants``
  (``Q8_0.quantize_blocks`` / ``dequantize_blocks``, ``Q4_K`` / ``Q5_K`` /
  ``Q6_K.dequantize_blocks``), the third-party library
  the reference's tools call (``qw35_cook_common.py:34-35``, ``:155-179``).
  Every K-quant and Q8_0 fixture is also checked, bit for bit, against the
  reference's own call site ``dequantize_chunk`` (``qw35_cook_common.py:155``)
  on the same rows.

Usage::

    python tests/golden/make_golden.py /path/to/reference

Writes ``gf4.npz``, ``q8_0.npz``, ``q4_k.npz``, ``q5_k.npz``, ``q6_k.npz`` beside
this script.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "tools"))
    import qw35_cook_common as cc  # the reference's own module
    from gguf.quants import Q4_K, Q5_K, Q6_K, Q8_0
    import gguf

    out_dir = Path(__file__).resolve().parent
    rng = np.random.default_rng(0)

    # ---- GF4: N(0, 0.02) rows plus hand-made edge groups --------------------
    rows = rng.normal(0.0, 0.02, size=(48, 512)).astype(np.float32)
    edge = np.zeros((8, 512), dtype=np.float32)
    edge[0, :8] = 0.0                                    # all-zero group -> scale 0
    edge[0, 8:16] = [1, -1, 0.5, -0.5, 0.25, 0, -0.75, 0.75]
    edge[1, :8] = [-0.03, 0.01, 0.02, 0.0, -0.01, 0.005, 0.03, -0.03]  # |max| tie, sign
    edge[2, :] = rng.normal(0.0, 40000.0, size=512)       # near e5m2 top range
    edge[3, :] = rng.normal(0.0, 1e-5, size=512)          # e5m2 subnormal scales
    edge[4, :] = rng.uniform(-1, 1, size=512) * np.repeat(10.0 ** rng.integers(-6, 3, size=64), 8)
    edge[5, ::8] = 7.0                                    # one big element per group
    edge[6, :] = np.float32(0.0123)                       # constant groups
    edge[7, :] = -np.abs(rng.normal(0.0, 0.02, size=512))
    rows = np.concatenate([rows, edge], axis=0)
    words, scale = cc.pack_gf4_prepared(rows, scale_search=False)
    groups = rows.reshape(rows.shape[0], -1, 8)
    _, x_hat = cc._gf4_quantize_with_scale(groups, scale)
    x_hat = x_hat.reshape(rows.shape).astype(np.float32)
    e5m2_all = cc.e5m2_byte_to_fp32(np.arange(256, dtype=np.uint8))
    bytes_all = cc.fp32_to_e5m2_byte(rng.normal(0, 1, size=4096).astype(np.float32) *
                                     (10.0 ** rng.integers(-7, 5, size=4096)).astype(np.float32))
    np.savez_compressed(out_dir / "gf4.npz", rows=rows, words=np.asarray(words, dtype=np.uint32),
                        scale=np.asarray(scale, dtype=np.float32), x_hat=x_hat,
                        e5m2_table=np.asarray(e5m2_all, dtype=np.float32),
                        e5m2_probe_in=(rng.normal(0, 1, size=1).astype(np.float32)),
                        e5m2_bytes=np.asarray(bytes_all, dtype=np.uint8))

    # ---- Q8_0: gguf-py quantize of N(0,1)*10^u rows, then its dequant --------
    x = (rng.normal(0, 1, size=(32, 256)) * 10.0 ** rng.integers(-3, 2, size=(32, 1))).astype(np.float32)
    q8 = Q8_0.quantize_blocks(x.reshape(-1, 32))
    q8_deq = Q8_0.dequantize_blocks(q8).reshape(32, 256).astype(np.float32)
    q8_rand = rng.integers(0, 256, size=(16 * 8, 34), dtype=np.uint16).astype(np.uint8)
    q8_rand[:, 0:2] = (np.abs(rng.normal(0, 0.02, size=(16 * 8, 1)))).astype(np.float16).view(np.uint8)
    q8_rand_deq = Q8_0.dequantize_blocks(q8_rand).reshape(16, 256).astype(np.float32)
    np.savez_compressed(out_dir / "q8_0.npz", x=x, raw=q8.reshape(-1), deq=q8_deq,
                        raw_rand=q8_rand.reshape(-1), deq_rand=q8_rand_deq)

    # ---- Q4_K: random blocks (any 144 bytes with finite d/dmin are valid) ----
    nb = 16 * 4
    q4 = rng.integers(0, 256, size=(nb, 144), dtype=np.uint16).astype(np.uint8)
    q4[:, 0:2] = np.abs(rng.normal(0, 0.02, size=(nb, 1))).astype(np.float16).view(np.uint8)
    q4[:, 2:4] = np.abs(rng.normal(0, 0.02, size=(nb, 1))).astype(np.float16).view(np.uint8)
    q4_deq = Q4_K.dequantize_blocks(q4).reshape(16, 1024).astype(np.float32)
    np.savez_compressed(out_dir / "q4_k.npz", raw=q4.reshape(-1), deq=q4_deq)

    # ---- Q5_K: random blocks with finite d/dmin ------------------------------
    q5 = rng.integers(0, 256, size=(nb, 176), dtype=np.uint16).astype(np.uint8)
    q5[:, 0:2] = np.abs(rng.normal(0, 0.02, size=(nb, 1))).astype(np.float16).view(np.uint8)
    q5[:, 2:4] = np.abs(rng.normal(0, 0.02, size=(nb, 1))).astype(np.float16).view(np.uint8)
    q5_deq = Q5_K.dequantize_blocks(q5).reshape(16, 1024).astype(np.float32)
    np.savez_compressed(out_dir / "q5_k.npz", raw=q5.reshape(-1), deq=q5_deq)

    # ---- Q6_K: random blocks (signed scales, signed finite d); gguf-py 0.19.0
    # has no Q6_K quantizer, so the fixture pins the dequantiser only ---------
    q6 = rng.integers(0, 256, size=(nb, 210), dtype=np.uint16).astype(np.uint8)
    q6[:, 208:210] = rng.normal(0, 0.002, size=(nb, 1)).astype(np.float16).view(np.uint8)
    q6_deq = Q6_K.dequantize_blocks(q6).reshape(16, 1024).astype(np.float32)
    np.savez_compressed(out_dir / "q6_k.npz", raw=q6.reshape(-1), deq=q6_deq)

    # the reference's own call site gives the same values
    for raw, tid, rows_, deq in ((q8_rand.reshape(16, -1), cc.Q8_0_TYPE, 16, q8_rand_deq),
                                 (q4.reshape(16, -1), cc.Q4_K_TYPE, 16, q4_deq),
                                 (q5.reshape(16, -1), cc.Q5_K_TYPE, 16, q5_deq),
                                 (q6.reshape(16, -1), cc.Q6_K_TYPE, 16, q6_deq)):
        ref = np.asarray(cc.dequantize_chunk(raw, tid, 0, rows_), dtype=np.float32)
        assert np.array_equal(ref.view(np.uint32), deq.view(np.uint32)), tid

    (out_dir / "PROVENANCE.txt").write_text(
        "Generated by tests/golden/make_golden.py from the reference's tools/qw35_cook_common.py\n"
        f"and gguf-py {getattr(gguf, '__version__', '0.19.0')} (gguf.quants). Seed 0.\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
