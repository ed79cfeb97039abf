"""Quantized matvec shape sweep (the reference benchmark's matvec sweep config).

    python -m qwowl35_b200.sweep [--codecs gf4,q8_0,q4_k,q5_k,q6_k] [--batches 1,8,32] [--out FILE.md]

For every codec x shape x batch: y[B][rows] = W x^T through the public ops API
(``ops.matvec``; 1-2 rows run the CUDA-core kernels, 3-64 rows the tcgen05
dequant-GEMM), x fp16 N(0, 1), weights drawn with the
synthetic model's code and scale distributions (qwowl35_b200.synth).  Each
point replays a CUDA graph of launches over rotating weight copies whose total
exceeds twice the 126 MB L2, so every launch streams its weights from HBM;
time = best of 3 replays / launches, CUDA events on the replaying stream.
Algorithmic bytes per launch = GGUF weight bytes + B*K*2 (x) + B*rows*4 (y).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

from . import ops, synth

SHAPES = ((12288, 4096), (4096, 12288), (4096, 4096), (1024, 4096), (248320, 4096))  # (rows, K)
CODECS = {"gf4": ops.GF4, "q8_0": ops.Q8_0, "q4_k": ops.Q4_K, "q5_k": ops.Q5_K, "q6_k": ops.Q6_K}
L2 = 126 << 20


def graph_us(fns, reps: int = 3) -> float:
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    cur = torch.cuda.current_stream()  # replay() launches on the current stream
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        g.replay()
        e1.record(cur)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e3 / len(fns))
    return best


def hbm_peak() -> tuple[float, str]:
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def point(name: str, t: int, rows: int, k: int, batches, gen, dev, peak: float) -> list[dict]:
    """Time ops.matvec for one codec and shape at each batch size (see the module doc)."""
    wb = ops.weight_bytes(t, rows, k)
    ncopy = max(2, min(64, (2 * L2) // wb + 1))
    ws = [ops.repack(t, synth.gen_tensor(gen, t, k, rows, "weight"), rows, k) for _ in range(ncopy)]
    out = []
    for B in batches:
        x = torch.randn(B, k, device=dev).to(torch.float16)
        y = torch.empty(B, rows, device=dev)
        fns = [(lambda w=w: ops.matvec(t, w, x, rows, k, y=y)) for w in ws] * max(1, 16 // ncopy)
        us = graph_us(fns)
        gbs = (wb + B * k * 2 + B * rows * 4) / us / 1e3
        out.append(dict(codec=name, rows=rows, k=k, batch=B, us=round(us, 2), gbs=round(gbs, 1),
                        frac=round(gbs / peak, 3), weight_bytes=wb))
    del ws
    torch.cuda.empty_cache()
    return out


def main(argv: list[str]) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--codecs", default="gf4,q8_0,q4_k,q5_k,q6_k")
    ap.add_argument("--batches", default="1,8,32")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    peak, kind = hbm_peak()
    gen = synth._Gen(11, dev)
    batches = [int(b) for b in a.batches.split(",")]
    rows_out = []
    for name in a.codecs.split(","):
        for rows, k in SHAPES:
            for r in point(name, CODECS[name], rows, k, batches, gen, dev, peak):
                rows_out.append(r)
                print(f"{name:5s} {k:6d}->{rows:<6d} B={r['batch']:2d}: {r['us']:9.2f} us  {r['gbs']:7.1f} GB/s  "
                      f"{r['frac']:5.3f} of {kind}", flush=True)
    if a.out:
        with open(a.out, "w") as f:
            f.write(f"| codec | K -> rows | batch | us / launch | GB/s (algorithmic) | of {kind} {peak:.0f} GB/s |\n")
            f.write("|---|---|---|---|---|---|\n")
            for r in rows_out:
                f.write(f"| {r['codec']} | {r['k']} -> {r['rows']} | {r['batch']} | {r['us']} | {r['gbs']} | {r['frac']} |\n")
    print(json.dumps({"sweep": rows_out}))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
