"""Quantized matvec shape sweep (the reference benchmark's matvec sweep config).

    python -m qwowl35_b200.sweep [--codecs gf4,q8_0,q4_k,q5_k,q6_k] [--batches 1,8,32] [--shapes 12288x4096]
                                 [--out FILE.md]
    python -m qwowl35_b200.sweep --case matvec_gf4_b1      # one ncu workload

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


# ---- named single-kernel workloads for ncu ---------------------------------
# ``python -m qwowl35_b200.sweep --case NAME`` runs the call the decode step makes
# for one kernel class once per rotating weight copy (the copies exceed the
# 126 MB L2, so a launch after the first two streams its weights from HBM);
# e.g. capture the third launch with ``ncu -k regex:dq_kernel -s 2 -c 1``.

B, H, F = 32, 4096, 12288


_GEN = {}


def _weight(type_id: int, rows: int, k: int, device) -> torch.Tensor:
    """Random weight with the synthetic model's code and scale distributions."""
    g = _GEN.setdefault(str(device), synth._Gen(7, device))
    return ops.repack(type_id, synth.gen_tensor(g, type_id, k, rows, "weight"), rows, k)


def gateup_gf4_b32(device) -> None:
    """FFN gate/up pair (GF4 2 x 12288 x 4096, batch 32): one dq_kernel launch each."""
    ws = [(_weight(ops.GF4, F, H, device), _weight(ops.GF4, F, H, device)) for _ in range(4)]
    x = torch.randn(B, H, device=device)
    for wg, wu in ws:
        ops.gate_up_swiglu(ops.GF4, wg, wu, x, F, H)


def matvec_q8_0_b32(device) -> None:
    """DeltaNet input projection (Q8_0 12352 x 4096, batch 32)."""
    ws = [_weight(ops.Q8_0, 12352, H, device) for _ in range(4)]
    x = torch.randn(B, H, device=device)
    y = torch.empty(B, 12352, device=device)
    for w in ws:
        ops.matvec(ops.Q8_0, w, x, 12352, H, y=y)


def gqa_b8_ctx4096(device) -> None:
    """GQA split-K decode (one attention layer) at batch 8, 4096 positions each,
    over 3 rotating KV pools (3 x 134 MB): the per-CTA work of the batch-32 step
    with a quarter of the grid (small enough for a full ncu capture)."""
    plane = 4 * 256 * 256  # f16 elements of one K (or V) plane of a chunk
    ctx, nch, B = 4096, 16, 8
    pools, tables = [], []
    for _ in range(3):
        pool = torch.randn(B * nch * 2 * plane, device=device).to(torch.float16)
        base = pool.data_ptr()
        tables.append(torch.tensor([[base + (s * nch + c) * 2 * plane * 2 for c in range(nch)] for s in range(B)],
                                   dtype=torch.int64, device=device))
        pools.append(pool)
    q, gate = torch.randn(B, 16, 256, device=device), torch.randn(B, 16, 256, device=device)
    lens = torch.full((B,), ctx, dtype=torch.int32, device=device)
    ws = ops.gqa_workspace(B, ctx, device)
    out = torch.empty(B, 4096, device=device)
    for t in tables:
        ops.gqa_decode(q, gate, lens, ctx, t, 0, plane * 2, ws=ws, out=out)


def gateup_gf4_b1(device) -> None:
    """FFN gate/up pair (GF4 2 x 12288 x 4096, batch 1): one mv_kernel launch each."""
    ws = [(_weight(ops.GF4, F, H, device), _weight(ops.GF4, F, H, device)) for _ in range(4)]
    x = torch.randn(1, H, device=device)
    for wg, wu in ws:
        ops.gate_up_swiglu(ops.GF4, wg, wu, x, F, H)


def matvec_gf4_b1(device) -> None:
    """FFN up-shaped GF4 matvec 12288 x 4096 at batch 1."""
    ws = [_weight(ops.GF4, F, H, device) for _ in range(8)]
    x = torch.randn(1, H, device=device).to(torch.float16)
    y = torch.empty(1, F, device=device)
    for w in ws:
        ops.matvec(ops.GF4, w, x, F, H, y=y)


def matvec_q8_0_b1(device) -> None:
    """DeltaNet input projection (Q8_0 12352 x 4096) at batch 1."""
    ws = [_weight(ops.Q8_0, 12352, H, device) for _ in range(8)]
    x = torch.randn(1, H, device=device)
    y = torch.empty(1, 12352, device=device)
    for w in ws:
        ops.matvec(ops.Q8_0, w, x, 12352, H, y=y)


def _deltanet(device, n: int) -> None:
    """One Gated DeltaNet decode step over n sequences, over rotating state sets
    (> 126 MB in total) so a launch streams its 4 MiB per sequence from HBM."""
    sets = max(3, (3 * (126 << 20)) // (n * 2 * 32 * 128 * 128 * 4) + 1)
    conv_w = torch.randn(8192, 4, device=device) * 0.3
    dt, a = torch.randn(32, device=device), -torch.exp(torch.randn(32, device=device) * 0.5)
    norm_w = torch.randn(128, device=device).abs()
    proj = torch.randn(n, 12352, device=device)
    for _ in range(sets):
        conv = torch.randn(n, 8192 * 3, device=device)
        ssm = torch.randn(n, 32 * 128 * 128, device=device) * 0.01
        ops.deltanet_step(proj, conv_w, dt, a, norm_w, conv, ssm)


def deltanet_b1(device) -> None:
    """Gated DeltaNet decode step for one sequence."""
    _deltanet(device, 1)


def deltanet_b32(device) -> None:
    """Gated DeltaNet decode step for 32 sequences."""
    _deltanet(device, 32)


def attn_pre_b32(device) -> None:
    """Attention preprocess (q/k RMS norm, NeoX RoPE, f16 K/V rows into the chunk) for 32 sequences."""
    plane = 4 * 256 * 256
    B = 32
    pool = torch.zeros(B * 2 * plane, device=device, dtype=torch.float16)
    table = torch.tensor([[pool.data_ptr() + s * 2 * plane * 2] for s in range(B)], dtype=torch.int64, device=device)
    qkv = torch.randn(B, 16 * 512 + 2048, device=device)
    qn, kn = torch.randn(256, device=device).abs(), torch.randn(256, device=device).abs()
    freq = torch.pow(1.0e7, -torch.arange(0, 64, 2, device=device, dtype=torch.float32) / 64.0)
    pos = torch.arange(B, dtype=torch.int32, device=device) * 7
    for _ in range(3):
        ops.attn_preprocess(qkv, qn, kn, freq, pos, table, 0, plane * 2)


CASES = {"gateup_gf4_b32": gateup_gf4_b32, "matvec_q8_0_b1": matvec_q8_0_b1, "deltanet_b1": deltanet_b1,
         "deltanet_b32": deltanet_b32, "attn_pre_b32": attn_pre_b32, "gateup_gf4_b1": gateup_gf4_b1, "matvec_gf4_b1": matvec_gf4_b1,
         "matvec_q8_0_b32": matvec_q8_0_b32, "gqa_b8_ctx4096": gqa_b8_ctx4096}



def main(argv: list[str]) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="", help="run one named ncu workload (" + ", ".join(CASES) + ") and exit")
    ap.add_argument("--shapes", default="", help="rowsxK list, e.g. 12288x4096 (default: all five)")
    ap.add_argument("--codecs", default="gf4,q8_0,q4_k,q5_k,q6_k")
    ap.add_argument("--batches", default="1,8,32")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    if a.case:
        CASES[a.case](dev)
        torch.cuda.synchronize()
        print("done")
        return 0
    shapes = [tuple(int(v) for v in sh.split("x")) for sh in a.shapes.split(",")] if a.shapes else SHAPES
    peak, kind = hbm_peak()
    gen = synth._Gen(11, dev)
    batches = [int(b) for b in a.batches.split(",")]
    rows_out = []
    for name in a.codecs.split(","):
        for rows, k in shapes:
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
