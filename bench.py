#!/usr/bin/env python3
"""Decode throughput of the Qwen3.5-9B-shaped hot path on B200.

Workload: 32 layers (24 Gated DeltaNet + 8 gated GQA),
hidden 4096, FFN 12288 in GF4, every other projection and the 248320-row
lm_head in Q8_0, greedy argmax head, 4096 positions of context per sequence,
a batch of --batch sequences per GPU (ragged-batch data parallel: each rank
owns its own sequences and a full weight replica, no collective).  A "step"
is one decode step of the whole batch.  Synthetic random-init weights
(qwowl35_b200.synth) -- there is no network for checkpoints.

Printed JSON line (rank 0):
  value     tok/s over all ranks, device-timed (CUDA events on the runtime's
            stream), inputs already resident, steps replayed back to back;
  e2e       the same metric through the public C ABI in a greedy loop:
            token ids host->device, argmax ids device->host every step;
  roofline  the step's dominant kernel, timed alone with CUDA events;
  cpu_baseline  the CPU oracle port on a bounded sample of the same batch
            (rank 0, N=1; RefSample).
--impl reference runs the reference's CPU rendering of the path (the oracle
port: the reference's own GPU code is Metal-only) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HBM_FALLBACK = 6650.0  # GB/s, pool fallback when MEASURED_PEAKS.json is absent


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK, "fallback"


# ---------------------------------------------------------------------------
# CPU leg: the oracle port on a bounded sample (test infrastructure; the
# product path never touches it)
# ---------------------------------------------------------------------------
def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="qw35clk", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(r[0] for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# the step's kernels timed alone (roofline of the dominant one)
# ---------------------------------------------------------------------------
# DRAM bytes (read + write) per launch measured by ncu for a kernel class of the
# table: one `--set full` capture of `python -m qwowl35_b200.sweep --case
# gateup_gf4_b32` (third launch, weights not in L2).
NCU_TRAFFIC = {
    "gate_up_swiglu GF4 12288x4096": 55032064,
}


def kernel_table(B: int, ctx: int, device):
    """Times each kernel class of the step alone and returns rows of
    (name, algorithmic bytes per launch, avg seconds per launch, launches per step).

    Each class is launched back to back inside one CUDA graph over rotating
    copies of its weights/state totalling well over the 126 MB L2, so every
    launch streams from HBM and host launch cost is excluded; CUDA events
    bracket the graph replay on the launching stream."""
    import torch

    from qwowl35_b200 import ops

    from qwowl35_b200 import synth

    gen = synth._Gen(1, device)

    def rnd_weight(t, rows, k):
        # the model's own code / scale distributions (decode cost depends on the scales)
        raw = synth.gen_tensor(gen, t, k, rows, "weight")
        return ops.repack(t, raw, rows, k)

    def graph_time(fns, reps=3):
        st = torch.cuda.Stream(device)
        with torch.cuda.stream(st):
            for f in fns:
                f()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for f in fns:
                f()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = 1e9
        for _ in range(reps):
            e0.record()
            g.replay()
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) / 1e3 / len(fns))
        del g
        return best

    def copies(nbytes):
        return max(2, min(12, (400 << 20) // max(nbytes, 1) + 1))

    H, F = 4096, 12288
    x = torch.randn(B, H, device=device)
    h = torch.randn(B, F, device=device)
    rows = []
    n = copies(2 * 25165824)
    wg = [rnd_weight(ops.GF4, F, H) for _ in range(n)]
    wu = [rnd_weight(ops.GF4, F, H) for _ in range(n)]
    rows.append(("gate_up_swiglu GF4 12288x4096", 2 * 25165824 + B * (H + F) * 4,
                 graph_time([lambda a=a, b=b: ops.gate_up_swiglu(ops.GF4, a, b, x, F, H) for a, b in zip(wg, wu)]),
                 32))
    del wg, wu
    y = torch.zeros(B, H, device=device)
    wd = [rnd_weight(ops.GF4, H, F) for _ in range(copies(25165824))]
    rows.append(("matvec GF4 4096x12288 +residual", 25165824 + B * (F * 4 + H * 8),
                 graph_time([lambda w=w: ops.matvec(ops.GF4, w, h, H, F, y=y, accumulate=True) for w in wd]), 32))
    del wd
    for r, cnt in ((12352, 24), (10240, 8)):
        wb = ops.weight_bytes(ops.Q8_0, r, H)
        ws = [rnd_weight(ops.Q8_0, r, H) for _ in range(copies(wb))]
        yy = torch.empty(B, r, device=device)
        rows.append((f"matvec Q8_0 {r}x4096", wb + B * (H + r) * 4,
                     graph_time([lambda w=w: ops.matvec(ops.Q8_0, w, x, r, H, y=yy) for w in ws]), cnt))
        del ws
    wb = ops.weight_bytes(ops.Q8_0, H, 4096)
    ws = [rnd_weight(ops.Q8_0, H, 4096) for _ in range(copies(wb))]
    rows.append(("matvec Q8_0 4096x4096 +residual", wb + B * H * 12,
                 graph_time([lambda w=w: ops.matvec(ops.Q8_0, w, x, H, 4096, y=y, accumulate=True) for w in ws]), 32))
    del ws
    wh = rnd_weight(ops.Q8_0, 248320, H)
    aw = ops.argmax_workspace(248320, B, device)
    tok = torch.empty(B, dtype=torch.int32, device=device)
    rows.append(("argmax head Q8_0 248320x4096", 1080688640 + B * H * 4,
                 graph_time([lambda: ops.argmax_head(ops.Q8_0, wh, x, 248320, H, ws=aw)] * 2), 1))
    del wh
    proj = torch.randn(B, 12352, device=device)
    conv_w = torch.randn(8192 * 4, device=device) * 0.3
    dt, a, nw = torch.zeros(32, device=device), -torch.ones(32, device=device), torch.ones(128, device=device)
    per = 2 * 32 * 128 * 128 * 4
    nst = copies(B * per // 2)
    conv = [torch.zeros(B, 8192 * 3, device=device) for _ in range(nst)]
    ssm = [torch.randn(B, 32 * 128 * 128, device=device) * 0.01 for _ in range(nst)]
    rows.append(("deltanet_step (cluster)", B * (per + 2 * 8192 * 3 * 4 + 12352 * 4 + 4096 * 4),
                 graph_time([lambda c=c, s_=s_: ops.deltanet_step(proj, conv_w, dt, a, nw, c, s_)
                             for c, s_ in zip(conv, ssm)]), 24))
    del conv, ssm
    plane = 4 * 256 * 256
    nch = (ctx + 255) // 256
    npool = copies(B * ctx * 4096)
    pools, tables = [], []
    for _ in range(npool):
        pool = torch.randn(B * nch * 2 * plane, device=device).to(torch.float16)
        base = pool.data_ptr()
        tables.append(torch.tensor([[base + (s_ * nch + c) * 2 * plane * 2 for c in range(nch)] for s_ in range(B)],
                                   dtype=torch.int64, device=device))
        pools.append(pool)
    q, gt = torch.randn(B, 16, 256, device=device), torch.randn(B, 16, 256, device=device)
    lens = torch.full((B,), ctx, dtype=torch.int32, device=device)
    aws = ops.gqa_workspace(B, ctx, device)
    out = torch.empty(B, 4096, device=device)
    rows.append((f"gqa split-K decode ctx {ctx} (+combine)", B * ctx * 4096 + B * 16 * 256 * 12,
                 graph_time([lambda t=t: ops.gqa_decode(q, gt, lens, ctx, t, 0, plane * 2, ws=aws, out=out)
                             for t in tables]), 8))
    del pools, tables
    torch.cuda.empty_cache()
    return rows


# ---------------------------------------------------------------------------
# BASELINE configs 1, 3 and 4 as kernel-level lines (each with its roofline
# fraction and a CPU-port baseline on a bounded sample)
# ---------------------------------------------------------------------------
CONFIG4_LENS = [131072, 512, 114894, 801, 14856, 4129, 43695, 1347, 64324, 10452, 76211, 7217, 5571, 40667,
                120045, 3977, 110329, 88427, 1371, 14980, 25512, 95448, 20527, 1072, 8095, 7907, 8202, 104175,
                3564, 1770, 9259, 17921]  # np.random.default_rng(4) log-uniform 512..131072, ends pinned


def config_lines(device, peak: float, kind: str):
    """Config 1: the GF4 12288 x 4096 up-projection at batch 1 (x fp16).
    Config 3: the DeltaNet recurrent core (prepared q/k/v, beta, log-decay) for
    1 and 64 sequences.  Config 4: one attention layer's GQA decode over 32
    sequences of 512..131072 positions in shuffled 256-position chunks.
    GPU: CUDA events over graph replays of rotating inputs larger than L2.
    CPU: the numpy oracle port on a sample (rows / sequences), scaled up."""
    import numpy as np
    import torch

    from oracle import ops as O
    from oracle import quants as Q
    from qwowl35_b200 import ops, synth, sweep

    out = {}
    cores = cpu_cores()
    # ---- config 1 -------------------------------------------------------------
    g = synth._Gen(0, device)
    pt = sweep.point("gf4", ops.GF4, 12288, 4096, [1], g, device, peak)[0]
    rng = np.random.default_rng(0)
    rows_s = 768  # 1/16 of the rows
    raw = Q.gen_weight(rng, Q.GF4_TYPE, rows_s, 4096)
    x = rng.standard_normal((1, 4096)).astype(np.float16).astype(np.float32)
    t0 = time.perf_counter()
    O.matvec(Q.dequant(Q.GF4_TYPE, raw, rows_s, 4096), x)
    cpu_s = (time.perf_counter() - t0) * (12288 / rows_s)
    b1 = 25165824 + 8192 + 49152
    out["config1"] = {"workload": "GF4 matvec 12288x4096, batch 1, x fp16", "unit": "GB/s",
                      "value": pt["gbs"], "us": pt["us"], "bytes": b1,
                      "roofline": {"bound": "hbm", "achieved": pt["gbs"], "peak": peak, "peak_kind": kind,
                                   "frac": pt["gbs"] / peak},
                      "cpu_baseline": {"value": b1 / cpu_s / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                                       "sample": f"{rows_s} of 12288 rows dequantised (metal semantics) and "
                                                 "multiplied in fp64 numpy, scaled to the whole matrix"}}
    # ---- config 3 -------------------------------------------------------------
    per = 4227072  # state R+W + q, k, v + out per sequence-layer
    rows3 = []
    for n in (1, 64):
        q = torch.randn(n, 16, 128, device=device)
        q = (q / q.norm(dim=-1, keepdim=True)).half()
        k = torch.randn(n, 16, 128, device=device)
        k = (k / k.norm(dim=-1, keepdim=True)).half()
        v = torch.randn(n, 32, 128, device=device).half()
        beta = torch.sigmoid(torch.randn(n, 32, device=device))
        gl = -torch.nn.functional.softplus(torch.randn(n, 32, device=device))
        nst = max(2, (400 << 20) // (n * 32 * 128 * 128 * 4) + 1)
        states = [torch.randn(n, 32, 128, 128, device=device) * 0.01 for _ in range(min(nst, 64))]
        fns = [(lambda S=S: ops.deltanet_core(q, k, v, beta, gl, S)) for S in states]
        us = sweep.graph_us(fns * max(1, 8 // len(fns)))
        gbs = n * per / us / 1e3
        rows3.append({"sequences": n, "us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3)})
        del states
    rng = np.random.default_rng(3)
    S = rng.normal(0, 0.01, (32, 128, 128))
    qq = rng.standard_normal((16, 128))
    qq /= np.linalg.norm(qq, axis=-1, keepdims=True)
    t0 = time.perf_counter()
    O.deltanet_core(S, qq, qq, rng.standard_normal((32, 128)), np.full(32, 0.5), np.full(32, -0.5), 0.0884)
    cpu3 = time.perf_counter() - t0
    out["config3"] = {"workload": "Gated DeltaNet recurrent core, one layer, ragged 1..64 sequences",
                      "unit": "GB/s", "value": rows3[-1]["gbs"], "rows": rows3,
                      "roofline": {"bound": "hbm", "achieved": rows3[-1]["gbs"], "peak": peak, "peak_kind": kind,
                                   "frac": rows3[-1]["gbs"] / peak},
                      "cpu_baseline": {"value": per / cpu3 / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                                       "sample": "one sequence-layer of the fp64 numpy oracle"}}
    # ---- config 4 -------------------------------------------------------------
    lens = CONFIG4_LENS
    plane = 4 * 256 * 256
    nch = [(L + 255) // 256 for L in lens]
    total = sum(nch)
    pool = torch.randn(total * 2 * plane, device=device).half()
    perm = np.random.default_rng(44).permutation(total)
    table = np.zeros((len(lens), max(nch)), dtype=np.int64)
    i = 0
    for s_, c in enumerate(nch):
        for j in range(c):
            table[s_, j] = pool.data_ptr() + int(perm[i]) * 2 * plane * 2
            i += 1
    tab = torch.from_numpy(table).to(device)
    qd, gd = torch.randn(len(lens), 16, 256, device=device), torch.randn(len(lens), 16, 256, device=device)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=device)
    ws = ops.gqa_workspace(len(lens), max(lens), device)
    o4 = torch.empty(len(lens), 4096, device=device)
    us4 = sweep.graph_us([lambda: ops.gqa_decode(qd, gd, lens_d, max(lens), tab, 0, plane * 2, ws=ws, out=o4)] * 4)
    b4 = 4096 * sum(lens) + len(lens) * 16 * 256 * 12
    del pool
    Ls = 8192  # CPU sample: one sequence of 8192 positions, scaled by the positions
    Kc = rng.standard_normal((Ls, 4, 256)).astype(np.float16)
    t0 = time.perf_counter()
    O.gqa_decode(rng.standard_normal((16, 256)), rng.standard_normal((16, 256)), Kc, Kc)
    cpu4 = (time.perf_counter() - t0) * sum(lens) / Ls
    out["config4"] = {"workload": "GQA decode, one layer, 32 sequences of 512..131072 positions (seed 4)",
                      "unit": "GB/s", "value": b4 / us4 / 1e3, "us": us4, "bytes": b4,
                      "roofline": {"bound": "hbm", "achieved": b4 / us4 / 1e3, "peak": peak, "peak_kind": kind,
                                   "frac": b4 / us4 / 1e3 / peak},
                      "cpu_baseline": {"value": b4 / cpu4 / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                                       "sample": f"one sequence of {Ls} positions in fp64 numpy, scaled by positions"}}
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def max_over_ranks(v: float, world: int, device) -> float:
    """The slowest rank's value (device-timed seconds): all_reduce(MAX) over the
    process group (NCCL on GPUs; gloo with a CPU device in the tests)."""
    if world == 1:
        return v
    import torch

    t = torch.tensor([v], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


class RefSample:
    """The reference arm's unit of work: one slice of one layer of the decode
    step for the whole batch (the same config as the GPU arm), rendered by
    the CPU oracle port (numpy, the host's BLAS threads).  A slice is 1/SLICES
    of the layer's matrix rows (dequantised, then multiplied by all B
    activation rows at once, as a batched engine reads weights once per step)
    plus the per-sequence mixer (DeltaNet step or attention at ctx positions)
    of B/SLICES sequences.  Step i takes layer i % 32 (attention when
    (i + 1) % 4 == 0), so a run of K steps covers the model's layer mix; the
    lm_head's slice is timed once.  The estimated decode step is
    SLICES * (24 mean DeltaNet slices + 8 mean attention slices + 1 head slice)."""

    SLICES = 16

    def __init__(self, B: int, ctx: int):
        import numpy as np

        from oracle import quants as Q
        self.np, self.Q = np, Q
        self.B, self.ctx = B, ctx
        rng = np.random.default_rng(0)
        H, F, S = 4096, 12288, self.SLICES
        self.rng = rng
        # the slice's rows of every matrix of a layer (GGUF bytes; dequantised per use)
        self.gate = Q.gen_weight(rng, Q.GF4_TYPE, F // S, H)
        self.up = Q.gen_weight(rng, Q.GF4_TYPE, F // S, H)
        self.down = Q.gen_weight(rng, Q.GF4_TYPE, H // S, F)
        self.proj_d = Q.gen_weight(rng, Q.Q8_0_TYPE, 12352 // S, H, 127.0)
        self.proj_a = Q.gen_weight(rng, Q.Q8_0_TYPE, 10240 // S, H, 127.0)
        self.outw = Q.gen_weight(rng, Q.Q8_0_TYPE, H // S, 4096, 127.0)
        self.head = Q.gen_weight(rng, Q.Q8_0_TYPE, 248320 // S, H, 127.0)
        self.x = rng.standard_normal((B, H))
        self.h = rng.standard_normal((B, F))
        nseq = max(1, B // S)
        self.nseq = nseq
        self.K = rng.standard_normal((ctx, 4, 256)).astype(np.float16)
        self.V = rng.standard_normal((ctx, 4, 256)).astype(np.float16)
        self.S = [rng.normal(0, 0.01, (32, 128, 128)) for _ in range(nseq)]

    def _mm(self, t, raw, rows, k, x):
        return x @ self.Q.dequant(t, raw, rows, k).T.astype(self.np.float64)

    def layer(self, attn: bool) -> float:
        from oracle import ops as O
        np, Q, H, F, S = self.np, self.Q, 4096, 12288, self.SLICES
        t0 = time.perf_counter()
        if attn:
            self._mm(Q.Q8_0_TYPE, self.proj_a, 10240 // S, H, self.x)
            for _ in range(self.nseq):
                p = self.rng.standard_normal(10240)
                q, gate, _, _ = O.attn_preprocess(p[:8192], p[8192:9216], p[9216:], np.ones(256), np.ones(256),
                                                  self.ctx - 1, O.rope_freqs())
                O.gqa_decode(q, gate, self.K, self.V)
        else:
            self._mm(Q.Q8_0_TYPE, self.proj_d, 12352 // S, H, self.x)
            for i in range(self.nseq):
                p = self.rng.standard_normal(12352)
                O.deltanet_step(p[:8192], np.ones((8192, 4)) * 0.3, np.zeros((8192, 3)), p[12288:12320],
                                p[12320:], np.zeros(32), -np.ones(32), self.S[i], p[8192:12288], np.ones(128))
        self._mm(Q.Q8_0_TYPE, self.outw, H // S, 4096, self.x)
        self._mm(Q.GF4_TYPE, self.gate, F // S, H, self.x)
        self._mm(Q.GF4_TYPE, self.up, F // S, H, self.x)
        self._mm(Q.GF4_TYPE, self.down, H // S, F, self.h)
        return time.perf_counter() - t0

    def head_slice(self) -> float:
        t0 = time.perf_counter()
        self._mm(self.Q.Q8_0_TYPE, self.head, 248320 // self.SLICES, 4096, self.x)
        return time.perf_counter() - t0

    def describe(self) -> str:
        return (f"per step: 1/{self.SLICES} of one layer (rows of every matrix dequantised and multiplied by "
                f"all {self.B} activation rows, plus the DeltaNet step / attention at ctx {self.ctx} for "
                f"{self.nseq} sequence(s)), layers rotating through the 24 DeltaNet + 8 attention mix, fp64 "
                f"numpy oracle port; decode step = {self.SLICES} x (24 DeltaNet + 8 attention + head) slices")


def run_reference(args, world):
    rank, _, _ = dist_env()
    if rank != 0:
        return
    cores = cpu_cores()
    ref = RefSample(args.batch, args.ctx_fill)
    head = ref.head_slice()
    t_delta, t_attn, times = [], [], []
    for i in range(args.warmup + args.steps):
        attn = (i + 1) % 4 == 0
        t = ref.layer(attn)
        if i >= args.warmup:
            (t_attn if attn else t_delta).append(t)
            times.append(t)
    if not t_attn:  # fewer than 4 timed steps: time one attention slice as well
        t_attn.append(ref.layer(True))
    if not t_delta:
        t_delta.append(ref.layer(False))
    step_s = RefSample.SLICES * (24 * sum(t_delta) / len(t_delta) + 8 * sum(t_attn) / len(t_attn) + head)
    tps = args.batch / step_s
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "step_unit": f"one 1/{RefSample.SLICES}-layer slice of the batch (see cpu_baseline.sample)",
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": workload_config(args, 1),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": ref.describe() + "; the reference's own decode path is Metal-only "
                                       "(unavailable on this box), so its kernels run as the numpy oracle port"},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


METRIC = "decode tok/s, Qwen3.5-9B-shape (GF4 FFN, Q8_0 projections+head), 4k ctx"


def workload_config(args, world):
    return {"workload": f"config5 full decode step, batch {args.batch}/GPU, ctx {args.ctx_fill}",
            "global_batch": args.batch * world, "seq_len": args.ctx_fill, "layers": args.layers,
            "ffn_codec": "gf4", "proj_codec": "q8_0", "head_codec": "q8_0", "vocab": 248320,
            "parallelism": f"dp{world} (ragged sequences per GPU, no collective)",
            "l2": "inputs larger than L2: every step streams 5.7 GB of weights plus state/KV"}


def run_ragged(args, rank, world, device, model, cfg):
    """BASELINE config 4's ragged batch through the full decode step: 32 sequences
    per GPU (global batch 32 * world) with context lengths log-uniform in
    512..131072, assigned to ranks by the step-bytes partitioner
    (qwowl35_b200.partition); each rank decodes only its own sequences, every
    sequence at its own position.  KV caches are synthetic (no prefill).
    Returns (tokens, device seconds of the slowest rank, detail dict)."""
    import numpy as np
    import torch

    from qwowl35_b200.partition import imbalance, log_uniform_lengths, partition
    from qwowl35_b200.runtime import LogitsMode, Runtime

    lens = log_uniform_lengths(32 * world, seed=4)
    parts = partition(lens, world)
    mine = [lens[i] for i in parts[rank]]
    n = len(mine)
    steps = args.ragged_steps
    rt = Runtime(model, ctx=max(mine) + steps + args.warmup + 8, max_seqs=max(n, 1))
    ids = [0] + [rt.seq_alloc() for _ in range(n - 1)]
    for k, (s_, L) in enumerate(zip(ids, mine)):
        rt.seq_fill_synthetic(s_, L, seed=1000 + parts[rank][k])
    pos = list(mine)
    tok = [int((7919 * (i + 1)) % cfg.vocab) for i in range(n)]
    for _ in range(args.warmup):
        rt.eval_batch(ids, tok, pos, LogitsMode.ARGMAX)
        pos = [p_ + 1 for p_ in pos]
    rt.sync()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ext = torch.cuda.ExternalStream(rt.stream(), device=device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(steps):
        rt.eval_batch(ids, tok, pos, LogitsMode.ARGMAX)
        pos = [p_ + 1 for p_ in pos]
    e1.record(ext)
    e1.synchronize()
    t = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, device)
    rt.close()
    detail = {"sequences": 32 * world, "lengths": "log-uniform 512..131072, seed 4",
              "partition": "greedy by per-step bytes (weights + state + KV)",
              "bytes_imbalance": round(imbalance(lens, parts), 4), "steps": steps,
              "kv_positions_total": int(np.sum(lens))}
    return 32 * world * steps, t, detail


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx-fill", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel roofline table")
    ap.add_argument("--ragged-steps", type=int, default=5,
                    help="steps of the ragged config-4 batch (32 sequences/GPU, 512..131072 positions); 0 skips it")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_env()

    if args.impl == "reference":
        run_reference(args, world)
        return

    import numpy as np
    import torch

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device)
    from qwowl35_b200 import synth
    from qwowl35_b200.runtime import LogitsMode, Runtime

    B = args.batch
    cfg = synth.ModelConfig(layers=args.layers)
    t0 = time.time()
    model = synth.build(cfg, seed=0, device=device)
    t_gen = time.time() - t0
    total_pos = args.ctx_fill + 2 * (args.warmup + args.steps) + args.steps + 8
    t0 = time.time()
    rt = Runtime(model, ctx=total_pos, max_seqs=B)
    t_load = time.time() - t0
    ids = [0] + [rt.seq_alloc() for _ in range(B - 1)]
    tok = (np.arange(B, dtype=np.uint32) * 7919) % cfg.vocab

    # context (untimed): every sequence gets ctx_fill positions of synthetic KV
    # (deterministic pseudo-random rows, no prefill); the recurrent state starts
    # at zero.  A decode step reads the same bytes either way.
    t0 = time.time()
    for k, s_ in enumerate(ids):
        rt.seq_fill_synthetic(s_, args.ctx_fill, seed=k)
    t_fill = time.time() - t0
    pos = args.ctx_fill

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()


    # ---- device-timed steps (inputs resident, no host reads inside) --------
    ext = torch.cuda.ExternalStream(rt.stream(), device=device)
    for _ in range(args.warmup):
        rt.eval_batch(ids, tok, [pos] * B, LogitsMode.ARGMAX)
        pos += 1
    rt.sync()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local if "CUDA_VISIBLE_DEVICES" not in os.environ else
                      int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])) as clk:
        ev0.record(ext)
        torch.cuda.nvtx.range_push("timed_steps")  # lets a profiler select just these launches
        for _ in range(args.steps):
            rt.eval_batch(ids, tok, [pos] * B, LogitsMode.ARGMAX)
            pos += 1
        torch.cuda.nvtx.range_pop()
        ev1.record(ext)
        ev1.synchronize()
    rt.sync()
    barrier()
    dev_s = max_over_ranks(ev0.elapsed_time(ev1) / 1e3, world, device)
    kernels = rt.last_step_kernels()
    value = B * world * args.steps / dev_s

    # ---- end to end through the C ABI: greedy loop, H2D ids, D2H argmax ----
    cur = tok.copy()
    for _ in range(args.warmup):
        rt.eval_batch(ids, cur, [pos] * B, LogitsMode.ARGMAX)
        cur, _ = rt.argmax_batch(B)
        pos += 1
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        rt.eval_batch(ids, cur, [pos] * B, LogitsMode.ARGMAX)
        cur, _ = rt.argmax_batch(B)
        pos += 1
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, device)
    barrier()

    # ---- batch 1 on the same runtime (sequence 0) ---------------------------
    for _ in range(3):
        rt.eval_batch([0], [1], [pos], LogitsMode.ARGMAX)
        pos += 1
    rt.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    n1 = min(args.steps, 8)
    torch.cuda.nvtx.range_push("timed_b1")
    for _ in range(n1):
        rt.eval_batch([0], [1], [pos], LogitsMode.ARGMAX)
        pos += 1
    torch.cuda.nvtx.range_pop()
    e1.record(ext)
    e1.synchronize()
    b1_s = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, device)
    rt.close()
    ragged = None
    if args.ragged_steps > 0:
        r_tok, r_s, r_detail = run_ragged(args, rank, world, device, model, cfg)
        ragged = dict(value=r_tok / r_s, unit="tok/s", ms_per_step=r_s / args.ragged_steps * 1e3, **r_detail)
    del model

    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_s / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (random-init, seed 0)",
            "config": workload_config(args, world), "clocks": clk.summary(),
            "e2e": {"value": B * world * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 16 * B,
                    "d2h_bytes_per_step": 8 * B},
            "gpu_launches": kernels * args.steps,
            "b1": {"value": world * n1 / b1_s, "unit": "tok/s", "ms_per_token": b1_s / n1 * 1e3},
            "ragged": ragged,
            "setup_s": {"generate": round(t_gen, 1), "upload": round(t_load, 1), "ctx_fill": round(t_fill, 1)}}

    if rank == 0 and not args.no_kernels:
        peak, kind = peaks()
        rows = kernel_table(B, args.ctx_fill, device)
        table = [{"kernel": n, "bytes": b, "us": t * 1e6, "per_step": c, "gbs": b / t / 1e9,
                  "frac": b / t / 1e9 / peak} for n, b, t, c in rows]
        dom = max(rows, key=lambda r: r[2] * r[3])
        achieved = dom[1] / dom[2] / 1e9
        line["roofline"] = {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": peak,
                            "peak_kind": kind, "unit": "GB/s", "frac": achieved / peak,
                            "traffic": NCU_TRAFFIC.get(dom[0]),
                            "bytes_per_launch": dom[1], "us_per_launch": dom[2] * 1e6}
        line["kernels"] = table
        # GEMV half of the metric: batch-1 matvec HBM throughput of the FFN
        # up-projection shape per codec (qwowl35_b200.sweep, x fp16)
        try:
            from qwowl35_b200 import ops as _ops, sweep
            g = synth._Gen(11, device)
            pts = []
            for name, t in (("gf4", _ops.GF4), ("q8_0", _ops.Q8_0), ("q4_k", _ops.Q4_K)):
                pts += sweep.point(name, t, 12288, 4096, [1], g, device, peak)
            line["gemv"] = {"shape": "K 4096 -> rows 12288, batch 1, x fp16", "unit": "GB/s",
                            "peak": peak, "peak_kind": kind,
                            "rows": [{"codec": r["codec"], "gbs": r["gbs"], "us": r["us"], "frac": r["frac"],
                                      "frac_of_8tbs": round(r["gbs"] / 8000.0, 3)} for r in pts]}
        except Exception as exc:  # the GEMV table never blocks the bench line
            line["gemv"] = {"error": str(exc)[:200]}
        try:
            line["configs"] = config_lines(device, peak, kind)
        except Exception as exc:
            line["configs"] = {"error": str(exc)[:200]}
    if rank == 0 and world == 1 and not args.no_cpu:
        ref = RefSample(B, args.ctx_fill)
        head = ref.head_slice()
        td = [ref.layer(False) for _ in range(3)]
        ta = [ref.layer(True)]
        step_s = RefSample.SLICES * (24 * sum(td) / len(td) + 8 * sum(ta) / len(ta) + head)
        line["cpu_baseline"] = {"value": B / step_s, "unit": "tok/s", "cores": cpu_cores(), "kind": "port",
                                "sample": ref.describe() + " (3 DeltaNet + 1 attention slice timed)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
