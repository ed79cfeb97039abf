"""Named single-kernel workloads for profiling (ncu) through the public ops API.

    python -m qwowl35_b200.profile_cases gateup_gf4_b32
    python -m qwowl35_b200.profile_cases matvec_q8_0_b32

Each case runs the call the decode step makes for one kernel class, over
enough rotating weight copies (> the 126 MB L2) that a launch after the first
two streams its weights from HBM; e.g. capture the third launch with
``ncu -k regex:dq_kernel -s 2 -c 1``.  Weights follow the synthetic model's
distributions (qwowl35_b200.synth); activations N(0, 1).
"""
from __future__ import annotations

import sys

import torch

from . import ops

B, H, F = 32, 4096, 12288


_GEN = {}


def _weight(type_id: int, rows: int, k: int, device) -> torch.Tensor:
    """Random weight with the synthetic model's code and scale distributions."""
    from . import synth
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


CASES = {"gateup_gf4_b32": gateup_gf4_b32, "matvec_q8_0_b32": matvec_q8_0_b32, "gqa_b8_ctx4096": gqa_b8_ctx4096}


def main(argv: list[str]) -> int:
    if len(argv) != 1 or argv[0] not in CASES:
        print("usage: python -m qwowl35_b200.profile_cases {" + "|".join(CASES) + "}", file=sys.stderr)
        return 2
    device = torch.device("cuda")
    CASES[argv[0]](device)
    torch.cuda.synchronize()
    print("done")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
