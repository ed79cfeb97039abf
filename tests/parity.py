"""Error measures shared by the GPU parity tests.

``relerr`` is the bar every CUDA-vs-oracle comparison is held to (fp32
accumulation, tolerance 1e-3 in the tests): the larger of
  * the norm-wise error  max|y - ref| / max|ref|, and
  * the per-element relative error  max |y_i - ref_i| / |ref_i| over the
    elements with |ref_i| > 1e-3 * max|ref|
so a row-local error on a small output cannot hide under the largest one.
``normerr`` is the norm-wise part alone, for the few checks that compare two
fp32 renderings of the same exact quantity at a much tighter bound.

``modelerr`` is the bar for the logits of whole decode steps (many layers):
fp32 rounding carried through the layers and the recurrent state reaches every
logit through the products of the head, and some tokens are ill-conditioned
(measured on the 4-layer test model against fp64: norm-wise error ~2e-7 on
most positions, up to 3e-5 on a few), so no fp32 implementation holds 1e-3
per element on logits near zero; there the per-element part applies to the
logits above 5% of the largest (the argmax candidates).
"""
import numpy as np

SIGNIFICANT = 1e-3  # elements below this fraction of max|ref| only count norm-wise


def normerr(y, ref) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def elemerr(y, ref, floor: float = SIGNIFICANT) -> float:
    y = np.asarray(y, dtype=np.float64).reshape(-1)
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    m = np.abs(ref) > floor * max(np.max(np.abs(ref)), 1e-30)
    if not m.any():
        return 0.0
    return float(np.max(np.abs(y[m] - ref[m]) / np.abs(ref[m])))


def relerr(y, ref) -> float:
    return max(normerr(y, ref), elemerr(y, ref))


MODEL_FLOOR = 0.05


def modelerr(y, ref) -> float:
    return max(normerr(y, ref), elemerr(y, ref, MODEL_FLOOR))
