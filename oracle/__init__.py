"""CPU oracle for the Qwen3.5-9B decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of the reference engine
(EmilioSchi/qwowl35) for the ops the CUDA library implements:

* ``quants``    -- GF4 / Q8_0 / Q4_K block formats: packing, dequantisation
                   and the synthetic weight generators of the benchmark configs.
* ``ops``       -- matvec, fused gate/up SwiGLU, RMS norms, the Gated DeltaNet
                   decode step, GQA decode attention over a chunk table and the
                   argmax head with its lowest-id tie rule.
* ``model``     -- a full decode step (embedding -> 3:1 DeltaNet/attention
                   stack -> head) over a synthetic model in cooked-GGUF layout.

It is a checker, never a product path: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may import
it.  The CUDA library never calls into it and has no CPU fallback.

Parity pinning: the GF4 packer / exact dequant and the Q4_K / Q8_0 dequant are
pinned bit-for-bit against golden vectors produced by the reference's own
``tools/qw35_cook_common.py`` and by gguf-py 0.19.0 (the third-party library
the reference calls for K-quants); see ``tests/golden/make_golden.py``.  The
Metal-kernel emulations (GF4 "metal" decode quirk, DeltaNet step, attention)
restate shader source that cannot execute off Apple hardware; they are pinned
only by hand-derived known-answer words and by internal consistency, i.e.
parity for those is unpinned by reference execution.
"""
