"""Full decode step of the synthetic model, restated in numpy (oracle, test-only).

Follows the reference's per-token order, encodeDecodeLayers
(qw35-server/src/metal/bridge/Qw35MetalRuntime.m:1170-1221):
embedding -> attn_norm -> [DeltaNet | gated attention] -> residual ->
post_attention_norm -> SwiGLU FFN -> residual -> ... -> output_norm -> head.
Layer il is full attention iff (il + 1) % interval == 0 (graph.rs:83).
Weights are read from the same host mapping the CUDA runtime uploads.
"""
from __future__ import annotations

import numpy as np

from . import ops as O
from . import quants as Q


class OracleModel:
    def __init__(self, synth, gf4_exact: bool = False, window: int = 0, sink: int = 0, tiled: bool = False,
                 kv_q8: bool = False):
        """tiled: weights as the reference's multi-token (tiled) path rounds them
        to half (GF4 element 4, K-quant values) -- the semantics of the batched
        tensor-core path (3 or more rows).  kv_q8: the KV cache holds q8_0
        blocks (kv_cache_type 1, qw35_attention.metal:425-793)."""
        self.tiled = tiled
        self.kv_q8 = kv_q8
        self.m = synth
        self.cfg = synth.cfg
        self.gf4_exact = gf4_exact
        self.window, self.sink = window, sink
        self._cache: dict[str, np.ndarray] = {}
        self.freq = O.rope_freqs(self.cfg.rope_base)
        self.reset()

    def reset(self):
        self.conv: dict[int, np.ndarray] = {}
        self.ssm: dict[int, np.ndarray] = {}
        self.k: dict[int, list] = {}
        self.v: dict[int, list] = {}
        for il in range(self.cfg.layers):
            if self._is_attn(il):
                self.k[il], self.v[il] = [], []
            else:
                self.conv[il] = np.zeros((8192, 3), dtype=np.float64)
                self.ssm[il] = np.zeros((32, 128, 128), dtype=np.float64)

    def _is_attn(self, il: int) -> bool:
        return (il + 1) % self.cfg.interval == 0

    def w(self, name: str) -> np.ndarray:
        if name not in self._cache:
            t, k, r, off, n = self.m.offsets[name]
            raw = self.m.buf[off:off + n]
            if t == Q.F32_TYPE:
                self._cache[name] = raw.view(np.float32).reshape(r, k) if r > 1 else raw.view(np.float32)
            else:
                self._cache[name] = Q.dequant(t, raw, r, k, gf4_exact=self.gf4_exact, tiled=self.tiled)
        return self._cache[name]

    def mv(self, name: str, x: np.ndarray) -> np.ndarray:
        """W[name] @ x for one activation row x (fp64)."""
        return O.matvec(self.w(name), x[None])[0]

    def embed(self, token: int) -> np.ndarray:
        t, k, r, off, n = self.m.offsets["token_embd.weight"]
        rb = n // r
        row = self.m.buf[off + token * rb: off + (token + 1) * rb]
        return Q.dequant(t, row, 1, k)[0].astype(np.float64)

    def step(self, token: int, pos: int):
        """Returns (logits [vocab] f64)."""
        eps = self.cfg.eps
        x = self.embed(token)
        for il in range(self.cfg.layers):
            p = f"blk.{il}."
            xn = O.rms_norm(x, self.w(p + "attn_norm.weight"), eps)
            if self._is_attn(il):
                q_full = self.mv(p + "attn_q.weight", xn)
                kk = self.mv(p + "attn_k.weight", xn)
                vv = self.mv(p + "attn_v.weight", xn)
                if self.kv_q8:
                    q, gate, kb, vb = O.attn_preprocess_q8_0(q_full, kk, vv, self.w(p + "attn_q_norm.weight"),
                                                             self.w(p + "attn_k_norm.weight"), pos, self.freq, eps)
                    krow, vrow = O.q8_0_kv_dequant(*kb), O.q8_0_kv_dequant(*vb)
                else:
                    q, gate, krow, vrow = O.attn_preprocess(q_full, kk, vv, self.w(p + "attn_q_norm.weight"),
                                                            self.w(p + "attn_k_norm.weight"), pos, self.freq, eps)
                self.k[il].append(krow)
                self.v[il].append(vrow)
                assert len(self.k[il]) == pos + 1, "oracle positions must be contiguous"
                K = np.stack(self.k[il])
                V = np.stack(self.v[il])
                core = O.gqa_decode(q, gate, K, V, self.window, self.sink).reshape(-1)
                x = x + self.mv(p + "attn_output.weight", core)
            else:
                qkv = self.mv(p + "attn_qkv.weight", xn)
                z = self.mv(p + "attn_gate.weight", xn)
                beta = self.mv(p + "ssm_beta.weight", xn)
                alpha = self.mv(p + "ssm_alpha.weight", xn)
                out, self.conv[il], self.ssm[il] = O.deltanet_step(
                    qkv, self.w(p + "ssm_conv1d.weight"), self.conv[il], beta, alpha, self.w(p + "ssm_dt.bias"),
                    self.w(p + "ssm_a"), self.ssm[il], z, self.w(p + "ssm_norm.weight"), eps)
                x = x + self.mv(p + "ssm_out.weight", out)
            xn = O.rms_norm(x, self.w(p + "post_attention_norm.weight"), eps)
            h = O.silu(self.mv(p + "ffn_gate.weight", xn)) * self.mv(p + "ffn_up.weight", xn)
            x = x + self.mv(p + "ffn_down.weight", h)
        xn = O.rms_norm(x, self.w("output_norm.weight"), eps)
        return self.mv("output.weight", xn)
