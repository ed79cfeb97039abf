"""Decode-path ops restated in numpy (oracle, test-only).

Every routine computes in float64 unless noted, following the reference's
Metal kernels step by step (file:line cited per function; paths relative to
the reference project root).
"""
from __future__ import annotations

import numpy as np

F64 = np.float64


def silu(x):
    """qw35_types.metal:40-42."""
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    """qw35_types.metal:44-46."""
    return 1.0 / (1.0 + np.exp(-x))


def softplus(x):
    """qw35_types.metal:66-68 (threshold 20)."""
    x = np.asarray(x, dtype=F64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


# --------------------------------------------------------------------------
# matvec family (qw35_gf4.metal:62-246, qw35_matvec.metal:171-683)
# --------------------------------------------------------------------------
def matvec(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """y[b, r] = sum_k w[r, k] * x[b, k] in fp64.  w: [R, K] dequantised, x: [B, K]."""
    return np.asarray(x, dtype=F64) @ np.asarray(w, dtype=F64).T


def gate_up_swiglu(wg: np.ndarray, wu: np.ndarray, x: np.ndarray) -> np.ndarray:
    """h = silu(Wg x) * (Wu x)  (qw35_gf4.metal:62-96)."""
    return silu(matvec(wg, x)) * matvec(wu, x)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """qw35_core.metal:14-48: x * rsqrt(mean(x^2) + eps) * w, per row."""
    x = np.asarray(x, dtype=F64)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * inv * np.asarray(w, dtype=F64)


def argmax_lowest(logits: np.ndarray) -> tuple[int, float]:
    """Largest logit; ties resolve to the smallest id (qw35_output.metal:141-182)."""
    v = np.asarray(logits)
    m = v.max()
    idx = int(np.flatnonzero(v == m)[0])
    return idx, float(m)


# --------------------------------------------------------------------------
# Gated DeltaNet decode step (qw35_ssm.metal:260-451)
# --------------------------------------------------------------------------
N_QK = 16
N_V = 32
DS = 128
CONV_CH = 2 * N_QK * DS + N_V * DS  # 8192


def deltanet_core(S, q, k, v, beta, g, scale):
    """Delta-rule state update + readout for one sequence.

    S [H, 128(v), 128(k)] float state (rows = value index), q/k [H_qk, 128]
    (already L2-normalised), v [H, 128], beta [H] (post-sigmoid), g [H]
    (log-decay; gate = exp(g)).  Head h reads qk group h % 16.  Returns
    (y [H, 128], S_new).  Mirrors qw35_ssm.metal:393-428: delta uses the OLD
    state, y = (gate * (S q) + delta * (k.q)) * scale.
    """
    S = np.asarray(S, dtype=F64)
    H = S.shape[0]
    nqk = q.shape[0]
    y = np.empty((H, S.shape[1]), dtype=F64)
    S_new = np.empty_like(S)
    for h in range(H):
        gi = h % nqk
        kh = np.asarray(k[gi], dtype=F64)
        qh = np.asarray(q[gi], dtype=F64)
        gate = np.exp(F64(g[h]))
        kd = S[h] @ kh
        qd = S[h] @ qh
        kq = float(kh @ qh)
        delta = (np.asarray(v[h], dtype=F64) - gate * kd) * F64(beta[h])
        S_new[h] = S[h] * gate + np.outer(delta, kh)
        y[h] = (gate * qd + delta * kq) * scale
    return y, S_new


def deltanet_step(qkv, conv_w, conv_state, beta_raw, alpha_raw, dt, a, S, z, norm_w,
                  eps: float = 1e-6, n_v: int = N_V):
    """Fused DeltaNet decode step for one layer and one sequence.

    qkv [8192] raw projection (q[16x128] | k[16x128] | v[32x128]), conv_w
    [8192, 4], conv_state [8192, 3], beta_raw/alpha_raw/dt/a [32], S
    [32,128,128], z [32*128], norm_w [128].  Returns (gated [32*128],
    conv_state_new, S_new).  Steps (qw35_ssm.metal:260-451):
      1. causal conv over (s0, s1, s2, x) with SiLU; state shifts left;
      2. q/k L2 normalised with max(norm, eps);
      3. beta = sigmoid(beta_raw); gate = exp(softplus(alpha_raw + dt) * a);
      4. delta-rule core (see deltanet_core), scale = 1/sqrt(128);
      5. out = y * rsqrt(mean(y^2) + eps) * norm_w * silu(z) per head.
    """
    qkv = np.asarray(qkv, dtype=F64)
    cs = np.asarray(conv_state, dtype=F64)
    cw = np.asarray(conv_w, dtype=F64)
    conv = silu(cs[:, 0] * cw[:, 0] + cs[:, 1] * cw[:, 1] + cs[:, 2] * cw[:, 2] + qkv * cw[:, 3])
    cs_new = np.stack([cs[:, 1], cs[:, 2], qkv], axis=1)
    q = conv[:N_QK * DS].reshape(N_QK, DS)
    k = conv[N_QK * DS:2 * N_QK * DS].reshape(N_QK, DS)
    v = conv[2 * N_QK * DS:].reshape(N_V, DS)[:n_v]
    qn = q / np.maximum(np.sqrt(np.sum(q * q, axis=1, keepdims=True)), eps)
    kn = k / np.maximum(np.sqrt(np.sum(k * k, axis=1, keepdims=True)), eps)
    beta = sigmoid(np.asarray(beta_raw, dtype=F64))
    g = softplus(np.asarray(alpha_raw, dtype=F64) + np.asarray(dt, dtype=F64)) * np.asarray(a, dtype=F64)
    y, S_new = deltanet_core(S, qn, kn, v, beta, g, 1.0 / np.sqrt(DS))
    inv = 1.0 / np.sqrt(np.mean(y * y, axis=1, keepdims=True) + eps)
    zz = np.asarray(z, dtype=F64).reshape(-1, DS)[:n_v]
    out = y * inv * np.asarray(norm_w, dtype=F64)[None, :] * silu(zz)
    return out.reshape(-1), cs_new, S_new


# --------------------------------------------------------------------------
# GQA attention (qw35_attention.metal:29-112, :211-292, :302-414)
# --------------------------------------------------------------------------
N_HEAD = 16
N_KV = 4
HD = 256
ROPE = 64
CHUNK = 256


def rope_freqs(base: float = 1.0e7, rope_dim: int = ROPE) -> np.ndarray:
    """freq[i] = base^(-2i/rope_dim) in fp32 (Qw35MetalRuntime.m:772-795)."""
    i = np.arange(rope_dim // 2, dtype=np.float32)
    return np.power(np.float32(base), -(i * np.float32(2.0)) / np.float32(rope_dim)).astype(np.float32)


def _norm_rope(x, w, pos, freq, eps):
    """Per-head RMS norm then NeoX RoPE on dims [0, rope) pairing d <-> d + rope/2."""
    x = np.asarray(x, dtype=F64)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    xn = x * inv * np.asarray(w, dtype=F64)
    half = len(freq)
    theta = (np.float32(pos) * freq.astype(np.float32)).astype(np.float32).astype(F64)
    c, s = np.cos(theta), np.sin(theta)
    out = xn.copy()
    x0 = xn[..., :half]
    x1 = xn[..., half:2 * half]
    out[..., :half] = x0 * c - x1 * s
    out[..., half:2 * half] = x0 * s + x1 * c
    return out


def attn_preprocess(q_full, k, v, q_norm_w, k_norm_w, pos, freq, eps=1e-6):
    """q_full [16, 512] (q | gate per head), k/v [4, 256] ->
    (q [16,256] f64, gate [16,256] f64, k_row f16 [4,256], v_row f16 [4,256]).
    qw35_attention.metal:29-112 (K/V cache written as f16, round-to-nearest-even)."""
    q_full = np.asarray(q_full, dtype=F64).reshape(N_HEAD, 2 * HD)
    q = _norm_rope(q_full[:, :HD], q_norm_w, pos, freq, eps)
    gate = q_full[:, HD:]
    kk = _norm_rope(np.asarray(k, dtype=F64).reshape(N_KV, HD), k_norm_w, pos, freq, eps)
    return q, gate, kk.astype(np.float16), np.asarray(v, dtype=F64).reshape(N_KV, HD).astype(np.float16)


def attended_positions(seq_len: int, window: int = 0, sink: int = 0) -> np.ndarray:
    """Sink + sliding-window index set (qw35_attention.metal:250-262)."""
    sink = max(0, min(sink, seq_len))
    if window <= 0 or sink + window >= seq_len:
        return np.arange(seq_len)
    return np.concatenate([np.arange(sink), np.arange(seq_len - window, seq_len)])


def gqa_decode(q, gate, K, V, window: int = 0, sink: int = 0, scale: float = 1.0 / 16.0):
    """One sequence: q/gate [16, 256], K/V [L, 4, 256] (f16 values) ->
    out [16, 256] = softmax(q.K * scale) V * sigmoid(gate).  fp64."""
    L = K.shape[0]
    t = attended_positions(L, window, sink)
    Kf = np.asarray(K, dtype=F64)[t]
    Vf = np.asarray(V, dtype=F64)[t]
    out = np.empty((N_HEAD, HD), dtype=F64)
    grp = N_HEAD // N_KV
    for h in range(N_HEAD):
        kvh = h // grp
        s = Kf[:, kvh, :] @ np.asarray(q[h], dtype=F64) * scale
        s = s - s.max()
        p = np.exp(s)
        out[h] = (p @ Vf[:, kvh, :]) / p.sum()
    if gate is not None:
        out = out * sigmoid(np.asarray(gate, dtype=F64))
    return out


# --------------------------------------------------------------------------
# q8_0 KV cache (qw35_attention.metal:425-793)
# --------------------------------------------------------------------------
def q8_0_kv_quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """fp32 rows [..., 32n] -> (d f16 [..., n], qs int8 [..., 32n]), one block
    per 32 values (qw35_q8_0_quantize_block, qw35_attention.metal:429-440):
    d = amax / 127 in fp32, id = 1 / d (0 for an all-zero block), qs =
    clamp(round(x * id), -127, 127) with rounding half away from zero; the
    codes use the fp32 d, the block stores half(d).  IEEE fp32 division and
    product here; the reference's shaders are built with Metal's default fast
    math (qw35-server/build.rs:150-156 passes no -fno-fast-math), so a value
    that lands exactly on a .5 boundary may round differently there."""
    x = np.asarray(x, dtype=np.float32)
    b = x.reshape(x.shape[:-1] + (-1, 32))
    amax = np.max(np.abs(b), axis=-1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    safe = np.where(d != 0, d, np.float32(1.0)).astype(np.float32)
    inv = np.where(d != 0, np.float32(1.0) / safe, np.float32(0.0)).astype(np.float32)
    y = (b * inv[..., None]).astype(np.float32).astype(F64)  # fp32 product, exact in f64
    q = np.sign(y) * np.floor(np.abs(y) + 0.5)               # round half away from zero
    qs = np.clip(q, -127, 127).astype(np.int8).reshape(x.shape)
    return d.astype(np.float16), qs


def q8_0_kv_dequant(d: np.ndarray, qs: np.ndarray) -> np.ndarray:
    """float(half d) * qs per block (qw35_q8_0_dequant_qi times the block's d,
    qw35_attention.metal:442-445, :670-682), fp64."""
    qs = np.asarray(qs)
    b = qs.reshape(qs.shape[:-1] + (-1, 32)).astype(F64)
    return (b * np.asarray(d, dtype=np.float16).astype(F64)[..., None]).reshape(qs.shape)


def attn_preprocess_q8_0(q_full, k, v, q_norm_w, k_norm_w, pos, freq, eps=1e-6):
    """q8_0 twin of attn_preprocess (qw35_attention.metal:452-533): K after
    norm + RoPE and V quantised per 32-value block -> (q, gate, (kd, kqs), (vd, vqs)).
    K is formed in fp64 and rounded to fp32 before quantisation (the kernel
    forms it in fp32, so a code can differ by one where the two fp32 values
    differ in the last place)."""
    q_full = np.asarray(q_full, dtype=F64).reshape(N_HEAD, 2 * HD)
    q = _norm_rope(q_full[:, :HD], q_norm_w, pos, freq, eps)
    gate = q_full[:, HD:]
    kk = _norm_rope(np.asarray(k, dtype=F64).reshape(N_KV, HD), k_norm_w, pos, freq, eps).astype(np.float32)
    vv = np.asarray(v, dtype=np.float32).reshape(N_KV, HD)
    return q, gate, q8_0_kv_quantize(kk), q8_0_kv_quantize(vv)


def gqa_decode_q8_0(q, gate, Kq, Vq, window: int = 0, sink: int = 0, scale: float = 1.0 / 16.0):
    """Decode attention over a q8_0 KV cache (qw35_attention_gqa_flash_decode_q8_0_f32,
    qw35_attention.metal:625-690): Kq / Vq = (d [L, 4, 8] f16, qs [L, 4, 256] int8),
    dequantised per block, then gqa_decode."""
    return gqa_decode(q, gate, q8_0_kv_dequant(*Kq), q8_0_kv_dequant(*Vq), window, sink, scale)


def kv_address(chunk_table: np.ndarray, t: int, chunk: int = CHUNK):
    """Chunk-table indexing: position t lives in chunk chunk_table[t // chunk] at row t % chunk."""
    return int(chunk_table[t // chunk]), t % chunk
