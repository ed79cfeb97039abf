"""Synthetic Qwen3.5-9B-shaped model in the cooked-GGUF tensor layout.

There is no network for checkpoints, so benchmarks and tests decode through
a random-init model written exactly the way the reference's loader hands
tensors to the runtime (qw35-server/src/metal/bridge.rs:260-338): one host
mapping, a table of ``qw35_metal_tensor_desc`` (dims[0] = K), GGUF type ids
(100 GF4, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K, 0 f32) and the reference's tensor names
(qw35-server/src/graph.rs:173-210).

Value distributions follow the benchmark configs: GF4 words carry uniform
3-bit codes and an e5m2 scale of |N(0, 0.02)|; Q8_0 blocks carry uniform
int8 codes in [-127, 127] and d = |N(0, 0.02)| / 127 (so the block maximum,
like the GF4 group maximum, is |N(0, 0.02)|); Q4_K blocks carry uniform
codes/6-bit scales and d, dmin = |N(0, 0.02)| / 64 (Q5_K: / 128); Q6_K blocks
carry uniform codes and int8 scales and d = |N(0, 0.02)| / 4096.  Norm weights are
|N(1, 0.1)|, ssm_a = -exp(N(0, 0.5)), ssm_dt.bias ~ N(0, 1),
ssm_conv1d ~ N(0, 0.3).

Large models are generated on the GPU with torch (plumbing only) and copied
into one pinned host buffer that plays the role of the mmapped file.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from ._lib import Hparams, TensorDesc

GF4, Q8_0, Q4_K, Q5_K, Q6_K, F32 = 100, 8, 12, 13, 14, 0
ALIGN = 32  # GGUF general.alignment


@dataclass
class ModelConfig:
    layers: int = 32
    hidden: int = 4096
    ffn: int = 12288
    vocab: int = 248320
    ffn_type: int = GF4
    proj_type: int = Q8_0
    head_type: int = Q8_0
    embd_type: int = Q8_0
    interval: int = 4
    eps: float = 1e-6
    rope_base: float = 1.0e7
    # per-tensor type overrides by name suffix (e.g. {"attn_v.weight": Q6_K}),
    # for the mixed-type layouts of the reference's source GGUFs
    overrides: dict = field(default_factory=dict)

    def hparams(self, window: int = 0, sink: int = 0) -> Hparams:
        h = Hparams()
        h.transformer_layers = self.layers
        h.embedding_length = self.hidden
        h.feed_forward_length = self.ffn
        h.attention_heads = 16
        h.attention_kv_heads = 4
        h.attention_key_length = 256
        h.attention_value_length = 256
        h.rope_dimension_count = 64
        h.rope_sections[:] = [11, 11, 10, 0]
        h.rope_freq_base = self.rope_base
        h.rms_epsilon = self.eps
        h.ssm_conv_kernel = 4
        h.ssm_state_size = 128
        h.ssm_group_count = 16
        h.ssm_time_step_rank = 32
        h.ssm_inner_size = 4096
        h.full_attention_interval = self.interval
        h.attn_window = window
        h.attn_sink = sink
        h.attn_gate = 1
        h.n_cls_out = 0
        return h


def tensor_plan(cfg: ModelConfig) -> list[tuple[str, int, tuple[int, int]]]:
    """(name, type, (K, rows)) for every tensor, in file order."""
    H, F = cfg.hidden, cfg.ffn
    t = [("token_embd.weight", cfg.embd_type, (H, cfg.vocab))]
    for il in range(cfg.layers):
        p = f"blk.{il}."
        t.append((p + "attn_norm.weight", F32, (H, 1)))
        if (il + 1) % cfg.interval == 0:
            t += [(p + "attn_q.weight", cfg.proj_type, (H, 16 * 512)),
                  (p + "attn_k.weight", cfg.proj_type, (H, 1024)),
                  (p + "attn_v.weight", cfg.proj_type, (H, 1024)),
                  (p + "attn_q_norm.weight", F32, (256, 1)),
                  (p + "attn_k_norm.weight", F32, (256, 1)),
                  (p + "attn_output.weight", cfg.proj_type, (4096, H))]
        else:
            t += [(p + "attn_qkv.weight", cfg.proj_type, (H, 8192)),
                  (p + "attn_gate.weight", cfg.proj_type, (H, 4096)),
                  (p + "ssm_beta.weight", cfg.proj_type, (H, 32)),
                  (p + "ssm_alpha.weight", cfg.proj_type, (H, 32)),
                  (p + "ssm_conv1d.weight", F32, (4, 8192)),
                  (p + "ssm_dt.bias", F32, (32, 1)),
                  (p + "ssm_a", F32, (32, 1)),
                  (p + "ssm_norm.weight", F32, (128, 1)),
                  (p + "ssm_out.weight", cfg.proj_type, (4096, H))]
        t += [(p + "post_attention_norm.weight", F32, (H, 1)),
              (p + "ffn_gate.weight", cfg.ffn_type, (H, F)),
              (p + "ffn_up.weight", cfg.ffn_type, (H, F)),
              (p + "ffn_down.weight", cfg.ffn_type, (F, H))]
    t += [("output_norm.weight", F32, (H, 1)), ("output.weight", cfg.head_type, (H, cfg.vocab))]
    if cfg.overrides:
        t = [(n, next((v for s, v in cfg.overrides.items() if n.endswith(s)), ty), dims) for n, ty, dims in t]
    return t


def nbytes(type_id: int, k: int, rows: int) -> int:
    if type_id == GF4:
        return rows * k // 2
    if type_id == Q8_0:
        return rows * k // 32 * 34
    if type_id == Q4_K:
        return rows * k // 256 * 144
    if type_id == Q5_K:
        return rows * k // 256 * 176
    if type_id == Q6_K:
        return rows * k // 256 * 210
    return rows * k * 4


# ---------------------------------------------------------------------------
# generators (torch on the GPU when available, numpy otherwise)
# ---------------------------------------------------------------------------
class _Gen:
    def __init__(self, seed: int, device):
        self.device = device
        if device is not None:
            import torch
            self.torch = torch
            self.g = torch.Generator(device=device)
            self.g.manual_seed(seed)
        else:
            self.rng = np.random.default_rng(seed)

    def bytes(self, n: int) -> np.ndarray:
        if self.device is None:
            return self.rng.integers(0, 256, size=n, dtype=np.uint8)
        t = self.torch.randint(0, 256, (n,), dtype=self.torch.uint8, device=self.device, generator=self.g)
        return t

    def normal(self, n: int, mean=0.0, std=1.0):
        if self.device is None:
            return self.rng.normal(mean, std, size=n).astype(np.float32)
        return self.torch.randn(n, device=self.device, generator=self.g) * std + mean

    def to_host(self, t) -> np.ndarray:
        return t if isinstance(t, np.ndarray) else t.cpu().numpy()


def _f16_bits(g: _Gen, x):
    if isinstance(x, np.ndarray):
        return x.astype(np.float16).view(np.uint16)
    return x.to(g.torch.float16).view(g.torch.int16)


def _e5m2(g: _Gen, x):
    """fp32 -> e5m2 byte (top byte of the fp16 bits + 0x80), as the cooker does."""
    if isinstance(x, np.ndarray):
        b = x.astype(np.float16).view(np.uint16).astype(np.uint32)
        return (((b + 0x80) >> 8) & 0xFF).astype(np.uint8)
    b = x.to(g.torch.float16).view(g.torch.int16).to(g.torch.int32) & 0xFFFF
    return (((b + 0x80) >> 8) & 0xFF).to(g.torch.uint8)


def gen_tensor(g: _Gen, type_id: int, k: int, rows: int, name: str):
    n = nbytes(type_id, k, rows)
    if type_id == GF4:
        raw = g.bytes(n)
        raw = raw.reshape(-1, 4)
        raw[:, 0] = _e5m2(g, abs(g.normal(rows * k // 8, 0.0, 0.02)))
        return raw.reshape(-1)
    if type_id == Q8_0:
        nb = rows * k // 32
        raw = g.bytes(n).reshape(nb, 34)
        d = _f16_bits(g, abs(g.normal(nb, 0.0, 0.02)) / 127.0)
        if isinstance(raw, np.ndarray):
            raw[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
            q = raw[:, 2:]
            q[q == 0x80] = 0x81
        else:
            raw[:, 0:2] = d.view(g.torch.uint8).reshape(nb, 2)
            q = raw[:, 2:]
            q[q == 0x80] = 0x81
        return raw.reshape(-1)
    if type_id in (Q4_K, Q5_K):
        nb = rows * k // 256
        raw = g.bytes(n).reshape(nb, 144 if type_id == Q4_K else 176)
        for off in (0, 2):
            d = _f16_bits(g, abs(g.normal(nb, 0.0, 0.02)) / (64.0 if type_id == Q4_K else 128.0))
            raw[:, off:off + 2] = d.view(np.uint8).reshape(nb, 2) if isinstance(raw, np.ndarray) \
                else d.view(g.torch.uint8).reshape(nb, 2)
        return raw.reshape(-1)
    if type_id == Q6_K:
        nb = rows * k // 256
        raw = g.bytes(n).reshape(nb, 210)
        d = _f16_bits(g, abs(g.normal(nb, 0.0, 0.02)) / 4096.0)
        raw[:, 208:210] = d.view(np.uint8).reshape(nb, 2) if isinstance(raw, np.ndarray) \
            else d.view(g.torch.uint8).reshape(nb, 2)
        return raw.reshape(-1)
    # f32 tensors
    cnt = rows * k
    if name.endswith("ssm_a"):
        v = -np.exp(g.to_host(g.normal(cnt, 0.0, 0.5)).astype(np.float64))
    elif name.endswith("ssm_dt.bias"):
        v = g.to_host(g.normal(cnt, 0.0, 1.0))
    elif name.endswith("ssm_conv1d.weight"):
        v = g.to_host(g.normal(cnt, 0.0, 0.3))
    else:
        v = np.abs(g.to_host(g.normal(cnt, 1.0, 0.1)))
    return np.asarray(v, dtype=np.float32).view(np.uint8)


@dataclass
class SynthModel:
    cfg: ModelConfig
    buf: np.ndarray                      # host "mapping" (uint8)
    descs: C.Array
    offsets: dict = field(default_factory=dict)   # name -> (type, K, rows, offset, nbytes)
    _names: list = field(default_factory=list)
    _pinned: object = None

    def tensor(self, name: str) -> np.ndarray:
        t, k, r, off, n = self.offsets[name]
        return self.buf[off:off + n]


def build(cfg: ModelConfig, seed: int = 0, device=None) -> SynthModel:
    """Generate the model.  device='cuda' generates on the GPU (fast for full size)."""
    plan = tensor_plan(cfg)
    offsets, off = {}, 0
    for name, t, (k, r) in plan:
        n = nbytes(t, k, r)
        offsets[name] = (t, k, r, off, n)
        off = (off + n + ALIGN - 1) // ALIGN * ALIGN
    total = off
    pinned = None
    if device is not None:
        import torch
        pinned = torch.empty(total, dtype=torch.uint8, pin_memory=True)
        buf = pinned.numpy()
    else:
        buf = np.zeros(total, dtype=np.uint8)
    g = _Gen(seed, device)
    for name, t, (k, r) in plan:
        _, _, _, o, n = offsets[name]
        data = gen_tensor(g, t, k, r, name)
        if isinstance(data, np.ndarray):
            buf[o:o + n] = data
        else:
            pinned[o:o + n].copy_(data, non_blocking=False)
    names = [name.encode() for name, _, _ in plan]
    descs = (TensorDesc * len(plan))()
    for i, (name, t, (k, r)) in enumerate(plan):
        _, _, _, o, n = offsets[name]
        d = descs[i]
        d.name = C.cast(C.c_char_p(names[i]), C.c_void_p)
        d.name_len = len(names[i])
        d.dims[0], d.dims[1] = k, r
        d.n_dims = 2 if r > 1 else 1
        d.type_id = t
        d.abs_offset = o
        d.bytes = n
        d.elements = k * r
    return SynthModel(cfg=cfg, buf=buf, descs=descs, offsets=offsets, _names=names, _pinned=pinned)
