"""Seeded synthetic inputs for the sparse-prefill layer (the benchmark's configs).

The reference measures its path on random Gaussian Q/K/V with Llama-3-8B head shapes
(``modal_rd/attn_bench.py:42-45``). These generators add RoPE tables (theta 500000, the Hugging
Face ``LlamaRotaryEmbedding`` default formula) and "planted" salient keys: for each KV head a few
key rows are set, in post-RoPE space, to 3x the mean of the last 64 post-RoPE query rows of that
head's query group, then rotated back so that the pipeline's own RoPE recreates them. Routing
must find those keys.

Every KV head draws from its own ``torch.Generator`` seeded with ``seed * 1_000_003 + kv_head``
on the CPU, so a rank that owns only some KV heads generates exactly its slice and every
machine with this torch version produces the same numbers.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

__all__ = ["LayerConfig", "CONFIGS", "rope_tables", "rope_reference_f32", "make_layer", "make_llama"]


@dataclass(frozen=True)
class LayerConfig:
    name: str
    n: int
    dtype: torch.dtype
    seed: int
    scale: float
    planted: int
    plant_lo: int
    plant_hi: int | None        # None -> n - window
    sink: int
    window: int
    vertical: int
    exact_tail: int
    n_route: int = 64
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    theta: float = 500000.0
    extra: dict = field(default_factory=dict)

    @property
    def scaling(self) -> float:
        return self.head_dim ** -0.5

    def attn_kwargs(self) -> dict:
        return dict(sink=self.sink, window=self.window, vertical=self.vertical,
                    exact_tail=self.exact_tail, n_route=self.n_route)


def _sweep(n, window):
    return LayerConfig(f"sweep_n{n}_w{window}", n, torch.bfloat16, 1, 0.5, 32, 64, None,
                       64, window, 512, 256)


CONFIGS = {
    # the reference's CPU-runnable case (fp32).
    "config1": LayerConfig("config1", 8192, torch.float32, 0, 1.0, 8, 64, 6000, 64, 2048, 128, 256),
    # the headline 128K Llama-3-8B-shaped layer (bf16).
    "config2": LayerConfig("config2", 131072, torch.bfloat16, 1, 0.5, 32, 64, None, 64, 16384, 512, 256),
}
# configs[4]'s attention layer at 1M tokens (64 planted keys per KV head): on one GPU, run as one
# rank's share of the 8-GPU head split (bench.py --config config5 --kv-shard R/8).
CONFIGS["config5"] = LayerConfig("config5", 1048576, torch.bfloat16, 1, 0.5, 64, 64, None, 64, 16384, 512, 256)
for _n in (16384, 32768, 65536, 131072, 262144, 524288):
    for _w in (4096, 16384):
        CONFIGS[f"sweep_n{_n}_w{_w}"] = _sweep(_n, _w)


def rope_tables(n, head_dim=128, theta=500000.0, dtype=torch.float32, start=0):
    """cos/sin ``[n, head_dim]`` exactly as ``LlamaRotaryEmbedding`` (default rope type) builds
    them: float32 ``inv_freq = 1 / theta ** (arange(0, d, 2) / d)``, ``freqs = pos * inv_freq``,
    ``emb = cat(freqs, freqs)``, then ``cos``/``sin`` cast to ``dtype``."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(start, start + n, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope_reference_f32(x, cos, sin):
    """float32 RoPE used only while generating inputs."""
    return x * cos + _rotate_half(x) * sin


def make_layer(cfg: LayerConfig, kv_heads=None, device="cpu"):
    """Pre-RoPE ``q [1, g*len(kv_heads), n, d]``, ``k, v [1, len(kv_heads), n, d]`` in ``cfg.dtype``,
    the RoPE tables ``cos, sin [1, n, d]`` and the planted positions ``[len(kv_heads), planted]``.

    ``kv_heads`` selects the KV heads to generate (default: all); Q heads follow their group."""
    n, d = cfg.n, cfg.head_dim
    g = cfg.heads // cfg.kv_heads
    kv_heads = list(range(cfg.kv_heads)) if kv_heads is None else list(kv_heads)
    hi = cfg.plant_hi if cfg.plant_hi is not None else n - cfg.window
    if hi <= cfg.plant_lo:  # window covers the whole prompt: plant anywhere past the sink
        hi = n
    cos32, sin32 = rope_tables(n, d, cfg.theta, torch.float32)
    q = torch.empty(1, g * len(kv_heads), n, d, dtype=cfg.dtype)
    k = torch.empty(1, len(kv_heads), n, d, dtype=cfg.dtype)
    v = torch.empty(1, len(kv_heads), n, d, dtype=cfg.dtype)
    planted = torch.empty(len(kv_heads), cfg.planted, dtype=torch.int64)
    last = min(64, n)
    for j, h in enumerate(kv_heads):
        gen = torch.Generator().manual_seed(cfg.seed * 1_000_003 + h)
        qh = torch.randn(g, n, d, generator=gen) * cfg.scale
        kh = torch.randn(n, d, generator=gen) * cfg.scale
        vh = torch.randn(n, d, generator=gen) * cfg.scale
        pos = torch.randint(cfg.plant_lo, hi, (cfg.planted,), generator=gen)
        q_last = rope_reference_f32(qh[:, n - last:], cos32[n - last:], sin32[n - last:])
        target = 3.0 * q_last.reshape(-1, d).mean(0)
        # Inverse rotation (RoPE is orthogonal): R(-theta) x = x*cos - rotate_half(x)*sin.
        kh[pos] = target[None, :] * cos32[pos] - _rotate_half(target[None, :].expand(len(pos), d)) * sin32[pos]
        q[0, j * g:(j + 1) * g] = qh.to(cfg.dtype)
        k[0, j] = kh.to(cfg.dtype)
        v[0, j] = vh.to(cfg.dtype)
        planted[j] = pos
    cos, sin = cos32.to(cfg.dtype)[None], sin32.to(cfg.dtype)[None]
    if device != "cpu":
        q, k, v, cos, sin = (t.to(device) for t in (q, k, v, cos, sin))
    return q, k, v, cos, sin, planted


def make_llama(n_layers: int = 32, seed: int = 2, device="cuda", dtype=torch.bfloat16):
    """Random-init Llama-3-8B architecture (hidden 4096, 32 Q / 8 KV heads, head_dim 128, SwiGLU
    14336, RMSNorm eps 1e-5, RoPE theta 500000, vocab 128256), weights ~ N(0, 0.02) from ``seed``:
    the model of the whole-model prefill configs. Built directly on ``device`` in ``dtype``."""
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=n_layers,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-5,
                      rope_theta=500000.0, max_position_embeddings=1 << 20, initializer_range=0.02,
                      tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    old = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            model = LlamaForCausalLM(cfg)
    finally:
        torch.set_default_dtype(old)
    return model.eval()

