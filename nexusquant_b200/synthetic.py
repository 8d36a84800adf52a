"""Seeded synthetic KV caches with the shapes of the benchmark configurations.

No public dataset is involved: keys are pre-RoPE N(0, 1) with four outlier
channels scaled by 8 (channels drawn once from seed S, shared by all layers and
heads), then split-half RoPE is applied at positions 0..T-1 in fp32; values are
N(0, 1).  Layer l draws from a CPU ``torch.Generator`` seeded ``S*1000 + l``;
synthetic queries for the real-attention scorer use ``S*1000 + 500 + l`` and are
rotated at positions T-nq .. T-1.

``device_layer`` draws the same distribution on the GPU (torch's CUDA
generator) for the large benchmark caches, where the CPU generator would take
minutes; those tensors are not bit-identical to the CPU ones and are used only
for throughput and size-independent checks.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch

DEFAULT_SEED = 1234


@dataclass(frozen=True)
class CacheConfig:
    name: str
    n_layers: int
    batch: int
    heads: int
    seq: int
    head_dim: int
    dtype: torch.dtype = torch.float16
    rope_base: float = 10000.0
    key_bits: int = 3
    value_bits: int = 2
    eviction_rate: float = 0.0
    sliding_window: int = 32
    scorer: str = "key-key"       # "key-key" | "real" | "none"
    protect_boundary: int = 0
    sharpen: bool = False
    n_queries: int = 64           # synthetic queries (real scorer)
    q_heads: int = 0              # query heads (real scorer); 0 = heads

    @property
    def fp16_bytes(self) -> int:
        """Bytes of the cache handed in, counted at 2 bytes per element (fp16-in)."""
        return self.n_layers * 2 * self.batch * self.heads * self.seq * self.head_dim * 2


# The five benchmark configurations (BASELINE.json "configs").
CONFIGS = {
    0: CacheConfig("cfg0_quant_only_k3v2_T512_fp32", 1, 1, 8, 512, 128, torch.float32,
                   key_bits=3, value_bits=2, scorer="none"),
    1: CacheConfig("cfg1_mistral7b_T4096_b4_quant_only_k3v2", 32, 4, 8, 4096, 128,
                   key_bits=3, value_bits=2, scorer="none", sharpen=True),
    2: CacheConfig("cfg2_phi3mini_T8192_b2_k3v2_evict35_real", 32, 2, 32, 8192, 96,
                   key_bits=3, value_bits=2, eviction_rate=0.35, scorer="real"),
    3: CacheConfig("cfg3_mistral7b_T32768_k2v2_evict60_keykey", 32, 1, 8, 32768, 128,
                   key_bits=2, value_bits=2, eviction_rate=0.60),
    4: CacheConfig("cfg4_llama3_70b_T131072_k2v2_evict80_protect2", 80, 1, 8, 131072, 128,
                   rope_base=500000.0, key_bits=2, value_bits=2, eviction_rate=0.80,
                   protect_boundary=2),
}


def outlier_channels(d: int, seed: int = DEFAULT_SEED) -> torch.Tensor:
    g0 = torch.Generator().manual_seed(seed)
    return torch.randperm(d, generator=g0)[:4]


def rope_inv_freq(d: int, base: float) -> torch.Tensor:
    return 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))


def apply_rope(x: torch.Tensor, base: float, offset: int = 0) -> torch.Tensor:
    """Split-half forward RoPE (pairs i, i + d/2) at positions offset.. (fp32)."""
    d = x.shape[-1]
    s = x.shape[-2]
    dh = d // 2
    pos = torch.arange(s, dtype=torch.float32) + offset
    fr = torch.outer(pos, rope_inv_freq(d, base)).to(x.device)
    c, sn = fr.cos(), fr.sin()
    x1, x2 = x[..., :dh], x[..., dh:]
    out = torch.empty_like(x)
    out[..., :dh] = x1 * c - x2 * sn
    out[..., dh:] = x1 * sn + x2 * c
    return out


def cpu_layer(cfg: CacheConfig, layer: int, seed: int = DEFAULT_SEED,
              batch: Optional[int] = None, heads: Optional[int] = None,
              seq: Optional[int] = None):
    """(K, V) of one layer on the CPU, deterministic for (seed, layer, shape)."""
    b = batch or cfg.batch
    h = heads or cfg.heads
    T = seq or cfg.seq
    d = cfg.head_dim
    g = torch.Generator().manual_seed(seed * 1000 + layer)
    k = torch.randn(b, h, T, d, generator=g)
    k[..., outlier_channels(d, seed)] *= 8.0
    k = apply_rope(k, cfg.rope_base)
    v = torch.randn(b, h, T, d, generator=g)
    return k.to(cfg.dtype), v.to(cfg.dtype)


def cpu_queries(cfg: CacheConfig, layer: int, seed: int = DEFAULT_SEED,
                batch: Optional[int] = None, q_heads: Optional[int] = None,
                seq: Optional[int] = None, n_queries: Optional[int] = None):
    """Synthetic real-scorer queries [b, Hq, nq, d] at positions T-nq .. T-1."""
    b = batch or cfg.batch
    hq = q_heads or cfg.q_heads or cfg.heads
    T = seq or cfg.seq
    nq = n_queries or cfg.n_queries
    g = torch.Generator().manual_seed(seed * 1000 + 500 + layer)
    q = torch.randn(b, hq, nq, cfg.head_dim, generator=g)
    return apply_rope(q, cfg.rope_base, offset=T - nq).to(cfg.dtype)


def device_layer(cfg: CacheConfig, layer: int, device, seed: int = DEFAULT_SEED,
                 out_k: Optional[torch.Tensor] = None, out_v: Optional[torch.Tensor] = None):
    """Same distribution as cpu_layer, drawn on `device` (fast; not bit-identical)."""
    b, h, T, d = cfg.batch, cfg.heads, cfg.seq, cfg.head_dim
    g = torch.Generator(device=device).manual_seed(seed * 1000 + layer)
    k = torch.randn(b, h, T, d, generator=g, device=device)
    k[..., outlier_channels(d, seed).to(device)] *= 8.0
    k = apply_rope(k, cfg.rope_base)
    v = torch.randn(b, h, T, d, generator=g, device=device, dtype=torch.float32)
    if out_k is not None:
        out_k.copy_(k)
        out_v.copy_(v)
        return out_k, out_v
    return k.to(cfg.dtype), v.to(cfg.dtype)


def device_queries(cfg: CacheConfig, layer: int, device, seed: int = DEFAULT_SEED,
                   n_queries: Optional[int] = None) -> torch.Tensor:
    """Same distribution as cpu_queries, drawn on `device` (fast; not bit-identical)."""
    b, hq, T = cfg.batch, cfg.q_heads or cfg.heads, cfg.seq
    nq = n_queries or cfg.n_queries
    g = torch.Generator(device=device).manual_seed(seed * 1000 + 500 + layer)
    q = torch.randn(b, hq, nq, cfg.head_dim, generator=g, device=device)
    return apply_rope(q, cfg.rope_base, offset=T - nq).to(cfg.dtype)
