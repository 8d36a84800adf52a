"""Split-half RoPE tables for the compress / dequantize kernels.

The kernels read cos/sin rows [p, head_dim/2] (fp32) at each token's position
instead of evaluating sin/cos on the device.  The rows are built on the host
with exactly the reference's fp32 formula (nexusquant/core/rope_utils.py:106-112:
``inv_freq = 1 / base ** (arange(0, d, 2) / d)``, ``freqs = outer(pos, inv_freq)``,
``cos/sin`` in fp32 on the CPU), so the rotation the kernels undo is bit-identical
to the one the reference computes.  A table is built once per (device, head_dim,
base, rope_scaling) and grown when a longer sequence arrives; it is a model
constant, like an inference engine's cos/sin cache.
"""
from __future__ import annotations

import math
import threading
from typing import Dict, Optional, Tuple

import torch


def inv_freq(d: int, base: float, rope_scaling: Optional[dict] = None) -> torch.Tensor:
    """fp32 inverse frequencies (rope_utils.py:106) with optional scaling (rope_utils.py:34-72)."""
    inv = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    if rope_scaling is None:
        return inv
    kind = rope_scaling.get("type", rope_scaling.get("rope_type", "linear"))
    factor = float(rope_scaling.get("factor", 1.0))
    if factor == 1.0:
        return inv
    if kind in ("linear", "dynamic"):
        return inv / factor
    if kind == "llama3":
        lo = float(rope_scaling.get("low_freq_factor", 1.0))
        hi = float(rope_scaling.get("high_freq_factor", 4.0))
        old = int(rope_scaling.get("original_max_position_embeddings", 8192))
        lo_w, hi_w = old / lo, old / hi
        out = []
        for f in inv:
            w = 2.0 * math.pi / f.item()
            if w < hi_w:
                out.append(f)
            elif w > lo_w:
                out.append(f / factor)
            else:
                sm = (old / w - lo) / (hi - lo)
                out.append((1.0 - sm) * f / factor + sm * f)
        return torch.stack(out)
    return inv


def host_tables(n_rows: int, d: int, base: float, rope_scaling: Optional[dict] = None):
    """(cos, sin) fp32 CPU tensors [n_rows, d/2] for positions 0..n_rows-1."""
    pos = torch.arange(n_rows, dtype=torch.float32)
    fr = torch.outer(pos, inv_freq(d, base, rope_scaling))
    return fr.cos().contiguous(), fr.sin().contiguous()


def _scaling_key(rope_scaling: Optional[dict]):
    if rope_scaling is None:
        return None
    return tuple(sorted((k, str(v)) for k, v in rope_scaling.items()))


class RopeCache:
    """Per-device cache of RoPE tables, grown in powers of two."""

    def __init__(self):
        self._tables: Dict[Tuple, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, d: int, base: float, rows: int,
            rope_scaling: Optional[dict] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        key = (str(device), d, float(base), _scaling_key(rope_scaling))
        with self._lock:
            cur = self._tables.get(key)
            if cur is None or cur[0].shape[0] < rows:
                n = 1
                while n < max(rows, 1):
                    n *= 2
                c, s = host_tables(n, d, base, rope_scaling)
                cur = (c.to(device, non_blocking=False), s.to(device, non_blocking=False))
                self._tables[key] = cur
            return cur

    def clear(self):
        with self._lock:
            self._tables.clear()


TABLES = RopeCache()
