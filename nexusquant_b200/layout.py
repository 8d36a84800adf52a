"""Compressed KV-cache layout.

Per layer (the CompressedPage fields of nexusquant/integrations/vllm_backend.py:73-101,
extended to [batch, heads, tokens]):
  k_codes / v_codes   uint8 [b, h, n_kept, packed_bytes(d_p, L)]   packed 2*lattice-point codes
  k_scales / v_scales fp16  [b, h, n_kept]                          per-vector scale amax/(L/2)
  positions           int32 [b, n_kept]  original token positions (shared by all layers)
Boundary-protected layers keep fp16 K/V of the kept tokens instead of codes.

Serialization (``to_bytes``) starts with the 24-byte NQC1 header of
nexusquant/core/compression_accounting.py:24-46 ('<4sHHHIBHBBxxxxx': magic,
n_layers, n_heads, head_dim, n_tokens, bits, pca_dims, use_delta, zstd_level),
followed by an 'NQB2' extension block (key/value bits per layer, d_p, batch,
rope base) and the raw tensors.
"""
from __future__ import annotations

import io
import struct
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np
import torch

from . import kernels as K

NQC1_MAGIC = b"NQC1"
NQC1_HEADER = "<4sHHHIBHBBxxxxx"
EXT_MAGIC = b"NQB2"


def nqc1_header(n_layers, n_heads, head_dim, n_tokens, bits, pca_dims=0, use_delta=False, zstd_level=22) -> bytes:
    return struct.pack(NQC1_HEADER, NQC1_MAGIC, n_layers, n_heads, head_dim, n_tokens, bits, pca_dims or 0,
                       int(use_delta), zstd_level)


@dataclass
class CompressedLayer:
    codes: Optional[K.LayerCodes] = None          # quantized layer
    k_fp16: Optional[torch.Tensor] = None         # protected layer (kept rows, fp16)
    v_fp16: Optional[torch.Tensor] = None

    @property
    def protected(self) -> bool:
        return self.codes is None

    def nbytes(self) -> int:
        if self.protected:
            return self.k_fp16.numel() * 2 + self.v_fp16.numel() * 2
        c = self.codes
        return sum(t.numel() * t.element_size() for t in (c.k_codes, c.v_codes, c.k_scales, c.v_scales)
                   if t is not None)


@dataclass
class CompressedKVCache:
    layers: List[CompressedLayer]
    positions: torch.Tensor          # int32 [b, n_kept]
    kept_count: torch.Tensor         # int32 [b]
    seq_len: int
    batch: int
    heads: int
    head_dim: int
    rope_base: float = 10000.0
    rope_scaling: Optional[dict] = None
    mask: Optional[torch.Tensor] = None  # float [b, seq_len] keep mask (1 = kept)

    @property
    def n_kept(self) -> int:
        return self.positions.shape[1]

    @property
    def head_dim_padded(self) -> int:
        return K.next_pow2(self.head_dim)

    def nbytes(self) -> int:
        return sum(l.nbytes() for l in self.layers) + self.positions.numel() * 4

    def fp16_bytes(self) -> int:
        return len(self.layers) * 2 * self.batch * self.heads * self.seq_len * self.head_dim * 2

    def compression_ratio(self) -> float:
        return self.fp16_bytes() / max(1, self.nbytes())

    def decompress(self, layers=None, sharpen: bool = False) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """fp16 (K, V) [b, h, n_kept, d] per layer; keys re-encoded at the stored positions,
        optionally multiplied by sqrt(1.05) (README.md:75, paper section 3.6)."""
        idx = range(len(self.layers)) if layers is None else layers
        q = [i for i in idx if not self.layers[i].protected]
        out = {}
        if q:
            ks, vs = K.decompress_layers([self.layers[i].codes for i in q], self.positions, head_dim=self.head_dim,
                                         count=self.kept_count, rope_base=self.rope_base,
                                         rope_scaling=self.rope_scaling,
                                         key_sharpen=K.SHARPEN if sharpen else 1.0)
            for i, kk, vv in zip(q, ks, vs):
                out[i] = (kk, vv)
        for i in idx:
            if self.layers[i].protected:
                out[i] = (self.layers[i].k_fp16, self.layers[i].v_fp16)
        return [out[i] for i in idx]

    def delta_stream(self) -> torch.Tensor:
        """int8 temporal deltas of the codes, streams ordered layer -> K, V -> batch -> head
        (nexusquant/core/compression_accounting.py:236-251), shape [streams, n_kept, d_p]."""
        parts = []
        for l in self.layers:
            if l.protected:
                continue
            c = l.codes
            parts.append(K.delta_codes(c.k_codes, self.head_dim_padded, c.key_levels).reshape(-1, self.n_kept,
                                                                                               self.head_dim_padded))
            parts.append(K.delta_codes(c.v_codes, self.head_dim_padded, c.value_levels).reshape(-1, self.n_kept,
                                                                                                 self.head_dim_padded))
        return torch.cat(parts, 0) if parts else torch.empty(0, dtype=torch.int8)

    # ------------------------------------------------------------ serialization
    def to_bytes(self) -> bytes:
        buf = io.BytesIO()
        kb = next((l.codes.key_levels for l in self.layers if not l.protected), 4).bit_length() - 1
        buf.write(nqc1_header(len(self.layers), self.heads, self.head_dim, self.n_kept, kb))
        buf.write(EXT_MAGIC)
        buf.write(struct.pack("<IIIIId", self.batch, self.seq_len, self.head_dim_padded, len(self.layers), 0,
                              float(self.rope_base)))
        for l in self.layers:
            if l.protected:
                buf.write(struct.pack("<BBB", 1, 0, 0))
            else:
                buf.write(struct.pack("<BBB", 0, l.codes.key_levels, l.codes.value_levels))

        def put(t: torch.Tensor):
            a = t.detach().contiguous().cpu().numpy()
            buf.write(a.tobytes())

        put(self.positions)
        put(self.kept_count)
        for l in self.layers:
            if l.protected:
                put(l.k_fp16); put(l.v_fp16)
            else:
                c = l.codes
                put(c.k_codes); put(c.v_codes); put(c.k_scales); put(c.v_scales)
        return buf.getvalue()

    @classmethod
    def from_bytes(cls, data: bytes, device="cuda") -> "CompressedKVCache":
        mv = memoryview(data)
        magic, n_layers, heads, head_dim, n_kept, _bits, _pca, _delta, _z = struct.unpack_from(NQC1_HEADER, mv, 0)
        if magic != NQC1_MAGIC:
            raise ValueError("not an NQC1 stream")
        off = struct.calcsize(NQC1_HEADER)
        if bytes(mv[off:off + 4]) != EXT_MAGIC:
            raise ValueError("missing NQB2 extension block")
        off += 4
        batch, seq_len, dp, nl2, _r, base = struct.unpack_from("<IIIIId", mv, off)
        off += struct.calcsize("<IIIIId")
        meta = []
        for _ in range(n_layers):
            meta.append(struct.unpack_from("<BBB", mv, off))
            off += 3

        def take(shape, dtype):
            nonlocal off
            n = int(np.prod(shape)) * np.dtype(dtype).itemsize
            a = np.frombuffer(mv[off:off + n], dtype=dtype).reshape(shape).copy()
            off += n
            return torch.from_numpy(a).to(device)

        positions = take((batch, n_kept), np.int32)
        kept_count = take((batch,), np.int32)
        layers = []
        for prot, kl, vl in meta:
            if prot:
                layers.append(CompressedLayer(k_fp16=take((batch, heads, n_kept, head_dim), np.float16),
                                              v_fp16=take((batch, heads, n_kept, head_dim), np.float16)))
            else:
                kc = take((batch, heads, n_kept, K.packed_bytes(dp, kl)), np.uint8)
                vc = take((batch, heads, n_kept, K.packed_bytes(dp, vl)), np.uint8)
                ksc = take((batch, heads, n_kept), np.float16)
                vsc = take((batch, heads, n_kept), np.float16)
                layers.append(CompressedLayer(codes=K.LayerCodes(kc, vc, ksc, vsc, kl, vl)))
        return cls(layers, positions, kept_count, seq_len, batch, heads, head_dim, rope_base=base)
