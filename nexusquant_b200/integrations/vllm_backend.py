"""Paged (vLLM-style) interface: nexusquant/integrations/vllm_backend.py on the B200 kernels.

Same names, arguments, page layout and errors as the reference module:

  CompressedPage                 vllm_backend.py:73-129   int8 codes (2 x lattice point), fp16 scales
  NexusQuantKVCompressor         vllm_backend.py:132-555  compress_page / decompress_page / nibble packing
  NexusQuantPagedAttention       vllm_backend.py:558-787  block pool, compress_and_cache, decode forward
  register_nexusquant_backend    vllm_backend.py:790-895
  compress_kv_pages / decompress_kv_pages / measure_compression_ratio   vllm_backend.py:968-1077

What runs on the device:
  * compress_page is one nq_compress_layers launch (inverse RoPE at the page positions ->
    Hadamard -> relaxed E8, the per-vector arithmetic of _quantize_perhead_with_scales) plus
    nq_unpack_codes into the int8 page layout; compress_kv_pages and compress_and_cache
    compress every token of the call in that one launch and then cut it into pages (tokens are
    independent, so the pages are identical to page-by-page compression).
  * decompress_page reads the int8 codes directly (the library's 16-level format is int8
    codes) through nq_decompress_layers; decompress_kv_pages is one launch for all pages.
  * NexusQuantPagedAttention.forward runs the fused compressed-domain decode attention
    (nq_attend_compressed) for all sequences in one launch at head_dim 128; other head
    dims decompress with nq_decompress_layers and attend with torch on the GPU.
  * pack_codes_nibble / unpack_codes_nibble are nq_pack_nibbles / nq_unpack_nibbles.

Tensors must be CUDA tensors: there is no CPU path.
"""
from __future__ import annotations

import dataclasses
import math
import warnings
from typing import List, Optional, Tuple

import torch

from .. import _native as N
from .. import kernels as K

_FP16_BYTES = 2


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


@dataclasses.dataclass
class CompressedPage:
    """One compressed KV block (vllm_backend.py:73-101): key/value codes int8
    (num_heads, num_valid, head_dim) holding 2 x the E8 lattice point, fp16 scales
    (num_heads, num_valid), int32 positions (num_valid,), num_valid."""

    key_codes: torch.Tensor
    value_codes: torch.Tensor
    key_scales: torch.Tensor
    value_scales: torch.Tensor
    positions: torch.Tensor
    num_valid: int

    @property
    def compressed_bytes(self) -> int:
        """int8 K and V codes + fp16 K and V scales + int32 positions (vllm_backend.py:105-117)."""
        n = self.num_valid
        h = self.key_codes.shape[0]
        d = self.key_codes.shape[2]
        return 2 * h * n * d + 2 * h * n * _FP16_BYTES + n * 4

    @property
    def uncompressed_bytes(self) -> int:
        """fp16 K and V of the same tokens (vllm_backend.py:119-129)."""
        n = self.num_valid
        h = self.key_codes.shape[0]
        d = self.key_codes.shape[2]
        return 2 * h * n * d * _FP16_BYTES


class NexusQuantKVCompressor:
    """Page-granular compressor (vllm_backend.py:132-555).

    Keys: inverse RoPE at the stored positions -> Hadamard -> E8 VQ; values: Hadamard -> E8 VQ.
    bits in (2, 3, 4) -> 4, 8, 16 levels; head_dim a power of two (64 or 128 on the B200 kernels).
    eviction_rate is stored as the reference stores it and, as there, not used by compress_page.
    """

    def __init__(self, head_dim: int = 128, bits: int = 2, eviction_rate: float = 0.0,
                 rope_base: float = 10000.0):
        if bits not in (2, 3, 4):
            raise ValueError(f"bits must be 2, 3, or 4 (got {bits})")
        if head_dim & (head_dim - 1) != 0:
            raise ValueError(f"head_dim must be a power of 2 (got {head_dim})")
        self.head_dim = head_dim
        self.bits = bits
        self.levels = 2 ** bits
        self.eviction_rate = eviction_rate
        self.rope_base = rope_base

    # ------------------------------------------------------------------ pages
    def _check_dims(self, d: int):
        if d != self.head_dim:
            raise ValueError(f"page head_dim {d} does not match the compressor's {self.head_dim}")
        if d not in (64, 128):
            raise NotImplementedError(f"head_dim {d}: the B200 page kernels support head_dim 64 and 128")

    def _compress_tokens(self, key: torch.Tensor, value: torch.Tensor, positions: torch.Tensor):
        """key / value (h, n, d) -> int8 codes (h, n, d) x2, fp16 scales (h, n) x2, int32 positions."""
        K._require_cuda(key, value)
        h, n, d = key.shape
        if value.shape != key.shape:
            raise ValueError(f"key page {tuple(key.shape)} and value page {tuple(value.shape)} differ")
        self._check_dims(d)
        dev = key.device
        pos = positions.to(device=dev, dtype=torch.int32).reshape(-1)
        if pos.numel() != n:
            raise ValueError(f"{pos.numel()} positions for {n} tokens")
        kc = torch.empty((h, n, d), dtype=torch.int8, device=dev)
        vc = torch.empty((h, n, d), dtype=torch.int8, device=dev)
        if n == 0:
            e = torch.empty((h, 0), dtype=torch.float16, device=dev)
            return kc, vc, e, e.clone(), pos
        lc = K.compress_layers([key.unsqueeze(0)], [value.unsqueeze(0)], key_levels=self.levels,
                               value_levels=self.levels, positions=pos[None], rope_base=self.rope_base)[0]
        s = _stream(dev)
        N.call("nq_unpack_codes", lc.k_codes.data_ptr(), h * n, d, self.levels, kc.data_ptr(), s)
        N.call("nq_unpack_codes", lc.v_codes.data_ptr(), h * n, d, self.levels, vc.data_ptr(), s)
        return kc, vc, lc.k_scales[0], lc.v_scales[0], pos

    def compress_page(self, key_page: torch.Tensor, value_page: torch.Tensor,
                      page_positions: torch.Tensor) -> CompressedPage:
        """Compress one page (num_heads, block_size, head_dim), fp16 / bf16 / fp32, at the given
        absolute positions (vllm_backend.py:344-396).  All tokens of the page are stored."""
        kc, vc, ks, vs, pos = self._compress_tokens(key_page, value_page, page_positions)
        return CompressedPage(key_codes=kc, value_codes=vc, key_scales=ks, value_scales=vs, positions=pos,
                              num_valid=key_page.shape[1])

    def _decompress(self, key_codes, value_codes, key_scales, value_scales, positions):
        """int8 codes (h, n, d) -> fp16 keys / values (h, n, d).  The codes are read as the
        library's 16-level (int8) format; |code| <= 16 as compress_page writes them."""
        K._require_cuda(key_codes, value_codes, key_scales, value_scales, positions)
        h, n, d = key_codes.shape
        self._check_dims(d)
        dev = key_codes.device
        if n == 0:
            e = torch.empty((h, 0, d), dtype=torch.float16, device=dev)
            return e, e.clone()
        lc = K.LayerCodes(key_codes.contiguous().view(torch.uint8)[None], value_codes.contiguous().view(torch.uint8)[None],
                          key_scales.to(torch.float16).contiguous()[None],
                          value_scales.to(torch.float16).contiguous()[None], 16, 16)
        ok, ov = K.decompress_layers([lc], positions.to(device=dev, dtype=torch.int32).reshape(1, -1),
                                     head_dim=d, rope_base=self.rope_base)
        return ok[0][0], ov[0][0]

    def decompress_page(self, compressed_page: CompressedPage) -> Tuple[torch.Tensor, torch.Tensor]:
        """(keys, values), both fp16 (num_heads, num_valid, head_dim) (vllm_backend.py:398-429)."""
        p = compressed_page
        return self._decompress(p.key_codes, p.value_codes, p.key_scales, p.value_scales, p.positions)

    def decompress_for_attention(self, compressed_page: CompressedPage, query: torch.Tensor) -> torch.Tensor:
        """Unnormalised logits query @ keys^T / sqrt(head_dim), fp32 (num_heads, q_len, num_valid)
        (vllm_backend.py:431-470).  The keys come from decompress_page (rounded to fp16), where
        the reference keeps them in fp32: logits agree within that rounding."""
        keys, _ = self.decompress_page(compressed_page)
        q = query.float()
        return torch.einsum("hqd,hsd->hqs", q, keys.float()) / math.sqrt(self.head_dim)

    # --------------------------------------------------------------- nibbles
    @staticmethod
    def pack_codes_nibble(codes: torch.Tensor) -> torch.Tensor:
        """int8 (..., d) -> uint8 (..., ceil(d/2)): byte = clamp(c_even + 8) | clamp(c_odd + 8) << 4,
        clamp to [0, 15], an odd d padded with a zero nibble (vllm_backend.py:476-513)."""
        K._require_cuda(codes)
        c = codes.to(torch.int8).contiguous()
        d = c.shape[-1]
        rows = c.numel() // d if d else 0
        out = torch.empty(c.shape[:-1] + ((d + 1) // 2,), dtype=torch.uint8, device=c.device)
        N.call("nq_pack_nibbles", c.data_ptr(), rows, d, out.data_ptr(), _stream(c.device))
        return out

    @staticmethod
    def unpack_codes_nibble(packed: torch.Tensor, original_d: int) -> torch.Tensor:
        """uint8 (..., ceil(original_d/2)) -> int8 (..., original_d), nibble - 8
        (vllm_backend.py:515-540)."""
        K._require_cuda(packed)
        p = packed.to(torch.uint8).contiguous()
        full = 2 * p.shape[-1]
        rows = p.numel() // p.shape[-1] if p.shape[-1] else 0
        out = torch.empty(p.shape[:-1] + (full,), dtype=torch.int8, device=p.device)
        N.call("nq_unpack_nibbles", p.data_ptr(), rows, full, out.data_ptr(), _stream(p.device))
        return out[..., :original_d]

    def compression_ratio(self, page: CompressedPage) -> float:
        """uncompressed / compressed bytes, all overhead counted (vllm_backend.py:542-555)."""
        if page.uncompressed_bytes == 0:
            return 1.0
        return page.uncompressed_bytes / page.compressed_bytes


def _split_pages(kc, vc, ks, vs, pos, bounds) -> List[CompressedPage]:
    return [CompressedPage(key_codes=kc[:, a:b].contiguous(), value_codes=vc[:, a:b].contiguous(),
                           key_scales=ks[:, a:b].contiguous(), value_scales=vs[:, a:b].contiguous(),
                           positions=pos[a:b].contiguous(), num_valid=b - a) for a, b in bounds]


class NexusQuantPagedAttention:
    """Compressed block pool and decode attention (vllm_backend.py:558-787)."""

    def __init__(self, compressor: NexusQuantKVCompressor):
        self.compressor = compressor
        self._block_pool: dict = {}
        self._next_block_id: int = 0

    def allocate_block(self) -> int:
        block_id = self._next_block_id
        self._next_block_id += 1
        return block_id

    def free_block(self, block_id: int) -> None:
        self._block_pool.pop(block_id, None)

    def is_block_compressed(self, block_id: int) -> bool:
        return block_id in self._block_pool

    def compress_and_cache(self, key: torch.Tensor, value: torch.Tensor, key_cache: dict, value_cache: dict,
                           slot_mapping: torch.Tensor) -> None:
        """Compress new tokens (total_tokens, num_heads, head_dim) into CompressedPages keyed by
        block id (vllm_backend.py:618-690): tokens are grouped by slot // block_size in order of
        first appearance and stored at position slot % block_size, block_size as
        _infer_block_size gives it.  All tokens are compressed in one launch."""
        if key.shape[0] == 0:
            return
        block_size = self._infer_block_size(slot_mapping)
        dev = key.device
        slots = slot_mapping.to(torch.int64)
        block_ids = (slots // block_size).tolist()
        offsets = (slots % block_size).to(device=dev, dtype=torch.int32)
        order: dict = {}
        for i, bid in enumerate(block_ids):
            order.setdefault(bid, []).append(i)
        perm = [i for toks in order.values() for i in toks]
        perm_t = torch.tensor(perm, dtype=torch.long, device=dev)
        k = key[perm_t].permute(1, 0, 2)
        v = value[perm_t].permute(1, 0, 2)
        kc, vc, ks, vs, pos = self.compressor._compress_tokens(k, v, offsets[perm_t])
        bounds, a = [], 0
        for toks in order.values():
            bounds.append((a, a + len(toks)))
            a += len(toks)
        for bid, page in zip(order.keys(), _split_pages(kc, vc, ks, vs, pos, bounds)):
            key_cache[bid] = page
            value_cache[bid] = page

    def forward(self, query: torch.Tensor, compressed_key_cache: dict, compressed_value_cache: dict,
                block_tables: List[List[int]], context_lens: torch.Tensor) -> torch.Tensor:
        """Decode attention, one query token per sequence (vllm_backend.py:692-765): for each
        sequence the pages of its block table that are present, concatenated and cut to
        context_lens[b] tokens; softmax(q K^T / sqrt(head_dim)) V; sequences with no tokens give
        zeros.  query (batch, num_heads, head_dim) fp16 with RoPE applied -> fp16 output."""
        K._require_cuda(query)
        b, h, d = query.shape
        dev = query.device
        ctx = [int(c) for c in context_lens.tolist()]
        seqs = []
        for bi in range(b):
            pages = [compressed_key_cache[i] for i in block_tables[bi] if i in compressed_key_cache]
            n = min(ctx[bi], sum(p.num_valid for p in pages)) if pages and ctx[bi] > 0 else 0
            seqs.append((pages, n))
        n_max = max([n for _, n in seqs] + [1])
        kc = torch.zeros((b, h, n_max, d), dtype=torch.int8, device=dev)
        vc = torch.zeros_like(kc)
        ks = torch.zeros((b, h, n_max), dtype=torch.float16, device=dev)
        vs = torch.zeros_like(ks)
        pos = torch.zeros((b, n_max), dtype=torch.int32, device=dev)
        for bi, (pages, n) in enumerate(seqs):
            if n == 0:
                continue
            kc[bi, :, :n] = torch.cat([p.key_codes for p in pages], 1)[:, :n]
            vc[bi, :, :n] = torch.cat([p.value_codes for p in pages], 1)[:, :n]
            ks[bi, :, :n] = torch.cat([p.key_scales for p in pages], 1)[:, :n]
            vs[bi, :, :n] = torch.cat([p.value_scales for p in pages], 1)[:, :n]
            pos[bi, :n] = torch.cat([p.positions for p in pages])[:n]
        count = torch.tensor([n for _, n in seqs], dtype=torch.int32, device=dev)
        if d == 128:
            lc = K.LayerCodes(kc.view(torch.uint8), vc.view(torch.uint8), ks, vs, 16, 16)
            return K.attend_compressed(query.to(torch.float16), lc, pos, count=count,
                                       rope_base=self.compressor.rope_base)
        # other head dims: decompress on the device, attend with torch
        out = torch.zeros((b, h, d), dtype=torch.float16, device=dev)
        for bi, (_, n) in enumerate(seqs):
            if n == 0:
                continue
            keys, values = self.compressor._decompress(kc[bi, :, :n], vc[bi, :, :n], ks[bi, :, :n],
                                                       vs[bi, :, :n], pos[bi, :n])
            logits = torch.einsum("hqd,hsd->hqs", query[bi].unsqueeze(1).float(), keys.float()) / math.sqrt(d)
            out[bi] = torch.einsum("hqs,hsd->hqd", torch.softmax(logits, -1), values.float()).squeeze(1).half()
        return out

    @staticmethod
    def _infer_block_size(slot_mapping: torch.Tensor) -> int:
        """The reference's heuristic, kept as written (vllm_backend.py:771-787): the first of
        4, 8, 16, 32 with (slot % bs).max() < bs, which is 4 for any non-empty mapping."""
        if slot_mapping.numel() == 0:
            return 16
        for bs in [4, 8, 16, 32]:
            if (slot_mapping % bs).max() < bs:
                return bs
        return 16


def _extract_head_dim(engine_config) -> int:
    """head_dim, or hidden_size // num_attention_heads, from the engine config (vllm_backend.py:862-883)."""
    for attr in ("model_config", "model", "hf_config", "config"):
        cfg = getattr(engine_config, attr, None)
        if cfg is not None:
            hd = getattr(cfg, "head_dim", None)
            if hd is not None:
                return int(hd)
            hs = getattr(cfg, "hidden_size", None)
            nh = getattr(cfg, "num_attention_heads", None)
            if hs is not None and nh is not None:
                return int(hs) // int(nh)
    warnings.warn("NexusQuant: could not auto-detect head_dim from engine_config. Defaulting to 128.  "
                  "Pass head_dim explicitly to avoid this.", RuntimeWarning, stacklevel=2)
    return 128


def _extract_rope_base(engine_config) -> float:
    """rope_theta from the engine config, else 10000 (vllm_backend.py:886-894)."""
    for attr in ("model_config", "model", "hf_config", "config"):
        cfg = getattr(engine_config, attr, None)
        if cfg is not None:
            base = getattr(cfg, "rope_theta", None)
            if base is not None:
                return float(base)
    return 10000.0


def register_nexusquant_backend(engine_config, bits: int = 2, rope_base: Optional[float] = None,
                                eviction_rate: float = 0.0) -> NexusQuantPagedAttention:
    """Build the compressor and paged attention for a vLLM engine (vllm_backend.py:790-859).

    The reference then wraps vLLM's attention forward with a function that always calls the
    original (vllm_backend.py:924-941), so serving is unchanged.  Here that pass-through is
    not installed; drive NexusQuantPagedAttention.compress_and_cache / forward from the
    serving loop.  Raises ImportError without vLLM, as the reference does."""
    try:
        import vllm  # noqa: F401
    except ImportError as exc:
        raise ImportError("vLLM is not installed. Install with: pip install vllm\n"
                          "NexusQuant works without vLLM for standalone use.") from exc
    head_dim = _extract_head_dim(engine_config)
    if rope_base is None:
        rope_base = _extract_rope_base(engine_config)
    compressor = NexusQuantKVCompressor(head_dim=head_dim, bits=bits, eviction_rate=eviction_rate,
                                        rope_base=rope_base)
    return NexusQuantPagedAttention(compressor=compressor)


def compress_kv_pages(key_cache: torch.Tensor, value_cache: torch.Tensor, position_ids: torch.Tensor,
                      block_size: int = 16, bits: int = 2, rope_base: float = 10000.0) -> List[CompressedPage]:
    """(num_heads, seq_len, head_dim) K / V -> pages of block_size tokens, the last one possibly
    shorter (vllm_backend.py:968-1007).  One compress launch for the whole sequence."""
    compressor = NexusQuantKVCompressor(head_dim=key_cache.shape[-1], bits=bits, rope_base=rope_base)
    seq_len = key_cache.shape[1]
    kc, vc, ks, vs, pos = compressor._compress_tokens(key_cache, value_cache, position_ids)
    bounds = [(s, min(s + block_size, seq_len)) for s in range(0, seq_len, block_size)]
    return _split_pages(kc, vc, ks, vs, pos, bounds)


def decompress_kv_pages(pages: List[CompressedPage], compressor: Optional[NexusQuantKVCompressor] = None,
                        bits: int = 2, rope_base: float = 10000.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Pages -> (keys, values) fp16 (num_heads, total_tokens, head_dim) (vllm_backend.py:1010-1046).
    One decompress launch for all pages."""
    if not pages:
        raise ValueError("pages list is empty")
    if compressor is None:
        compressor = NexusQuantKVCompressor(head_dim=pages[0].key_codes.shape[-1], bits=bits, rope_base=rope_base)
    return compressor._decompress(torch.cat([p.key_codes for p in pages], 1),
                                  torch.cat([p.value_codes for p in pages], 1),
                                  torch.cat([p.key_scales for p in pages], 1),
                                  torch.cat([p.value_scales for p in pages], 1),
                                  torch.cat([p.positions for p in pages]))


def measure_compression_ratio(pages: List[CompressedPage], compressor: Optional[NexusQuantKVCompressor] = None,
                              bits: int = 2) -> dict:
    """ratio, compressed_mb, uncompressed_mb, bits over a list of pages (vllm_backend.py:1049-1077)."""
    total_compressed = sum(p.compressed_bytes for p in pages)
    total_uncompressed = sum(p.uncompressed_bytes for p in pages)
    if total_compressed == 0:
        return {"ratio": 1.0, "compressed_mb": 0.0, "uncompressed_mb": 0.0, "bits": bits}
    return {"ratio": total_uncompressed / total_compressed, "compressed_mb": total_compressed / (1024 * 1024),
            "uncompressed_mb": total_uncompressed / (1024 * 1024), "bits": bits}
