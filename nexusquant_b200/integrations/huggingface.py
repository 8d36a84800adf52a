"""HuggingFace integration: the ``nexusquant_evict`` context manager.

Same arguments, presets and hook semantics as the reference
(nexusquant/integrations/huggingface.py:510-807): the DynamicLayer.update /
DynamicSlidingWindowLayer.update methods of transformers are wrapped so that the
first prefill chunk of every layer is compressed once, in place, with the
layer's own keys as the scoring input (a one-layer cache per call).  The
compression itself runs on the B200 kernels (nexusquant_b200.pipeline).

One deliberate difference: with scorer="real" the importance computed before
the prefill is actually used by the hook (the reference's hook raises, because
NexusQuantEvict.compress demands a model it is never given).
"""
from __future__ import annotations

import time
import warnings
from contextlib import contextmanager
from typing import Optional

import torch

from ..pipeline import NexusQuantEvict, NexusQuantEvictTruncate

# Presets of the reference (nexusquant/integrations/huggingface.py:510-515).
_EVICT_PRESETS = {
    "high": {"eviction_rate": 0.35, "bits": 2, "key_bits": 3},
    "balanced": {"eviction_rate": 0.60, "bits": 2},
    "max": {"eviction_rate": 0.80, "bits": 2},
    "asym": {"eviction_rate": 0.60, "bits": 2, "key_bits": 3},
}


def _detect_model_config(model):
    """head_dim, num_layers, rope_base, num_kv_heads, rope_scaling of a HF model
    (nexusquant/integrations/huggingface.py:105-133)."""
    config = model.config
    text_config = getattr(config, "text_config", config)
    head_dim = getattr(text_config, "head_dim", None)
    if head_dim is None:
        head_dim = getattr(text_config, "hidden_size", 4096) // getattr(text_config, "num_attention_heads", 32)
    num_kv_heads = getattr(text_config, "num_key_value_heads", None)
    if num_kv_heads is None:
        num_kv_heads = getattr(text_config, "num_attention_heads", 32)
    rope_base = getattr(text_config, "rope_theta", None)
    if rope_base is None:
        rp = getattr(text_config, "rope_parameters", None) or {}
        rope_base = rp.get("rope_theta", 10000.0) if isinstance(rp, dict) else 10000.0
    return {
        "head_dim": head_dim,
        "num_layers": getattr(text_config, "num_hidden_layers", 32),
        "rope_base": rope_base,
        "num_kv_heads": num_kv_heads,
        "rope_scaling": getattr(text_config, "rope_scaling", None),
    }


class _CompressionStats:
    """Counts layers compressed and the fp16 bytes vs. the bytes of the compressed form
    (codes + fp16 scales, or fp16 for protected layers) of the kept tokens."""

    def __init__(self, bits: int):
        self.bits = bits
        self.reset()

    def reset(self):
        self.total_original_bytes = 0
        self.total_compressed_bytes = 0
        self.layers_compressed = 0
        self.start_time = time.time()

    def record(self, original_elems: int, compressed_bytes: float):
        self.total_original_bytes += original_elems * 2
        self.total_compressed_bytes += compressed_bytes
        self.layers_compressed += 1

    @property
    def compression_ratio(self) -> float:
        return 1.0 if self.total_compressed_bytes == 0 else self.total_original_bytes / self.total_compressed_bytes

    @property
    def memory_saved_mb(self) -> float:
        return (self.total_original_bytes - self.total_compressed_bytes) / (1024 * 1024)

    def summary(self) -> str:
        return "\n".join([
            "", "--- NexusQuant Compression Stats ---",
            f"  Compression ratio:    {self.compression_ratio:.1f}x",
            f"  Memory saved:         {self.memory_saved_mb:.1f} MB",
            f"  Layers compressed:    {self.layers_compressed}",
            f"  Wall time:            {time.time() - self.start_time:.2f}s",
            "------------------------------------"])


def _bytes_of_kept(n_kept: int, heads: int, batch: int, d: int, key_bits: int, value_bits: int) -> float:
    d_p = 1 << (d - 1).bit_length()

    def pb(bits):
        return d_p / 2 if bits <= 2 else (d_p * 5 / 8 if bits == 3 else d_p)

    return batch * heads * n_kept * (pb(key_bits) + pb(value_bits) + 4)


@contextmanager
def nexusquant_evict(model, eviction_rate=0.6, quality: str = "balanced", sliding_window: int = 32,
                     obs_window: int = 32, bits: int = 2, key_bits: int = None, value_bits: int = None,
                     truncate: bool = False, scorer: str = "key-key", input_ids=None, protected_layers: set = None,
                     protect_boundary=0, min_context_for_compression: int = 0, soft_eviction: bool = False,
                     adaptive_context: bool = False, protected_positions: Optional[torch.Tensor] = None,
                     compress_layers: str = "all", layer_bit_profile: str = "uniform", verbose: bool = True):
    """Compress the KV cache of every layer on its first prefill (see module docstring).

    Yields the compressor; ``compressor.last_mask`` (masking) or
    ``compressor.next_position`` (truncate=True) is set on the first prefill.
    """
    if quality in _EVICT_PRESETS:
        preset = _EVICT_PRESETS[quality]
        eviction_rate = preset["eviction_rate"]
        bits = preset["bits"]
        if key_bits is None and "key_bits" in preset:
            key_bits = preset["key_bits"]
        if value_bits is None and "value_bits" in preset:
            value_bits = preset["value_bits"]
    if scorer == "real":
        attn_impl = getattr(model.config, "_attn_implementation", None)
        if attn_impl != "eager":
            raise ValueError(
                f"scorer='real' requires attn_implementation='eager' but model reports "
                f"attn_implementation={attn_impl!r}. SDPA suppresses attention weights silently. "
                "Reload with: AutoModelForCausalLM.from_pretrained(..., attn_implementation='eager')")
        if input_ids is None:
            raise ValueError("scorer='real' requires input_ids to be passed to nexusquant_evict(). "
                             "These are the (batch, seq) token ids for the prefix.")
    cfg = _detect_model_config(model)
    if hasattr(model, "_offload_cache"):
        warnings.warn("NexusQuantEvict detected KV cache offloading (_offload_cache); the compression hooks "
                      "intercept DynamicCache layer updates and may not fire for offloaded cache writes.",
                      stacklevel=3)
    cls = NexusQuantEvictTruncate if truncate else NexusQuantEvict
    compressor = cls(head_dim=cfg["head_dim"], bits=bits, key_bits=key_bits, value_bits=value_bits,
                     eviction_rate=eviction_rate, sliding_window=sliding_window, obs_window=obs_window,
                     rope_base=cfg["rope_base"], rope_scaling=cfg["rope_scaling"], scorer=scorer,
                     protected_layers=protected_layers, protect_boundary=protect_boundary,
                     min_context_for_compression=min_context_for_compression, soft_eviction=soft_eviction,
                     adaptive_context=adaptive_context, protected_positions=protected_positions,
                     compress_layers=compress_layers, layer_bit_profile=layer_bit_profile)
    if compress_layers == "global_only":
        compressor.set_model_config(model.config)
    compressor.last_mask = None
    compressor.next_position = None
    cached_importance = compressor._score_importance_real(model, input_ids) if scorer == "real" else None
    stats = _CompressionStats(bits=bits)

    from transformers.cache_utils import DynamicLayer, DynamicSlidingWindowLayer
    orig_dl = DynamicLayer.update
    orig_dsw = DynamicSlidingWindowLayer.update

    class _SingleLayerCache:
        def __init__(self, k, v):
            self.key_cache = [k]
            self.value_cache = [v]

    def make_hook(original):
        def hooked_update(self, key_states, value_states, cache_kwargs=None):
            keys, values = original(self, key_states, value_states, cache_kwargs)
            if getattr(keys, "_nq_compressed", False):
                return keys, values
            incoming = key_states.shape[-2]
            existing = keys.shape[-2] - incoming
            if incoming < 2:
                return keys, values
            if existing > 0 and incoming < max(existing * 0.1, 8):
                return keys, values
            single = _SingleLayerCache(keys, values)
            imp = cached_importance
            if truncate:
                _, nxt = compressor.compress(single, importance=imp)
                compressor.next_position = nxt
                n_kept = nxt
            else:
                _, mask = compressor.compress(single, importance=imp)
                compressor.last_mask = mask
                n_kept = int(mask[0].sum().item())
            new_k, new_v = single.key_cache[0], single.value_cache[0]
            new_k._nq_compressed = True
            self.keys = new_k
            self.values = new_v
            b, h, _, d = keys.shape
            stats.record(keys.numel() + values.numel(),
                         _bytes_of_kept(n_kept, h, b, d, compressor.key_bits, compressor.value_bits))
            return new_k, new_v
        return hooked_update

    DynamicLayer.update = make_hook(orig_dl)
    DynamicSlidingWindowLayer.update = make_hook(orig_dsw)
    if verbose:
        kb, vb = compressor.key_bits, compressor.value_bits
        label = f"K={kb}-bit/V={vb}-bit E8" if kb != vb else f"{kb}-bit E8"
        ev = "auto" if eviction_rate == "auto" else f"{eviction_rate:.0%}"
        print(f"NexusQuantEvict (B200): activating (eviction={ev}, {label}, sliding_window={sliding_window}, "
              f"mode={'truncate' if truncate else 'mask'}, scorer={scorer})", flush=True)
    try:
        yield compressor
    finally:
        DynamicLayer.update = orig_dl
        DynamicSlidingWindowLayer.update = orig_dsw
        if verbose:
            print(stats.summary(), flush=True)
