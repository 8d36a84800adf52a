"""nexusquant_b200: B200-native post-prefill KV-cache compression (NexusQuant-compatible API).

    from nexusquant_b200 import compress_kv_cache, nexusquant_evict
    compress_kv_cache(past_key_values, mode="quant_only", rope_base=10000.0)
    with nexusquant_evict(model, quality="balanced"):
        model.generate(...)

The math runs in hand-written sm_100a CUDA kernels behind a C ABI
(include/nexusquant_b200.h, nexusquant_b200/_lib/libnexusquant_b200.so);
there is no CPU fallback.
"""
__version__ = "0.1.0"

from .pipeline import (  # noqa: F401
    NexusQuantSimple,
    NexusQuantQuantOnly,
    NexusQuantEvict,
    NexusQuantEvictTruncate,
    compress_kv_cache,
    compress_cache_layers,
)
from .layout import CompressedKVCache, CompressedLayer  # noqa: F401
from .integrations.huggingface import nexusquant_evict, _EVICT_PRESETS  # noqa: F401
from . import kernels  # noqa: F401

__all__ = [
    "NexusQuantSimple", "NexusQuantQuantOnly", "NexusQuantEvict", "NexusQuantEvictTruncate",
    "compress_kv_cache", "compress_cache_layers", "nexusquant_evict", "CompressedKVCache",
    "CompressedLayer", "kernels",
]
