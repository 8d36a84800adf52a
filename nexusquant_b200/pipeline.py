"""Host side of the post-prefill KV-cache compression path.

Mirrors the reference's compressor API (nexusquant/pipeline.py, v0.5.0):
``NexusQuantSimple`` (:103), ``NexusQuantQuantOnly`` (:171), ``NexusQuantEvict``
(:535), ``NexusQuantEvictTruncate`` (:1247) and ``compress_kv_cache`` (:1409),
with the same constructor arguments, return values and errors.  The per-layer
torch loops of the reference are replaced by one native launch per step
(score -> select -> compress all layers), see nexusquant_b200/kernels.py.

Two layouts:
  layout="fake_quant" (default, the reference's behaviour): reconstructed fp16
      K/V of the original shape are written back into the cache, evicted rows
      zeroed (or, for the truncating compressor, removed).
  layout="compressed": a CompressedKVCache (packed codes, fp16 scales, kept
      positions) is returned instead and the cache is left untouched.
"""
from __future__ import annotations

import math
from typing import Any, List, Optional, Sequence, Union

import torch

from . import kernels as K
from .layout import CompressedKVCache, CompressedLayer


# --------------------------------------------------------------------------- cache access
def _get_layer_kv(past_key_values, layer_idx):
    """(keys, values) of a layer: .key_cache/.value_cache lists, else .layers[l].keys/.values
    (nexusquant/pipeline.py:25-41)."""
    if hasattr(past_key_values, "key_cache") and hasattr(past_key_values, "value_cache"):
        return past_key_values.key_cache[layer_idx], past_key_values.value_cache[layer_idx]
    layer = past_key_values.layers[layer_idx]
    return getattr(layer, "keys"), getattr(layer, "values")


def _set_layer_kv(past_key_values, layer_idx, keys, values):
    """Write a layer back (nexusquant/pipeline.py:44-59)."""
    if hasattr(past_key_values, "key_cache") and hasattr(past_key_values, "value_cache"):
        past_key_values.key_cache[layer_idx] = keys
        past_key_values.value_cache[layer_idx] = values
        return
    layer = past_key_values.layers[layer_idx]
    setattr(layer, "keys", keys)
    setattr(layer, "values", values)


def _num_layers(past_key_values):
    if hasattr(past_key_values, "key_cache"):
        return len(past_key_values.key_cache)
    return len(past_key_values.layers)


def _swa_layers_from_config(model_config) -> set:
    """SWA layer detection of NexusQuantEvict.set_model_config (nexusquant/pipeline.py:646-691)."""
    cfg = getattr(model_config, "text_config", model_config)
    swa = set()
    n_layers = getattr(cfg, "num_hidden_layers", 32)
    pattern = getattr(cfg, "sliding_window_pattern", None)
    if pattern is not None:
        for i in range(n_layers):
            if (i + 1) % pattern != 0:
                swa.add(i)
    layer_types = getattr(cfg, "layer_types", None)
    if layer_types is not None and not swa:
        for i, lt in enumerate(layer_types):
            if lt in ("sliding_window", "local", "swa", "sliding_attention"):
                swa.add(i)
    n_shared = getattr(cfg, "num_kv_shared_layers", 0)
    if n_shared > 0 and not swa:
        for i in range(n_layers - n_shared, n_layers):
            swa.add(i)
    return swa


def n_keep_for(seq: int, sliding_window: int, eviction_rate: float) -> int:
    """max(1, int(prefix * (1.0 - rate))) in IEEE double, as pipeline.py:918-920."""
    prefix = max(seq - sliding_window, 0)
    return max(1, int(prefix * (1.0 - eviction_rate)))


def kept_capacity(seq: int, sliding_window: int, n_keep: int, n_protected: int = 0) -> int:
    """Number of kept tokens per batch row (exact without protected positions, else an upper bound)."""
    if seq <= 0:
        return 0
    prefix = max(seq - sliding_window, 0)
    win_lo = max(0, seq - sliding_window) if sliding_window > 0 else seq
    w = seq - win_lo
    bos = 1 if win_lo > 0 else 0
    k = min(n_keep, prefix - 1) if prefix > 1 and n_keep > 0 else 0
    return min(seq, k + w + bos + n_protected)


def _group_layers(tensors: Sequence[torch.Tensor], idx: Sequence[int]):
    """Group layer indices whose tensors share shape, dtype, device and strides (one launch each)."""
    groups = {}
    for i in idx:
        t = tensors[i]
        key = (tuple(t.shape), t.dtype, str(t.device), tuple(t.stride()))
        groups.setdefault(key, []).append(i)
    return list(groups.values())


def _mask_from_kept(kept_idx: torch.Tensor, kept_count: torch.Tensor, seq: int) -> torch.Tensor:
    b, cap = kept_idx.shape
    valid = torch.arange(cap, device=kept_idx.device)[None, :] < kept_count[:, None].long()
    mask = torch.zeros(b, seq + 1, dtype=torch.float32, device=kept_idx.device)
    idx = torch.where(valid, kept_idx.long(), torch.full_like(kept_idx.long(), seq))
    mask.scatter_(1, idx, 1.0)
    return mask[:, :seq].contiguous()


def compress_cache_layers(keys: Sequence[torch.Tensor], values: Sequence[torch.Tensor], *,
                          key_levels: Union[int, Sequence[int]], value_levels: Union[int, Sequence[int]],
                          kept_idx: Optional[torch.Tensor] = None, kept_count: Optional[torch.Tensor] = None,
                          n_kept: Optional[int] = None, protected: Sequence[int] = (),
                          rope_base: float = 10000.0, rope_scaling: Optional[dict] = None,
                          position_offset: int = 0, mask: Optional[torch.Tensor] = None,
                          device: Optional[Union[int, str, torch.device]] = None, result_on_host: bool = False,
                          out: Optional[CompressedKVCache] = None, group_layers: int = 8) -> CompressedKVCache:
    """Compress a whole cache to the compressed layout: quantized layers in one launch per
    shape group, protected layers gathered to fp16.

    The layers may sit in pinned host memory (pass ``device=``, default the current CUDA
    device): only the kept rows then cross PCIe.  With ``result_on_host`` the compressed cache
    is returned in pinned host memory, layer group by layer group (``group_layers`` layers
    each), the copy of one group overlapping the gather and compression of the next; ``out``
    (a cache this function returned before, same shapes) is written into instead of
    allocating new host buffers."""
    L = len(keys)
    k0 = keys[0]
    b, h, seq, d = k0.shape
    host_in = not k0.is_cuda
    if host_in:
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = k0.device
    if kept_idx is None:
        n_kept = seq if n_kept is None else n_kept
        kept_idx = torch.arange(n_kept, dtype=torch.int32, device=dev).expand(b, n_kept).contiguous()
        if kept_count is None:
            kept_count = torch.full((b,), n_kept, dtype=torch.int32, device=dev)
    else:
        n_kept = kept_idx.shape[1] if n_kept is None else n_kept
        kept_idx = kept_idx[:, :n_kept].contiguous()
    if kept_count is None:
        kept_count = torch.full((b,), n_kept, dtype=torch.int32, device=dev)
    positions = kept_idx if position_offset == 0 else (kept_idx + position_offset)
    klv = K._levels_list(key_levels, L)
    vlv = K._levels_list(value_levels, L)
    prot = set(protected)
    quant = [i for i in range(L) if i not in prot]
    if result_on_host:
        return _compress_to_host(keys, values, quant, sorted(i for i in prot if i < L), klv, vlv, kept_idx,
                                 kept_count, n_kept, positions, rope_base, rope_scaling, mask, dev, group_layers, out)
    layers: List[Optional[CompressedLayer]] = [None] * L
    for grp in _group_layers(keys, quant):
        codes = K.compress_layers([keys[i] for i in grp], [values[i] for i in grp],
                                  key_levels=[klv[i] for i in grp], value_levels=[vlv[i] for i in grp],
                                  kept_idx=kept_idx, kept_count=kept_count, positions=positions,
                                  rope_base=rope_base, rope_scaling=rope_scaling, device=dev if host_in else None)
        for i, c in zip(grp, codes):
            layers[i] = CompressedLayer(codes=c)
    for i in sorted(prot):
        if i >= L:
            continue
        layers[i] = CompressedLayer(
            k_fp16=K.gather_rows(keys[i], kept_idx, n_kept, kept_count, device=dev if host_in else None),
            v_fp16=K.gather_rows(values[i], kept_idx, n_kept, kept_count, device=dev if host_in else None))
    return CompressedKVCache(layers, positions.to(torch.int32), kept_count, seq, b, h, d, rope_base=rope_base,
                             rope_scaling=rope_scaling, mask=mask)


_COPY_STREAMS = {}


def _copy_stream(dev: torch.device) -> torch.cuda.Stream:
    s = _COPY_STREAMS.get(str(dev))
    if s is None:
        s = _COPY_STREAMS[str(dev)] = torch.cuda.Stream(dev)
    return s


def _pinned_like(t: torch.Tensor) -> torch.Tensor:
    return torch.empty(t.shape, dtype=t.dtype, pin_memory=True)


def _compress_to_host(keys, values, quant, prot, klv, vlv, kept_idx, kept_count, n_kept, positions, rope_base,
                      rope_scaling, mask, dev, group_layers, out) -> CompressedKVCache:
    """compress_cache_layers(result_on_host=True): per group of layers, gather + compress on the
    current stream, then copy the group's codes to pinned host memory on a second stream while
    the next group is processed.  Device buffers of a group are released to the caching
    allocator only after their copy (record_stream)."""
    L = len(keys)
    b, h, seq, d = keys[0].shape
    comp = torch.cuda.current_stream(dev)
    cp = _copy_stream(dev)
    host_in = not keys[0].is_cuda
    layers: List[Optional[CompressedLayer]] = [None] * L if out is None else list(out.layers)

    def to_host(src: torch.Tensor, dst: Optional[torch.Tensor]) -> torch.Tensor:
        if dst is None:
            dst = _pinned_like(src)
        elif dst.shape != src.shape or dst.dtype != src.dtype:
            raise ValueError("out= does not match the shapes of this cache")
        dst.copy_(src, non_blocking=True)
        src.record_stream(cp)
        return dst

    def flush(done: List[int], made: dict):
        ev = torch.cuda.Event()
        ev.record(comp)
        cp.wait_event(ev)
        with torch.cuda.stream(cp):
            for i in done:
                prev = layers[i]
                if i in made and isinstance(made[i], K.LayerCodes):
                    c = made[i]
                    pc = prev.codes if prev is not None and not prev.protected else None
                    layers[i] = CompressedLayer(codes=K.LayerCodes(
                        to_host(c.k_codes, pc.k_codes if pc else None), to_host(c.v_codes, pc.v_codes if pc else None),
                        to_host(c.k_scales, pc.k_scales if pc else None),
                        to_host(c.v_scales, pc.v_scales if pc else None), c.key_levels, c.value_levels))
                else:
                    kf, vf = made[i]
                    pk_ = prev.k_fp16 if prev is not None and prev.protected else None
                    pv_ = prev.v_fp16 if prev is not None and prev.protected else None
                    layers[i] = CompressedLayer(k_fp16=to_host(kf, pk_), v_fp16=to_host(vf, pv_))

    # protected layers first: their fp16 rows are the largest copies back, and issued first
    # they travel while the quantized groups are gathered and compressed
    for i in prot:
        kf = K.gather_rows(keys[i], kept_idx, n_kept, kept_count, device=dev if host_in else None)
        vf = K.gather_rows(values[i], kept_idx, n_kept, kept_count, device=dev if host_in else None)
        flush([i], {i: (kf, vf)})
    groups = [quant[i:i + group_layers] for i in range(0, len(quant), max(1, group_layers))]
    for grp in groups:
        for sub in _group_layers(keys, grp):
            codes = K.compress_layers([keys[i] for i in sub], [values[i] for i in sub],
                                      key_levels=[klv[i] for i in sub], value_levels=[vlv[i] for i in sub],
                                      kept_idx=kept_idx, kept_count=kept_count, positions=positions,
                                      rope_base=rope_base, rope_scaling=rope_scaling,
                                      device=dev if host_in else None)
            flush(sub, dict(zip(sub, codes)))
    done = torch.cuda.Event()
    done.record(cp)
    comp.wait_event(done)  # the caller's stream (and a synchronize on it) covers the copies
    pos_h = out.positions if out is not None else torch.empty((b, n_kept), dtype=torch.int32, pin_memory=True)
    cnt_h = out.kept_count if out is not None else torch.empty((b,), dtype=torch.int32, pin_memory=True)
    pos_h.copy_(positions.to(torch.int32), non_blocking=True)
    cnt_h.copy_(kept_count.to(torch.int32), non_blocking=True)
    return CompressedKVCache(layers, pos_h, cnt_h, seq, b, h, d, rope_base=rope_base, rope_scaling=rope_scaling,
                             mask=mask)


# --------------------------------------------------------------------------- compressors
class _QuantBase:
    """Shared fake-quant / compressed-layout driver for the no-eviction compressors."""

    def _compress_all(self, past_key_values, skip: set, key_levels: int, value_levels: int):
        n_layers = _num_layers(past_key_values)
        ks, vs = zip(*[_get_layer_kv(past_key_values, l) for l in range(n_layers)]) if n_layers else ((), ())
        todo = [l for l in range(n_layers) if l not in skip]
        if self.layout == "compressed":
            return compress_cache_layers(list(ks), list(vs), key_levels=key_levels, value_levels=value_levels,
                                         protected=sorted(skip), rope_base=self.rope_base,
                                         rope_scaling=self.rope_scaling)
        for grp in _group_layers(ks, todo):
            outs_k = [torch.empty(ks[l].shape, dtype=torch.float16, device=ks[l].device) for l in grp]
            outs_v = [torch.empty(vs[l].shape, dtype=torch.float16, device=vs[l].device) for l in grp]
            K.compress_layers([ks[l] for l in grp], [vs[l] for l in grp], key_levels=key_levels,
                              value_levels=value_levels, rope_base=self.rope_base, rope_scaling=self.rope_scaling,
                              emit_codes=False, recon_k=outs_k, recon_v=outs_v,
                              key_sharpen=K.SHARPEN if self.sharpen else 1.0)
            for l, ok, ov in zip(grp, outs_k, outs_v):
                _set_layer_kv(past_key_values, l, ok, ov)
        return past_key_values


class NexusQuantSimple(_QuantBase):
    """RoPE removal + Hadamard + E8 (nexusquant/pipeline.py:103-168), same bits for K and V."""

    def __init__(self, head_dim: int = 128, bits: int = 3, rope_base: float = 10000.0,
                 rope_scaling: dict = None, merge_pct: float = 0.0, layout: str = "fake_quant",
                 sharpen: bool = False):
        if merge_pct:
            raise NotImplementedError("merge_pct > 0 (token merging) is not part of the B200 compression path")
        self.head_dim = head_dim
        self.bits = bits
        self.levels = 2 ** bits
        self.rope_base = rope_base
        self.rope_scaling = rope_scaling
        self.merge_pct = merge_pct
        self.layout = layout
        self.sharpen = sharpen

    @property
    def H(self) -> torch.Tensor:
        """The orthonormal Hadamard matrix the kernels apply (for inspection only)."""
        n = K.next_pow2(self.head_dim)
        h = torch.ones(1, 1)
        while h.shape[0] < n:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
        return h / math.sqrt(n)

    def compress(self, past_key_values) -> Any:
        return self._compress_all(past_key_values, set(), self.levels, self.levels)


class NexusQuantQuantOnly(_QuantBase):
    """Quantization only (nexusquant/pipeline.py:171-265).  ``key_bits`` / ``value_bits``
    extend the reference's single ``bits`` (K3V2 = key_bits=3, value_bits=2)."""

    def __init__(self, bits: int = 3, rope_base: float = 10000.0, rope_scaling: dict = None,
                 compress_layers: str = "all", key_bits: Optional[int] = None, value_bits: Optional[int] = None,
                 layout: str = "fake_quant", sharpen: bool = False):
        self.bits = bits
        self.levels = 2 ** bits
        self.key_bits = key_bits if key_bits is not None else bits
        self.value_bits = value_bits if value_bits is not None else bits
        self.rope_base = rope_base
        self.rope_scaling = rope_scaling
        self.compress_layers = compress_layers
        self.layout = layout
        self.sharpen = sharpen
        self._swa_layer_indices = None

    def set_model_config(self, model_config):
        if self.compress_layers != "global_only":
            return
        self._swa_layer_indices = _swa_layers_from_config(model_config)

    def compress(self, past_key_values) -> Any:
        skip = self._swa_layer_indices or set()
        return self._compress_all(past_key_values, skip, 2 ** self.key_bits, 2 ** self.value_bits)


class NexusQuantEvict:
    """Token eviction + quantization (nexusquant/pipeline.py:535-1244); same arguments."""

    def __init__(self, head_dim: int = 128, bits: int = 2, key_bits: int = None, value_bits: int = None,
                 eviction_rate: Union[float, str] = 0.6, sliding_window: int = 32, obs_window: int = 32,
                 rope_base: float = 10000.0, rope_scaling: dict = None, scorer: str = "key-key",
                 protected_layers: set = None, protect_boundary: Union[int, str] = 0,
                 min_context_for_compression: int = 0, soft_eviction: bool = False,
                 adaptive_context: bool = False, protected_positions: Optional[torch.Tensor] = None,
                 compress_layers: str = "all", layer_bit_profile: str = "uniform",
                 distance_graduated: bool = False, merge_eviction: bool = False,
                 layout: str = "fake_quant", sharpen: bool = False, device=None, result_on_host: bool = False,
                 group_layers: int = 8):
        if scorer not in ("key-key", "real"):
            raise ValueError(f"scorer must be 'key-key' or 'real', got {scorer!r}")
        if not (isinstance(eviction_rate, (int, float)) or eviction_rate == "auto"):
            raise ValueError(f"eviction_rate must be a float in [0, 1] or 'auto', got {eviction_rate!r}")
        if not (isinstance(protect_boundary, int) or protect_boundary == "auto"):
            raise ValueError(f"protect_boundary must be a non-negative int or 'auto', got {protect_boundary!r}")
        if layout not in ("fake_quant", "compressed"):
            raise ValueError(f"layout must be 'fake_quant' or 'compressed', got {layout!r}")
        self.head_dim = head_dim
        self.bits = bits
        self.key_bits = key_bits if key_bits is not None else bits
        self.value_bits = value_bits if value_bits is not None else bits
        self.key_levels = 2 ** self.key_bits
        self.value_levels = 2 ** self.value_bits
        self.levels = 2 ** bits
        self.eviction_rate = eviction_rate
        self.sliding_window = sliding_window
        self.obs_window = obs_window
        self.rope_base = rope_base
        self.rope_scaling = rope_scaling
        self.scorer = scorer
        self.protected_layers = set(protected_layers) if protected_layers else set()
        self.protect_boundary = protect_boundary
        self.min_context_for_compression = min_context_for_compression
        self.soft_eviction = soft_eviction
        self.adaptive_context = adaptive_context
        self.protected_positions = protected_positions
        self.compress_layers = compress_layers
        self.layer_bit_profile = layer_bit_profile
        self.distance_graduated = distance_graduated
        self.merge_eviction = merge_eviction
        self.layout = layout
        self.sharpen = sharpen
        # caches in pinned host memory: the device that compresses them, and whether the
        # compressed cache comes back to pinned host memory (layout="compressed" only)
        self.device = device
        self.result_on_host = result_on_host
        self.group_layers = group_layers
        self._host_out: Optional[CompressedKVCache] = None
        self._swa_layer_indices = None
        self.last_compressed: Optional[CompressedKVCache] = None

    # ----------------------------------------------------------------- config
    def set_model_config(self, model_config):
        if self.compress_layers != "global_only":
            return
        self._swa_layer_indices = _swa_layers_from_config(model_config)

    def _reusable_host_out(self, n_layers: int, b: int, cap: int) -> Optional[CompressedKVCache]:
        """The previous host-resident result, written into again when the shapes agree (pinned host
        allocation is slow); the caller must be done with it before compressing again."""
        o = self._host_out
        if not self.result_on_host or o is None:
            return None
        if len(o.layers) != n_layers or o.batch != b or o.n_kept != cap:
            return None
        return o

    def _find_scoring_layer(self, past_key_values, n_layers: int) -> int:
        """First global layer for hybrid models, else 0 (nexusquant/pipeline.py:726-738)."""
        if self.compress_layers == "global_only" and self._swa_layer_indices:
            for l in range(n_layers):
                if l not in self._swa_layer_indices:
                    return l
        return 0

    def _resolve_layer_levels(self, layer_idx: int, n_layers: int):
        """Graduated bit profile (nexusquant/pipeline.py:740-754)."""
        if self.layer_bit_profile == "graduated":
            boundary_count = max(1, int(n_layers * 0.15))
            if layer_idx < boundary_count or layer_idx >= n_layers - boundary_count:
                return 8, 8
        return self.key_levels, self.value_levels

    # ---------------------------------------------------------------- scoring
    def _score_importance(self, keys: torch.Tensor) -> torch.Tensor:
        """Key-key importance on the device (nexusquant/pipeline.py:756-782) -> (b, seq) fp32."""
        return K.score_keykey(keys, self.obs_window)

    def _score_importance_real(self, model, input_ids: torch.Tensor) -> torch.Tensor:
        """Real attention importance (nexusquant/pipeline.py:784-836): per layer, the causal
        softmax of every query against every key, summed over queries, averaged over heads,
        then averaged over layers.  The forward pass only records each layer's rotated queries
        and keys; the column sums run on the tensor-core scorer in blocks of 64 queries, so no
        (b, H, T, T) attention tensor is ever formed.  Models whose attention does not call a
        module-level ``apply_rotary_pos_emb`` use the reference's eager-attention route."""
        imp = _real_importance_recorded(model, input_ids)
        if imp is not None:
            return imp
        with torch.no_grad():
            out = model(input_ids, use_cache=False, output_attentions=True)
        attentions = out.attentions
        if attentions is None or len(attentions) == 0 or attentions[0] is None:
            raise RuntimeError(
                "output_attentions=True returned None. Load the model with attn_implementation='eager' to get "
                "real attention weights. SDPA (the default) suppresses attention weight output regardless of "
                "this flag.")
        b, seq = input_ids.shape
        importance = torch.zeros(b, seq, dtype=torch.float32, device=input_ids.device)
        for layer_attn in attentions:
            importance += layer_attn.float().sum(dim=2).mean(dim=1)
        return importance / len(attentions)

    def _compute_adaptive_eviction_rate(self, importance: torch.Tensor, seq: int) -> float:
        """Entropy-based rate in [0.1, 0.7] (nexusquant/pipeline.py:838-861)."""
        probs = importance[0] / (importance[0].sum() + 1e-8)
        entropy = -(probs * (probs + 1e-8).log()).sum().item()
        max_entropy = math.log(max(seq, 2))
        rate = 0.7 - 0.5 * (entropy / max_entropy)
        return max(0.1, min(0.7, rate))

    def _auto_detect_boundary(self, past_key_values) -> int:
        """2 when the first/last layers' keys are >2x brighter than the middle (pipeline.py:863-893)."""
        if hasattr(self, "_auto_boundary_cached"):
            return self._auto_boundary_cached
        n_layers = _num_layers(past_key_values)
        if n_layers < 6:
            self._auto_boundary_cached = 0
            return 0
        k_first, _ = _get_layer_kv(past_key_values, 0)
        k_last, _ = _get_layer_kv(past_key_values, n_layers - 1)
        k_mid, _ = _get_layer_kv(past_key_values, n_layers // 2)
        mag_b = (k_first.float().abs().mean() + k_last.float().abs().mean()) / 2
        mag_m = k_mid.float().abs().mean()
        self._auto_boundary_cached = 2 if (mag_b / (mag_m + 1e-8)).item() > 2.0 else 0
        return self._auto_boundary_cached

    def _skip_layers(self, past_key_values, n_layers: int) -> set:
        n_protect = (self._auto_detect_boundary(past_key_values) if self.protect_boundary == "auto"
                     else int(self.protect_boundary))
        skip = set(self.protected_layers)
        if n_protect > 0:
            for i in range(min(n_protect, n_layers)):
                skip.add(i)
                skip.add(n_layers - 1 - i)
        if self.compress_layers == "global_only" and self._swa_layer_indices:
            skip.update(self._swa_layer_indices)
        return skip

    def _resolve_rate(self, importance, seq: int) -> float:
        rate = (self._compute_adaptive_eviction_rate(importance, seq) if self.eviction_rate == "auto"
                else float(self.eviction_rate))
        if self.adaptive_context:
            if seq < 256:
                rate = 0.0
            elif seq < 512:
                rate *= 0.5
            elif seq < 1024:
                rate *= 0.75
        return rate

    def _keep_set(self, importance: torch.Tensor, seq: int, eviction_rate: float):
        """(kept_idx [b, cap], kept_count [b], cap) on the device."""
        if self.distance_graduated and max(seq - self.sliding_window, 0) > 1:
            prefix = max(seq - self.sliding_window, 0)
            ramp = torch.linspace(0.0, 1.0, prefix - 1, device=importance.device)
            importance = importance.clone()
            importance[:, 1:prefix] = importance[:, 1:prefix] + ramp * importance[:, 1:prefix].max() * 0.25
        nk = n_keep_for(seq, self.sliding_window, eviction_rate)
        prot = self.protected_positions
        n_prot = 0 if prot is None else len(prot)
        idx, cnt = K.select_keep(importance, self.sliding_window, nk, prot)
        cap = kept_capacity(seq, self.sliding_window, nk, n_prot)
        return idx, cnt, cap

    def _build_keep_mask(self, importance: torch.Tensor, seq: int, eviction_rate: float = None) -> torch.Tensor:
        """(b, seq) bool keep mask (nexusquant/pipeline.py:895-959), computed on the device."""
        if eviction_rate is None:
            eviction_rate = self.eviction_rate
        if not isinstance(eviction_rate, (int, float)):
            raise ValueError(
                f"_build_keep_mask requires a resolved float eviction_rate, got {eviction_rate!r}. "
                "If self.eviction_rate == 'auto', resolve it via _compute_adaptive_eviction_rate() first.")
        idx, cnt, _ = self._keep_set(importance, seq, float(eviction_rate))
        return _mask_from_kept(idx, cnt, seq) > 0

    # --------------------------------------------------------------- compress
    def _importance(self, past_key_values, n_layers, model, input_ids, importance):
        if importance is not None:
            return importance
        score_layer = self._find_scoring_layer(past_key_values, n_layers)
        k_score, _ = _get_layer_kv(past_key_values, score_layer)
        if self.scorer == "real":
            if model is None or input_ids is None:
                raise ValueError(
                    "scorer='real' requires model and input_ids to be passed to compress(). "
                    "Also ensure the model was loaded with attn_implementation='eager'.")
            return self._score_importance_real(model, input_ids)
        return self._score_importance(k_score)

    def _compute_device(self, k_score: torch.Tensor) -> torch.device:
        if k_score.is_cuda:
            return k_score.device
        if self.layout != "compressed":
            raise ValueError("a cache in host memory needs layout='compressed' (the fake-quant layout writes "
                             "fp16 tensors of the original shape back into the cache)")
        if not k_score.is_pinned():
            raise RuntimeError("a cache in host memory must be in pinned memory")
        dev = torch.device(self.device) if self.device is not None else torch.device("cuda")
        return torch.device("cuda", torch.cuda.current_device()) if dev.index is None else dev

    def compress(self, past_key_values, model=None, input_ids=None, importance: Optional[torch.Tensor] = None):
        """Evict + quantize.  Returns (past_key_values, prefix_attention_mask (b, seq) float) in the
        fake-quant layout, or (CompressedKVCache, mask) with layout="compressed".  With
        layout="compressed" the cache may sit in pinned host memory: the scoring layer's keys are
        copied to ``device``, only kept rows of the other layers cross PCIe, and with
        ``result_on_host`` the compressed cache comes back in pinned host memory."""
        n_layers = _num_layers(past_key_values)
        score_layer = self._find_scoring_layer(past_key_values, n_layers)
        k_score, _ = _get_layer_kv(past_key_values, score_layer)
        device = self._compute_device(k_score)
        host_in = not k_score.is_cuda
        b, _, seq, _ = k_score.shape
        if importance is None and host_in:
            if self.scorer == "real":
                raise ValueError("scorer='real' with a host-resident cache: pass importance=")
            importance = self._score_importance(k_score.to(device, non_blocking=True))
        importance = self._importance(past_key_values, n_layers, model, input_ids, importance)
        importance = importance.to(device)
        rate = self._resolve_rate(importance, seq)
        kept_idx, kept_count, cap = self._keep_set(importance, seq, rate)
        mask = _mask_from_kept(kept_idx, kept_count, seq)
        skip = self._skip_layers(past_key_values, n_layers)
        if self.min_context_for_compression > 0 and seq < self.min_context_for_compression:
            return past_key_values, torch.ones(b, seq, device=device)
        levels = [self._resolve_layer_levels(l, n_layers) for l in range(n_layers)]
        ks, vs = zip(*[_get_layer_kv(past_key_values, l) for l in range(n_layers)])
        if self.merge_eviction and not self.soft_eviction:
            if host_in:
                raise NotImplementedError("merge_eviction with a host-resident cache")
            # value merging before hard eviction (pipeline.py:1185-1187), on copies of the
            # full-length layers as the reference writes merged clones into the cache
            vs = [v.clone() if v.shape[2] == seq else v for v in vs]
            K.merge_evicted_values(vs, mask > 0, importance)
        if self.layout == "compressed":
            if self.soft_eviction:
                raise NotImplementedError("soft_eviction has no compressed layout (all tokens stay visible)")
            out = compress_cache_layers(list(ks), list(vs), key_levels=[lv[0] for lv in levels],
                                        value_levels=[lv[1] for lv in levels], kept_idx=kept_idx,
                                        kept_count=kept_count, n_kept=cap, protected=sorted(skip),
                                        rope_base=self.rope_base, rope_scaling=self.rope_scaling, mask=mask,
                                        device=device, result_on_host=self.result_on_host,
                                        out=self._reusable_host_out(n_layers, b, cap),
                                        group_layers=self.group_layers)
            if self.result_on_host:
                self._host_out = out
            self.last_compressed = out
            return out, mask
        todo = [l for l in range(n_layers) if l not in skip]
        sharpen = K.SHARPEN if self.sharpen else 1.0
        if self.soft_eviction:
            ones = torch.ones(b, seq, dtype=torch.float32, device=device)
            ev_order = torch.argsort(mask, dim=1, stable=True).to(torch.int32)  # evicted (0) first, ascending
            ev_count = (seq - kept_count).to(torch.int32)
            for l in skip:
                _set_layer_kv(past_key_values, l, ks[l].half(), vs[l].half())
            for grp in _group_layers(ks, todo):
                ok = [torch.empty(ks[l].shape, dtype=torch.float16, device=device) for l in grp]
                ov = [torch.empty(vs[l].shape, dtype=torch.float16, device=device) for l in grp]
                common = dict(rope_base=self.rope_base, rope_scaling=self.rope_scaling, emit_codes=False,
                              recon_k=ok, recon_v=ov, key_sharpen=sharpen)
                K.compress_layers([ks[l] for l in grp], [vs[l] for l in grp],
                                  key_levels=[levels[l][0] for l in grp], value_levels=[levels[l][1] for l in grp],
                                  kept_idx=kept_idx[:, :cap], kept_count=kept_count, **common)
                K.compress_layers([ks[l] for l in grp], [vs[l] for l in grp], key_levels=2, value_levels=2,
                                  kept_idx=ev_order, kept_count=ev_count, **common)
                for l, a, c in zip(grp, ok, ov):
                    _set_layer_kv(past_key_values, l, a, c)
            return past_key_values, ones
        mask4 = mask[:, None, :, None]
        for l in skip:
            if l < n_layers:
                _set_layer_kv(past_key_values, l, (ks[l].float() * mask4[:, :, :ks[l].shape[2]]).half(),
                              (vs[l].float() * mask4[:, :, :vs[l].shape[2]]).half())
        for grp in _group_layers(ks, todo):
            seq_l = ks[grp[0]].shape[2]
            ok = [torch.zeros(ks[l].shape, dtype=torch.float16, device=device) for l in grp]
            ov = [torch.zeros(vs[l].shape, dtype=torch.float16, device=device) for l in grp]
            kidx, kcnt, kcap = kept_idx[:, :cap], kept_count, cap
            if seq_l != seq:  # shorter (sliding-window) layer: keep set clipped to its length
                kidx, kcnt, kcap = _clip_keep(kept_idx, kept_count, cap, seq_l)
            K.compress_layers([ks[l] for l in grp], [vs[l] for l in grp],
                              key_levels=[levels[l][0] for l in grp], value_levels=[levels[l][1] for l in grp],
                              kept_idx=kidx, kept_count=kcnt, rope_base=self.rope_base,
                              rope_scaling=self.rope_scaling, emit_codes=False, recon_k=ok, recon_v=ov,
                              key_sharpen=sharpen)
            for l, a, c in zip(grp, ok, ov):
                _set_layer_kv(past_key_values, l, a, c)
        return past_key_values, mask


def _rotary_module(model):
    """The modeling module whose attention calls a module-level apply_rotary_pos_emb, if any."""
    import sys
    for m in model.modules():
        name = type(m).__name__
        if name.endswith("Attention"):
            mod = sys.modules.get(type(m).__module__)
            if mod is not None and callable(getattr(mod, "apply_rotary_pos_emb", None)):
                return mod
    return None


def _real_importance_recorded(model, input_ids: torch.Tensor, block: int = 64) -> Optional[torch.Tensor]:
    """Importance of _score_importance_real from recorded per-layer queries and keys (see there);
    None when the model's rotary embedding cannot be intercepted."""
    mod = _rotary_module(model)
    if mod is None:
        return None
    orig = mod.apply_rotary_pos_emb
    rec = []

    def recording(q, k, *args, **kwargs):
        qe, ke = orig(q, k, *args, **kwargs)
        rec.append((qe.detach(), ke.detach()))
        return qe, ke

    mod.apply_rotary_pos_emb = recording
    try:
        with torch.no_grad():
            model(input_ids, use_cache=False)
    finally:
        mod.apply_rotary_pos_emb = orig
    if not rec:
        return None
    b, T = input_ids.shape
    imp = torch.zeros(b, T, dtype=torch.float32, device=input_ids.device)
    for q, k in rec:
        if q.shape[2] != T or k.shape[2] != T:
            return None  # not a plain prefill of the whole sequence
        q = q.to(input_ids.device)
        k = k.to(input_ids.device)
        for q0 in range(0, T, block):
            q1 = min(T, q0 + block)  # keys past the block's last query are masked: leave them out
            part = K.score_attention(q[:, :, q0:q1], k[:, :, :q1], q0)
            imp[:, :q1] += part
    return imp / len(rec)


def _clip_keep(kept_idx, kept_count, cap, seq_l):
    idx = kept_idx[:, :cap].long()
    valid = (torch.arange(cap, device=idx.device)[None] < kept_count[:, None].long()) & (idx < seq_l)
    cnt = valid.sum(1).to(torch.int32)
    order = torch.argsort((~valid).to(torch.int8), dim=1, stable=True)
    out = torch.gather(idx, 1, order).to(torch.int32)
    return out.contiguous(), cnt, cap


class NexusQuantEvictTruncate(NexusQuantEvict):
    """Physical truncation with contiguous RoPE re-encoding (nexusquant/pipeline.py:1247-1406).
    Returns (past_key_values, n_kept)."""

    def compress(self, past_key_values, importance: Optional[torch.Tensor] = None):
        n_layers = _num_layers(past_key_values)
        score_layer = self._find_scoring_layer(past_key_values, n_layers)
        k_score, _ = _get_layer_kv(past_key_values, score_layer)
        b, _, seq, _ = k_score.shape
        if b > 1:
            raise ValueError(
                f"NexusQuantEvictTruncate does not support batch_size > 1 (got {b}). "
                "Physical truncation requires identical sequence lengths across batch elements. "
                "Use NexusQuantEvict (masking, not truncation) for batched inference.")
        if importance is None:
            importance = self._score_importance(k_score)
        rate = self._resolve_rate(importance, seq)
        kept_idx, kept_count, cap = self._keep_set(importance, seq, rate)
        n_kept = int(kept_count[0].item())
        skip = self._skip_layers(past_key_values, n_layers)
        if self.min_context_for_compression > 0 and seq < self.min_context_for_compression:
            return past_key_values, seq
        kidx = kept_idx[:, :n_kept].contiguous()
        ks, vs = zip(*[_get_layer_kv(past_key_values, l) for l in range(n_layers)])
        levels = [self._resolve_layer_levels(l, n_layers) for l in range(n_layers)]
        if self.layout == "compressed":
            out = compress_cache_layers(list(ks), list(vs), key_levels=[lv[0] for lv in levels],
                                        value_levels=[lv[1] for lv in levels], kept_idx=kidx,
                                        kept_count=kept_count, n_kept=n_kept, protected=sorted(skip),
                                        rope_base=self.rope_base, rope_scaling=self.rope_scaling)
            self.last_compressed = out
            return out, n_kept
        for l in sorted(skip):
            if l < n_layers:
                _set_layer_kv(past_key_values, l, K.gather_rows(ks[l], kidx, n_kept),
                              K.gather_rows(vs[l], kidx, n_kept))
        todo = [l for l in range(n_layers) if l not in skip]
        for grp in _group_layers(ks, todo):
            dev = ks[grp[0]].device
            h, d = ks[grp[0]].shape[1], ks[grp[0]].shape[3]
            ok = [torch.empty((b, h, n_kept, d), dtype=torch.float16, device=dev) for _ in grp]
            ov = [torch.empty((b, h, n_kept, d), dtype=torch.float16, device=dev) for _ in grp]
            K.compress_layers([ks[l] for l in grp], [vs[l] for l in grp],
                              key_levels=[levels[l][0] for l in grp], value_levels=[levels[l][1] for l in grp],
                              kept_idx=kidx, rope_base=self.rope_base, rope_scaling=self.rope_scaling,
                              emit_codes=False, recon_k=ok, recon_v=ov, recon_rows="kept",
                              key_sharpen=K.SHARPEN if self.sharpen else 1.0)
            for l, a, c in zip(grp, ok, ov):
                _set_layer_kv(past_key_values, l, a, c)
        if hasattr(past_key_values, "_seen_tokens"):
            past_key_values._seen_tokens = n_kept
        return past_key_values, n_kept


def compress_kv_cache(past_key_values, mode: str = "simple", head_dim: int = 128, **kwargs) -> Any:
    """Convenience entry (nexusquant/pipeline.py:1409-1468).

    mode "simple" (default) and "quant_only" run on the B200 kernels; "quant_only"
    additionally accepts key_bits / value_bits and layout="compressed".  The
    calibration modes "max" / "asymmetric" and the deprecated "fast" mode are not
    part of this compression path and raise NotImplementedError.
    """
    if mode == "simple":
        nq = NexusQuantSimple(head_dim=head_dim, bits=kwargs.get("bits", 3),
                              rope_base=kwargs.get("rope_base", 10000.0),
                              rope_scaling=kwargs.get("rope_scaling", None),
                              merge_pct=kwargs.get("merge_pct", 0.0),
                              layout=kwargs.get("layout", "fake_quant"), sharpen=kwargs.get("sharpen", False))
        return nq.compress(past_key_values)
    if mode == "quant_only":
        nq = NexusQuantQuantOnly(bits=kwargs.get("bits", 3), rope_base=kwargs.get("rope_base", 10000.0),
                                 rope_scaling=kwargs.get("rope_scaling", None),
                                 key_bits=kwargs.get("key_bits"), value_bits=kwargs.get("value_bits"),
                                 layout=kwargs.get("layout", "fake_quant"), sharpen=kwargs.get("sharpen", False))
        return nq.compress(past_key_values)
    if mode in ("fast", "max", "asymmetric"):
        raise NotImplementedError(f"mode={mode!r} is outside the B200 compression path "
                                  "(use 'simple' or 'quant_only')")
    raise ValueError(f"Unknown mode: {mode}. Use 'simple', 'fast', 'max', 'asymmetric', or 'quant_only'.")
