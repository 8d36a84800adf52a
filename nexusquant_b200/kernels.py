"""Torch-tensor front end of the native kernels.

These functions take CUDA tensors, allocate outputs with torch, and call the
C ABI (nexusquant_b200/_native.py -> libnexusquant_b200.so) on the current CUDA
stream.  They replace the reference's GPU entry points in
nexusquant/kernels/e8_triton.py (e8_quantize_perhead :478, e8_encode :525,
e8_decode :574) and the torch math the pipelines run per layer.

Tensors are [batch, heads, tokens, head_dim] with a unit innermost stride.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Union

import torch

from . import _native as N
from .rope import TABLES

_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
SHARPEN = math.sqrt(1.05)  # key sharpening factor (README.md:75; paper section 3.6)


def next_pow2(n: int) -> int:
    p = 1
    while p < n:
        p *= 2
    return p


def packed_bytes(d_p: int, levels: int) -> int:
    n = N.load().nq_packed_bytes(d_p, levels)
    if n < 0:
        raise ValueError(f"unsupported levels={levels} / d_p={d_p}")
    return n


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("nexusquant_b200 kernels need CUDA tensors (there is no CPU path)")


def _rowmajor(t: torch.Tensor) -> torch.Tensor:
    if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]):
        t = t.contiguous()
    return t


@dataclass
class LayerCodes:
    """Compressed form of one layer (CompressedPage fields, nexusquant/integrations/vllm_backend.py:73-101)."""
    k_codes: Optional[torch.Tensor]
    v_codes: Optional[torch.Tensor]
    k_scales: Optional[torch.Tensor]  # fp16
    v_scales: Optional[torch.Tensor]
    key_levels: int
    value_levels: int
    k_scales_f32: Optional[torch.Tensor] = None
    v_scales_f32: Optional[torch.Tensor] = None


def _levels_list(v: Union[int, Sequence[int]], n: int) -> List[int]:
    return [int(v)] * n if isinstance(v, int) else [int(x) for x in v]


def compress_layers(ks: Sequence[Optional[torch.Tensor]], vs: Sequence[Optional[torch.Tensor]], *,
                    key_levels: Union[int, Sequence[int]], value_levels: Union[int, Sequence[int]],
                    kept_idx: Optional[torch.Tensor] = None, kept_count: Optional[torch.Tensor] = None,
                    n_kept: Optional[int] = None, positions: Optional[torch.Tensor] = None,
                    rope_base: float = 10000.0, rope_scaling: Optional[dict] = None,
                    emit_codes: bool = True, emit_scales_f32: bool = False,
                    recon_k: Optional[Sequence[Optional[torch.Tensor]]] = None,
                    recon_v: Optional[Sequence[Optional[torch.Tensor]]] = None,
                    recon_rows: str = "source", recon_positions: Optional[torch.Tensor] = None,
                    key_sharpen: float = 1.0, rope_rows: Optional[int] = None,
                    codes_out: Optional[Sequence[LayerCodes]] = None, rotate: bool = True,
                    device: Optional[torch.device] = None, stage_host_rows: bool = True,
                    _rows_known: bool = False) -> List[LayerCodes]:
    """Compress several layers that share one keep set in a single kernel launch.

    ks / vs   : per-layer [b, h, T, d] tensors (same shape, dtype, strides); None skips that half.
    kept_idx  : int32 [b, n_kept] ascending source token indices (None = all T tokens).
    positions : int32 [b, n_kept] RoPE positions of the kept tokens (None = the token index).
    recon_k/v : optional fp16 outputs receiving the fake-quant reconstruction; rows are the
                source index (recon_rows="source", masked layout) or j (recon_rows="kept",
                truncated layout, keys re-encoded at position j unless recon_positions given).
    codes_out : optional preallocated outputs (LayerCodes per layer) to write into.
    stage_host_rows : with fp16 layers in pinned host memory, a keep set and no reconstruction
                outputs, first gather the kept rows into device memory (``gather_rows``) and
                compress them from there with the kept indices as RoPE positions.  The codes
                are identical; the gather reads the scattered rows across PCIe about twice as
                fast as the compress kernel does.  False reads them inside the compress kernel.
    Returns one LayerCodes per layer.
    """
    L = len(ks)
    ref = next((t for t in list(ks) + list(vs) if t is not None), None)
    if ref is None:
        return []
    host_in = not ref.is_cuda
    if host_in:
        # layers in pinned host memory: the kernel reads only the kept rows, over PCIe
        if not all(t.is_pinned() for t in list(ks) + list(vs) if t is not None):
            raise RuntimeError("host-resident layers must be in pinned memory")
        if device is None:
            raise ValueError("device= is required when the layers are in host memory")
        dev = torch.device(device)
    else:
        _require_cuda(ref)
        dev = ref.device
    _require_cuda(kept_idx, kept_count, positions)
    if (host_in and stage_host_rows and kept_idx is not None and ref.dtype == torch.float16
            and recon_k is None and recon_v is None):
        return _compress_host_staged(ks, vs, dev, key_levels=key_levels, value_levels=value_levels,
                                     kept_idx=kept_idx, kept_count=kept_count, positions=positions,
                                     rope_base=rope_base, rope_scaling=rope_scaling, emit_codes=emit_codes,
                                     emit_scales_f32=emit_scales_f32, key_sharpen=key_sharpen,
                                     rope_rows=rope_rows, codes_out=codes_out, rotate=rotate)
    b, h, T, d = ref.shape
    if ref.dtype not in _DTYPES:
        raise TypeError(f"unsupported cache dtype {ref.dtype}")
    dp = next_pow2(d)
    if kept_idx is not None:
        kept_idx = kept_idx.to(device=dev, dtype=torch.int32).contiguous()
        n_kept = kept_idx.shape[1]
    elif n_kept is None:
        n_kept = T
    if kept_count is not None:
        kept_count = kept_count.to(device=dev, dtype=torch.int32).contiguous()
    if positions is not None:
        positions = positions.to(device=dev, dtype=torch.int32).contiguous()
    if recon_positions is not None:
        recon_positions = recon_positions.to(device=dev, dtype=torch.int32).contiguous()
    klv = _levels_list(key_levels, L)
    vlv = _levels_list(value_levels, L)
    ks = [None if t is None else _rowmajor(t) for t in ks]
    vs = [None if t is None else _rowmajor(t) for t in vs]
    stride_src = next(t for t in ks + vs if t is not None)
    for t in ks + vs:
        if t is not None and (t.shape != ref.shape or t.dtype != ref.dtype or t.stride() != stride_src.stride()):
            raise ValueError("all layers of one compress call must share shape, dtype and strides")
    any_key = any(t is not None for t in ks)
    rows_needed = rope_rows or T
    if positions is not None and positions.numel() and not _rows_known:
        rows_needed = max(rows_needed, int(positions.max().item()) + 1)
    cos = sin = None
    if any_key:
        cos, sin = TABLES.get(dev, d, rope_base, max(rows_needed, n_kept), rope_scaling)

    outs: List[LayerCodes] = []
    arr = (N.LayerIO * L)()
    rk = list(recon_k) if recon_k is not None else [None] * L
    rv = list(recon_v) if recon_v is not None else [None] * L
    out_ref = next((t for t in rk + rv if t is not None), None)
    for l in range(L):
        k, v = ks[l], vs[l]
        if codes_out is not None:
            lc = codes_out[l]
        else:
            lc = LayerCodes(None, None, None, None, klv[l], vlv[l])
            if emit_codes:
                if k is not None:
                    lc.k_codes = torch.empty((b, h, n_kept, packed_bytes(dp, klv[l])), dtype=torch.uint8, device=dev)
                    lc.k_scales = torch.empty((b, h, n_kept), dtype=torch.float16, device=dev)
                if v is not None:
                    lc.v_codes = torch.empty((b, h, n_kept, packed_bytes(dp, vlv[l])), dtype=torch.uint8, device=dev)
                    lc.v_scales = torch.empty((b, h, n_kept), dtype=torch.float16, device=dev)
            if emit_scales_f32:
                if k is not None:
                    lc.k_scales_f32 = torch.empty((b, h, n_kept), dtype=torch.float32, device=dev)
                if v is not None:
                    lc.v_scales_f32 = torch.empty((b, h, n_kept), dtype=torch.float32, device=dev)
        outs.append(lc)
        for t in (rk[l], rv[l]):
            if t is not None and (t.dtype != torch.float16 or t.stride() != out_ref.stride()):
                raise ValueError("reconstruction outputs must be fp16 with identical strides")
        e = arr[l]
        e.k, e.v = _ptr(k), _ptr(v)
        e.k_codes, e.v_codes = _ptr(lc.k_codes), _ptr(lc.v_codes)
        e.k_scales, e.v_scales = _ptr(lc.k_scales), _ptr(lc.v_scales)
        e.k_scales_f32, e.v_scales_f32 = _ptr(lc.k_scales_f32), _ptr(lc.v_scales_f32)
        e.k_out, e.v_out = _ptr(rk[l]), _ptr(rv[l])
        e.key_levels, e.value_levels = klv[l], vlv[l]

    p = N.CompressParams()
    p.batch, p.heads, p.seq, p.head_dim, p.head_dim_padded, p.n_kept = b, h, T, d, dp, n_kept
    p.kept_idx, p.kept_count, p.positions = _ptr(kept_idx), _ptr(kept_count), _ptr(positions)
    p.rope_cos, p.rope_sin = _ptr(cos), _ptr(sin)
    p.rope_rows = 0 if cos is None else cos.shape[0]
    p.in_dtype = _DTYPES[ref.dtype]
    st = stride_src.stride()
    p.in_stride_b, p.in_stride_h, p.in_stride_t = st[0], st[1], st[2]
    if out_ref is not None:
        os_ = out_ref.stride()
        p.out_stride_b, p.out_stride_h, p.out_stride_t = os_[0], os_[1], os_[2]
    p.out_row_mode = 1 if recon_rows == "kept" else 0
    p.out_positions = _ptr(recon_positions)
    p.key_sharpen = float(key_sharpen)
    p.rotate = int(bool(rotate))
    p.inputs_host = int(host_in)
    p.error_flag = None
    p.layers = ctypes.cast(arr, ctypes.POINTER(N.LayerIO))
    p.n_layers = L
    N.call("nq_compress_layers", ctypes.byref(p), _stream(dev))
    return outs


_STAGE = {}
_STAGE_LIMIT = 2 << 30  # bytes of staged rows per compress launch


def _stage_buffer(dev: torch.device, nelem: int) -> torch.Tensor:
    """fp16 staging buffer for kept rows, one per (device, stream): calls on one stream are
    ordered, so reuse across them is safe."""
    key = (str(dev), torch.cuda.current_stream(dev).cuda_stream)
    cur = _STAGE.get(key)
    if cur is None or cur.numel() < nelem:
        _STAGE.pop(key, None)
        cur = torch.empty(nelem, dtype=torch.float16, device=dev)
        _STAGE[key] = cur
    return cur


def _compress_host_staged(ks, vs, dev, *, key_levels, value_levels, kept_idx, kept_count, positions, rope_base,
                          rope_scaling, emit_codes, emit_scales_f32, key_sharpen, rope_rows, codes_out,
                          rotate) -> List[LayerCodes]:
    """Host-resident fp16 layers: gather each layer's kept rows into device memory, then
    compress the gathered rows (kept index j, RoPE position kept_idx[b, j] unless positions
    are given).  Layers go in chunks of at most _STAGE_LIMIT staged bytes."""
    L = len(ks)
    ref = next(t for t in list(ks) + list(vs) if t is not None)
    b, h, T, d = ref.shape
    kept_idx = kept_idx.to(device=dev, dtype=torch.int32).contiguous()
    n_kept = kept_idx.shape[1]
    if kept_count is not None:
        kept_count = kept_count.to(device=dev, dtype=torch.int32).contiguous()
    rows_known = positions is None  # kept indices are below T, like the unstaged path assumes
    pos = kept_idx if positions is None else positions
    klv, vlv = _levels_list(key_levels, L), _levels_list(value_levels, L)
    per_layer = b * h * n_kept * d
    halves = [(k is not None) + (v is not None) for k, v in zip(ks, vs)]
    chunk = max(1, _STAGE_LIMIT // max(1, 2 * 2 * per_layer))
    outs: List[LayerCodes] = []
    for l0 in range(0, L, chunk):
        l1 = min(L, l0 + chunk)
        buf = _stage_buffer(dev, max(1, sum(halves[l0:l1])) * per_layer)
        sk, sv, o = [], [], 0
        for l in range(l0, l1):
            for src, dst in ((ks[l], sk), (vs[l], sv)):
                if src is None:
                    dst.append(None)
                    continue
                st = buf[o * per_layer:(o + 1) * per_layer].view(b, h, n_kept, d)
                o += 1
                gather_rows(src, kept_idx, n_kept, kept_count, out=st, device=dev)
                dst.append(st)
        outs += compress_layers(sk, sv, key_levels=klv[l0:l1], value_levels=vlv[l0:l1], kept_count=kept_count,
                                n_kept=n_kept, positions=pos, rope_base=rope_base, rope_scaling=rope_scaling,
                                emit_codes=emit_codes, emit_scales_f32=emit_scales_f32, key_sharpen=key_sharpen,
                                rope_rows=rope_rows or T, rotate=rotate,
                                codes_out=None if codes_out is None else codes_out[l0:l1],
                                _rows_known=rows_known)
    return outs


def decompress_layers(codes: Sequence[LayerCodes], positions: torch.Tensor, *, head_dim: int,
                      count: Optional[torch.Tensor] = None, rope_base: float = 10000.0,
                      rope_scaling: Optional[dict] = None, key_sharpen: float = 1.0,
                      out_k: Optional[Sequence[torch.Tensor]] = None,
                      out_v: Optional[Sequence[torch.Tensor]] = None, rope_rows: Optional[int] = None):
    """Dequantize layers to fp16 [b, h, n, head_dim]; keys re-encoded at `positions` [b, n].
    rope_rows: RoPE table rows to use when every position is known to be below it; None reads
    positions.max() (a host synchronisation) to size the table."""
    L = len(codes)
    if L == 0:
        return [], []
    ref = next(t for t in (codes[0].k_codes, codes[0].v_codes) if t is not None)
    _require_cuda(ref, positions, count)
    dev = ref.device
    b, h, n, _ = ref.shape
    dp = next_pow2(head_dim)
    positions = positions.to(device=dev, dtype=torch.int32).contiguous()
    if count is not None:
        count = count.to(device=dev, dtype=torch.int32).contiguous()
    if rope_rows is not None:
        rows = int(rope_rows)
    else:
        rows = int(positions.max().item()) + 1 if positions.numel() else 1
    cos, sin = TABLES.get(dev, head_dim, rope_base, rows, rope_scaling)
    ok = list(out_k) if out_k is not None else [None] * L
    ov = list(out_v) if out_v is not None else [None] * L
    arr = (N.DLayerIO * L)()
    for l, lc in enumerate(codes):
        if lc.k_codes is not None and ok[l] is None:
            ok[l] = torch.empty((b, h, n, head_dim), dtype=torch.float16, device=dev)
        if lc.v_codes is not None and ov[l] is None:
            ov[l] = torch.empty((b, h, n, head_dim), dtype=torch.float16, device=dev)
        e = arr[l]
        e.k_codes, e.v_codes = _ptr(lc.k_codes), _ptr(lc.v_codes)
        e.k_scales, e.v_scales = _ptr(lc.k_scales), _ptr(lc.v_scales)
        e.k_out, e.v_out = _ptr(ok[l]), _ptr(ov[l])
        e.key_levels, e.value_levels = lc.key_levels, lc.value_levels
    out_ref = next(t for t in ok + ov if t is not None)
    for t in ok + ov:
        if t is not None and t.stride() != out_ref.stride():
            raise ValueError("dequantize outputs must share strides")
    p = N.DecompressParams()
    p.batch, p.heads, p.n_tokens, p.head_dim, p.head_dim_padded = b, h, n, head_dim, dp
    p.count, p.positions = _ptr(count), _ptr(positions)
    p.rope_cos, p.rope_sin, p.rope_rows = _ptr(cos), _ptr(sin), cos.shape[0]
    s = out_ref.stride()
    p.out_stride_b, p.out_stride_h, p.out_stride_t = s[0], s[1], s[2]
    p.key_sharpen = float(key_sharpen)
    p.layers = ctypes.cast(arr, ctypes.POINTER(N.DLayerIO))
    p.n_layers = L
    N.call("nq_decompress_layers", ctypes.byref(p), _stream(dev))
    return ok, ov


_WS = {}


def _workspace(device, nbytes: int) -> torch.Tensor:
    key = str(device)
    cur = _WS.get(key)
    if cur is None or cur.numel() < nbytes:
        cur = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        _WS[key] = cur
    return cur


def score_keykey(k: torch.Tensor, obs_window: int = 32, head_range=None, per_head: bool = False) -> torch.Tensor:
    """Key-key importance (nexusquant/pipeline.py:756-782) -> fp32 [b, T] (or [b, Hr, T] per head)."""
    _require_cuda(k)
    k = _rowmajor(k)
    b, h, T, d = k.shape
    h0, h1 = head_range if head_range is not None else (0, h)
    ws_n = N.load().nq_score_keykey_workspace_size(b, h1 - h0, T, obs_window)
    ws = _workspace(k.device, ws_n)
    out = torch.empty((b, h1 - h0, T) if per_head else (b, T), dtype=torch.float32, device=k.device)
    st = k.stride()
    N.call("nq_score_keykey", k.data_ptr(), _DTYPES[k.dtype], b, h, T, d, st[0], st[1], st[2], obs_window, h0, h1,
           int(per_head), out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(k.device))
    return out


def check_device_errors(device=None) -> int:
    """Synchronize the device's current stream and raise NexusQuantError (NQ_ERR_TIMEOUT) if a
    bounded device-side wait expired since the last check (the scorer's or the decode
    attention's results are then not valid); clears the device's error word.  Returns 0."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    bits = ctypes.c_int32(0)
    with torch.cuda.device(dev):
        st = N.load().nq_device_error(ctypes.byref(bits), _stream(dev))
    N.check("nq_device_error", st)
    return bits.value


def reduce_heads(per_head: torch.Tensor, divisor: float, out: Optional[torch.Tensor] = None,
                 accumulate: bool = False) -> torch.Tensor:
    _require_cuda(per_head)
    per_head = per_head.contiguous()
    b, H, T = per_head.shape
    if out is None:
        out = torch.empty((b, T), dtype=torch.float32, device=per_head.device)
    N.call("nq_reduce_heads", per_head.data_ptr(), b, H, T, float(divisor), int(accumulate), out.data_ptr(),
           _stream(per_head.device))
    return out


def score_attention(q: torch.Tensor, k: torch.Tensor, q_pos0: int, out: Optional[torch.Tensor] = None,
                    accumulate: bool = False) -> torch.Tensor:
    """Causal softmax column sums of q [b, Hq, nq, d] against k [b, H, T, d], mean over query heads."""
    _require_cuda(q, k)
    q = _rowmajor(q)
    k = _rowmajor(k)
    b, hq, nq, d = q.shape
    _, h, T, _ = k.shape
    if q.dtype != k.dtype:
        q = q.to(k.dtype)
    ws_n = N.load().nq_score_attention_workspace_size(b, hq, nq, T)
    ws = _workspace(k.device, ws_n)
    if out is None:
        out = torch.zeros((b, T), dtype=torch.float32, device=k.device)
    qs, ks_ = q.stride(), k.stride()
    N.call("nq_score_attention", q.data_ptr(), k.data_ptr(), _DTYPES[k.dtype], b, hq, h, nq, T, d, qs[0], qs[1],
           qs[2], ks_[0], ks_[1], ks_[2], int(q_pos0), int(accumulate), out.data_ptr(), ws.data_ptr(), ws.numel(),
           _stream(k.device))
    return out


def select_keep(importance: torch.Tensor, sliding_window: int, n_keep: int,
                protected_positions: Optional[torch.Tensor] = None):
    """Keep set (nexusquant/pipeline.py:895-959) -> (kept_idx int32 [b, T], kept_count int32 [b])."""
    _require_cuda(importance)
    imp = importance.to(torch.float32).contiguous()
    b, T = imp.shape
    idx = torch.empty((b, max(T, 1)), dtype=torch.int32, device=imp.device)
    cnt = torch.empty((b,), dtype=torch.int32, device=imp.device)
    prot = None
    n_prot = 0
    if protected_positions is not None and len(protected_positions) > 0:
        pp = sorted({int(p) for p in protected_positions if 0 <= int(p) < T})
        n_prot = len(pp)
        if n_prot:
            prot = torch.tensor(pp, dtype=torch.int32, device=imp.device)
    N.call("nq_select_keep", imp.data_ptr(), b, T, int(sliding_window), int(n_keep), _ptr(prot), n_prot,
           idx.data_ptr(), cnt.data_ptr(), None, 0, _stream(imp.device))
    return idx, cnt


def gather_rows(x: torch.Tensor, kept_idx: Optional[torch.Tensor], n_kept: int,
                kept_count: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                device: Optional[torch.device] = None) -> torch.Tensor:
    """fp16 copy of the kept rows: out[b, h, j] = x[b, h, kept_idx[b, j]].  x may be in pinned
    host memory (pass device=): only the kept rows then cross PCIe."""
    _require_cuda(kept_idx, kept_count)
    if x.is_cuda:
        dev = x.device
        x = _rowmajor(x)
    else:
        if not x.is_pinned() or device is None:
            raise RuntimeError("host-resident input must be pinned, with device= given")
        dev = torch.device(device)
    b, h, T, d = x.shape
    if out is None:
        out = torch.empty((b, h, n_kept, d), dtype=torch.float16, device=dev)
    if kept_idx is not None:
        kept_idx = kept_idx.to(dtype=torch.int32).contiguous()
    s, o = x.stride(), out.stride()
    N.call("nq_gather_rows", x.data_ptr(), _DTYPES[x.dtype], b, h, d, s[0], s[1], s[2], _ptr(kept_idx),
           _ptr(kept_count), n_kept, out.data_ptr(), o[0], o[1], o[2], _stream(dev))
    return out


def merge_nearest(unit: torch.Tensor, evict_pos: torch.Tensor, kept_pos: torch.Tensor, *,
                  tensor_cores: bool = True) -> torch.Tensor:
    """nearest[i] = argmax_j unit[evict_pos[i]] . unit[kept_pos[j]] (first j on ties) for fp32 unit
    rows [seq, d]: nq_merge_nearest_unit (d = 128, tensor-core screening with an exact
    re-check) or nq_merge_nearest (the exact fp32 kernel)."""
    _require_cuda(unit)
    unit = unit.contiguous()
    ev = evict_pos.to(device=unit.device, dtype=torch.int32).contiguous()
    kp = kept_pos.to(device=unit.device, dtype=torch.int32).contiguous()
    out = torch.empty(ev.numel(), dtype=torch.int32, device=unit.device)
    fn = "nq_merge_nearest_unit" if tensor_cores else "nq_merge_nearest"
    N.call(fn, unit.data_ptr(), unit.shape[1], ev.data_ptr(), ev.numel(), kp.data_ptr(), kp.numel(), out.data_ptr(),
           _stream(unit.device))
    return out


def merge_evicted_values(vs: Sequence[torch.Tensor], keep_mask: torch.Tensor, importance: torch.Tensor,
                         nearest_out: Optional[List[torch.Tensor]] = None) -> None:
    """Merge eviction, in place on ``vs`` (nexusquant/pipeline.py:961-1048): for every batch
    element, each evicted token's values are added into the kept token whose value centroid
    (mean over layers and heads) is most cosine-similar, weighted by
    imp[e] / (imp[s] + imp[e] + 1e-8).  Layers whose sequence length differs from the mask's
    are skipped, as the reference skips sliding-window layers.  ``nearest_out`` (optional list)
    receives, per batch element, the chosen kept index of every evicted token (or None)."""
    b, T = keep_mask.shape
    layers = [v for v in vs if v.shape[2] == T]
    _require_cuda(keep_mask, importance, *layers)
    if nearest_out is not None:
        nearest_out.clear()
    if not layers:
        if nearest_out is not None:
            nearest_out.extend([None] * b)
        return
    ref = layers[0]
    dev = ref.device
    d = ref.shape[3]
    for v in layers:
        if v.shape[0] != b or v.shape[3] != d or v.dtype not in _DTYPES or v.stride(3) != 1:
            raise ValueError("merge eviction needs [b, h, T, d] value layers with a common d and unit inner stride")
    imp = importance.to(device=dev, dtype=torch.float32)
    stream = _stream(dev)
    # runs of consecutive layers sharing heads, dtype and strides go in one call, in layer order
    runs = []
    for v in layers:
        key = (v.shape[1], v.dtype, v.stride(1), v.stride(2))
        if runs and runs[-1][0] == key:
            runs[-1][1].append(v)
        else:
            runs.append((key, [v]))
    acc = torch.empty((T, d), dtype=torch.float32, device=dev)
    for bi in range(b):
        km = keep_mask[bi].to(dev)
        evict = torch.nonzero(~km).flatten().to(torch.int32)
        kept = torch.nonzero(km).flatten().to(torch.int32)
        n_e, n_k = evict.numel(), kept.numel()
        if n_e == 0 or n_k == 0:
            if nearest_out is not None:
                nearest_out.append(None)
            continue
        first = True
        for (h, dt, sh, st), vl in runs:
            ptrs = (ctypes.c_void_p * len(vl))(*[v[bi].data_ptr() for v in vl])
            N.call("nq_merge_centroid_accumulate", ptrs, len(vl), _DTYPES[dt], h, T, d, sh, st, 0 if first else 1,
                   acc.data_ptr(), stream)
            first = False
        N.call("nq_merge_centroid_normalize", acc.data_ptr(), T, d, len(layers), acc.data_ptr(), stream)
        nearest = torch.empty(n_e, dtype=torch.int32, device=dev)
        # unit rows at head_dim 128: tensor-core screening + exact re-check (same choices)
        N.call("nq_merge_nearest_unit" if d == 128 else "nq_merge_nearest", acc.data_ptr(), d, evict.data_ptr(),
               n_e, kept.data_ptr(), n_k, nearest.data_ptr(), stream)
        order = torch.argsort(nearest, stable=True)
        seg_evicted = evict[order].contiguous()
        seg_start = torch.zeros(n_k + 1, dtype=torch.int32, device=dev)
        seg_start[1:] = torch.cumsum(torch.bincount(nearest, minlength=n_k), 0).to(torch.int32)
        imp_b = imp[bi].contiguous()
        for (h, dt, sh, st), vl in runs:
            ptrs = (ctypes.c_void_p * len(vl))(*[v[bi].data_ptr() for v in vl])
            N.call("nq_merge_apply", ptrs, len(vl), _DTYPES[dt], h, T, d, sh, st, imp_b.data_ptr(), kept.data_ptr(),
                   n_k, seg_start.data_ptr(), seg_evicted.data_ptr(), stream)
        if nearest_out is not None:
            nearest_out.append(nearest)


def delta_codes(codes: torch.Tensor, head_dim_padded: int, levels: int) -> torch.Tensor:
    """Temporal delta (nexusquant/core/temporal_codec.py:30-52) of packed codes [..., n, pb] -> int8 [..., n, d_p]."""
    _require_cuda(codes)
    codes = codes.contiguous()
    *lead, n, pb = codes.shape
    streams = 1
    for x in lead:
        streams *= x
    out = torch.empty((*lead, n, head_dim_padded), dtype=torch.int8, device=codes.device)
    N.call("nq_delta_codes", codes.data_ptr(), streams, n, head_dim_padded, int(levels), out.data_ptr(),
           _stream(codes.device))
    return out


def code_histogram(codes: torch.Tensor, head_dim_padded: int, levels: int,
                   counts: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Histogram of the doubled lattice codes of packed rows [..., pb]: int32 [2L + 1] with
    counts[c + L] = number of codes equal to c (accumulated into ``counts`` when given)."""
    _require_cuda(codes)
    codes = codes.contiguous()
    rows = codes.numel() // max(codes.shape[-1], 1)
    if counts is None:
        counts = torch.zeros(2 * levels + 1, dtype=torch.int32, device=codes.device)
    N.call("nq_code_histogram", codes.data_ptr(), rows, head_dim_padded, int(levels), counts.data_ptr(),
           _stream(codes.device))
    return counts


def code_symbols(codes: torch.Tensor, head_dim_padded: int, levels: int, half: bool) -> torch.Tensor:
    """rANS symbols (nexusquant/core/entropy_coder.py:35-75) of packed rows [..., pb] ->
    uint8 [..., d_p]: c + L with half-integer coordinates present, else c / 2 + L / 2."""
    _require_cuda(codes)
    codes = codes.contiguous()
    *lead, pb = codes.shape
    rows = codes.numel() // max(pb, 1)
    out = torch.empty((*lead, head_dim_padded), dtype=torch.uint8, device=codes.device)
    N.call("nq_code_symbols", codes.data_ptr(), rows, head_dim_padded, int(levels), int(bool(half)),
           out.data_ptr(), _stream(codes.device))
    return out


# ---------------------------------------------------------------------------
# Names of the reference's GPU wrappers (nexusquant/kernels/e8_triton.py)
# ---------------------------------------------------------------------------
def e8_encode(x: torch.Tensor, levels: int = 4):
    """Per-vector E8 encode of rows x [..., d] (no RoPE) -> (codes int8 [..., d_p], fp32 scales [...]).
    Replaces e8_encode (nexusquant/kernels/e8_triton.py:525-571)."""
    *lead, d = x.shape
    rows = x.reshape(1, 1, -1, d)
    lc = compress_layers([None], [rows], key_levels=levels, value_levels=levels, emit_scales_f32=True,
                         rotate=False)[0]
    codes = unpack_codes(lc.v_codes, next_pow2(d), levels)[..., :(d + 7) // 8 * 8]
    return codes.reshape(*lead, -1), lc.v_scales_f32.reshape(*lead)


def unpack_codes(packed: torch.Tensor, d_p: int, levels: int) -> torch.Tensor:
    """Packed rows [..., pb] -> int8 codes [..., d_p] (first row of a delta stream is the codes)."""
    n = packed.shape[-2] if packed.dim() >= 2 else 1
    lead = packed.shape[:-2]
    d = delta_codes(packed.reshape(-1, 1, packed.shape[-1]), d_p, levels)
    return d.reshape(*lead, n, d_p) if packed.dim() >= 2 else d.reshape(d_p)


def e8_quantize_perhead(x: torch.Tensor, levels: int = 4) -> torch.Tensor:
    """Quantize-dequantize rows x [..., d] with one scale per row (no rotation), as
    E8Lattice.quantize_perhead (nexusquant/core/e8_lattice.py:97-124) and the Triton
    e8_quantize_perhead (nexusquant/kernels/e8_triton.py:478).  fp16 result."""
    *lead, d = x.shape
    rows = x.reshape(1, 1, -1, d)
    out = torch.empty(rows.shape, dtype=torch.float16, device=x.device)
    compress_layers([None], [rows], key_levels=levels, value_levels=levels, emit_codes=False, recon_v=[out],
                    rotate=False)
    return out.reshape(*lead, d)


def attend_compressed(q: torch.Tensor, codes: LayerCodes, positions: torch.Tensor, *,
                      count: Optional[torch.Tensor] = None, rope_base: float = 10000.0,
                      rope_scaling: Optional[dict] = None, key_sharpen: float = 1.0,
                      scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                      rope_rows: Optional[int] = None) -> torch.Tensor:
    """Decode attention over one compressed layer (NexusQuantPagedAttention.forward,
    vllm_backend.py:692-765) without materialising fp16 K/V.

    q         : fp16 [b, hq, 128], one query token per sequence (RoPE already applied).
    codes     : LayerCodes of the layer ([b, h, n, pb] codes, [b, h, n] fp16 scales); hq / h in {1,2,4,8}.
    positions : int32 [b, n] RoPE positions of the stored keys.
    rope_rows : RoPE table rows to use when every position is known to be below it; None reads
                positions.max() (a host synchronisation) to size the table.
    Returns fp16 [b, hq, 128] = softmax(q K^T * scale) V with K, V as decompress_layers gives them."""
    _require_cuda(q, positions, count)
    b, hq, d = q.shape
    _, h, n, _ = codes.k_codes.shape
    dev = q.device
    if q.dtype != torch.float16:
        raise TypeError("query must be fp16")
    q = q if q.stride(-1) == 1 else q.contiguous()
    positions = positions.to(device=dev, dtype=torch.int32).contiguous()
    if count is not None:
        count = count.to(device=dev, dtype=torch.int32).contiguous()
    if rope_rows is not None:
        rows = int(rope_rows)
    else:
        rows = int(positions.max().item()) + 1 if positions.numel() else 1
    cos, sin = TABLES.get(dev, d, rope_base, rows, rope_scaling)
    if out is None:
        out = torch.empty((b, hq, d), dtype=torch.float16, device=dev)
    ws = _workspace(dev, N.load().nq_attend_compressed_workspace_size(b, hq, h, n))
    p = N.AttendParams()
    p.batch, p.q_heads, p.heads, p.head_dim, p.head_dim_padded, p.n_tokens = b, hq, h, d, next_pow2(d), n
    p.count, p.q = _ptr(count), q.data_ptr()
    p.q_stride_b, p.q_stride_h = q.stride(0), q.stride(1)
    p.k_codes, p.v_codes = codes.k_codes.data_ptr(), codes.v_codes.data_ptr()
    p.k_scales, p.v_scales = codes.k_scales.data_ptr(), codes.v_scales.data_ptr()
    p.key_levels, p.value_levels = codes.key_levels, codes.value_levels
    p.positions, p.rope_cos, p.rope_sin, p.rope_rows = positions.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0]
    p.key_sharpen = float(key_sharpen)
    p.scale = 0.0 if scale is None else float(scale)
    p.out, p.out_stride_b, p.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    N.call("nq_attend_compressed", ctypes.byref(p), ws.data_ptr(), ws.numel(), _stream(dev))
    return out
