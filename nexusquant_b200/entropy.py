"""Entropy coding of the lattice codes: a host post-step outside the compression hot path.

The reference measures its compressed size by temporal-delta coding the E8 coordinates
and compressing them with zstd at level 22 (zlib when the ``zstandard`` module is missing):

  compress_indices / decompress_indices   nexusquant/core/temporal_codec.py:76-130
      header '<IIBBxx' (n_elements, n_tokens, use_delta, compressor 1 = zstd / 0 = zlib),
      then the zstd or zlib payload of the (optionally delta-coded) int8 coordinates
  temporal_delta_encode / decode          nexusquant/core/temporal_codec.py:30-71
  accounting order                        nexusquant/core/compression_accounting.py:49-62,
                                          :296-312 (streams (layer, K|V, head) x tokens x
                                          coords, delta along tokens, one zstd frame)

Here the delta of every (layer, K|V, batch, head) stream is taken on the device from the
packed codes (``kernels.delta_codes``, one launch per tensor); only the byte compressor runs
on the host.  zstd comes from the system libzstd through ctypes (the ``zstandard`` Python
package is not required); without libzstd, or with ``codec="zlib"``, the zlib fallback of
the reference is used, with the same header.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import struct
import time
import zlib
from typing import Dict, Optional

import numpy as np
import torch

from . import kernels as K

HEADER = "<IIBBxx"          # temporal_codec.py:105
HEADER_BYTES = struct.calcsize(HEADER)
COMPRESSOR_ZLIB, COMPRESSOR_ZSTD = 0, 1


# ------------------------------------------------------------------------- libzstd
class _Zstd:
    """Minimal ctypes binding of the one-shot libzstd API (ZSTD_compress / ZSTD_decompress)."""

    _ZSTD_c_compressionLevel = 100
    _ZSTD_c_nbWorkers = 400
    _ZSTD_e_end = 2

    def __init__(self):
        name = ctypes.util.find_library("zstd") or "libzstd.so.1"
        L = ctypes.CDLL(name)
        sz, vp, ci = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int
        L.ZSTD_compressBound.argtypes, L.ZSTD_compressBound.restype = [sz], sz
        L.ZSTD_isError.argtypes, L.ZSTD_isError.restype = [sz], ctypes.c_uint
        L.ZSTD_getErrorName.argtypes, L.ZSTD_getErrorName.restype = [sz], ctypes.c_char_p
        L.ZSTD_decompress.argtypes, L.ZSTD_decompress.restype = [vp, sz, vp, sz], sz
        L.ZSTD_getFrameContentSize.argtypes = [vp, sz]
        L.ZSTD_getFrameContentSize.restype = ctypes.c_ulonglong
        L.ZSTD_versionNumber.restype = ctypes.c_uint
        L.ZSTD_createCCtx.restype = vp
        L.ZSTD_freeCCtx.argtypes = [vp]
        L.ZSTD_CCtx_setParameter.argtypes, L.ZSTD_CCtx_setParameter.restype = [vp, ci, ci], sz
        L.ZSTD_compress2.argtypes, L.ZSTD_compress2.restype = [vp, vp, sz, vp, sz], sz
        self.L = L
        self.version = L.ZSTD_versionNumber()

    def _check(self, r: int, what: str) -> int:
        if self.L.ZSTD_isError(r):
            raise RuntimeError(f"{what}: {self.L.ZSTD_getErrorName(r).decode()}")
        return r

    def compress(self, raw: bytes, level: int, threads: int = 0) -> bytes:
        cap = self.L.ZSTD_compressBound(len(raw))
        dst = ctypes.create_string_buffer(cap)
        cctx = self.L.ZSTD_createCCtx()
        if not cctx:
            raise MemoryError("ZSTD_createCCtx failed")
        try:
            self._check(self.L.ZSTD_CCtx_setParameter(cctx, self._ZSTD_c_compressionLevel, int(level)), "level")
            if threads > 1:
                # libzstd builds without multithreading reject this; compress single-threaded then
                if self.L.ZSTD_isError(self.L.ZSTD_CCtx_setParameter(cctx, self._ZSTD_c_nbWorkers, int(threads))):
                    pass
            n = self._check(self.L.ZSTD_compress2(cctx, dst, cap, raw, len(raw)), "ZSTD_compress2")
        finally:
            self.L.ZSTD_freeCCtx(cctx)
        return dst.raw[:n]

    def decompress(self, payload: bytes) -> bytes:
        size = self.L.ZSTD_getFrameContentSize(payload, len(payload))
        if size >= (1 << 63):
            raise RuntimeError("zstd frame without a content size")
        dst = ctypes.create_string_buffer(max(int(size), 1))
        n = self._check(self.L.ZSTD_decompress(dst, int(size), payload, len(payload)), "ZSTD_decompress")
        return dst.raw[:n]


_ZSTD: Optional[_Zstd] = None
_ZSTD_TRIED = False


def zstd() -> Optional[_Zstd]:
    """The libzstd binding, or None when the system has no libzstd."""
    global _ZSTD, _ZSTD_TRIED
    if not _ZSTD_TRIED:
        _ZSTD_TRIED = True
        try:
            _ZSTD = _Zstd()
        except OSError:
            _ZSTD = None
    return _ZSTD


# -------------------------------------------------------------------- delta coding
def temporal_delta_encode(coords: np.ndarray, n_tokens: int) -> np.ndarray:
    """Delta along tokens of a flat int8 array laid out [n_tokens, n_per_token]
    (temporal_codec.py:30-52; returned unchanged when it does not reshape cleanly)."""
    coords = np.asarray(coords, dtype=np.int8)
    n = coords.size
    if n_tokens <= 0 or n % n_tokens or (n // n_tokens) % 8:
        return coords
    r = coords.reshape(n_tokens, -1)
    d = np.empty_like(r)
    d[0] = r[0]
    np.subtract(r[1:], r[:-1], out=d[1:])   # int8 wrap-around, as numpy does in the reference
    return d.reshape(-1)


def temporal_delta_decode(delta: np.ndarray, n_tokens: int) -> np.ndarray:
    """Inverse of temporal_delta_encode (temporal_codec.py:55-71: cumulative sum along tokens)."""
    delta = np.asarray(delta, dtype=np.int8)
    n = delta.size
    if n_tokens <= 0 or n % n_tokens:
        return delta
    return np.cumsum(delta.reshape(n_tokens, -1), axis=0).astype(np.int8).reshape(-1)


# ------------------------------------------------------------------- byte streams
def _compress_payload(raw: bytes, level: int, codec: str, threads: int):
    z = zstd() if codec in ("auto", "zstd") else None
    if codec == "zstd" and z is None:
        raise RuntimeError("codec='zstd' requested but libzstd is not available")
    if z is not None:
        return z.compress(raw, min(level, 22), threads), COMPRESSOR_ZSTD
    return zlib.compress(raw, min(level, 9)), COMPRESSOR_ZLIB


def compress_indices(coords: np.ndarray, n_tokens: int, use_delta: bool = True, level: int = 22,
                     codec: str = "auto", threads: int = 0) -> bytes:
    """Header '<IIBBxx' + zstd (codec 'auto'/'zstd') or zlib ('zlib') payload of the
    int8 coordinates, optionally temporal-delta coded first (temporal_codec.py:76-106)."""
    data = np.asarray(coords, dtype=np.int8).reshape(-1)
    n_el = data.size
    if use_delta:
        data = temporal_delta_encode(data, n_tokens)
    payload, comp = _compress_payload(data.tobytes(), level, codec, threads)
    return struct.pack(HEADER, n_el, n_tokens, int(use_delta), comp) + payload


def decompress_indices(data: bytes) -> np.ndarray:
    """Inverse of compress_indices (temporal_codec.py:109-130)."""
    n_el, n_tokens, use_delta, comp = struct.unpack_from("<IIBB", data)
    payload = data[HEADER_BYTES:]
    if comp == COMPRESSOR_ZSTD:
        z = zstd()
        if z is None:
            raise RuntimeError("stream is zstd-compressed but libzstd is not available")
        raw = z.decompress(payload)
    else:
        raw = zlib.decompress(payload)
    out = np.frombuffer(raw, dtype=np.int8).copy()
    if out.size != n_el:
        raise ValueError(f"stream holds {out.size} coordinates, header says {n_el}")
    return temporal_delta_decode(out, n_tokens) if use_delta else out


# ------------------------------------------------------------- cache-level report
def delta_streams(cache, layers=None, max_tokens: Optional[int] = None) -> np.ndarray:
    """Delta-coded int8 codes of a CompressedKVCache in the accounting order of
    compression_accounting.py:296-312: streams (layer, K|V, batch, head), each the delta
    along its kept tokens of the [tokens, d_p] codes, concatenated.  The delta runs on the
    device from the packed codes; boundary-protected layers carry no codes and are skipped.
    ``max_tokens`` bounds the tokens per stream (a sample)."""
    parts = []
    cnt = cache.kept_count.cpu().tolist()
    idx = range(len(cache.layers)) if layers is None else layers
    for li in idx:
        c = cache.layers[li].codes
        if c is None:
            continue
        for packed, lev in ((c.k_codes, c.key_levels), (c.v_codes, c.value_levels)):
            b, h, n, _ = packed.shape
            for bi in range(b):
                m = min(cnt[bi], n) if max_tokens is None else min(cnt[bi], n, max_tokens)
                if m <= 0:
                    continue
                src = packed[bi, :, :m]
                if not src.is_cuda:  # a host-resident cache: the slice goes to the device for the delta
                    src = src.to(torch.device("cuda", torch.cuda.current_device()))
                d = K.delta_codes(src, cache.head_dim_padded, lev)  # [h, m, d_p]
                parts.append(d.cpu().numpy().reshape(-1))
    return np.concatenate(parts) if parts else np.zeros((0,), np.int8)


def entropy_report(cache, level: int = 22, codec: str = "auto", threads: int = 0, layers=None,
                   max_tokens: Optional[int] = None) -> Dict[str, float]:
    """Entropy-coded size of the cache's lattice codes (the reference's reported host
    post-step): delta streams on the device, then one zstd (or zlib) frame on the host.
    Sizes of the scales, protected fp16 layers and the NQC1 header are added as stored."""
    t0 = time.perf_counter()
    d = delta_streams(cache, layers, max_tokens)
    t1 = time.perf_counter()
    payload, comp = _compress_payload(d.tobytes(), level, codec, threads)
    t2 = time.perf_counter()
    n = int(d.size)
    out = {
        "codec": "zstd" if comp == COMPRESSOR_ZSTD else "zlib",
        "level": min(level, 22 if comp == COMPRESSOR_ZSTD else 9),
        "symbols": n,
        "index_raw_bytes": n,
        "index_compressed_bytes": len(payload) + HEADER_BYTES,
        "bits_per_symbol": (8.0 * (len(payload) + HEADER_BYTES) / n) if n else 0.0,
        "delta_seconds": t1 - t0,
        "host_seconds": t2 - t1,
        "sampled": layers is not None or max_tokens is not None,
    }
    return out
