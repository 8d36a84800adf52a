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
import math
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


# ------------------------------------------------------------------------------ rANS
# The reference's rANS container for E8 lattice codes (nexusquant/core/entropy_coder.py):
#   header '<IBBI' (n_groups, levels, has_half, n_symbols), '<III' section lengths,
#   frequency table ('<H' alphabet size, '<H' per symbol), fp16 scale per 8-group,
#   rANS words ('<H', 32-bit state, 16-bit renormalisation, 12-bit table).
# The symbol mapping and the histogram over every code run on the device
# (kernels.code_histogram / kernels.code_symbols); the table normalisation is a few dozen
# numbers and the state loop is serial, both on the host (the loop in native code).
RANS_PROB_BITS = 12
RANS_M = 1 << RANS_PROB_BITS
RANS_HEADER = "<IBBI"
RANS_LENGTHS = "<III"


def rans_freq_table(counts: np.ndarray) -> np.ndarray:
    """Normalised frequencies summing to 4096 from symbol counts, as _build_freq_table
    (entropy_coder.py:175-243): every seen symbol gets 1, the rest of the budget is shared
    by floor(count / total * remaining), leftovers go to the largest fractional parts in
    numpy argsort order (the same sort calls, so ties break the same way)."""
    counts = np.asarray(counts, dtype=np.int64)
    a = counts.size
    total = int(counts.sum())
    if total == 0:
        freqs = np.full(a, RANS_M // a, dtype=np.int64)
        freqs[0] += RANS_M - int(freqs.sum())
        return freqs
    seen = counts > 0
    n_seen = int(seen.sum())
    freqs = np.zeros(a, dtype=np.int64)
    freqs[seen] = 1
    remaining = RANS_M - n_seen
    seen_idx = np.where(seen)[0]
    if remaining > 0:
        share = (counts[seen].astype(np.float64) / total) * remaining
        extra = np.floor(share).astype(np.int64)
        freqs[seen] += extra
        diff = int(RANS_M - freqs.sum())
        if diff > 0:
            order = seen_idx[np.argsort(-(share - extra))]
            for i in range(diff):
                freqs[order[i % len(order)]] += 1
        elif diff < 0:
            order = seen_idx[np.argsort(counts[seen])]
            removed = 0
            for j in order:
                while freqs[j] > 1 and removed < -diff:
                    freqs[j] -= 1
                    removed += 1
                if removed >= -diff:
                    break
    elif remaining < 0:  # more seen symbols than table slots: unreachable for alphabets <= 33
        order = seen_idx[np.argsort(-counts[seen])]
        freqs[:] = 0
        freqs[order[:RANS_M]] = 1
    if int(freqs.sum()) != RANS_M:
        raise ValueError(f"frequency table sums to {int(freqs.sum())}, not {RANS_M}")
    return freqs


def rans_encode(symbols: np.ndarray, freqs: np.ndarray) -> np.ndarray:
    """rANS words (uint16, stream order) of uint8 symbols (_rans_encode, entropy_coder.py:246-295);
    the state loop runs in the native library."""
    from . import _native as N
    sym = np.ascontiguousarray(symbols, dtype=np.uint8).reshape(-1)
    fr = np.ascontiguousarray(freqs, dtype=np.uint32)
    out = np.empty(sym.size + 2, dtype=np.uint16)
    n_out = ctypes.c_int64(0)
    N.call("nq_rans_encode", sym.ctypes.data, sym.size, fr.ctypes.data, fr.size, out.ctypes.data, out.size,
           ctypes.byref(n_out))
    return out[:n_out.value].copy()


def rans_decode(words: np.ndarray, n_symbols: int, freqs: np.ndarray) -> np.ndarray:
    """Inverse of rans_encode (_rans_decode, entropy_coder.py:298-345)."""
    from . import _native as N
    w = np.ascontiguousarray(words, dtype=np.uint16)
    fr = np.ascontiguousarray(freqs, dtype=np.uint32)
    out = np.empty(int(n_symbols), dtype=np.uint8)
    N.call("nq_rans_decode", w.ctypes.data, w.size, out.size, fr.ctypes.data, fr.size, out.ctypes.data)
    return out


def rans_pack_e8(symbols: np.ndarray, counts: np.ndarray, has_half: bool, levels: int,
                 group_scales: np.ndarray) -> bytes:
    """The encode_e8 byte stream (entropy_coder.py:405-452) from symbols already mapped,
    their counts over the alphabet and one fp16 scale per 8-group."""
    sym = np.ascontiguousarray(symbols, dtype=np.uint8).reshape(-1)
    freqs = rans_freq_table(counts)
    words = rans_encode(sym, freqs)
    scales = np.ascontiguousarray(group_scales, dtype=np.float16).reshape(-1)
    n_groups = scales.size
    if sym.size != 8 * n_groups:
        raise ValueError(f"{sym.size} symbols for {n_groups} groups of 8")
    ftab = struct.pack("<H", freqs.size) + freqs.astype("<u2").tobytes()
    sc = scales.astype("<f2").tobytes()
    wd = words.astype("<u2").tobytes()
    return (struct.pack(RANS_HEADER, n_groups, int(levels), int(bool(has_half)), sym.size) +
            struct.pack(RANS_LENGTHS, len(ftab), len(sc), len(wd)) + ftab + sc + wd)


def rans_encode_e8(packed: torch.Tensor, row_scales: torch.Tensor, head_dim_padded: int, levels: int,
                   timings: Optional[dict] = None) -> bytes:
    """encode_e8 (entropy_coder.py:405-452) of packed code rows [..., pb] with one fp16
    scale per row [...]: the stream the reference writes for quantized = code / 2 * scale and
    that row's scale repeated over its 8-groups.  Histogram and symbols on the device;
    ``timings`` (if given) accumulates 'device_seconds' (passes + copies) and 'host_seconds'."""
    t0 = time.perf_counter()
    cnt = K.code_histogram(packed, head_dim_padded, levels).cpu().numpy().astype(np.int64)
    has_half = bool(cnt[1::2].sum() > 0)   # L is even: bin c + L is odd exactly for odd (half-integer) c
    sym = K.code_symbols(packed, head_dim_padded, levels, has_half).cpu().numpy()
    alpha = cnt if has_half else cnt[0::2]
    g = head_dim_padded // 8
    sc = row_scales.reshape(-1, 1).expand(-1, g).reshape(-1).cpu().numpy()
    t1 = time.perf_counter()
    blob = rans_pack_e8(sym, alpha, has_half, levels, sc)
    if timings is not None:
        timings["device_seconds"] = timings.get("device_seconds", 0.0) + t1 - t0
        timings["host_seconds"] = timings.get("host_seconds", 0.0) + time.perf_counter() - t1
    return blob


def rans_report(cache, layers=None, max_tokens: Optional[int] = None) -> Dict[str, float]:
    """rANS-coded size (encode_e8 container, one stream per (layer, K|V, batch) of the kept
    tokens) of a CompressedKVCache's codes; ``layers`` / ``max_tokens`` sample it."""
    cnt = cache.kept_count.cpu().tolist()
    idx = range(len(cache.layers)) if layers is None else layers
    dev = torch.device("cuda", torch.cuda.current_device())
    tm: dict = {}
    n_sym = n_bytes = 0
    for li in idx:
        c = cache.layers[li].codes
        if c is None:
            continue
        for packed, scales, lev in ((c.k_codes, c.k_scales, c.key_levels), (c.v_codes, c.v_scales, c.value_levels)):
            n = packed.shape[2]
            for bi in range(packed.shape[0]):
                m = min(cnt[bi], n) if max_tokens is None else min(cnt[bi], n, max_tokens)
                if m <= 0:
                    continue
                blob = rans_encode_e8(packed[bi, :, :m].to(dev), scales[bi, :, :m].to(dev),
                                      cache.head_dim_padded, lev, tm)
                n_sym += packed.shape[1] * m * cache.head_dim_padded
                n_bytes += len(blob)
    return {"symbols": n_sym, "stream_bytes": n_bytes,
            "bits_per_symbol": 8.0 * n_bytes / n_sym if n_sym else 0.0,
            "device_seconds": tm.get("device_seconds", 0.0), "host_seconds": tm.get("host_seconds", 0.0),
            "host_msymbols_per_s": n_sym / tm["host_seconds"] / 1e6 if tm.get("host_seconds") else 0.0}


def rans_decode_e8(data: bytes):
    """Inverse of the encode_e8 stream (decode_e8, entropy_coder.py:455-500) ->
    (doubled lattice codes int8 [n_groups * 8], fp16 scales [n_groups])."""
    off = 0
    n_groups, levels, has_half, n_sym = struct.unpack_from(RANS_HEADER, data, off)
    off += struct.calcsize(RANS_HEADER)
    flen, slen, rlen = struct.unpack_from(RANS_LENGTHS, data, off)
    off += struct.calcsize(RANS_LENGTHS)
    a = struct.unpack_from("<H", data, off)[0]
    freqs = np.frombuffer(data, dtype="<u2", count=a, offset=off + 2).astype(np.uint32)
    off += flen
    scales = np.frombuffer(data, dtype="<f2", count=slen // 2, offset=off).copy()
    off += slen
    words = np.frombuffer(data, dtype="<u2", count=rlen // 2, offset=off)
    sym = rans_decode(words, n_sym, freqs).astype(np.int32)
    codes = (sym - levels) if has_half else 2 * (sym - levels // 2)
    return codes.astype(np.int8), scales


def measure_entropy_counts(counts: np.ndarray, alphabet_size: Optional[int] = None) -> Dict[str, float]:
    """measure_entropy (entropy_coder.py:89-131) from per-symbol counts instead of the symbol
    stream: Shannon bits per symbol, the uniform code's bits, their ratio, the symbol count and
    the number of distinct symbols, with the reference's numpy operations in its order."""
    counts = np.asarray(counts, dtype=np.int64)
    n = int(counts.sum())
    if n == 0:
        return {"entropy_bps": 0, "uniform_bps": 0, "compression_ratio": 1.0, "n_symbols": 0, "n_unique": 0}
    seen = np.nonzero(counts)[0]            # ascending, as np.unique returns them
    c = counts[seen]
    probs = c / n
    entropy = -np.sum(probs * np.log2(probs + 1e-30))
    if alphabet_size is None:
        alphabet_size = int(seen.max()) + 1
    uniform_bps = math.log2(max(alphabet_size, 2))
    return {"entropy_bps": float(entropy), "uniform_bps": float(uniform_bps),
            "compression_ratio": float(uniform_bps / max(entropy, 0.01)), "n_symbols": int(n),
            "n_unique": int(seen.size)}


def e8_entropy_stats(packed: torch.Tensor, head_dim_padded: int, levels: int) -> Dict[str, float]:
    """measure_e8_entropy (entropy_coder.py:134-159) of packed code rows [..., pb]: the
    histogram is taken on the device (kernels.code_histogram), the statistics on the host."""
    cnt = K.code_histogram(packed, head_dim_padded, levels).cpu().numpy().astype(np.int64)
    has_half = bool(cnt[1::2].sum() > 0)
    alpha = cnt if has_half else cnt[0::2]
    return measure_entropy_counts(alpha, alpha.size)
