"""Python side of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this module.  The product package (nexusquant_b200) never does.

It wraps the C restatement in nq_oracle.c (per-vector arithmetic, bit-exact with
the CUDA kernels) and restates, in numpy, the host-side steps of the reference
pipeline (jagmarques/nexusquant v0.5.0):

  rope tables          nexusquant/core/rope_utils.py:106-112 (+ scaling :34-72)
  keep mask            nexusquant/pipeline.py:895-959 (_build_keep_mask)
  key-key importance   nexusquant/pipeline.py:756-782 (_score_importance)
  real-attention score nexusquant/pipeline.py:826-836 applied to synthetic queries
  n_keep formula       nexusquant/pipeline.py:918-920 (IEEE double, as written)
  merge eviction       nexusquant/pipeline.py:961-1048 (_apply_merge_eviction)
  nibble packing       nexusquant/integrations/vllm_backend.py:476-540
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libnq_oracle.so")
_lib = None


def build() -> str:
    """Compile nq_oracle.c into oracle/_build (gcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "nq_oracle.c")
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        L.nqo_quantize.argtypes = [P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P, P,
                                   ctypes.c_int, P, P, P]
        L.nqo_quantize_ex.argtypes = [P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P, P,
                                      ctypes.c_int, P, P, P, ctypes.c_int]
        L.nqo_dequantize.argtypes = [P, P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P, P,
                                     ctypes.c_float, P]
        L.nqo_pack.argtypes = [P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P]
        L.nqo_unpack.argtypes = [P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P]
        L.nqo_delta.argtypes = [P, ctypes.c_long, ctypes.c_long, ctypes.c_int, P]
        L.nqo_attn_colsum.argtypes = [P, P, ctypes.c_int, ctypes.c_long, ctypes.c_int, P,
                                      ctypes.c_double, P]
        L.nqo_packed_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        L.nqo_packed_bytes.restype = ctypes.c_int
        L.nqo_hadamard_entry.argtypes = [ctypes.c_int]
        L.nqo_hadamard_entry.restype = ctypes.c_float
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def next_pow2(n: int) -> int:
    p = 1
    while p < n:
        p *= 2
    return p


# --------------------------------------------------------------------------- rope
def rope_inv_freq(d: int, base: float, rope_scaling=None):
    """inv_freq exactly as rope_utils.py:106 (fp32 torch pow + reciprocal)."""
    import torch
    inv = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    if rope_scaling is not None:
        kind = rope_scaling.get("type", rope_scaling.get("rope_type", "linear"))
        factor = float(rope_scaling.get("factor", 1.0))
        if factor != 1.0:
            if kind in ("linear", "dynamic"):
                inv = inv / factor
            elif kind == "llama3":
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
                inv = torch.stack(out)
    return inv


def rope_tables(positions, d: int, base: float, rope_scaling=None):
    """cos/sin rows [len(positions), d/2] float32 (rope_utils.py:109-112)."""
    import torch
    inv = rope_inv_freq(d, base, rope_scaling)
    pos = torch.as_tensor(np.asarray(positions), dtype=torch.float32)
    fr = torch.outer(pos, inv)
    return fr.cos().numpy().astype(np.float32), fr.sin().numpy().astype(np.float32)


# ---------------------------------------------------------------- quantization
def quantize(x, d_p: int, levels: int, cos=None, sin=None, want_nrm=False, rotate=True):
    """x [n, d] -> (codes [n, d_p] int8, scales [n] f32[, nrm [n, d_p] f32]).
    rotate=False quantizes the rows as given (E8Lattice.quantize_perhead, e8_lattice.py:97-124)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, d = x.shape
    codes = np.empty((n, d_p), np.int8)
    scales = np.empty((n,), np.float32)
    nrm = np.empty((n, d_p), np.float32) if want_nrm else None
    c = s = None
    if cos is not None:
        c = np.ascontiguousarray(cos, dtype=np.float32)
        s = np.ascontiguousarray(sin, dtype=np.float32)
        assert c.shape == (n, d // 2)
    lib().nqo_quantize_ex(_p(x), n, d, d_p, _p(c), _p(s), levels, _p(codes), _p(scales), _p(nrm), int(rotate))
    return (codes, scales, nrm) if want_nrm else (codes, scales)


def dequantize(codes, scales, d: int, cos=None, sin=None, sharpen: float = 1.0):
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    n, d_p = codes.shape
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty((n, d), np.float32)
    c = s = None
    if cos is not None:
        c = np.ascontiguousarray(cos, dtype=np.float32)
        s = np.ascontiguousarray(sin, dtype=np.float32)
    lib().nqo_dequantize(_p(codes), _p(sc), n, d, d_p, _p(c), _p(s), sharpen, _p(out))
    return out


def packed_bytes(d_p: int, levels: int) -> int:
    return lib().nqo_packed_bytes(d_p, levels)


def pack(codes, levels: int):
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    n, d_p = codes.shape
    out = np.empty((n, packed_bytes(d_p, levels)), np.uint8)
    lib().nqo_pack(_p(codes), n, d_p, levels, _p(out))
    return out


def unpack(packed, d_p: int, levels: int):
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    n = packed.shape[0]
    out = np.empty((n, d_p), np.int8)
    lib().nqo_unpack(_p(packed), n, d_p, levels, _p(out))
    return out


def delta(codes):
    """codes [S, T, d_p] int8 -> temporal delta along T."""
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    S, T, dp = codes.shape
    out = np.empty_like(codes)
    lib().nqo_delta(_p(codes), S, T, dp, _p(out))
    return out


# -------------------------------------------------------------------- scoring
def attn_colsum(Q, K, scale: float, qpos=None):
    """Column sums of row-softmax(Q K^T * scale) (float64), optional causal positions."""
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    nq, d = Q.shape
    T = K.shape[0]
    col = np.zeros((T,), np.float64)
    qp = None if qpos is None else np.ascontiguousarray(qpos, dtype=np.int64)
    lib().nqo_attn_colsum(_p(Q), _p(K), nq, T, d, _p(qp), float(scale), _p(col))
    return col


def keykey_importance(K, obs_window: int = 32):
    """K [b, h, T, d] -> importance [b, T] (pipeline.py:756-782), float64."""
    K = np.asarray(K, dtype=np.float32)
    b, h, T, d = K.shape
    obs = min(obs_window, T)
    scale = float(np.float32(d ** -0.5))
    imp = np.zeros((b, T), np.float64)
    for bi in range(b):
        acc = np.zeros((T,), np.float64)
        for hi in range(h):
            acc += attn_colsum(K[bi, hi, T - obs:], K[bi, hi], scale)
        imp[bi] = acc / h
    return imp


def real_importance(Qs, Ks, q_pos0: int):
    """Restated real-attention scorer: per layer, causal softmax of the synthetic
    queries (positions q_pos0 ..) against that layer's keys, column-summed over
    queries, averaged over heads; summed over layers and divided by their count
    (pipeline.py:826-836).  Qs/Ks: lists of [b, H, nq, d] / [b, H, T, d]."""
    n_layers = len(Ks)
    b, H, T, d = Ks[0].shape
    scale = float(np.float32(d ** -0.5))
    imp = np.zeros((b, T), np.float64)
    for Q, K in zip(Qs, Ks):
        nq = Q.shape[2]
        qpos = np.arange(q_pos0, q_pos0 + nq)
        for bi in range(b):
            acc = np.zeros((T,), np.float64)
            for hi in range(H):
                acc += attn_colsum(Q[bi, hi], K[bi, hi], scale, qpos)
            imp[bi] += acc / H
    return imp / n_layers


# ------------------------------------------------------------------- selection
def n_keep_for(T: int, sliding_window: int, rate: float) -> int:
    prefix = max(T - sliding_window, 0)
    return max(1, int(prefix * (1.0 - rate)))


def keep_mask(importance, T: int, sliding_window: int, rate: float, protected_positions=None):
    """(b, T) bool keep mask; top-k ties resolved toward the lower index."""
    imp = np.asarray(importance)
    b = imp.shape[0]
    prefix = max(T - sliding_window, 0)
    nk = n_keep_for(T, sliding_window, rate)
    m = np.zeros((b, T), bool)
    m[:, 0] = True
    if sliding_window > 0 and T > 0:
        m[:, max(0, T - sliding_window):] = True
    if prefix > 1 and nk > 0:
        k = min(nk, prefix - 1)
        for bi in range(b):
            sc = imp[bi, 1:prefix]
            order = np.lexsort((np.arange(sc.shape[0]), -sc))  # value desc, index asc
            m[bi, order[:k] + 1] = True
    if protected_positions is not None:
        for p in protected_positions:
            p = int(p)
            if 0 <= p < T:
                m[:, p] = True
    return m


def threshold_ambiguous(importance, T: int, sliding_window: int, rate: float, rel: float = 1e-6):
    """(b, T) bool: prefix positions whose importance lies within `rel` (relative)
    of the top-k threshold -- their kept/evicted status is excluded from exact
    comparison (tie order and ulp-level score differences)."""
    imp = np.asarray(importance, dtype=np.float64)
    b = imp.shape[0]
    prefix = max(T - sliding_window, 0)
    nk = n_keep_for(T, sliding_window, rate)
    amb = np.zeros((b, T), bool)
    if prefix > 1:
        k = min(nk, prefix - 1)
        for bi in range(b):
            sc = imp[bi, 1:prefix]
            thr = np.sort(sc)[::-1][k - 1]
            near = np.abs(sc - thr) <= rel * max(abs(thr), 1e-30)
            if k < sc.shape[0]:
                nxt = np.sort(sc)[::-1][k]
                near |= np.abs(sc - nxt) <= rel * max(abs(nxt), 1e-30)
            amb[bi, 1:prefix] = near
    return amb


# ---------------------------------------------------------- boundary detection
def boundary_groups(nrm_ref, nrm_mine=None, levels: int = 8, tol: float = 1e-6):
    """Per 8-group flags of inputs within `tol` of an E8 decision boundary.

    nrm_* : [n, d_p] normalised inputs (x / sc).  A group is ambiguous when
      - its two normalised vectors differ and some coordinate lies within tol of
        a rounding boundary of either candidate (k + 1/2 for A, k for B) or of
        the clamp, or two gaps are within tol of each other; or
      - |d_half - d_int| < tol (the candidate choice itself is a near tie).
    """
    x = np.asarray(nrm_ref, dtype=np.float64).reshape(-1, 8)
    a = np.round(x)
    g = np.abs(x - a)
    odd = (a.sum(1) % 2) != 0
    b = np.round(np.float32(x) - np.float32(0.5)).astype(np.float64) + 0.5
    d_int = (g ** 2).sum(1) + np.where(odd, 1.0 - 2.0 * g.min(1), 0.0)
    d_half = ((x - b) ** 2).sum(1)
    amb = np.abs(d_half - d_int) < tol
    if nrm_mine is not None:
        y = np.asarray(nrm_mine, dtype=np.float64).reshape(-1, 8)
        differs = (x != y).any(1)
        fr = x - np.floor(x)
        near_round = (np.abs(fr - 0.5) < tol) | (fr < tol) | (fr > 1 - tol)
        gs = np.sort(g, 1)
        near_gap = (gs[:, 1] - gs[:, 0]) < tol
        amb |= differs & (near_round.any(1) | near_gap)
    return amb.reshape(np.asarray(nrm_ref).shape[0], -1)


# ----------------------------------------------------------------- merge eviction
def merge_unit_centroids(vs_b):
    """Unit-norm value centroids of one batch element (nexusquant/pipeline.py:996-1020):
    mean over heads per layer, summed over the layers in order, divided by their count,
    then x / max(||x||, 1e-12).  vs_b: list of [h, T, d] arrays (full-length layers only)."""
    acc = None
    for v in vs_b:
        m = v.astype(np.float32).mean(axis=0, dtype=np.float32)
        acc = m if acc is None else (acc + m).astype(np.float32)
    c = (acc / np.float32(len(vs_b))).astype(np.float32)
    n = np.sqrt((c.astype(np.float64) ** 2).sum(-1)).astype(np.float32)
    return (c / np.maximum(n, np.float32(1e-12))[:, None]).astype(np.float32)


def merge_similarity(unit, evict_pos, kept_pos):
    """Cosine similarity [n_evict, n_kept] (pipeline.py:1016-1023), in float64 so that the
    tests can tell a genuine argmax from a near tie."""
    return unit[evict_pos].astype(np.float64) @ unit[kept_pos].astype(np.float64).T


def merge_apply(vs_b, imp_b, evict_pos, kept_pos, nearest):
    """The accumulation loop of pipeline.py:1026-1048 for one batch element, on float32 copies:
    for each evicted position in ascending order, v[:, s] = fl32(v[:, s] + fl32(w32 * v[:, e]))
    with w32 = float32(imp_e / (imp_s + imp_e + 1e-8)) evaluated in double (Python floats) --
    torch casts the Python scalar to float32 before the multiply.  Returns new arrays in the
    input dtype."""
    out = []
    for v in vs_b:
        f = v.astype(np.float32)
        for ei, e in enumerate(evict_pos):
            s_ = kept_pos[nearest[ei]]
            ie, is_ = float(imp_b[e]), float(imp_b[s_])
            w = np.float32(ie / (is_ + ie + 1e-8))
            f[:, s_, :] = (f[:, s_, :] + (f[:, e, :] * w).astype(np.float32)).astype(np.float32)
        out.append(f.astype(v.dtype))
    return out


def merge_values(vs, keep_mask_, importance, nearest=None):
    """Whole merge step over [b, h, T, d] layers (pipeline.py:977-1048).  Layers of another
    length are returned unchanged.  nearest: optional per-batch argmax override (to replay a
    device choice that differs from this one only on a near tie).  Returns (layers, nearest)."""
    b, T = keep_mask_.shape
    out = [np.array(v, copy=True) for v in vs]
    full = [i for i, v in enumerate(vs) if v.shape[2] == T]
    chosen = []
    for bi in range(b):
        km = keep_mask_[bi].astype(bool)
        ev, kp = np.nonzero(~km)[0], np.nonzero(km)[0]
        if ev.size == 0 or kp.size == 0 or not full:
            chosen.append(None)
            continue
        if nearest is not None and nearest[bi] is not None:
            nr = np.asarray(nearest[bi])
        else:
            unit = merge_unit_centroids([vs[i][bi] for i in full])
            nr = merge_similarity(unit, ev, kp).argmax(axis=1)
        chosen.append(nr)
        merged = merge_apply([out[i][bi] for i in full], importance[bi], ev, kp, nr)
        for i, m in zip(full, merged):
            out[i][bi] = m
    return out, chosen


# ------------------------------------------------------------------- page nibbles
def pack_codes_nibble(codes):
    """vllm_backend.py:476-513: c = clamp(code + 8, 0, 15); an odd last dim is padded with a
    0 nibble; byte = c_even | c_odd << 4."""
    c = np.clip(np.asarray(codes).astype(np.int32) + 8, 0, 15)
    if c.shape[-1] % 2:
        c = np.concatenate([c, np.zeros(c.shape[:-1] + (1,), np.int32)], axis=-1)
    return ((c[..., 0::2] & 0xF) | ((c[..., 1::2] & 0xF) << 4)).astype(np.uint8)


def unpack_codes_nibble(packed, original_d: int):
    """vllm_backend.py:515-540: low nibble then high nibble, minus 8, first original_d."""
    p = np.asarray(packed).astype(np.int32)
    both = np.stack([p & 0xF, (p >> 4) & 0xF], axis=-1).reshape(p.shape[:-1] + (-1,))
    return (both[..., :original_d] - 8).astype(np.int8)
