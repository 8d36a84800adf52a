"""The C-ABI library loads and exports every symbol include/nexusquant_b200.h declares.
Host-side argument validation is checked too (it runs before any CUDA call)."""
import ctypes
import os
import re

import pytest

from nexusquant_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nexusquant_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nq_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_header_symbols():
    lib = N.load()
    names = header_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    assert set(N.EXPORTED) == set(names)


def test_abi_version_and_status_strings():
    lib = N.load()
    assert lib.nq_abi_version() == 2
    assert lib.nq_status_string(0) == b"ok"
    assert lib.nq_status_string(-6).startswith(b"pointer")
    assert lib.nq_packed_bytes(128, 8) == 80
    assert lib.nq_packed_bytes(128, 4) == 64
    assert lib.nq_packed_bytes(128, 2) == 64
    assert lib.nq_packed_bytes(128, 16) == 128
    assert lib.nq_packed_bytes(64, 8) == 40
    assert lib.nq_packed_bytes(128, 3) == -1


def _params(**kw):
    p = N.CompressParams()
    arr = (N.LayerIO * 1)()
    arr[0].key_levels = arr[0].value_levels = 4
    p.batch, p.heads, p.seq, p.head_dim, p.head_dim_padded, p.n_kept = 1, 1, 16, 128, 128, 16
    p.in_stride_b, p.in_stride_h, p.in_stride_t = 16 * 128, 16 * 128, 128
    p.layers = ctypes.cast(arr, ctypes.POINTER(N.LayerIO))
    p.n_layers = 1
    for k, v in kw.items():
        setattr(p, k, v)
    return p, arr


def test_compress_validation_without_gpu():
    lib = N.load()
    assert lib.nq_compress_layers(None, None) == -1
    p, arr = _params(head_dim=100)
    assert lib.nq_compress_layers(ctypes.byref(p), None) == -2          # unsupported head_dim
    p, arr = _params(head_dim=96, head_dim_padded=96)
    assert lib.nq_compress_layers(ctypes.byref(p), None) == -2          # d_p must be a power of two
    p, arr = _params(in_stride_t=100)
    assert lib.nq_compress_layers(ctypes.byref(p), None) == -6          # row not 16-byte aligned
    p, arr = _params(n_kept=32)
    assert lib.nq_compress_layers(ctypes.byref(p), None) == -1          # n_kept > seq without kept_idx
    p, arr = _params()
    arr[0].v = 16
    arr[0].value_levels = 3
    assert lib.nq_compress_layers(ctypes.byref(p), None) == -1          # levels must be 2, 4, 8, 16
    p, arr = _params(n_kept=0)
    assert lib.nq_compress_layers(ctypes.byref(p), None) == 0           # empty: no work, no launch


def test_other_entry_validation_without_gpu():
    lib = N.load()
    assert lib.nq_select_keep(None, 1, 10, 2, 3, None, 0, None, None, None, 0, None) == -1
    assert lib.nq_score_keykey(None, 0, 1, 1, 1, 128, 0, 0, 0, 32, 0, 1, 0, None, None, 0, None) == -1
    assert lib.nq_score_keykey(16, 0, 1, 1, 8, 80, 0, 0, 0, 32, 0, 1, 0, 16, None, 0, None) == -2
    assert lib.nq_score_keykey(16, 0, 1, 2, 8, 128, 0, 0, 0, 32, 0, 1, 0, 16, None, 0, None) == -5  # no workspace
    assert lib.nq_score_attention(16, 16, 0, 1, 3, 2, 4, 8, 128, 0, 0, 0, 0, 0, 0, 0, 0, 16, None, 0, None) == -1
    assert lib.nq_delta_codes(None, 1, 1, 128, 4, None, None) == -1
    assert lib.nq_gather_rows(16, 0, 1, 1, 12, 0, 0, 0, None, None, 1, 16, 0, 0, 0, None) == -1
    assert lib.nq_reduce_heads(16, 1, 1, 1, 0.0, 0, 16, None) == -1
    assert lib.nq_score_keykey_workspace_size(1, 8, 131072, 32) > 4 * 8 * 131072


def test_missing_library_fails_loudly(tmp_path):
    saved = N._lib
    try:
        N._lib = None
        with pytest.raises(ImportError):
            N.load(str(tmp_path / "nope.so"))
    finally:
        N._lib = saved
