"""nq_score_keykey_noalloc: key-key importance for callers that cannot allocate
device memory when they score (code inside an allocator or memory pool, engines
that reserve all device memory up front, bindings without cudaMalloc).

Called through the C ABI and compared with nq_score_keykey (caller-provided
workspace) on two consecutive calls, since every call reuses the library's one
built-in scratch array.  Kept in a file of its own, collected last."""
import ctypes

import numpy as np
import pytest
import torch

from nexusquant_b200 import _native as N
from nexusquant_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def _reference_scores(lib, k, per_head, h0, h1):
    b, h, T, d = k.shape
    dt = _CODE[k.dtype]
    ws_n = lib.nq_score_keykey_workspace_size(b, h1 - h0, T, 32)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=DEV)
    out = torch.empty((b, h1 - h0, T) if per_head else (b, T), dtype=torch.float32, device=DEV)
    st = k.stride()
    s = torch.cuda.current_stream().cuda_stream
    N.check("nq_score_keykey", lib.nq_score_keykey(k.data_ptr(), dt, b, h, T, d, st[0], st[1], st[2], 32, h0, h1,
                                                   int(per_head), out.data_ptr(), ws.data_ptr(), ws_n, s))
    return out


def _noalloc_scores(lib, k, per_head, h0, h1):
    b, h, T, d = k.shape
    dt = _CODE[k.dtype]
    out = torch.empty((b, h1 - h0, T) if per_head else (b, T), dtype=torch.float32, device=DEV)
    st = k.stride()
    s = torch.cuda.current_stream().cuda_stream
    N.check("nq_score_keykey_noalloc", lib.nq_score_keykey_noalloc(k.data_ptr(), dt, b, h, T, d, st[0], st[1],
                                                                   st[2], 32, h0, h1, int(per_head),
                                                                   out.data_ptr(), s))
    return out


@pytest.mark.parametrize("per_head,h0,h1", [(0, 0, 8), (1, 2, 5)])
def test_noalloc_matches_workspace_entry_two_calls(per_head, h0, h1):
    lib = N.load()
    # two different inputs in a row: the second call must not see the first call's scratch
    for layer, seq in ((0, 4096), (1, 1500)):
        k, _ = syn.cpu_layer(syn.CacheConfig("na", 1, 1, 8, seq, 128), layer)
        k = k.to(DEV)
        ref = _reference_scores(lib, k, per_head, h0, h1)
        got = _noalloc_scores(lib, k, per_head, h0, h1)
        torch.cuda.synchronize()
        assert np.allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=5e-5, atol=1e-8)


@pytest.mark.parametrize("dtype,d", [(torch.float32, 128), (torch.bfloat16, 96), (torch.float16, 64),
                                     (torch.float32, 96)])
def test_noalloc_other_dtypes_and_head_dims(dtype, d):
    """fp32 runs the CUDA-core scorer, fp16/bf16 the tensor-core one; both carve the same array."""
    lib = N.load()
    for layer, seq in ((2, 2048), (3, 777)):
        k, _ = syn.cpu_layer(syn.CacheConfig("na", 1, 2, 4, seq, d), layer)
        k = k.to(DEV, dtype)
        ref = _reference_scores(lib, k, 0, 0, 4)
        got = _noalloc_scores(lib, k, 0, 0, 4)
        torch.cuda.synchronize()
        assert np.allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=5e-5, atol=1e-8)


def test_noalloc_at_documented_capacity():
    """One 131072-token, 8-head, head_dim-128 layer fits in the built-in scratch (6 MiB of 8)."""
    lib = N.load()
    g = torch.Generator(device=DEV).manual_seed(5)
    for _ in range(2):
        k = torch.randn((1, 8, 131072, 128), generator=g, device=DEV).half()
        ref = _reference_scores(lib, k, 0, 0, 8)
        got = _noalloc_scores(lib, k, 0, 0, 8)
        torch.cuda.synchronize()
        assert np.allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=5e-5, atol=1e-8)


def test_noalloc_rejects_oversize():
    lib = N.load()
    k = torch.empty((1, 8, 16, 128), dtype=torch.float16, device=DEV)
    out = torch.empty(1, dtype=torch.float32, device=DEV)
    # 8 heads x 1M tokens of column sums alone need 32 MiB > the built-in 8 MiB
    st = lib.nq_score_keykey_noalloc(k.data_ptr(), 0, 1, 8, 1 << 20, 128, 0, 0, 0, 32, 0, 8, 0, out.data_ptr(),
                                     None)
    assert st == -7
    assert b"scratch" in lib.nq_status_string(st)
