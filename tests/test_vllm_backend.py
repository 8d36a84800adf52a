"""Paged interface (nexusquant/integrations/vllm_backend.py) on the B200 kernels.

Pinned to the reference's own compress_page / decompress_page / pack_codes_nibble outputs
(tests/golden/golden.npz "dq_*"), and checked for the properties the reference's page helpers
have: paging a sequence equals compressing each page, decompress_kv_pages equals the page-by-
page decompression, and the paged decode attention equals decompress_page followed by the
reference's fp32 softmax attention (vllm_backend.py:728-763).
"""
import math
import types

import numpy as np
import pytest
import torch

from nexusquant_b200 import synthetic as syn
from nexusquant_b200.integrations import vllm_backend as VB
from tests.parity import REL_L2_TOL, rel_l2

DEV = "cuda:0"


# ----------------------------------------------------------------------------- CPU


def test_oracle_nibbles_match_reference(golden, orc):
    assert np.array_equal(orc.pack_codes_nibble(golden["dq_k_codes"]), golden["dq_k_nibble"])
    assert np.array_equal(orc.unpack_codes_nibble(golden["dq_k_nibble"], 128), golden["dq_k_codes"])
    odd = np.array([[-9, 3, 7, 20, -4]], np.int8)  # clamps and an odd length
    assert np.array_equal(orc.pack_codes_nibble(odd), np.array([[0 | (11 << 4), 15 | (15 << 4), 4]], np.uint8))


def test_page_accounting():
    h, n, d = 4, 10, 128
    p = VB.CompressedPage(torch.zeros(h, n, d, dtype=torch.int8), torch.zeros(h, n, d, dtype=torch.int8),
                          torch.zeros(h, n, dtype=torch.float16), torch.zeros(h, n, dtype=torch.float16),
                          torch.zeros(n, dtype=torch.int32), n)
    assert p.compressed_bytes == 2 * h * n * d + 2 * h * n * 2 + 4 * n
    assert p.uncompressed_bytes == 4 * h * n * d
    comp = VB.NexusQuantKVCompressor(head_dim=128, bits=2)
    assert comp.compression_ratio(p) == p.uncompressed_bytes / p.compressed_bytes
    m = VB.measure_compression_ratio([p, p], bits=2)
    assert m["ratio"] == p.uncompressed_bytes / p.compressed_bytes and m["bits"] == 2
    assert VB.measure_compression_ratio([])["ratio"] == 1.0


def test_compressor_argument_errors():
    with pytest.raises(ValueError, match="bits must be 2, 3, or 4"):
        VB.NexusQuantKVCompressor(bits=5)
    with pytest.raises(ValueError, match="power of 2"):
        VB.NexusQuantKVCompressor(head_dim=96)
    with pytest.raises(ValueError, match="pages list is empty"):
        VB.decompress_kv_pages([])


def test_infer_block_size_as_reference():
    assert VB.NexusQuantPagedAttention._infer_block_size(torch.tensor([], dtype=torch.int64)) == 16
    assert VB.NexusQuantPagedAttention._infer_block_size(torch.tensor([0, 17, 35])) == 4


def test_register_backend_reads_engine_config():
    cfg = types.SimpleNamespace(model_config=types.SimpleNamespace(head_dim=128, rope_theta=500000.0))
    pa = VB.register_nexusquant_backend(cfg, bits=3)
    assert isinstance(pa, VB.NexusQuantPagedAttention)
    assert (pa.compressor.head_dim, pa.compressor.levels, pa.compressor.rope_base) == (128, 8, 500000.0)
    cfg = types.SimpleNamespace(model_config=types.SimpleNamespace(hidden_size=4096, num_attention_heads=64))
    assert VB.register_nexusquant_backend(cfg).compressor.head_dim == 64
    with pytest.warns(RuntimeWarning):
        assert VB._extract_head_dim(types.SimpleNamespace()) == 128


# ----------------------------------------------------------------------------- GPU


def _dq_page():
    kk, vv = syn.cpu_layer(syn.CacheConfig("dq", 1, 1, 2, 24, 128), 11)
    pos = torch.tensor([0, 3, 4, 9, 10, 11, 20, 31, 40, 41, 42, 50, 63, 64, 65, 70, 71, 72, 80, 81, 90, 99,
                        100, 127], dtype=torch.int32)
    return kk[0], vv[0], pos


@pytest.mark.gpu
def test_compress_decompress_page_match_reference(golden):
    k, v, pos = _dq_page()
    comp = VB.NexusQuantKVCompressor(head_dim=128, bits=2, rope_base=10000.0)
    page = comp.compress_page(k.to(DEV), v.to(DEV), pos.to(DEV))
    assert page.num_valid == 24 and page.key_codes.dtype == torch.int8
    assert np.array_equal(page.key_codes.cpu().numpy().reshape(-1, 128), golden["dq_k_codes"])
    assert np.array_equal(page.value_codes.cpu().numpy().reshape(-1, 128), golden["dq_v_codes"])
    assert np.array_equal(page.key_scales.cpu().numpy().reshape(-1), golden["dq_k_scales16"])
    assert np.array_equal(page.value_scales.cpu().numpy().reshape(-1), golden["dq_v_scales16"])
    dk, dv = comp.decompress_page(page)
    # bit-exact against the oracle's dequantize; the reference inverts the Hadamard with a
    # matmul (other rounding), so against its output the bar is the relative L2 tolerance
    from oracle import oracle as orc
    cos, sin = orc.rope_tables(pos.numpy(), 128, 10000.0)
    okr = orc.dequantize(golden["dq_k_codes"], golden["dq_k_scales16"].astype(np.float32), 128,
                         np.tile(cos, (2, 1)), np.tile(sin, (2, 1))).astype(np.float16)
    ovr = orc.dequantize(golden["dq_v_codes"], golden["dq_v_scales16"].astype(np.float32), 128).astype(np.float16)
    assert np.array_equal(dk.cpu().numpy().reshape(-1, 128), okr)
    assert np.array_equal(dv.cpu().numpy().reshape(-1, 128), ovr)
    assert rel_l2(dk.cpu().numpy(), golden["dq_k_out"]) < REL_L2_TOL
    assert rel_l2(dv.cpu().numpy(), golden["dq_v_out"]) < REL_L2_TOL
    assert np.array_equal(comp.pack_codes_nibble(page.key_codes).cpu().numpy().reshape(-1, 64), golden["dq_k_nibble"])
    # decompress_for_attention: logits of the decompressed keys against the reference formula
    q = torch.randn(2, 3, 128, device=DEV)
    lg = comp.decompress_for_attention(page, q)
    ref = torch.einsum("hqd,hsd->hqs", q, dk.float()) / math.sqrt(128)
    assert torch.allclose(lg, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("bits,d", [(3, 128), (4, 128), (2, 64), (4, 64)])
def test_page_codes_equal_library_codes(orc, bits, d):
    """Unpacked page codes are the library's packed codes, coordinate for coordinate."""
    from nexusquant_b200 import kernels as K
    g = torch.Generator().manual_seed(bits * d)
    k = torch.randn(3, 37, d, generator=g).half().to(DEV)
    v = torch.randn(3, 37, d, generator=g).half().to(DEV)
    pos = torch.arange(5, 5 + 37 * 3, 3, dtype=torch.int32, device=DEV)
    comp = VB.NexusQuantKVCompressor(head_dim=d, bits=bits, rope_base=500000.0)
    page = comp.compress_page(k, v, pos)
    lc = K.compress_layers([k[None]], [v[None]], key_levels=2 ** bits, value_levels=2 ** bits, positions=pos[None],
                           rope_base=500000.0)[0]
    for codes, packed in ((page.key_codes, lc.k_codes), (page.value_codes, lc.v_codes)):
        ref = orc.unpack(packed.cpu().numpy().reshape(-1, packed.shape[-1]), d, 2 ** bits)
        assert np.array_equal(codes.cpu().numpy().reshape(-1, d), ref)
    # decompress_page = the library's dequantize of the same codes
    dk, dv = comp.decompress_page(page)
    ok, ov = K.decompress_layers([lc], pos[None], head_dim=d, rope_base=500000.0)
    assert torch.equal(dk, ok[0][0]) and torch.equal(dv, ov[0][0])


@pytest.mark.gpu
@pytest.mark.parametrize("d", [7, 128, 129])
def test_nibble_pack_unpack_vs_oracle(orc, d):
    rng = np.random.default_rng(d)
    codes = rng.integers(-20, 21, size=(5, d)).astype(np.int8)
    p = VB.NexusQuantKVCompressor.pack_codes_nibble(torch.from_numpy(codes).to(DEV))
    assert np.array_equal(p.cpu().numpy(), orc.pack_codes_nibble(codes))
    u = VB.NexusQuantKVCompressor.unpack_codes_nibble(p, d)
    assert np.array_equal(u.cpu().numpy(), orc.unpack_codes_nibble(orc.pack_codes_nibble(codes), d))


@pytest.mark.gpu
def test_kv_pages_equal_page_by_page():
    g = torch.Generator().manual_seed(1)
    h, T, d = 4, 50, 128
    k = torch.randn(h, T, d, generator=g).half().to(DEV)
    v = torch.randn(h, T, d, generator=g).half().to(DEV)
    pos = torch.arange(100, 100 + T, dtype=torch.int32, device=DEV)
    pages = VB.compress_kv_pages(k, v, pos, block_size=16, bits=3, rope_base=10000.0)
    assert [p.num_valid for p in pages] == [16, 16, 16, 2]
    comp = VB.NexusQuantKVCompressor(head_dim=d, bits=3, rope_base=10000.0)
    for i, p in enumerate(pages):
        q = comp.compress_page(k[:, 16 * i:16 * i + p.num_valid], v[:, 16 * i:16 * i + p.num_valid],
                               pos[16 * i:16 * i + p.num_valid])
        for a, b in ((p.key_codes, q.key_codes), (p.value_codes, q.value_codes), (p.key_scales, q.key_scales),
                     (p.value_scales, q.value_scales), (p.positions, q.positions)):
            assert torch.equal(a, b)
    dk, dv = VB.decompress_kv_pages(pages, comp)
    per = [comp.decompress_page(p) for p in pages]
    assert torch.equal(dk, torch.cat([a for a, _ in per], 1)) and torch.equal(dv, torch.cat([b for _, b in per], 1))


def _ref_forward(comp, query, cache, block_tables, context_lens):
    """NexusQuantPagedAttention.forward as the reference writes it (vllm_backend.py:728-763)."""
    b, h, d = query.shape
    out = torch.zeros_like(query)
    for bi in range(b):
        n = int(context_lens[bi])
        pages = [cache[i] for i in block_tables[bi] if i in cache]
        if n == 0 or not pages:
            continue
        kv = [comp.decompress_page(p) for p in pages]
        keys = torch.cat([a for a, _ in kv], 1)[:, :n]
        values = torch.cat([c for _, c in kv], 1)[:, :n]
        lg = torch.einsum("hqd,hsd->hqs", query[bi].unsqueeze(1).float(), keys.float()) / math.sqrt(d)
        out[bi] = torch.einsum("hqs,hsd->hqd", torch.softmax(lg, -1), values.float()).squeeze(1).half()
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("d", [128, 64])
def test_paged_attention_cache_and_forward(d):
    g = torch.Generator().manual_seed(d)
    h = 4
    comp = VB.NexusQuantKVCompressor(head_dim=d, bits=2, rope_base=10000.0)
    pa = VB.NexusQuantPagedAttention(comp)
    blocks = [pa.allocate_block() for _ in range(6)]
    assert blocks == list(range(6)) and not pa.is_block_compressed(0)
    # 3 sequences: blocks [0, 1, 2] (10 tokens), [3, 4] (7 tokens), [5] (unused); block size is
    # inferred as 4, so slot = block * 4 + offset
    slots, toks = [], 0
    for blk, n in ((0, 4), (1, 4), (2, 2), (3, 4), (4, 3)):
        slots += [blk * 4 + o for o in range(n)]
        toks += n
    key = torch.randn(toks, h, d, generator=g).half().to(DEV)
    value = torch.randn(toks, h, d, generator=g).half().to(DEV)
    cache = {}
    pa.compress_and_cache(key, value, cache, cache, torch.tensor(slots, dtype=torch.int64, device=DEV))
    assert sorted(cache) == [0, 1, 2, 3, 4]
    assert [cache[i].num_valid for i in range(5)] == [4, 4, 2, 4, 3]
    # each block equals compress_page of its tokens at positions slot % 4
    first = comp.compress_page(key[:4].permute(1, 0, 2), value[:4].permute(1, 0, 2),
                               torch.arange(4, dtype=torch.int32, device=DEV))
    assert torch.equal(cache[0].key_codes, first.key_codes) and torch.equal(cache[0].value_scales, first.value_scales)
    query = torch.randn(3, h, d, generator=g).half().to(DEV)
    tables = [[0, 1, 2], [3, 4, 9], [5]]
    ctx = torch.tensor([9, 7, 4])
    out = pa.forward(query, cache, cache, tables, ctx)
    ref = _ref_forward(comp, query, cache, tables, ctx)
    assert out.shape == query.shape and out.dtype == torch.float16
    assert torch.count_nonzero(out[2]) == 0  # no compressed block -> zeros, as the reference
    assert rel_l2(out.float().cpu().numpy(), ref.float().cpu().numpy()) < 2e-3
