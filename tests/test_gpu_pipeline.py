"""GPU: the reference-facing API (NexusQuantEvict, NexusQuantEvictTruncate,
compress_kv_cache, nexusquant_evict) against outputs of the reference pipelines
recorded in tests/golden/golden.npz."""
import numpy as np
import pytest
import torch

import nexusquant_b200 as nq
from nexusquant_b200 import synthetic as syn
from tests.parity import REL_L2_TOL, golden_str, rel_l2, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


class FakeCache:
    def __init__(self, ks, vs):
        self.key_cache = list(ks)
        self.value_cache = list(vs)


def _pipe_layers(golden, n=3):
    cfgp = syn.CacheConfig("pipe", 3, 2, 2, 96, 128)
    ks, vs = zip(*[syn.cpu_layer(cfgp, l) for l in range(3)])
    if sha(torch.stack(ks)) != golden_str(golden, "pipe_sha"):
        pytest.skip("generator drift")
    return list(ks[:n]), list(vs[:n])


def _close(out, ref, tol=REL_L2_TOL):
    out = out.float().cpu().numpy()
    assert out.shape == ref.shape
    assert rel_l2(out, ref) < tol


def test_evict_mask_and_outputs(golden):
    ks, vs = _pipe_layers(golden)
    cache = FakeCache([k.to(DEV) for k in ks], [v.to(DEV) for v in vs])
    ev = nq.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, protect_boundary=1)
    out, mask = ev.compress(cache)
    assert out is cache
    assert np.array_equal(mask.cpu().numpy(), golden["pipe_evict_mask"])
    for l in range(3):
        assert cache.key_cache[l].dtype == torch.float16
        _close(cache.key_cache[l], golden[f"pipe_evict_k{l}"])
        _close(cache.value_cache[l], golden[f"pipe_evict_v{l}"])
    # protected layers (0 and 2 with protect_boundary=1): exact fp16 copies, evicted rows zeroed
    for l in (0, 2):
        assert np.array_equal(cache.key_cache[l].cpu().numpy(), golden[f"pipe_evict_k{l}"])


def test_quant_only_k3(golden):
    ks, vs = _pipe_layers(golden, 1)
    cache = FakeCache([ks[0].to(DEV)], [vs[0].to(DEV)])
    nq.compress_kv_cache(cache, mode="quant_only", bits=3)
    _close(cache.key_cache[0], golden["pipe_qo_k0"])
    _close(cache.value_cache[0], golden["pipe_qo_v0"])


def test_simple_mode_default(golden):
    ks, vs = _pipe_layers(golden, 1)
    cache = FakeCache([ks[0][:1].to(DEV)], [vs[0][:1].to(DEV)])
    res = nq.compress_kv_cache(cache)
    assert res is cache
    _close(cache.key_cache[0], golden["pipe_simple_k0"])
    _close(cache.value_cache[0], golden["pipe_simple_v0"])


def test_truncate(golden):
    ks, vs = _pipe_layers(golden, 2)
    cache = FakeCache([k[:1].to(DEV) for k in ks], [v[:1].to(DEV) for v in vs])
    tr = nq.NexusQuantEvictTruncate(bits=2, key_bits=3, eviction_rate=0.5, sliding_window=10)
    _, nxt = tr.compress(cache)
    assert isinstance(nxt, int) and nxt == int(golden["pipe_trunc_next"][0])
    for l in range(2):
        _close(cache.key_cache[l], golden[f"pipe_trunc_k{l}"])
        _close(cache.value_cache[l], golden[f"pipe_trunc_v{l}"])
    with pytest.raises(ValueError):
        tr.compress(FakeCache([ks[0].to(DEV)], [vs[0].to(DEV)]))  # batch 2


def test_soft_eviction(golden):
    ks, vs = _pipe_layers(golden, 1)
    cache = FakeCache([ks[0].to(DEV)], [vs[0].to(DEV)])
    ev = nq.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, soft_eviction=True)
    _, mask = ev.compress(cache)
    assert mask.sum().item() == mask.numel()
    _close(cache.key_cache[0], golden["pipe_soft_k0"])
    _close(cache.value_cache[0], golden["pipe_soft_v0"])


def test_compressed_layout_roundtrip(golden):
    """layout='compressed': the CompressedKVCache dequantizes to the fake-quant rows (up to
    the fp16 rounding of the stored scales) and survives to_bytes/from_bytes."""
    ks, vs = _pipe_layers(golden)
    ev = nq.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, protect_boundary=1,
                            layout="compressed")
    cc, mask = ev.compress(FakeCache([k.to(DEV) for k in ks], [v.to(DEV) for v in vs]))
    assert isinstance(cc, nq.CompressedKVCache)
    kept = np.nonzero(golden["pipe_evict_mask"][0])[0]
    assert int(cc.kept_count[0]) == len(kept)
    assert np.array_equal(cc.positions[0, :len(kept)].cpu().numpy(), kept)
    dec = cc.decompress()
    ref = golden["pipe_evict_k1"][0][:, kept]
    assert rel_l2(dec[1][0][0].float().cpu().numpy(), ref) < 2e-3
    assert np.array_equal(dec[0][0][0].cpu().numpy(), golden["pipe_evict_k0"][0][:, kept])
    blob = cc.to_bytes()
    assert blob[:4] == b"NQC1"
    back = nq.CompressedKVCache.from_bytes(blob, device=DEV)
    d2 = back.decompress()
    assert all(torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) for a, b in zip(dec, d2))
    # 2 of the 3 layers are fp16-protected here, so the whole-cache ratio is modest
    assert cc.compression_ratio() > 1.5
    assert cc.layers[1].nbytes() == 2 * 2 * len(kept) * (64 + 64 + 2 + 2)


def test_min_context_and_adaptive(golden):
    ks, vs = _pipe_layers(golden, 1)
    cache = FakeCache([ks[0].to(DEV)], [vs[0].to(DEV)])
    k_before = cache.key_cache[0].clone()
    ev = nq.NexusQuantEvict(eviction_rate=0.8, min_context_for_compression=200)
    _, mask = ev.compress(cache)
    assert mask.sum().item() == mask.numel() and torch.equal(cache.key_cache[0], k_before)
    ev = nq.NexusQuantEvict(eviction_rate=0.8, sliding_window=4, adaptive_context=True)
    _, mask = ev.compress(FakeCache([ks[0].to(DEV)], [vs[0].to(DEV)]))
    assert mask.sum().item() == mask.numel()


def test_hf_hook_tiny_llama():
    """nexusquant_evict on a tiny random Llama: every layer compressed once on prefill; layer 0
    (whose input does not depend on earlier compression) equals NexusQuantEvict applied to
    the uncompressed cache."""
    pytest.importorskip("transformers")
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=512)
    model = LlamaForCausalLM(cfg).to(DEV, torch.float16).eval()
    ids = torch.randint(0, 128, (1, 90), device=DEV)
    with torch.no_grad():
        plain = model(ids, use_cache=True).past_key_values
    with nq.nexusquant_evict(model, quality="balanced", verbose=False) as comp:
        with torch.no_grad():
            hooked = model(ids, use_cache=True).past_key_values
    assert comp.last_mask is not None and comp.last_mask.shape == (1, 90)
    k, v = plain.layers[0].keys, plain.layers[0].values
    ref = nq.NexusQuantEvict(head_dim=64, bits=2, eviction_rate=0.6, sliding_window=32, rope_base=comp.rope_base)
    c = FakeCache([k.clone()], [v.clone()])
    ref.compress(c)
    assert torch.equal(hooked.layers[0].keys, c.key_cache[0])
    assert torch.equal(hooked.layers[0].values, c.value_cache[0])
    n_kept = int(comp.last_mask.sum().item())
    for l in range(3):
        hk = hooked.layers[l].keys
        assert hk.dtype == torch.float16 and hk.shape == (1, 2, 90, 64)
        assert int((hk.abs().sum(-1) != 0).sum(-1).max().item()) == n_kept


def test_evict_host_cache_through_api_matches_device():
    """NexusQuantEvict(layout="compressed") on a cache in pinned host memory, result copied back
    to pinned host memory group by group, equals the device-resident call bit for bit; a second
    call writes into the first call's host buffers."""
    cfg = syn.CacheConfig("host", 6, 2, 4, 600, 128, key_bits=2, value_bits=2, eviction_rate=0.7)
    ks, vs = zip(*[syn.cpu_layer(cfg, l) for l in range(6)])
    ref, mask_d = nq.NexusQuantEvict(bits=2, eviction_rate=0.7, protect_boundary=1, layout="compressed").compress(
        FakeCache([k.to(DEV) for k in ks], [v.to(DEV) for v in vs]))
    host = FakeCache([k.pin_memory() for k in ks], [v.pin_memory() for v in vs])
    ev = nq.NexusQuantEvict(bits=2, eviction_rate=0.7, protect_boundary=1, layout="compressed", device=DEV,
                            result_on_host=True, group_layers=2)
    first = None
    for _ in range(2):
        out, mask_h = ev.compress(host)
        torch.cuda.synchronize()
        assert torch.equal(mask_h.cpu(), mask_d.cpu())
        assert torch.equal(out.positions, ref.positions.cpu()) and out.positions.is_pinned()
        for lo, lr in zip(out.layers, ref.layers):
            assert lo.protected == lr.protected
            if lo.protected:
                pairs = [(lo.k_fp16, lr.k_fp16), (lo.v_fp16, lr.v_fp16)]
            else:
                pairs = [(getattr(lo.codes, f), getattr(lr.codes, f)) for f in ("k_codes", "v_codes", "k_scales",
                                                                                  "v_scales")]
            for a, b in pairs:
                assert not a.is_cuda and a.is_pinned() and torch.equal(a, b.cpu())
        if first is None:
            first = out.layers[2].codes.k_codes.data_ptr()
        else:
            assert out.layers[2].codes.k_codes.data_ptr() == first


def test_real_scorer_on_model_without_attention_matrix():
    """scorer='real' on a tiny Llama: the recorded-queries tensor-core route gives the reference's
    eager-attention importance (fp32 model: within 1e-5) and the same keep mask, and at T = 8192 it
    runs without forming a (b, H, T, T) attention tensor."""
    pytest.importorskip("transformers")
    from transformers import LlamaConfig, LlamaForCausalLM
    from nexusquant_b200.pipeline import _real_importance_recorded
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=8192,
                      attn_implementation="eager")
    model = LlamaForCausalLM(cfg).to(DEV, torch.float32).eval()
    ids = torch.randint(0, 128, (2, 300), device=DEV)
    ours = _real_importance_recorded(model, ids)
    assert ours is not None
    with torch.no_grad():
        att = model(ids, use_cache=False, output_attentions=True).attentions
    ref = sum(a.float().sum(dim=2).mean(dim=1) for a in att) / len(att)   # pipeline.py:826-835
    assert torch.allclose(ours, ref, rtol=1e-5, atol=1e-6)
    ev = nq.NexusQuantEvict(head_dim=64, bits=2, eviction_rate=0.5, sliding_window=16, scorer="real")
    m_ours = ev._build_keep_mask(ours, 300, 0.5)
    m_ref = ev._build_keep_mask(ref, 300, 0.5)
    assert torch.equal(m_ours, m_ref)
    # long prefill (SDPA forward): memory stays far below one layer's attention tensor
    ids = torch.randint(0, 128, (1, 8192), device=DEV)
    cfg.attn_implementation = "sdpa"
    sdpa = LlamaForCausalLM(cfg)
    sdpa.load_state_dict(model.state_dict())
    model = sdpa.to(DEV, torch.float16).eval()

    def peak_of(fn):
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        out = fn()
        torch.cuda.synchronize()
        return out, torch.cuda.max_memory_allocated() - base

    with torch.no_grad():
        _, fwd = peak_of(lambda: model(ids, use_cache=False).logits)
    imp, ours = peak_of(lambda: _real_importance_recorded(model, ids))
    assert imp.shape == (1, 8192) and torch.isfinite(imp).all()
    # beyond the forward pass itself: the recorded queries/keys and the scorer's workspace, far
    # below one fp32 (1, 4, T, T) attention tensor (1 GiB)
    assert ours - fwd < 128 << 20, (ours, fwd)
