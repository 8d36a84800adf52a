"""GPU parity at the exact shape of every benchmark configuration.

Each case builds one layer of the configuration's synthetic cache on the CPU (seeded,
bit-reproducible), runs the configuration's keep-set path on the GPU (key-key or
real-attention scorer, then the top-k select), compresses and dequantizes the layer with the
CUDA kernels, and checks against the CPU oracle:

  * importance within rtol 5e-5 (the oracle scores in float64);
  * the keep set equal to the oracle's keep mask on the GPU importance, and equal to the
    mask on the oracle's importance except tokens within 1e-4 (relative) of the top-k
    threshold, twice the scorer's rtol (the count of such flips is printed);
  * packed code bytes and fp16 scales bit-exact, fp16 dequantized rows bit-exact;
  * the fraction of 8-groups whose normalised input lies within 1e-6 of an E8 decision
    boundary (the groups the comparison against the reference would exclude) is printed.
"""
import numpy as np
import pytest
import torch

from nexusquant_b200 import kernels as K
from nexusquant_b200 import synthetic as syn
from nexusquant_b200.pipeline import kept_capacity, n_keep_for
from tests.parity import BOUNDARY_TOL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _keep_set(orc, cfg, k0, layers_q=None, layers_k=None):
    """GPU importance + keep set for the configuration, checked against the oracle.
    Returns (kept [b, n] int64 numpy, kept_idx device, kept_count device, n_cap)."""
    b, h, T, d = k0.shape
    if cfg.eviction_rate == 0.0:
        kept = np.tile(np.arange(T), (b, 1))
        return kept, None, None, T
    if cfg.scorer == "real":
        acc = torch.zeros(b, T, device=DEV)
        for q, k in zip(layers_q, layers_k):
            K.score_attention(q.to(DEV), k.to(DEV), T - q.shape[2], out=acc, accumulate=True)
        imp = (acc / len(layers_k)).cpu().numpy()
        oimp = orc.real_importance([q.float().numpy() for q in layers_q], [k.float().numpy() for k in layers_k],
                                   T - layers_q[0].shape[2])
    else:
        imp = K.score_keykey(k0.to(DEV), 32).cpu().numpy()
        oimp = orc.keykey_importance(k0.float().numpy(), 32)
    assert np.allclose(imp, oimp, rtol=5e-5, atol=1e-8)
    nk = n_keep_for(T, cfg.sliding_window, cfg.eviction_rate)
    idx, cnt = K.select_keep(torch.as_tensor(imp, device=DEV), cfg.sliding_window, nk)
    cap = kept_capacity(T, cfg.sliding_window, nk)
    m_gpu = orc.keep_mask(imp, T, cfg.sliding_window, cfg.eviction_rate)
    m_orc = orc.keep_mask(oimp, T, cfg.sliding_window, cfg.eviction_rate)
    amb = orc.threshold_ambiguous(oimp, T, cfg.sliding_window, cfg.eviction_rate, rel=1e-4)
    idx_h, cnt_h = idx.cpu().numpy(), cnt.cpu().numpy()
    kept = np.zeros((b, cap), np.int64)
    flips = 0
    for bi in range(b):
        assert cnt_h[bi] == cap == m_gpu[bi].sum()
        assert np.array_equal(idx_h[bi, :cap], np.nonzero(m_gpu[bi])[0])
        diff = m_gpu[bi] != m_orc[bi]
        assert not (diff & ~amb[bi]).any(), f"keep sets differ off the threshold in batch {bi}"
        flips += int(diff.sum())
        kept[bi] = idx_h[bi, :cap]
    print(f"[{cfg.name}] kept {cap}/{T} tokens; {int(amb.sum())} tokens within 1e-4 of the threshold, "
          f"{flips} of them kept/evicted differently than on the float64 oracle importance")
    return kept, idx[:, :cap].contiguous(), cnt, cap


def _layer_parity(orc, cfg, k, v, kept, kidx, kcnt, n_cap):
    b, h, T, d = k.shape
    dp = K.next_pow2(d)
    lk, lv = 2 ** cfg.key_bits, 2 ** cfg.value_bits
    sharpen = K.SHARPEN if cfg.sharpen else 1.0
    kd, vd = k.to(DEV), v.to(DEV)
    lc = K.compress_layers([kd], [vd], key_levels=lk, value_levels=lv, kept_idx=kidx, kept_count=kcnt,
                           n_kept=n_cap, rope_base=cfg.rope_base, rope_rows=T)[0]
    pos = torch.as_tensor(kept, dtype=torch.int32, device=DEV)
    ok, ov = K.decompress_layers([lc], pos, head_dim=d, count=kcnt, rope_base=cfg.rope_base,
                                 key_sharpen=sharpen)
    del kd, vd
    # oracle on the kept rows, in [b, h, n] order
    kr = np.stack([k[bi, :, kept[bi]].float().numpy() for bi in range(b)]).reshape(-1, d)
    vr = np.stack([v[bi, :, kept[bi]].float().numpy() for bi in range(b)]).reshape(-1, d)
    cos = np.zeros((b, h, n_cap, d // 2), np.float32)
    sin = np.zeros_like(cos)
    for bi in range(b):
        c, s = orc.rope_tables(kept[bi], d, cfg.rope_base)
        cos[bi], sin[bi] = c[None], s[None]
    cos, sin = cos.reshape(-1, d // 2), sin.reshape(-1, d // 2)
    kc, ks, knrm = orc.quantize(kr, dp, lk, cos, sin, want_nrm=True)
    vc, vs, vnrm = orc.quantize(vr, dp, lv, want_nrm=True)
    assert np.array_equal(lc.k_codes.cpu().numpy().reshape(-1, K.packed_bytes(dp, lk)), orc.pack(kc, lk))
    assert np.array_equal(lc.v_codes.cpu().numpy().reshape(-1, K.packed_bytes(dp, lv)), orc.pack(vc, lv))
    k16 = lc.k_scales.cpu().numpy().reshape(-1)
    v16 = lc.v_scales.cpu().numpy().reshape(-1)
    assert np.array_equal(k16, ks.astype(np.float16)) and np.array_equal(v16, vs.astype(np.float16))
    okr = orc.dequantize(kc, k16.astype(np.float32), d, cos, sin, sharpen=sharpen).astype(np.float16)
    ovr = orc.dequantize(vc, v16.astype(np.float32), d).astype(np.float16)
    assert np.array_equal(ok[0].cpu().numpy().reshape(-1, d), okr)
    assert np.array_equal(ov[0].cpu().numpy().reshape(-1, d), ovr)
    n_groups = kc.size // 8 + vc.size // 8
    amb = int(orc.boundary_groups(knrm, None, lk, BOUNDARY_TOL).sum() +
              orc.boundary_groups(vnrm, None, lv, BOUNDARY_TOL).sum())
    print(f"[{cfg.name}] {n_groups} groups bit-exact vs the oracle; {amb} ({amb / n_groups:.2e}) lie within "
          f"{BOUNDARY_TOL:g} of a decision boundary (excluded against the reference)")
    return n_groups, amb


@pytest.mark.parametrize("cid", [1, 3, 4])
def test_config_layer_parity(orc, cid):
    """Configs 1 (b4 T4096 K3V2 quant-only, sharpening), 3 (T32768 K2V2 key-key 60 %) and 4
    (T131072 RoPE base 5e5 K2V2 key-key 80 %): one full layer at the configuration's shape."""
    cfg = syn.CONFIGS[cid]
    k, v = syn.cpu_layer(cfg, 0)
    kept, kidx, kcnt, cap = _keep_set(orc, cfg, k)
    if cid == 4:
        assert cap == 26240
    _layer_parity(orc, cfg, k, v, kept, kidx, kcnt, cap)


def test_config2_real_scorer_layer_parity(orc):
    """Config 2: Phi-3-mini shape (b2, 32 heads, d96 zero-padded to 128, T8192), keep set from
    the tcgen05 real-attention scorer over 64 synthetic causal queries of two layers."""
    cfg = syn.CONFIGS[2]
    ks, vs, qs = [], [], []
    for l in range(2):
        k, v = syn.cpu_layer(cfg, l)
        ks.append(k)
        vs.append(v)
        qs.append(syn.cpu_queries(cfg, l))
    kept, kidx, kcnt, cap = _keep_set(orc, cfg, ks[0], qs, ks)
    _layer_parity(orc, cfg, ks[1], vs[1], kept, kidx, kcnt, cap)


@pytest.mark.parametrize("heads", [1, 2, 4])
def test_config4_head_slice_parity(orc, heads):
    """The per-rank shapes of config 4's head-sharded runs at 8, 4 and 2 GPUs (1, 2 and 4 KV
    heads per rank: head groups of 1, 2 and 4 in the compress and dequantize tiles), RoPE base
    5e5, K2V2 after the key-key keep set, at T = 16384 so the oracle finishes in seconds."""
    cfg = syn.CacheConfig("cfg4_slice", 2, 1, heads, 16384, 128, rope_base=500000.0, key_bits=2, value_bits=2,
                          eviction_rate=0.8)
    k, v = syn.cpu_layer(cfg, 0)
    kept, kidx, kcnt, cap = _keep_set(orc, cfg, k)
    _layer_parity(orc, cfg, k, v, kept, kidx, kcnt, cap)
