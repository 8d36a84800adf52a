"""GPU parity: the CUDA kernels (through the C ABI) against the CPU oracle and the
reference's golden outputs.  Lattice codes, packed bytes, fp16 scales and kept
indices must be bit-exact against the oracle; against the reference, only groups
on a decision boundary may differ.  Reconstructions: relative L2 <= 1e-3."""
import numpy as np
import pytest
import torch

from nexusquant_b200 import kernels as K
from nexusquant_b200 import synthetic as syn
from nexusquant_b200.rope import host_tables
from tests.parity import REL_L2_TOL, check_codes_vs_reference, golden_str, rel_l2, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _oracle_layer(orc, k, v, kept, levels_k, levels_v, base=10000.0, positions=None):
    """Oracle codes/scales for layer tensors k, v [b, h, T, d] (CPU) at kept [b, n] indices."""
    b, h, T, d = k.shape
    dp = orc.next_pow2(d)
    kept = np.asarray(kept)
    pos = kept if positions is None else np.asarray(positions)
    out = {}
    kr = np.stack([k[bi, :, kept[bi]].float().numpy() for bi in range(b)])  # [b, h, n, d]
    vr = np.stack([v[bi, :, kept[bi]].float().numpy() for bi in range(b)])
    n = kept.shape[1]
    cos = np.zeros((b, h, n, d // 2), np.float32)
    sin = np.zeros_like(cos)
    for bi in range(b):
        c, s = orc.rope_tables(pos[bi], d, base)
        cos[bi] = c[None]
        sin[bi] = s[None]
    kc, ks = orc.quantize(kr.reshape(-1, d), dp, levels_k, cos.reshape(-1, d // 2), sin.reshape(-1, d // 2))
    vc, vs = orc.quantize(vr.reshape(-1, d), dp, levels_v)
    out["k_codes"], out["k_scales"] = kc, ks
    out["v_codes"], out["v_scales"] = vc, vs
    out["k_packed"] = orc.pack(kc, levels_k).reshape(b, h, n, -1)
    out["v_packed"] = orc.pack(vc, levels_v).reshape(b, h, n, -1)
    out["cos"], out["sin"] = cos.reshape(-1, d // 2), sin.reshape(-1, d // 2)
    return out


def _run_compress(k, v, kept, lk, lv, dtype=torch.float16, base=10000.0):
    kd, vd = k.to(DEV, dtype), v.to(DEV, dtype)
    kidx = torch.as_tensor(np.asarray(kept), dtype=torch.int32, device=DEV)
    return K.compress_layers([kd], [vd], key_levels=lk, value_levels=lv, kept_idx=kidx, rope_base=base,
                             emit_scales_f32=True)[0]


@pytest.mark.parametrize("heads", [3, 6])  # partial head groups (2 + 1, 4 + 2)
@pytest.mark.parametrize("d", [128, 96, 64])
@pytest.mark.parametrize("lk,lv", [(8, 4), (4, 4), (16, 2), (2, 8)])
def test_compress_bit_exact_vs_oracle(orc, d, lk, lv, heads):
    cfg = syn.CacheConfig("t", 1, 2, heads, 77, d)
    k, v = syn.cpu_layer(cfg, 5)
    rng = np.random.default_rng(d + lk)
    kept = np.stack([np.sort(rng.choice(77, 37, replace=False)) for _ in range(2)])
    lc = _run_compress(k, v, kept, lk, lv)
    o = _oracle_layer(orc, k, v, kept, lk, lv)
    torch.cuda.synchronize()
    assert np.array_equal(lc.k_codes.cpu().numpy(), o["k_packed"])
    assert np.array_equal(lc.v_codes.cpu().numpy(), o["v_packed"])
    assert np.array_equal(lc.k_scales_f32.cpu().numpy().reshape(-1), o["k_scales"])
    assert np.array_equal(lc.v_scales_f32.cpu().numpy().reshape(-1), o["v_scales"])
    assert np.array_equal(lc.k_scales.cpu().numpy().reshape(-1), o["k_scales"].astype(np.float16))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_compress_input_dtypes(orc, dtype):
    cfg = syn.CacheConfig("t", 1, 1, 8, 64, 128, dtype=torch.float32)
    k, v = syn.cpu_layer(cfg, 2)
    k, v = k.to(dtype), v.to(dtype)
    kept = np.arange(64)[None]
    lc = _run_compress(k, v, kept, 8, 4, dtype=dtype)
    o = _oracle_layer(orc, k, v, kept, 8, 4)
    assert np.array_equal(lc.k_codes.cpu().numpy(), o["k_packed"])
    assert np.array_equal(lc.v_codes.cpu().numpy(), o["v_packed"])


def test_config0_codes_vs_reference(golden, orc):
    """Config 0 exactly: GPU codes equal the reference's codes (fixture from the reference)."""
    k0, v0 = syn.cpu_layer(syn.CONFIGS[0], 0)
    if sha(k0) != golden_str(golden, "cfg0_k_sha"):
        pytest.skip("generator drift")
    lc = K.compress_layers([k0.to(DEV)], [v0.to(DEV)], key_levels=8, value_levels=4, emit_scales_f32=True)[0]
    kp = lc.k_codes.cpu().numpy().reshape(-1, 80)
    vp = lc.v_codes.cpu().numpy().reshape(-1, 64)
    kc = orc.unpack(kp, 128, 8)
    vc = orc.unpack(vp, 128, 4)
    rk = orc.unpack(golden["cfg0_k_codes_packed"], 128, 8)
    rv = orc.unpack(golden["cfg0_v_codes_packed"], 128, 4)
    ex_k, n_k = check_codes_vs_reference(orc, kc, rk, golden["cfg0_k_diff_nrm_ref"], golden["cfg0_k_diff_vecs"],
                                         128, 8, label="cfg0 K")
    ex_v, n_v = check_codes_vs_reference(orc, vc, rv, golden["cfg0_v_diff_nrm_ref"], golden["cfg0_v_diff_vecs"],
                                         128, 4, label="cfg0 V")
    assert ex_k + ex_v == 0  # config 0 matches the reference in every one of its 131072 groups
    assert np.allclose(lc.k_scales_f32.cpu().numpy().reshape(-1), golden["cfg0_k_scales"], rtol=1e-6, atol=0)


def test_fake_quant_recon_vs_oracle_and_reference(golden, orc):
    k0, v0 = syn.cpu_layer(syn.CONFIGS[0], 0)
    kd, vd = k0.to(DEV), v0.to(DEV)
    ok = torch.empty(k0.shape, dtype=torch.float16, device=DEV)
    ov = torch.empty(v0.shape, dtype=torch.float16, device=DEV)
    lc = K.compress_layers([kd], [vd], key_levels=8, value_levels=4, recon_k=[ok], recon_v=[ov],
                           emit_scales_f32=True)[0]
    kept = np.arange(512)[None]
    o = _oracle_layer(orc, k0, v0, kept, 8, 4)
    kr = orc.dequantize(o["k_codes"], o["k_scales"], 128, o["cos"], o["sin"]).astype(np.float16)
    vr = orc.dequantize(o["v_codes"], o["v_scales"], 128).astype(np.float16)
    assert np.array_equal(ok.cpu().numpy().reshape(-1, 128), kr)
    assert np.array_equal(ov.cpu().numpy().reshape(-1, 128), vr)
    if sha(k0) == golden_str(golden, "cfg0_k_sha"):
        assert rel_l2(ok[:, :2].cpu().numpy(), golden["cfg0_fq_k"]) < REL_L2_TOL
        assert rel_l2(ov[:, :2].cpu().numpy(), golden["cfg0_fq_v"]) < REL_L2_TOL


@pytest.mark.parametrize("sharpen", [1.0, K.SHARPEN])
def test_decompress_vs_oracle_and_page_path(golden, orc, sharpen):
    pos = golden["dq_pos"]
    h = golden["dq_k_codes"].shape[0] // len(pos)
    n = len(pos)
    kc = torch.as_tensor(orc.pack(golden["dq_k_codes"], 4).reshape(1, h, n, 64), device=DEV)
    vc = torch.as_tensor(orc.pack(golden["dq_v_codes"], 4).reshape(1, h, n, 64), device=DEV)
    ks = torch.as_tensor(golden["dq_k_scales16"].reshape(1, h, n), device=DEV)
    vs = torch.as_tensor(golden["dq_v_scales16"].reshape(1, h, n), device=DEV)
    lc = K.LayerCodes(kc, vc, ks, vs, 4, 4)
    ok, ov = K.decompress_layers([lc], torch.as_tensor(pos[None], device=DEV), head_dim=128, key_sharpen=sharpen)
    cos, sin = orc.rope_tables(pos, 128, 10000.0)
    okr = orc.dequantize(golden["dq_k_codes"], golden["dq_k_scales16"].astype(np.float32), 128,
                         np.tile(cos, (h, 1)), np.tile(sin, (h, 1)), sharpen=sharpen).astype(np.float16)
    ovr = orc.dequantize(golden["dq_v_codes"], golden["dq_v_scales16"].astype(np.float32), 128).astype(np.float16)
    assert np.array_equal(ok[0].cpu().numpy().reshape(-1, 128), okr)
    assert np.array_equal(ov[0].cpu().numpy().reshape(-1, 128), ovr)
    ref_k = golden["dq_k_out"].reshape(-1, 128).astype(np.float32) * sharpen
    assert rel_l2(ok[0].cpu().numpy().reshape(-1, 128), ref_k) < REL_L2_TOL
    assert rel_l2(ov[0].cpu().numpy().reshape(-1, 128), golden["dq_v_out"].reshape(-1, 128)) < REL_L2_TOL


@pytest.mark.parametrize("d,lk", [(128, 8), (96, 8), (64, 4), (128, 16)])
def test_compress_decompress_roundtrip_vs_oracle(orc, d, lk):
    cfg = syn.CacheConfig("t", 1, 2, 4, 50, d)
    k, v = syn.cpu_layer(cfg, 9)
    kept = np.stack([np.arange(0, 50, 2), np.arange(1, 50, 2)])
    lc = _run_compress(k, v, kept, lk, 4)
    ok, ov = K.decompress_layers([lc], torch.as_tensor(kept, device=DEV), head_dim=d)
    o = _oracle_layer(orc, k, v, kept, lk, 4)
    k16 = lc.k_scales.cpu().numpy().reshape(-1).astype(np.float32)
    v16 = lc.v_scales.cpu().numpy().reshape(-1).astype(np.float32)
    kr = orc.dequantize(o["k_codes"], k16, d, o["cos"], o["sin"]).astype(np.float16)
    vr = orc.dequantize(o["v_codes"], v16, d).astype(np.float16)
    assert np.array_equal(ok[0].cpu().numpy().reshape(-1, d), kr)
    assert np.array_equal(ov[0].cpu().numpy().reshape(-1, d), vr)


def test_kept_count_ragged_rows(orc):
    """Rows past kept_count[b] are neither read nor written."""
    cfg = syn.CacheConfig("t", 1, 2, 2, 40, 128)
    k, v = syn.cpu_layer(cfg, 1)
    kept = np.stack([np.arange(20), np.arange(20) * 2])
    cnt = torch.tensor([20, 13], dtype=torch.int32, device=DEV)
    kd, vd = k.to(DEV), v.to(DEV)
    codes = [K.LayerCodes(torch.full((2, 2, 20, 64), 0xAB, dtype=torch.uint8, device=DEV),
                          torch.full((2, 2, 20, 64), 0xAB, dtype=torch.uint8, device=DEV),
                          torch.zeros((2, 2, 20), dtype=torch.float16, device=DEV),
                          torch.zeros((2, 2, 20), dtype=torch.float16, device=DEV), 4, 4)]
    K.compress_layers([kd], [vd], key_levels=4, value_levels=4, kept_idx=torch.as_tensor(kept, device=DEV),
                      kept_count=cnt, codes_out=codes)
    o = _oracle_layer(orc, k, v, kept, 4, 4)
    got = codes[0].k_codes.cpu().numpy()
    assert np.array_equal(got[0], o["k_packed"][0])
    assert np.array_equal(got[1, :, :13], o["k_packed"][1, :, :13])
    assert (got[1, :, 13:] == 0xAB).all()


def test_no_rotation_mode_matches_quantize_perhead(orc):
    """rotate=False is E8Lattice.quantize_perhead / e8_encode (no Hadamard): bit-exact vs the oracle."""
    x = torch.randn(300, 128, generator=torch.Generator().manual_seed(4)) * 3
    codes, scales = K.e8_encode(x.to(DEV), levels=8)
    oc, osc = orc.quantize(x.numpy(), 128, 8, rotate=False)
    assert np.array_equal(codes.cpu().numpy(), oc)
    assert np.array_equal(scales.cpu().numpy(), osc)
    q = K.e8_quantize_perhead(x.to(DEV), levels=8).cpu().numpy()
    ref = (oc.astype(np.float32) * (osc[:, None] * np.float32(0.5))).astype(np.float16)
    assert np.array_equal(q, ref)


@pytest.mark.parametrize("levels", [2, 4, 8, 16])
def test_step_direction_at_tiny_gaps(orc, levels):
    """The A step moves toward x (e8_lattice.py:42-43) even where fl(x - 1/2) rounds onto a
    half-way point: x just below 0 (a = 0, e < 0) and x = -1 + 2^-24 (a = -1, e > 0), each the
    smallest gap of an odd-sum group that keeps the integer candidate."""
    half = levels / 2
    g1 = [-1e-9, 0.1, 0.1, 0.1, 0.9, 0.1, 0.1, 0.1]
    g2 = [-1.0 + 2.0 ** -24, 0.1, 0.1, 0.1, 0.1, 0.1, 0.1, 0.1]
    row = np.zeros(128, np.float32)
    row[0:8], row[8:16], row[16] = g1, g2, half  # amax = L/2: scale 1, x / scale = x
    x = torch.from_numpy(np.stack([row, -row, row[::-1].copy()]))
    codes, scales = K.e8_encode(x.to(DEV), levels=levels)
    oc, osc = orc.quantize(x.numpy(), 128, levels, rotate=False)
    assert np.array_equal(scales.cpu().numpy(), osc)
    assert np.array_equal(codes.cpu().numpy(), oc)
    assert oc[0, 0] == -2 and oc[0, 8] == 0  # stepped down from 0, up from -1
    # many such rows: more flagged vectors than a CTA queues, so whole shares are redone exactly
    xs = torch.from_numpy(np.tile(np.stack([row, -row, row[::-1].copy()]), (70, 1)))
    xs[1::3] *= torch.linspace(0.5, 2.0, xs[1::3].shape[0])[:, None]
    codes, scales = K.e8_encode(xs.to(DEV), levels=levels)
    oc, osc = orc.quantize(xs.numpy(), 128, levels, rotate=False)
    assert np.array_equal(scales.cpu().numpy(), osc)
    assert np.array_equal(codes.cpu().numpy(), oc)


# ----------------------------------------------------------------- scoring + select
def test_keykey_importance_vs_oracle_and_reference(golden, orc):
    cfg = syn.CacheConfig("score", 1, 2, 4, 300, 128)
    k, _ = syn.cpu_layer(cfg, 0)
    imp = K.score_keykey(k.to(DEV), 32).cpu().numpy()
    o = orc.keykey_importance(k.float().numpy(), 32)
    assert np.allclose(imp, o, rtol=5e-5, atol=1e-8)
    if sha(k) == golden_str(golden, "score_k_sha"):
        assert np.allclose(imp, golden["score_importance"], rtol=5e-5, atol=1e-8)
    # head-range partials reduce to the same mean
    ph = K.score_keykey(k.to(DEV), 32, head_range=(1, 3), per_head=True)
    ph0 = K.score_keykey(k.to(DEV), 32, head_range=(0, 1), per_head=True)
    ph3 = K.score_keykey(k.to(DEV), 32, head_range=(3, 4), per_head=True)
    full = K.reduce_heads(torch.cat([ph0, ph, ph3], 1), 4.0).cpu().numpy()
    assert np.array_equal(full, imp)


def test_real_scorer_vs_oracle(golden, orc):
    cfg = syn.CacheConfig("real", 2, 1, 4, 256, 96, rope_base=10000.0)
    Ks = [syn.cpu_layer(cfg, l)[0] for l in range(2)]
    Qs = [syn.cpu_queries(cfg, l, n_queries=64) for l in range(2)]
    acc = torch.zeros(1, 256, device=DEV)
    for q, k in zip(Qs, Ks):
        K.score_attention(q.to(DEV), k.to(DEV), 256 - 64, out=acc, accumulate=True)
    imp = (acc / 2).cpu().numpy()
    o = orc.real_importance([q.float().numpy() for q in Qs], [k.float().numpy() for k in Ks], 256 - 64)
    assert np.allclose(imp, o, rtol=5e-5, atol=1e-8)
    assert np.allclose(imp, golden["real_importance"], rtol=5e-5, atol=1e-8)


def _check_select(orc, imp, T, sw, rate, prot=None):
    from nexusquant_b200.pipeline import kept_capacity, n_keep_for
    nk = n_keep_for(T, sw, rate)
    idx, cnt = K.select_keep(torch.as_tensor(imp, device=DEV), sw, nk, prot)
    m = orc.keep_mask(imp, T, sw, rate, prot)
    idx, cnt = idx.cpu().numpy(), cnt.cpu().numpy()
    for bi in range(imp.shape[0]):
        assert cnt[bi] == m[bi].sum()
        assert np.array_equal(idx[bi, :cnt[bi]], np.nonzero(m[bi])[0])
        if prot is None:
            assert cnt[bi] == kept_capacity(T, sw, nk)


def test_select_matches_oracle_and_reference(golden, orc):
    for i, (T, sw, r) in enumerate(golden["sel_cases"]):
        imp = golden[f"sel{i}_imp"]
        _check_select(orc, imp, int(T), int(sw), float(r))
        nk_ref = golden[f"sel{i}_mask"]
        from nexusquant_b200.pipeline import n_keep_for
        idx, cnt = K.select_keep(torch.as_tensor(imp, device=DEV), int(sw), n_keep_for(int(T), int(sw), float(r)))
        amb = orc.threshold_ambiguous(imp, int(T), int(sw), float(r))
        for bi in range(imp.shape[0]):
            m = np.zeros(int(T), bool)
            m[idx[bi, :cnt[bi]].cpu().numpy()] = True
            assert np.array_equal(m[~amb[bi]], nk_ref[bi][~amb[bi]])
    _check_select(orc, golden["selprot_imp"], 120, 8, 0.8, [1, 2, 3, 50, 51, 999])
    _check_select(orc, golden["selties_imp"], 100, 4, 0.5)


@pytest.mark.parametrize("T,sw,rate", [(131072, 32, 0.8), (32768, 32, 0.6), (8192, 32, 0.35), (5000, 0, 0.5),
                                       (70000, 32, 0.0)])
def test_select_large(orc, T, sw, rate):
    rng = np.random.default_rng(T)
    imp = rng.random((1, T)).astype(np.float32)
    imp[0, rng.choice(T, 50)] = 0.5  # exact ties near the middle
    _check_select(orc, imp, T, sw, rate)


@pytest.mark.parametrize("case", ["all_equal", "few_values", "negative", "protected_ties", "ragged_batch"])
def test_select_adversarial(orc, case):
    rng = np.random.default_rng(7)
    prot = None
    if case == "all_equal":
        T, sw, rate = 9001, 16, 0.5
        imp = np.full((1, T), 0.25, np.float32)
    elif case == "few_values":
        T, sw, rate = 20000, 32, 0.3
        imp = rng.integers(0, 5, (2, T)).astype(np.float32)
    elif case == "negative":
        T, sw, rate = 12345, 7, 0.6
        imp = (rng.standard_normal((1, T)) * 1e-3).astype(np.float32)
        imp[0, ::97] = -0.0
        imp[0, 1::97] = 0.0
    elif case == "protected_ties":
        T, sw, rate = 10000, 32, 0.5
        imp = rng.integers(0, 3, (1, T)).astype(np.float32)
        prot = list(range(0, T, 37))
    else:
        T, sw, rate = 4099, 3, 0.45
        imp = rng.random((3, T)).astype(np.float32)
        imp[1] = np.round(imp[1] * 8) / 8
        prot = [5, 4098, 2000]
    _check_select(orc, imp, T, sw, rate, prot)


def test_gather_and_delta(orc):
    cfg = syn.CacheConfig("t", 1, 1, 2, 30, 128)
    k, v = syn.cpu_layer(cfg, 3)
    kept = np.array([[0, 3, 4, 9, 29]])
    g = K.gather_rows(k.to(DEV), torch.as_tensor(kept, device=DEV, dtype=torch.int32), 5)
    assert torch.equal(g.cpu(), k[:, :, kept[0]])
    lc = _run_compress(k, v, kept, 8, 4)
    for packed, lv in ((lc.k_codes, 8), (lc.v_codes, 4)):
        d = K.delta_codes(packed, 128, lv).cpu().numpy()
        codes = orc.unpack(packed.cpu().numpy().reshape(-1, packed.shape[-1]), 128, lv).reshape(2, 5, 128)
        assert np.array_equal(d.reshape(2, 5, 128), orc.delta(codes))


def test_host_resident_inputs_match_device(orc):
    """Layers in pinned host memory: compress and gather read only the kept rows across PCIe
    and give the same bytes as device-resident layers; pageable memory is refused."""
    cfg = syn.CacheConfig("t", 1, 2, 4, 300, 128)
    k, v = syn.cpu_layer(cfg, 4)
    kd, vd = k.to(DEV), v.to(DEV)
    hk, hv = k.pin_memory(), v.pin_memory()
    rng = np.random.default_rng(3)
    kept = torch.as_tensor(np.stack([np.sort(rng.choice(300, 111, replace=False)) for _ in range(2)]),
                           dtype=torch.int32, device=DEV)
    ref = K.compress_layers([kd], [vd], key_levels=8, value_levels=4, kept_idx=kept)[0]
    got = K.compress_layers([hk], [hv], key_levels=8, value_levels=4, kept_idx=kept, device=DEV)[0]
    for a, b in ((ref.k_codes, got.k_codes), (ref.v_codes, got.v_codes), (ref.k_scales, got.k_scales),
                 (ref.v_scales, got.v_scales)):
        assert torch.equal(a, b)
    direct = K.compress_layers([hk], [hv], key_levels=8, value_levels=4, kept_idx=kept, device=DEV,
                               stage_host_rows=False)[0]
    for a, b in ((ref.k_codes, direct.k_codes), (ref.v_codes, direct.v_codes), (ref.k_scales, direct.k_scales),
                 (ref.v_scales, direct.v_scales)):
        assert torch.equal(a, b)
    assert torch.equal(K.gather_rows(kd, kept, 111), K.gather_rows(hk, kept, 111, device=DEV))
    with pytest.raises(RuntimeError):
        K.compress_layers([k], [v], key_levels=8, value_levels=4, kept_idx=kept, device=DEV)  # not pinned
    from nexusquant_b200 import _native as N
    with pytest.raises(RuntimeError):  # the C ABI itself refuses pageable host memory
        N.call("nq_gather_rows", k.data_ptr(), 0, 2, 4, 128, *k.stride()[:3], kept.data_ptr(), None, 111,
               torch.empty((2, 4, 111, 128), dtype=torch.float16, device=DEV).data_ptr(), 4 * 111 * 128,
               111 * 128, 128, None)


@pytest.mark.parametrize("explicit_positions", [False, True])
def test_host_staged_compress_ragged_chunks(explicit_positions, monkeypatch):
    """Staged host path (kept rows gathered into device memory, then compressed) against the
    kernel reading the host rows itself and against device-resident layers: ragged kept
    counts, a missing half, explicit positions and staging split into several chunks."""
    cfg = syn.CacheConfig("t", 1, 2, 3, 400, 128)
    layers = [syn.cpu_layer(cfg, l) for l in range(5)]
    assert layers[0][0].dtype == torch.float16
    rng = np.random.default_rng(5)
    n_kept = 150
    kept = torch.as_tensor(np.stack([np.sort(rng.choice(400, n_kept, replace=False)) for _ in range(2)]),
                           dtype=torch.int32, device=DEV)
    cnt = torch.tensor([150, 97], dtype=torch.int32, device=DEV)
    pos = (kept + 1000) if explicit_positions else None
    ks = [k for k, _ in layers]
    vs = [v for _, v in layers]
    vs[2] = None
    hks = [k.pin_memory() for k in ks]
    hvs = [None if v is None else v.pin_memory() for v in vs]
    dks = [k.to(DEV) for k in ks]
    dvs = [None if v is None else v.to(DEV) for v in vs]
    kw = dict(key_levels=[4, 8, 16, 2, 4], value_levels=4, kept_idx=kept, kept_count=cnt, positions=pos)
    ref = K.compress_layers(dks, dvs, **kw)
    monkeypatch.setattr(K, "_STAGE_LIMIT", 2 * 2 * 2 * 3 * n_kept * 128 * 2)  # two layers per chunk
    staged = K.compress_layers(hks, hvs, device=DEV, **kw)
    direct = K.compress_layers(hks, hvs, device=DEV, stage_host_rows=False, **kw)
    for got in (staged, direct):
        for a, b in zip(ref, got):
            for bi in range(2):
                n = int(cnt[bi])
                for x, y in ((a.k_codes, b.k_codes), (a.v_codes, b.v_codes), (a.k_scales, b.k_scales),
                             (a.v_scales, b.v_scales)):
                    if x is None:
                        assert y is None
                        continue
                    assert torch.equal(x[bi, :, :n], y[bi, :, :n])


def _attend_ref(q, ok, ov, count, scale):
    """NexusQuantPagedAttention.forward restated in torch (fp32 softmax over fp16 K/V)."""
    b, hq, d = q.shape
    h = ok.shape[1]
    out = torch.zeros_like(q)
    for bi in range(b):
        n = int(count[bi])
        if n == 0:
            continue
        k = ok[bi, :, :n].float().repeat_interleave(hq // h, 0)
        v = ov[bi, :, :n].float().repeat_interleave(hq // h, 0)
        w = torch.softmax(torch.einsum("hd,hnd->hn", q[bi].float(), k) * scale, -1)
        out[bi] = torch.einsum("hn,hnd->hd", w, v).to(torch.float16)
    return out


@pytest.mark.parametrize("lk,lv,g,sharpen", [(4, 4, 1, 1.0), (8, 4, 2, K.SHARPEN), (16, 16, 4, 1.0), (2, 8, 8, 1.0)])
def test_attend_compressed_vs_decompress_then_attention(orc, lk, lv, g, sharpen):
    """Decode attention over the compressed layout equals dequantize + the reference attention."""
    cfg = syn.CacheConfig("t", 1, 2, 2, 700, 128)
    k, v = syn.cpu_layer(cfg, 6)
    rng = np.random.default_rng(lk + g)
    kept = np.stack([np.sort(rng.choice(700, 333, replace=False)) for _ in range(2)])
    lc = _run_compress(k, v, kept, lk, lv)
    pos = torch.as_tensor(kept, dtype=torch.int32, device=DEV)
    count = torch.tensor([333, 150], dtype=torch.int32, device=DEV)  # ragged second sequence
    ok, ov = K.decompress_layers([lc], pos, head_dim=128, count=count, key_sharpen=sharpen)
    q = (torch.randn(2, 2 * g, 128, generator=torch.Generator().manual_seed(g)) * 0.3).to(torch.float16).to(DEV)
    got = K.attend_compressed(q, lc, pos, count=count, key_sharpen=sharpen)
    ref = _attend_ref(q, ok[0], ov[0], count.cpu(), 128 ** -0.5)
    assert rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < REL_L2_TOL
    again = K.attend_compressed(q, lc, pos, count=count, key_sharpen=sharpen)
    assert torch.equal(got, again)  # deterministic


def test_attend_compressed_empty_layer_zeroes_strided_output():
    """No stored tokens: every query row of a strided output is zeroed, and nothing else."""
    codes = K.LayerCodes(torch.zeros((2, 2, 0, 64), dtype=torch.uint8, device=DEV),
                         torch.zeros((2, 2, 0, 64), dtype=torch.uint8, device=DEV),
                         torch.zeros((2, 2, 0), dtype=torch.float16, device=DEV),
                         torch.zeros((2, 2, 0), dtype=torch.float16, device=DEV), 4, 4)
    q = torch.ones((2, 4, 128), dtype=torch.float16, device=DEV)
    big = torch.full((2, 5, 160), 7.0, dtype=torch.float16, device=DEV)   # rows of 160, 5 per batch
    out = big[:, :4, :128]
    K.attend_compressed(q, codes, torch.zeros((2, 0), dtype=torch.int32, device=DEV), out=out, rope_rows=1)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
    assert bool((big[:, 4] == 7).all()) and bool((big[:, :4, 128:] == 7).all())


def test_positions_past_the_rope_table_are_clamped():
    """A stored position at or past the RoPE table (a caller's rope_rows too small) reads the
    table's last row instead of memory past it: the output equals that of the clamped positions."""
    from nexusquant_b200.rope import TABLES
    cfg = syn.CacheConfig("t", 1, 1, 2, 64, 128)
    k, v = syn.cpu_layer(cfg, 2)
    base = 12345.0  # a table of its own, sized by this test
    pos = torch.arange(64, dtype=torch.int32, device=DEV)[None]
    lc = K.compress_layers([k.to(DEV)], [v.to(DEV)], key_levels=4, value_levels=4, positions=pos,
                           rope_base=base, rope_rows=64)[0]
    rows = TABLES.get(torch.device(DEV), 128, base, 16)[0].shape[0]
    far = pos.clone()
    far[0, 40:] += rows + 1000
    q = torch.randn(1, 4, 128, device=DEV).half()
    got = K.attend_compressed(q, lc, far, rope_base=base, rope_rows=rows)
    want = K.attend_compressed(q, lc, far.clamp(max=rows - 1), rope_base=base, rope_rows=rows)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("d,kl,vl,sharpen,rows", [(128, 4, 4, 1.0, "source"), (128, 8, 4, K.SHARPEN, "kept"),
                                                   (64, 4, 16, 1.0, "kept"), (64, 8, 8, K.SHARPEN, "source")])
def test_fake_quant_recon_kept_rows(orc, d, kl, vl, sharpen, rows):
    """Fake-quant reconstruction of fp16 layers through a keep set (each thread of a vector's
    pair rebuilds its own half): bit-exact against the oracle's dequantize with the fp32
    scales, keys re-encoded at the source position (masked layout) or at the kept index j
    (truncated layout), sharpened or not."""
    b, h, T = 2, 3, 700
    g = torch.Generator().manual_seed(17 + d + kl)
    k = (torch.randn(b, h, T, d, generator=g)).half()
    v = (torch.randn(b, h, T, d, generator=g)).half()
    n = 300
    kept = np.stack([np.sort(np.random.default_rng(bi).choice(T, n, replace=False)) for bi in range(b)])
    kidx = torch.as_tensor(kept, dtype=torch.int32, device=DEV)
    cnt = torch.full((b,), n, dtype=torch.int32, device=DEV)
    shape_o = (b, h, T if rows == "source" else n, d)
    ok = torch.zeros(shape_o, dtype=torch.float16, device=DEV)
    ov = torch.zeros(shape_o, dtype=torch.float16, device=DEV)
    lc = K.compress_layers([k.to(DEV)], [v.to(DEV)], key_levels=kl, value_levels=vl, kept_idx=kidx, kept_count=cnt,
                           n_kept=n, recon_k=[ok], recon_v=[ov], recon_rows=rows, key_sharpen=sharpen,
                           emit_scales_f32=True, rope_rows=T)[0]
    okh, ovh = ok.cpu().numpy(), ov.cpu().numpy()
    for bi in range(b):
        kr = k[bi][:, kept[bi]].float().numpy().reshape(-1, d)
        vr = v[bi][:, kept[bi]].float().numpy().reshape(-1, d)
        c_in, s_in = orc.rope_tables(kept[bi], d, 10000.0)
        kc, _ = orc.quantize(kr, d, kl, np.tile(c_in, (h, 1)), np.tile(s_in, (h, 1)))
        vc, _ = orc.quantize(vr, d, vl)
        ks32 = lc.k_scales_f32[bi].cpu().numpy().reshape(-1)
        vs32 = lc.v_scales_f32[bi].cpu().numpy().reshape(-1)
        opos = kept[bi] if rows == "source" else np.arange(n)
        c_out, s_out = orc.rope_tables(opos, d, 10000.0)
        kx = orc.dequantize(kc, ks32, d, np.tile(c_out, (h, 1)), np.tile(s_out, (h, 1)), sharpen=sharpen)
        vx = orc.dequantize(vc, vs32, d).astype(np.float16)
        sel = kept[bi] if rows == "source" else np.arange(n)
        assert np.array_equal(okh[bi][:, sel].reshape(-1, d), kx.astype(np.float16))
        assert np.array_equal(ovh[bi][:, sel].reshape(-1, d), vx)
