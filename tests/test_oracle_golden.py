"""Pin the CPU oracle against the reference's own outputs (tests/golden/golden.npz).

The fixtures were produced by running jagmarques/nexusquant v0.5.0 on seeded
inputs (tests/golden/make_golden.py).  No GPU needed.
"""
import numpy as np
import pytest
import torch

from nexusquant_b200 import synthetic as syn
from nexusquant_b200.rope import host_tables, inv_freq
from tests.parity import REL_L2_TOL, check_codes_vs_reference, golden_str, rel_l2, sha


def test_hadamard_entries(golden, orc):
    for n, e in zip(golden["hadamard_sizes"], golden["hadamard_entries"]):
        assert np.float32(orc.lib().nqo_hadamard_entry(int(n))) == e


@pytest.mark.parametrize("name,d,base", [("r128", 128, 10000.0), ("r96", 96, 10000.0),
                                          ("r128b5e5", 128, 500000.0)])
def test_rope_tables_bit_identical(golden, orc, name, d, base):
    pos = golden[f"{name}_pos"]
    c_ref, s_ref = golden[f"{name}_cos"], -golden[f"{name}_negsin"]
    c_o, s_o = orc.rope_tables(pos, d, base)
    assert np.array_equal(c_o, c_ref) and np.array_equal(s_o, s_ref)
    # the product's host tables (rows 0..n-1) agree at the same positions
    hc, hs = host_tables(int(pos.max()) + 1, d, base)
    assert np.array_equal(hc.numpy()[pos], c_ref) and np.array_equal(hs.numpy()[pos], s_ref)


def test_llama3_rope_scaling(golden):
    sc = {"type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
    assert np.array_equal(inv_freq(128, 500000.0, sc).numpy(), golden["llama3_inv_freq"])


def _cfg0_inputs(golden):
    k0, v0 = syn.cpu_layer(syn.CONFIGS[0], 0)
    if sha(k0) != golden_str(golden, "cfg0_k_sha") or sha(v0) != golden_str(golden, "cfg0_v_sha"):
        pytest.skip("torch CPU generator output differs from the fixture's (different torch build)")
    return k0, v0


def test_oracle_config0_codes_match_reference(golden, orc):
    """Config 0 (b1 h8 T512 d128 fp32, K3V2): every lattice code equal to the reference's."""
    k0, v0 = _cfg0_inputs(golden)
    cos, sin = orc.rope_tables(np.arange(512), 128, 10000.0)
    kx = k0[0].float().reshape(-1, 128).numpy()
    kc, ks = orc.quantize(kx, 128, 8, np.tile(cos, (8, 1)), np.tile(sin, (8, 1)))
    vc, vs = orc.quantize(v0[0].float().reshape(-1, 128).numpy(), 128, 4)
    assert np.array_equal(orc.pack(kc, 8), golden["cfg0_k_codes_packed"])
    assert np.array_equal(orc.pack(vc, 4), golden["cfg0_v_codes_packed"])
    # fp32 scales agree to an ulp or two (butterfly vs dense GEMM rounding of amax)
    assert np.allclose(ks, golden["cfg0_k_scales"], rtol=1e-6, atol=0)
    assert np.allclose(vs, golden["cfg0_v_scales"], rtol=1e-6, atol=0)


def test_oracle_config0_fake_quant_matches_reference(golden, orc):
    """Oracle quantize + dequantize (fp32 scales) vs NexusQuantEvict(rate 0, K3V2) output."""
    k0, v0 = _cfg0_inputs(golden)
    cos, sin = orc.rope_tables(np.arange(512), 128, 10000.0)
    cr, sr = np.tile(cos, (2, 1)), np.tile(sin, (2, 1))
    kx = k0[0, :2].float().reshape(-1, 128).numpy()
    kc, ks = orc.quantize(kx, 128, 8, cr, sr)
    kr = orc.dequantize(kc, ks, 128, cr, sr).astype(np.float16)
    vc, vs = orc.quantize(v0[0, :2].float().reshape(-1, 128).numpy(), 128, 4)
    vr = orc.dequantize(vc, vs, 128).astype(np.float16)
    ref_k = golden["cfg0_fq_k"].reshape(-1, 128)
    ref_v = golden["cfg0_fq_v"].reshape(-1, 128)
    assert rel_l2(kr, ref_k) < REL_L2_TOL and rel_l2(vr, ref_v) < REL_L2_TOL
    # fp16 outputs are identical except for last-bit differences of a few percent of elements
    assert np.mean(kr != ref_k) < 0.05 and np.mean(vr != ref_v) < 0.05


@pytest.mark.parametrize("levels", [2, 4, 8, 16])
@pytest.mark.parametrize("kind", ["v", "k"])
def test_oracle_edge_vectors(golden, orc, levels, kind):
    """Zero, constant, ramp, huge/tiny and one-hot vectors at every level count."""
    x = golden["edge_x"]
    cos = sin = None
    if kind == "k":
        cos, sin = orc.rope_tables(np.arange(x.shape[0]) * int(golden["edge_pos_stride"][0]), 128, 10000.0)
    codes, scales, nrm = orc.quantize(x, 128, levels, cos, sin, want_nrm=True)
    p = f"edge_{kind}{levels}"
    n_ex, n = check_codes_vs_reference(orc, codes, golden[f"{p}_codes"], golden[f"{p}_diff_nrm_ref"],
                                       golden[f"{p}_diff_vecs"], 128, levels, nrm, label=p)
    assert n_ex <= 4
    assert np.allclose(scales, golden[f"{p}_scales"], rtol=1e-6, atol=1e-12)


@pytest.mark.parametrize("name,d", [("d96", 96), ("d64", 64)])
def test_oracle_head_dims(golden, orc, name, d):
    """head_dim 96 (zero-padded to 128 after RoPE, the config-2 restatement) and 64."""
    cfg = syn.CacheConfig(name, 1, 1, 3, 41, d)
    k, v = syn.cpu_layer(cfg, 3)
    if sha(k) != golden_str(golden, f"{name}_k_sha"):
        pytest.skip("generator drift")
    dp = orc.next_pow2(d)
    cos, sin = orc.rope_tables(np.arange(41), d, 10000.0)
    kc, ks = orc.quantize(k[0].float().reshape(-1, d).numpy(), dp, 8, np.tile(cos, (3, 1)), np.tile(sin, (3, 1)))
    vc, vs = orc.quantize(v[0].float().reshape(-1, d).numpy(), dp, 4)
    assert np.array_equal(kc, golden[f"{name}_k_codes"]) and np.array_equal(vc, golden[f"{name}_v_codes"])
    assert np.allclose(ks, golden[f"{name}_k_scales"], rtol=1e-6, atol=0)
    assert np.allclose(vs, golden[f"{name}_v_scales"], rtol=1e-6, atol=0)


def test_oracle_dequantize_matches_decompress_page(golden, orc):
    pos = golden["dq_pos"]
    cos, sin = orc.rope_tables(pos, 128, 10000.0)
    h = golden["dq_k_codes"].shape[0] // len(pos)
    cr, sr = np.tile(cos, (h, 1)), np.tile(sin, (h, 1))
    k = orc.dequantize(golden["dq_k_codes"], golden["dq_k_scales16"].astype(np.float32), 128, cr, sr)
    v = orc.dequantize(golden["dq_v_codes"], golden["dq_v_scales16"].astype(np.float32), 128)
    ref_k = golden["dq_k_out"].reshape(-1, 128)
    ref_v = golden["dq_v_out"].reshape(-1, 128)
    assert rel_l2(k.astype(np.float16), ref_k) < REL_L2_TOL
    assert rel_l2(v.astype(np.float16), ref_v) < REL_L2_TOL


def test_oracle_nibble_pack_matches_reference(golden, orc):
    assert np.array_equal(orc.pack(golden["dq_k_codes"], 4), golden["dq_k_nibble"])
    for lv in (4, 8, 16):
        c = golden["edge_v%d_codes" % lv]
        assert np.array_equal(orc.unpack(orc.pack(c, lv), 128, lv), c)


def test_oracle_delta_matches_temporal_codec(golden, orc):
    codes = golden["delta_codes"]  # (h, s, d)
    d = orc.delta(codes)
    assert np.array_equal(d[0], golden["delta_ref"])
    assert np.array_equal(np.cumsum(d.astype(np.int64), axis=1).astype(np.int8), codes)


def test_n_keep_formula(golden):
    from nexusquant_b200.pipeline import kept_capacity, n_keep_for
    for (T, sw, r), cnt in zip(golden["nkeep_cases"], golden["nkeep_counts"]):
        T, sw = int(T), int(sw)
        assert kept_capacity(T, sw, n_keep_for(T, sw, float(r))) == cnt
    # config 4: 131040 * (1 - 0.8) evaluates to 26207.99.. in IEEE double
    assert n_keep_for(131072, 32, 0.8) == 26207


def test_oracle_keep_masks(golden, orc):
    cases = golden["sel_cases"]
    for i, (T, sw, r) in enumerate(cases):
        imp = golden[f"sel{i}_imp"]
        m = orc.keep_mask(imp, int(T), int(sw), float(r))
        amb = orc.threshold_ambiguous(imp, int(T), int(sw), float(r))
        ref = golden[f"sel{i}_mask"]
        assert np.array_equal(m[~amb], ref[~amb]), f"case {i}"
        assert m.sum() == ref.sum()
    m = orc.keep_mask(golden["selprot_imp"], 120, 8, 0.8, [1, 2, 3, 50, 51, 999])
    assert np.array_equal(m, golden["selprot_mask"])


def test_oracle_keep_mask_ties(golden, orc):
    """Exact ties: same number kept; the lower-index rule may pick other tied tokens than torch.topk."""
    imp = golden["selties_imp"]
    m = orc.keep_mask(imp, 100, 4, 0.5)
    ref = golden["selties_mask"]
    assert m.sum() == ref.sum()
    vals = np.unique(imp[0, 1:96][(m != ref)[0, 1:96]])
    assert len(vals) <= 1  # differences only inside one tied value class


def test_oracle_keykey_importance(golden, orc):
    cfg = syn.CacheConfig("score", 1, 2, 4, 300, 128)
    k, _ = syn.cpu_layer(cfg, 0)
    if sha(k) != golden_str(golden, "score_k_sha"):
        pytest.skip("generator drift")
    imp = orc.keykey_importance(k.float().numpy(), 32)
    ref = golden["score_importance"]
    # the reference scores in fp32 (einsum + softmax): ~1e-5 relative error vs exact
    assert np.allclose(imp, ref, rtol=5e-5, atol=1e-8)
    m = orc.keep_mask(imp, 300, 16, 0.6)
    amb = orc.threshold_ambiguous(ref, 300, 16, 0.6)
    assert np.array_equal(m[~amb], golden["score_mask"][~amb])


def test_oracle_real_importance(golden, orc):
    cfg = syn.CacheConfig("real", 2, 1, 4, 256, 96, rope_base=10000.0)
    Ks = [syn.cpu_layer(cfg, l)[0] for l in range(2)]
    if sha(torch.stack(Ks)) != golden_str(golden, "real_sha"):
        pytest.skip("generator drift")
    Qs = [syn.cpu_queries(cfg, l, n_queries=64) for l in range(2)]
    imp = orc.real_importance([q.float().numpy() for q in Qs], [k.float().numpy() for k in Ks], 256 - 64)
    assert np.allclose(imp, golden["real_importance"], rtol=5e-5, atol=1e-8)


# ----------------------------------------------------- reference test_core invariants
def test_e8_properties(orc):
    """Ports of tests/test_core.py:20-88 on the oracle."""
    rng = np.random.default_rng(42)
    x = rng.standard_normal((200, 128)).astype(np.float32)
    c2, s2 = orc.quantize(x, 128, 4)
    c4, s4 = orc.quantize(x, 128, 16)
    H = np.array([[1.0]])
    while H.shape[0] < 128:
        H = np.block([[H, H], [H, -H]])
    H /= np.sqrt(128)
    rec2 = (c2 * 0.5 * s2[:, None]) @ H.T
    rec4 = (c4 * 0.5 * s4[:, None]) @ H.T
    e2, e4 = np.mean((x - rec2) ** 2), np.mean((x - rec4) ** 2)
    assert e4 < e2 and np.sqrt(e2) < 1.0
    g = c2.reshape(-1, 8)
    integer = (g % 2 == 0).all(1)
    # integer-coset groups are on D8 unless the clamp moved a coordinate
    assert np.all(((g[integer] // 2).sum(1) % 2 == 0) | (np.abs(g[integer]) == 4).any(1))
    assert np.abs(c2).max() <= 4 and np.abs(c4).max() <= 16
