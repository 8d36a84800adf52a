"""Generate the golden fixtures in tests/golden/ from the reference implementation.

Run in a container that has the reference checked out (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref /path/to/nexusquant
    (--part merge / entropy / rans regenerates only merge.npz / entropy.npz / rans.npz)

The reference is jagmarques/nexusquant v0.5.0.  Every fixture is produced by the
reference's own functions on seeded inputs (nexusquant_b200.synthetic or small
hand-built edge cases); inputs that the tests can regenerate bit-identically
(torch CPU generator) are stored only as a SHA-256 digest, the rest are stored.

For lattice codes the fixture also records which 8-groups differ between the
reference and the C oracle, together with the reference's normalised inputs for
those groups, so the tests can re-verify that every difference is a boundary
case (within 1e-6 of a decision boundary).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from nexusquant_b200 import synthetic as syn  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def sha(t) -> str:
    a = t.detach().cpu().contiguous().numpy() if isinstance(t, torch.Tensor) else np.ascontiguousarray(t)
    return hashlib.sha256(a.tobytes()).hexdigest()


class FakeCache:
    def __init__(self, ks, vs):
        self.key_cache = list(ks)
        self.value_cache = list(vs)


def ref_codes_page(NQC, k, v, positions, bits, base):
    """Codes via the reference's code-emitting path (vllm_backend.compress_page)."""
    comp = NQC(head_dim=k.shape[-1], bits=bits, rope_base=base)
    page = comp.compress_page(k, v, positions)
    return page


def ref_codes_direct(NQC, hadamard_matrix, rope_remove, x, positions, d_p, levels, base, is_key):
    """Reference components composed as the pipelines do, with zero padding of a
    non-power-of-two head_dim to d_p after RoPE removal (config-2 restatement).
    x: [h, s, d] float32.  Returns codes [h*s, d_p], fp32 scales, nrm [h*s, d_p]."""
    import torch.nn.functional as F
    h, s, d = x.shape
    if is_key:
        x = rope_remove(x, positions, base)
    if d_p != d:
        x = F.pad(x, (0, d_p - d))
    H = hadamard_matrix(d_p)
    rot = torch.einsum('hsd,de->hse', x, H.float())
    codes, scales = NQC._quantize_perhead_with_scales(rot, levels)
    flat = rot.reshape(h * s, d_p)
    amax = flat.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    nrm = flat / (amax / (levels / 2))
    return codes.reshape(h * s, d_p).numpy(), scales.reshape(-1).numpy(), nrm.numpy()


def diff_record(prefix, codes_ref, nrm_ref, x_rows, d_p, levels, cos=None, sin=None):
    """Compare the oracle with reference codes; record differing groups."""
    oc, osc, onrm = orc.quantize(x_rows, d_p, levels, cos, sin, want_nrm=True)
    G = d_p // 8
    cr = codes_ref.reshape(-1, G, 8)
    co = oc.reshape(-1, G, 8)
    diff = np.nonzero((cr != co).any(-1).reshape(-1))[0]
    vec = np.unique(diff // G)
    out = {
        f"{prefix}_diff_groups": diff.astype(np.int64),
        f"{prefix}_diff_vecs": vec.astype(np.int64),
        f"{prefix}_diff_nrm_ref": nrm_ref.reshape(-1, d_p)[vec].astype(np.float32),
    }
    if len(vec):
        amb = orc.boundary_groups(nrm_ref.reshape(-1, d_p)[vec], onrm[vec], levels)
        flat_amb = {int(v) * G + gi for j, v in enumerate(vec) for gi in range(G) if amb[j, gi]}
        bad = [int(gidx) for gidx in diff if int(gidx) not in flat_amb]
        print(f"  {prefix}: {len(diff)} differing groups of {cr.shape[0] * G}, "
              f"{len(bad)} not explained by a boundary")
        if bad:
            raise SystemExit(f"oracle mismatch not at a boundary in {prefix}: {bad[:10]}")
    else:
        print(f"  {prefix}: 0 differing groups of {cr.shape[0] * G}")
    return out


def make_merge(P) -> dict:
    """Merge eviction (pipeline.py:961-1048) run by the reference itself: the merged values of
    _apply_merge_eviction on a cache with one shorter (skipped) layer, and the fake-quant output
    of a full compress(merge_eviction=True).  Written to merge.npz."""
    fx = {}
    cfg = syn.CacheConfig("merge", 4, 2, 2, 96, 128)
    ks_, vs_ = zip(*[syn.cpu_layer(cfg, l, seq=(64 if l == 2 else None)) for l in range(4)])
    ev = P.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, merge_eviction=True)
    imp = ev._score_importance(ks_[0].float())
    mask = ev._build_keep_mask(imp, 96, eviction_rate=0.6)
    cache = FakeCache([k.clone() for k in ks_], [v.clone() for v in vs_])
    ev._apply_merge_eviction(cache, mask, imp, 4)
    fx["merge_importance"] = imp.numpy()
    fx["merge_mask"] = mask.numpy()
    fx["merge_in_sha"] = np.frombuffer(sha(torch.cat([t.reshape(-1) for t in ks_ + vs_])).encode(), np.uint8)
    for l in range(4):
        fx[f"merge_v{l}"] = cache.value_cache[l].numpy()
    # full pipeline on the three full-length layers, boundary layers 0 and 2 kept at fp16
    ev = P.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, protect_boundary=1, merge_eviction=True)
    idx = [0, 1, 3]
    cache = FakeCache([ks_[l].clone() for l in idx], [vs_[l].clone() for l in idx])
    _, pm = ev.compress(cache)
    fx["merge_pipe_mask"] = pm.numpy()
    for i in range(3):
        fx[f"merge_pipe_k{i}"] = cache.key_cache[i].numpy()
        fx[f"merge_pipe_v{i}"] = cache.value_cache[i].numpy()
    return fx


def entropy_coords():
    """Seeded int8 lattice codes with temporal correlation (a random walk along 96 tokens of
    16 streams x 128 coordinates, clipped to [-4, 4]); regenerated bit-identically by the tests."""
    rng = np.random.default_rng(20240601)
    steps = rng.integers(-1, 2, size=(96, 16 * 128))
    return np.clip(np.cumsum(steps, axis=0), -4, 4).astype(np.int8).reshape(-1), 96


def make_entropy() -> dict:
    """temporal_codec.compress_indices (temporal_codec.py:76-106) run by the reference itself, with
    and without the temporal delta.  Without the zstandard module the reference writes zlib
    streams (compressor 0), which is what a container without it records."""
    from nexusquant.core import temporal_codec as TC
    coords, n_tokens = entropy_coords()
    fx = {"coords_sha": np.frombuffer(sha(coords).encode(), np.uint8), "n_tokens": np.int64(n_tokens),
          "has_zstd": np.int64(int(TC._HAS_ZSTD))}
    for use_delta in (True, False):
        blob = TC.compress_indices(coords, n_tokens, use_delta=use_delta)
        fx[f"stream_delta{int(use_delta)}"] = np.frombuffer(blob, np.uint8)
        fx[f"delta{int(use_delta)}_roundtrip"] = np.int64(int(np.array_equal(TC.decompress_indices(blob), coords)))
    return fx


RANS_CASES = (("l4", 4, 48, 0), ("l4even", 4, 48, 1), ("l2", 2, 40, 0), ("l8", 8, 24, 0), ("l16", 16, 24, 0),
              ("zero", 4, 8, 2))


def rans_case(levels, rows, kind, seed=7):
    """Seeded E8 codes of ``rows`` Gaussian rows (d = d_p = 128) from the C oracle's quantizer,
    with fp16 scales; kind 1 clears the low bit (integer coordinates only), kind 2 zeroes all."""
    rng = np.random.default_rng(seed + 131 * levels + rows)
    x = rng.standard_normal((rows, 128)).astype(np.float32)
    codes, scales = orc.quantize(x, 128, levels)
    if kind == 1:
        codes = (codes & ~1).astype(np.int8)
    elif kind == 2:
        codes = np.zeros_like(codes)
    return codes, scales.astype(np.float16)


def make_rans() -> dict:
    """entropy_coder.encode_e8 (entropy_coder.py:405-452) run by the reference on
    quantized = code / 2 * scale with the row's fp16 scale repeated over its 8-groups,
    decode_e8's round trip, and measure_e8_entropy's statistics (entropy_coder.py:134-159)."""
    from nexusquant.core import entropy_coder as EC
    fx = {}
    for name, levels, rows, kind in RANS_CASES:
        codes, s16 = rans_case(levels, rows, kind)
        sc = np.repeat(s16.astype(np.float32), 128 // 8)
        q = torch.from_numpy(codes.astype(np.float32).reshape(-1, 8) / 2.0 * sc[:, None])
        blob = EC.encode_e8(q, torch.from_numpy(sc), levels=levels)
        dq, ds = EC.decode_e8(blob)
        fx[f"{name}_codes"] = codes
        fx[f"{name}_scales"] = s16
        fx[f"{name}_levels"] = np.int64(levels)
        fx[f"{name}_stream"] = np.frombuffer(blob, np.uint8)
        fx[f"{name}_roundtrip"] = np.int64(int(torch.equal(dq.reshape(-1, 8).float(), q)))
        st = EC.measure_e8_entropy(q, torch.from_numpy(sc), levels=levels)
        fx[f"{name}_entropy"] = np.array([st["entropy_bps"], st["uniform_bps"], st["compression_ratio"],
                                          st["n_symbols"], st["n_unique"]], np.float64)
    return fx


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NQ_REFERENCE"),
                    help="checkout of the reference (or set NQ_REFERENCE)")
    ap.add_argument("--part", choices=["all", "merge", "entropy", "rans"], default="all",
                    help="merge: write only merge.npz (merge eviction fixtures); entropy: only entropy.npz; "
                         "rans: only rans.npz")
    args = ap.parse_args()
    if not args.ref:
        ap.error("--ref (or NQ_REFERENCE) must name the reference checkout")
    sys.path.insert(0, args.ref)
    if args.part == "entropy":
        out = os.path.join(HERE, "entropy.npz")
        np.savez_compressed(out, **make_entropy())
        print("wrote", out, os.path.getsize(out), "bytes")
        return
    if args.part == "rans":
        out = os.path.join(HERE, "rans.npz")
        np.savez_compressed(out, **make_rans())
        print("wrote", out, os.path.getsize(out), "bytes")
        return
    if args.part == "merge":
        from nexusquant import pipeline as P
        torch.set_num_threads(8)
        out = os.path.join(HERE, "merge.npz")
        np.savez_compressed(out, **make_merge(P))
        print("wrote", out, os.path.getsize(out), "bytes")
        return
    from nexusquant.core.hadamard import hadamard_matrix
    from nexusquant.core.e8_lattice import E8Lattice
    from nexusquant.core import rope_utils
    from nexusquant.core.temporal_codec import temporal_delta_encode
    from nexusquant.integrations.vllm_backend import NexusQuantKVCompressor as NQC
    from nexusquant import pipeline as P
    from nexusquant.integrations import huggingface as HF

    torch.set_num_threads(8)
    fx = {}

    # ---------------------------------------------------------------- constants
    fx["hadamard_sizes"] = np.array([8, 16, 32, 64, 128, 256], np.int64)
    fx["hadamard_entries"] = np.array([hadamard_matrix(n).abs().max().item() for n in fx["hadamard_sizes"]],
                                      np.float32)
    fx["presets_json"] = np.frombuffer(repr(sorted(HF._EVICT_PRESETS.items())).encode(), np.uint8)
    # n_keep formula at the configs' sizes (float artefacts included)
    cases = [(512, 32, 0.0), (4096, 32, 0.0), (8192, 32, 0.35), (32768, 32, 0.6), (131072, 32, 0.8),
             (100, 10, 0.5), (60, 8, 0.9), (33, 32, 0.5), (32, 32, 0.5), (1, 32, 0.5)]
    fx["nkeep_cases"] = np.array(cases, np.float64)
    nk = []
    for T, sw, r in cases:
        ev = P.NexusQuantEvict(eviction_rate=r, sliding_window=int(sw))
        imp = torch.arange(int(T), dtype=torch.float32).flip(0).unsqueeze(0) + 1.0
        m = ev._build_keep_mask(imp, int(T), eviction_rate=r)
        nk.append(int(m.sum()))
    fx["nkeep_counts"] = np.array(nk, np.int64)

    # ------------------------------------------------------------- rope tables
    for name, d, base, pos in [("r128", 128, 10000.0, np.arange(64)),
                               ("r96", 96, 10000.0, np.arange(64)),
                               ("r128b5e5", 128, 500000.0, np.array([0, 1, 77, 4095, 32767, 131071]))]:
        hk = torch.zeros(1, len(pos), d)
        # recover the reference's cos/sin via inverse_rope_at_positions on unit vectors
        e1 = torch.zeros(1, len(pos), d); e1[..., 0] = 1.0
        r = rope_utils.inverse_rope_at_positions(e1, torch.tensor(pos), base=base)
        fx[f"{name}_cos0"] = r[0, :, 0].numpy()          # x1*c -> cos of freq 0
        fx[f"{name}_pos"] = pos.astype(np.int64)
        c, s = orc.rope_tables(pos, d, base)
        e = torch.zeros(1, len(pos), d); e[..., :d // 2] = 1.0
        r1 = rope_utils.inverse_rope_at_positions(e, torch.tensor(pos), base=base)
        fx[f"{name}_cos"] = r1[0, :, :d // 2].numpy()
        fx[f"{name}_negsin"] = r1[0, :, d // 2:].numpy()
        del hk
    sc = {"type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
    fx["llama3_inv_freq"] = rope_utils._apply_rope_scaling(
        1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128)), sc).numpy()

    # -------------------------------------------- lattice codes: config 0 exactly
    cfg0 = syn.CONFIGS[0]
    k0, v0 = syn.cpu_layer(cfg0, 0)
    fx["cfg0_k_sha"] = np.frombuffer(sha(k0).encode(), np.uint8)
    fx["cfg0_v_sha"] = np.frombuffer(sha(v0).encode(), np.uint8)
    pos = torch.arange(cfg0.seq, dtype=torch.int32)
    kc, ks, kn = ref_codes_direct(NQC, hadamard_matrix, NQC._rope_remove_page, k0[0].float(), pos, 128, 8,
                                  cfg0.rope_base, True)
    vc, vs, vn = ref_codes_direct(NQC, hadamard_matrix, NQC._rope_remove_page, v0[0].float(), pos, 128, 4,
                                  cfg0.rope_base, False)
    # the page path (vllm_backend.compress_page) must give the same codes
    pg = ref_codes_page(NQC, k0[0], v0[0], pos, 3, cfg0.rope_base)
    assert np.array_equal(pg.key_codes.reshape(-1, 128).numpy(), kc)
    fx["cfg0_k_codes_packed"] = orc.pack(kc, 8)
    fx["cfg0_v_codes_packed"] = orc.pack(vc, 4)
    fx["cfg0_k_scales"] = ks.astype(np.float32)
    fx["cfg0_v_scales"] = vs.astype(np.float32)
    cos, sin = orc.rope_tables(np.arange(cfg0.seq), 128, cfg0.rope_base)
    kx = k0[0].float().reshape(-1, 128).numpy()
    cosr = np.tile(cos, (cfg0.heads, 1)); sinr = np.tile(sin, (cfg0.heads, 1))
    fx.update(diff_record("cfg0_k", kc, kn, kx, 128, 8, cosr, sinr))
    fx.update(diff_record("cfg0_v", vc, vn, v0[0].float().reshape(-1, 128).numpy(), 128, 4))
    # fake-quant pipeline output on config 0 (K3V2 quant-only == evict with rate 0)
    ev = P.NexusQuantEvict(eviction_rate=0.0, key_bits=3, value_bits=2, sliding_window=32,
                           rope_base=cfg0.rope_base)
    cache = FakeCache([k0.clone()], [v0.clone()])
    _, mask = ev.compress(cache)
    fx["cfg0_fq_k"] = cache.key_cache[0][:, :2].numpy()     # heads 0-1 keep the fixture small
    fx["cfg0_fq_v"] = cache.value_cache[0][:, :2].numpy()

    # ---------------------------------------- lattice codes: edge-case vectors
    g = torch.Generator().manual_seed(7)
    rows = [torch.zeros(128), torch.ones(128), -torch.ones(128), torch.full((128,), 1e-3),
            torch.arange(128, dtype=torch.float32) - 63.5, torch.randn(128, generator=g) * 1e4,
            torch.randn(128, generator=g) * 1e-4]
    e = torch.zeros(128); e[5] = 3.0; rows.append(e)
    e = torch.zeros(128); e[0] = 1.0; e[64] = -1.0; rows.append(e)
    rows += [torch.randn(128, generator=g) for _ in range(57)]
    edge = torch.stack(rows).half().float()
    fx["edge_x"] = edge.numpy()
    for lv in (2, 4, 8, 16):
        c, s, n = ref_codes_direct(NQC, hadamard_matrix, NQC._rope_remove_page, edge.unsqueeze(0),
                                   torch.arange(edge.shape[0]), 128, lv, 10000.0, False)
        fx[f"edge_v{lv}_codes"] = c
        fx[f"edge_v{lv}_scales"] = s
        fx.update(diff_record(f"edge_v{lv}", c, n, edge.numpy(), 128, lv))
        ck, sk, nk_ = ref_codes_direct(NQC, hadamard_matrix, NQC._rope_remove_page, edge.unsqueeze(0),
                                       torch.arange(edge.shape[0]) * 37, 128, lv, 10000.0, True)
        fx[f"edge_k{lv}_codes"] = ck
        fx[f"edge_k{lv}_scales"] = sk
        cs, sn = orc.rope_tables(np.arange(edge.shape[0]) * 37, 128, 10000.0)
        fx.update(diff_record(f"edge_k{lv}", ck, nk_, edge.numpy(), 128, lv, cs, sn))
    fx["edge_pos_stride"] = np.array([37], np.int64)

    # --------------------------------- head_dim 96 restatement and head_dim 64
    for d, name in ((96, "d96"), (64, "d64")):
        cfg = syn.CacheConfig(name, 1, 1, 3, 41, d)
        k, v = syn.cpu_layer(cfg, 3)
        dp = orc.next_pow2(d)
        p = torch.arange(41, dtype=torch.int32)
        kc, ks, kn = ref_codes_direct(NQC, hadamard_matrix, NQC._rope_remove_page, k[0].float(), p, dp, 8,
                                      10000.0, True)
        vc, vs, vn = ref_codes_direct(NQC, hadamard_matrix, NQC._rope_remove_page, v[0].float(), p, dp, 4,
                                      10000.0, False)
        fx[f"{name}_k_codes"], fx[f"{name}_k_scales"] = kc, ks
        fx[f"{name}_v_codes"], fx[f"{name}_v_scales"] = vc, vs
        cs, sn = orc.rope_tables(np.arange(41), d, 10000.0)
        fx.update(diff_record(f"{name}_k", kc, kn, k[0].float().reshape(-1, d).numpy(), dp, 8,
                              np.tile(cs, (3, 1)), np.tile(sn, (3, 1))))
        fx.update(diff_record(f"{name}_v", vc, vn, v[0].float().reshape(-1, d).numpy(), dp, 4))
        fx[f"{name}_k_sha"] = np.frombuffer(sha(k).encode(), np.uint8)

    # --------------------------------------------------- dequantize (page path)
    comp = NQC(head_dim=128, bits=2, rope_base=10000.0)
    kk, vv = syn.cpu_layer(syn.CacheConfig("dq", 1, 1, 2, 24, 128), 11)
    pos = torch.tensor([0, 3, 4, 9, 10, 11, 20, 31, 40, 41, 42, 50, 63, 64, 65, 70, 71, 72, 80, 81, 90, 99,
                        100, 127], dtype=torch.int32)
    page = comp.compress_page(kk[0], vv[0], pos)
    dk, dv = comp.decompress_page(page)
    fx["dq_pos"] = pos.numpy().astype(np.int64)
    fx["dq_k_codes"] = page.key_codes.reshape(-1, 128).numpy()
    fx["dq_v_codes"] = page.value_codes.reshape(-1, 128).numpy()
    fx["dq_k_scales16"] = page.key_scales.reshape(-1).numpy()
    fx["dq_v_scales16"] = page.value_scales.reshape(-1).numpy()
    fx["dq_k_out"] = dk.numpy()
    fx["dq_v_out"] = dv.numpy()
    fx["dq_k_nibble"] = NQC.pack_codes_nibble(page.key_codes).reshape(-1, 64).numpy()
    # temporal delta on codes laid out (streams, tokens, coords)
    codes_st = page.key_codes.numpy()  # (h, s, d)
    fx["delta_codes"] = codes_st
    fx["delta_ref"] = temporal_delta_encode(codes_st[0].reshape(-1), codes_st.shape[1]).reshape(
        codes_st.shape[1], -1)

    # ------------------------------------------------------ key-key importance
    cfgs = syn.CacheConfig("score", 1, 2, 4, 300, 128)
    ksc, _ = syn.cpu_layer(cfgs, 0)
    ev = P.NexusQuantEvict(eviction_rate=0.6, sliding_window=16)
    imp = ev._score_importance(ksc.float())
    fx["score_k_sha"] = np.frombuffer(sha(ksc).encode(), np.uint8)
    fx["score_importance"] = imp.numpy()
    fx["score_mask"] = ev._build_keep_mask(imp, 300, eviction_rate=0.6).numpy()

    # ---------------------------------------------------- keep-mask edge cases
    sel = []
    rng = np.random.default_rng(3)
    for i, (T, sw, r) in enumerate([(200, 16, 0.6), (64, 8, 0.5), (40, 32, 0.5), (33, 32, 0.9),
                                    (16, 32, 0.5), (1, 32, 0.5), (500, 0, 0.3), (128, 4, 0.0),
                                    (300, 32, 0.999)]):
        imp = torch.tensor(rng.random((2, T)).astype(np.float32))
        ev = P.NexusQuantEvict(eviction_rate=r, sliding_window=sw)
        m = ev._build_keep_mask(imp, T, eviction_rate=r)
        fx[f"sel{i}_imp"] = imp.numpy()
        fx[f"sel{i}_mask"] = m.numpy()
        sel.append((T, sw, r))
    # ties: many equal scores; record torch.topk's own choice for reference
    imp = torch.tensor(np.repeat(np.array([[0.5, 0.25]], np.float32), 50, axis=1))
    ev = P.NexusQuantEvict(eviction_rate=0.5, sliding_window=4)
    fx["selties_imp"] = imp.numpy()
    fx["selties_mask"] = ev._build_keep_mask(imp, 100, eviction_rate=0.5).numpy()
    # protected positions
    ev = P.NexusQuantEvict(eviction_rate=0.8, sliding_window=8,
                           protected_positions=torch.tensor([1, 2, 3, 50, 51, 999]))
    imp = torch.tensor(rng.random((2, 120)).astype(np.float32))
    fx["selprot_imp"] = imp.numpy()
    fx["selprot_mask"] = ev._build_keep_mask(imp, 120, eviction_rate=0.8).numpy()
    fx["sel_cases"] = np.array(sel, np.float64)

    # --------------------------------------------------------- pipeline outputs
    cfgp = syn.CacheConfig("pipe", 3, 2, 2, 96, 128)
    ks_, vs_ = zip(*[syn.cpu_layer(cfgp, l) for l in range(3)])
    fx["pipe_sha"] = np.frombuffer(sha(torch.stack(ks_)).encode(), np.uint8)
    # (a) evict K2V2 60 %, sw 16, protect_boundary 1 (layers 0 and 2 fp16)
    ev = P.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, protect_boundary=1)
    cache = FakeCache([k.clone() for k in ks_], [v.clone() for v in vs_])
    _, mask = ev.compress(cache)
    fx["pipe_evict_mask"] = mask.numpy()
    for l in range(3):
        fx[f"pipe_evict_k{l}"] = cache.key_cache[l].numpy()
        fx[f"pipe_evict_v{l}"] = cache.value_cache[l].numpy()
    # (b) quant-only (compress_kv_cache mode="quant_only", bits=3)
    cache = FakeCache([k.clone() for k in ks_[:1]], [v.clone() for v in vs_[:1]])
    P.compress_kv_cache(cache, mode="quant_only", bits=3)
    fx["pipe_qo_k0"] = cache.key_cache[0].numpy()
    fx["pipe_qo_v0"] = cache.value_cache[0].numpy()
    # (c) simple mode (the default of compress_kv_cache), batch 1
    cache = FakeCache([ks_[0][:1].clone()], [vs_[0][:1].clone()])
    P.compress_kv_cache(cache)
    fx["pipe_simple_k0"] = cache.key_cache[0].numpy()
    fx["pipe_simple_v0"] = cache.value_cache[0].numpy()
    # (d) truncation, batch 1, K3V2
    tr = P.NexusQuantEvictTruncate(bits=2, key_bits=3, eviction_rate=0.5, sliding_window=10)
    cache = FakeCache([k[:1].clone() for k in ks_[:2]], [v[:1].clone() for v in vs_[:2]])
    _, nxt = tr.compress(cache)
    fx["pipe_trunc_next"] = np.array([nxt], np.int64)
    for l in range(2):
        fx[f"pipe_trunc_k{l}"] = cache.key_cache[l].numpy()
        fx[f"pipe_trunc_v{l}"] = cache.value_cache[l].numpy()
    # (e) soft eviction (1-bit for evicted tokens)
    ev = P.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, soft_eviction=True)
    cache = FakeCache([ks_[0].clone()], [vs_[0].clone()])
    _, mask = ev.compress(cache)
    fx["pipe_soft_k0"] = cache.key_cache[0].numpy()
    fx["pipe_soft_v0"] = cache.value_cache[0].numpy()

    # ------------------------------------------- real-attention scorer (restated)
    cfgr = syn.CacheConfig("real", 2, 1, 4, 256, 96, rope_base=10000.0)
    Ks = [syn.cpu_layer(cfgr, l)[0] for l in range(2)]
    Qs = [syn.cpu_queries(cfgr, l, n_queries=64) for l in range(2)]
    imp = torch.zeros(1, 256)
    for Q, K in zip(Qs, Ks):
        att = torch.einsum('bhqd,bhkd->bhqk', Q.float(), K.float()) * (96 ** -0.5)
        qpos = torch.arange(256 - 64, 256)
        causal = torch.arange(256)[None, :] > qpos[:, None]
        att = att.masked_fill(causal, float('-inf')).softmax(-1)
        imp += att.sum(dim=2).mean(dim=1)      # pipeline.py:826-834
    imp = imp / 2                                # pipeline.py:835
    fx["real_importance"] = imp.numpy()
    fx["real_sha"] = np.frombuffer(sha(torch.stack(Ks)).encode(), np.uint8)

    out = os.path.join(HERE, "golden.npz")
    np.savez_compressed(out, **fx)
    print("wrote", out, os.path.getsize(out), "bytes")
    out = os.path.join(HERE, "merge.npz")
    np.savez_compressed(out, **make_merge(P))
    print("wrote", out, os.path.getsize(out), "bytes")
    out = os.path.join(HERE, "entropy.npz")
    np.savez_compressed(out, **make_entropy())
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
