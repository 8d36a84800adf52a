"""Merge eviction (NexusQuantEvict(merge_eviction=True), nexusquant/pipeline.py:961-1048).

CPU: the oracle's restatement reproduces the reference's merged values bit for bit
(tests/golden/merge.npz, written by the reference's own _apply_merge_eviction).
GPU: the device path (centroids -> fused similarity argmax -> in-place accumulation) against
the oracle -- the same nearest survivor for every evicted token (a different choice is only
accepted on a near tie) and bit-identical merged values -- and the reference-facing pipeline
against the reference's compress(merge_eviction=True) output.
"""
import os

import numpy as np
import pytest
import torch

from nexusquant_b200 import synthetic as syn
from tests.parity import REL_L2_TOL, golden_str, rel_l2, sha

HERE = os.path.dirname(os.path.abspath(__file__))
DEV = "cuda:0"
NEAR_TIE = 1e-5  # cosine gap under which fp32 summation order may pick either survivor


@pytest.fixture(scope="module")
def mg():
    return np.load(os.path.join(HERE, "golden", "merge.npz"))


def _fixture_layers(mg):
    cfg = syn.CacheConfig("merge", 4, 2, 2, 96, 128)
    ks, vs = zip(*[syn.cpu_layer(cfg, l, seq=(64 if l == 2 else None)) for l in range(4)])
    if sha(torch.cat([t.reshape(-1) for t in ks + vs])) != golden_str(mg, "merge_in_sha"):
        pytest.skip("generator drift")
    return list(ks), list(vs)


def test_oracle_merge_matches_reference(mg, orc):
    _, vs = _fixture_layers(mg)
    out, near = orc.merge_values([v.numpy() for v in vs], mg["merge_mask"], mg["merge_importance"])
    for l in range(4):
        assert np.array_equal(out[l], mg[f"merge_v{l}"]), f"layer {l}"
    assert np.array_equal(out[2], vs[2].numpy())  # the shorter layer is skipped
    assert all(n is not None for n in near)


def test_oracle_merge_weights_are_fp32_products(orc):
    """w is rounded to fp32 before the multiply, and product and sum are separately rounded
    (torch scalar semantics) -- a double-precision product would differ here."""
    v = np.zeros((1, 1, 3, 8), np.float32)
    v[0, 0, 0] = 1.0
    v[0, 0, 1] = np.float32(1.0009765625)   # evicted
    imp = np.array([[0.7, 0.3, 1.0]], np.float32)
    mask = np.array([[True, False, True]])
    out, near = orc.merge_values([v], mask, imp, nearest=[np.array([0])])
    w = np.float32(float(imp[0, 1]) / (float(imp[0, 0]) + float(imp[0, 1]) + 1e-8))
    assert np.array_equal(out[0][0, 0, 0], np.float32(1.0) + (v[0, 0, 1] * w).astype(np.float32))


# ----------------------------------------------------------------------------- GPU


def _check_against_oracle(orc, vs_dev, vs_cpu, mask, imp):
    from nexusquant_b200 import kernels as K
    near_dev = []
    K.merge_evicted_values(vs_dev, torch.as_tensor(mask, device=DEV), torch.as_tensor(imp, device=DEV),
                           nearest_out=near_dev)
    torch.cuda.synchronize()
    b, T = mask.shape
    full = [i for i, v in enumerate(vs_cpu) if v.shape[2] == T]
    for bi in range(b):
        ev, kp = np.nonzero(~mask[bi])[0], np.nonzero(mask[bi])[0]
        if ev.size == 0 or kp.size == 0 or not full:
            assert near_dev[bi] is None
            continue
        nd = near_dev[bi].cpu().numpy()
        unit = orc.merge_unit_centroids([vs_cpu[i][bi] for i in full])
        S = orc.merge_similarity(unit, ev, kp)
        no = S.argmax(axis=1)
        diff = np.nonzero(nd != no)[0]
        gap = S[diff, no[diff]] - S[diff, nd[diff]]
        assert np.all(gap < NEAR_TIE), f"batch {bi}: {diff.size} different survivors, max gap {gap.max()}"
    ref, _ = orc.merge_values(vs_cpu, mask, imp, nearest=[None if n is None else n.cpu().numpy() for n in near_dev])
    for i, (a, r) in enumerate(zip(vs_dev, ref)):
        assert np.array_equal(a.cpu().numpy(), r), f"layer {i}"
    return near_dev


@pytest.mark.gpu
def test_merge_kernels_match_reference_fixture(mg, orc):
    from nexusquant_b200 import kernels as K
    _, vs = _fixture_layers(mg)
    vd = [v.to(DEV) for v in vs]
    K.merge_evicted_values(vd, torch.as_tensor(mg["merge_mask"], device=DEV),
                           torch.as_tensor(mg["merge_importance"], device=DEV))
    for l in range(4):
        assert np.array_equal(vd[l].cpu().numpy(), mg[f"merge_v{l}"]), f"layer {l}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,d,T,heads", [(torch.float16, 128, 300, [2, 2, 3, 2]),
                                            (torch.bfloat16, 64, 257, [4, 4]),
                                            (torch.float32, 96, 130, [1, 2]),
                                            (torch.float16, 128, 2000, [8, 8])])
def test_merge_kernels_vs_oracle(orc, dtype, d, T, heads):
    g = torch.Generator().manual_seed(T + d)
    b = 2
    vs = [torch.randn(b, h, T, d, generator=g).to(dtype) for h in heads]
    vs.append(torch.randn(b, heads[0], T // 2, d, generator=g).to(dtype))  # shorter layer: skipped
    rng = np.random.default_rng(T)
    mask = rng.random((b, T)) < 0.3
    mask[:, 0] = True
    mask[:, -16:] = True
    imp = rng.random((b, T)).astype(np.float32)
    if dtype == torch.bfloat16:
        vs_cpu = [v.float().numpy() for v in vs]  # exact widening; results compared in fp32
    else:
        vs_cpu = [v.numpy() for v in vs]
    vd = [v.to(DEV) for v in vs]
    if dtype == torch.bfloat16:
        # the oracle rounds to the input dtype: replay bf16 rounding through torch
        from nexusquant_b200 import kernels as K
        near = []
        K.merge_evicted_values(vd, torch.as_tensor(mask, device=DEV), torch.as_tensor(imp, device=DEV),
                               nearest_out=near)
        ref, _ = orc.merge_values(vs_cpu, mask, imp, nearest=[n.cpu().numpy() for n in near])
        for a, r in zip(vd, ref):
            assert torch.equal(a.cpu(), torch.from_numpy(r).to(torch.bfloat16))
        # and the chosen survivors agree with the oracle's
        for bi in range(b):
            ev, kp = np.nonzero(~mask[bi])[0], np.nonzero(mask[bi])[0]
            unit = orc.merge_unit_centroids([vs_cpu[i][bi] for i in range(len(heads))])
            S = orc.merge_similarity(unit, ev, kp)
            nd = near[bi].cpu().numpy()
            assert np.all(S.max(1) - S[np.arange(len(ev)), nd] < NEAR_TIE)
    else:
        _check_against_oracle(orc, vd, vs_cpu, mask, imp)
    assert torch.equal(vd[-1].cpu(), vs[-1])


@pytest.mark.gpu
def test_merge_nothing_evicted_is_identity():
    from nexusquant_b200 import kernels as K
    v = torch.randn(1, 2, 50, 128).half().to(DEV)
    before = v.clone()
    near = []
    K.merge_evicted_values([v], torch.ones(1, 50, dtype=torch.bool, device=DEV), torch.rand(1, 50, device=DEV),
                           nearest_out=near)
    assert near == [None] and torch.equal(v, before)


@pytest.mark.gpu
def test_evict_with_merge_matches_reference_pipeline(mg):
    import nexusquant_b200 as nq

    class FakeCache:
        def __init__(self, ks, vs):
            self.key_cache = list(ks)
            self.value_cache = list(vs)

    ks, vs = _fixture_layers(mg)
    idx = [0, 1, 3]
    orig = [vs[l].to(DEV) for l in idx]
    cache = FakeCache([ks[l].to(DEV) for l in idx], [o.clone() for o in orig])
    inputs = list(cache.value_cache)
    ev = nq.NexusQuantEvict(bits=2, eviction_rate=0.6, sliding_window=16, protect_boundary=1, merge_eviction=True)
    _, mask = ev.compress(cache)
    assert np.array_equal(mask.cpu().numpy(), mg["merge_pipe_mask"])
    for i in range(3):
        out_k = cache.key_cache[i].float().cpu().numpy()
        out_v = cache.value_cache[i].float().cpu().numpy()
        assert rel_l2(out_k, mg[f"merge_pipe_k{i}"]) < REL_L2_TOL
        assert rel_l2(out_v, mg[f"merge_pipe_v{i}"]) < REL_L2_TOL
    # boundary layers (0 and 2) stay fp16: merged values with evicted rows zeroed.  The
    # pipeline scores importance on the device (within rtol 5e-5 of the reference's), so the
    # merge weights -- and an occasional fp16 ulp -- may differ; with the reference's own
    # importance the merge is bit-exact (test_merge_kernels_match_reference_fixture).
    m = mg["merge_pipe_mask"][:, None, :, None] > 0
    for i in (0, 2):
        out_v = cache.value_cache[i].float().cpu().numpy()
        ref_v = mg[f"merge_pipe_v{i}"].astype(np.float32)
        assert np.array_equal(out_v * ~m, np.zeros_like(out_v)) and np.array_equal(ref_v * ~m, np.zeros_like(ref_v))
        assert np.allclose(out_v, ref_v, rtol=2e-3, atol=1e-4)
    # the caller's tensors are not modified (the reference merges into clones)
    for a, o in zip(inputs, orig):
        assert torch.equal(a, o)


def _unit_rows(seq, seed, d=128, structured=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(seq, d, generator=g)
    if structured:  # correlated rows: a few directions plus noise, like averaged value rows
        base = torch.randn(8, d, generator=g)
        x = base[torch.randint(0, 8, (seq,), generator=g)] + 0.3 * x
    return torch.nn.functional.normalize(x, dim=1)


@pytest.mark.gpu
@pytest.mark.parametrize("seed,seq,structured", [(0, 5000, False), (1, 20011, True), (2, 777, True), (3, 300, False)])
def test_nearest_unit_equals_exact_kernel(seed, seq, structured):
    """Tensor-core screening + exact re-check picks exactly the exact kernel's indices."""
    from nexusquant_b200 import kernels as K
    u = _unit_rows(seq, seed, structured=structured).to(DEV)
    g = torch.Generator().manual_seed(100 + seed)
    perm = torch.randperm(seq, generator=g)
    nk = max(1, seq // 5 + seed)
    kept, ev = perm[:nk].sort().values, perm[nk:].sort().values
    a = K.merge_nearest(u, ev, kept, tensor_cores=True)
    b = K.merge_nearest(u, ev, kept, tensor_cores=False)
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_nearest_unit_ties_overflow_nan_and_non_unit_rows():
    """Exact ties (first index wins), more near-ties than candidate slots (exact fallback),
    a NaN evicted row (index 0, as torch.argmax) and a non-unit evicted row."""
    from nexusquant_b200 import kernels as K
    seq = 3000
    u = _unit_rows(seq, 7)
    target = u[0].clone()
    g = torch.Generator().manual_seed(11)
    for i in range(1, 41):  # 40 kept rows within ~1e-6 of the first evicted row's direction
        u[100 + i] = torch.nn.functional.normalize(target + 1e-6 * torch.randn(128, generator=g), dim=0)
    u[200] = target
    u[201] = target                      # exact tie between kept rows 200 and 201
    u[5] = float("nan")                  # NaN evicted row
    u[6] = 2.0 * u[6]                    # not a unit row
    u = u.to(DEV)
    ev = torch.tensor([0, 5, 6] + list(range(1000, 1400)))
    kept = torch.tensor(list(range(100, 142)) + [200, 201] + list(range(2000, 2600)))
    a = K.merge_nearest(u, ev, kept, tensor_cores=True)
    b = K.merge_nearest(u, ev, kept, tensor_cores=False)
    bad = (a != b).nonzero().flatten().tolist()
    assert not bad, (bad[:8], a[bad[:8]].tolist(), b[bad[:8]].tolist())
    assert int(a[1]) == 0
