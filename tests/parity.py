"""Shared parity helpers for the tests (oracle-side checks and tolerances)."""
from __future__ import annotations

import hashlib

import numpy as np

# Reconstructed K/V tolerance of the north star: relative L2 per tensor.
REL_L2_TOL = 1e-3
# Kept-token / lattice decisions within this distance of a boundary are excluded.
BOUNDARY_TOL = 1e-6


def sha(a) -> str:
    import torch
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu().contiguous().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def golden_str(g, key) -> str:
    return bytes(g[key]).decode()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def check_codes_vs_reference(orc, codes_mine, codes_ref, nrm_ref_rows, diff_vecs, d_p, levels, nrm_mine=None,
                             label=""):
    """Codes must equal the reference's except in 8-groups that sit on a decision boundary.

    codes_*: [n, d_p] int8.  diff_vecs / nrm_ref_rows: the vectors whose groups the
    fixture generator found to differ, with the reference's normalised inputs.
    Returns (n_excluded_groups, n_groups)."""
    G = d_p // 8
    cm = np.asarray(codes_mine).reshape(-1, G, 8)
    cr = np.asarray(codes_ref).reshape(-1, G, 8)
    bad = np.nonzero((cm != cr).any(-1))
    allowed = {}
    for j, v in enumerate(np.asarray(diff_vecs)):
        amb = orc.boundary_groups(nrm_ref_rows[j:j + 1], None if nrm_mine is None else nrm_mine[int(v)][None],
                                  levels)[0]
        allowed[int(v)] = amb
    unexplained = []
    for v, g in zip(*bad):
        ok = int(v) in allowed and bool(allowed[int(v)][g])
        if not ok:
            unexplained.append((int(v), int(g)))
    assert not unexplained, f"{label}: {len(unexplained)} groups differ off-boundary, e.g. {unexplained[:5]}"
    return len(bad[0]), cm.shape[0] * G
