"""rANS container of the lattice codes (nexusquant_b200/entropy.py, native nq_rans_encode /
nq_rans_decode, device nq_code_histogram / nq_code_symbols) against the reference's own
entropy_coder.encode_e8 streams (tests/golden/rans.npz, made by make_golden.py --part rans).

CPU tests map codes to symbols here (the reference's rule, entropy_coder.py:35-75), then
check the host half -- frequency table, native state loop, container layout -- byte for
byte.  GPU tests run the whole path from packed codes in HBM."""
import os

import numpy as np
import pytest

from nexusquant_b200 import entropy as E
from tests.golden.make_golden import RANS_CASES, rans_case

FIX = os.path.join(os.path.dirname(__file__), "golden", "rans.npz")
NAMES = [c[0] for c in RANS_CASES]


@pytest.fixture(scope="module")
def fx():
    return np.load(FIX)


def _symbols(codes, levels):
    c = codes.astype(np.int32).reshape(-1)
    half = bool((c & 1).any())
    sym = np.clip(c + levels, 0, 2 * levels) if half else np.clip(c // 2 + levels // 2, 0, levels)
    return sym.astype(np.uint8), half, (2 * levels + 1 if half else levels + 1)


@pytest.mark.parametrize("name", NAMES)
def test_inputs_regenerate(fx, name):
    case = [c for c in RANS_CASES if c[0] == name][0]
    codes, s16 = rans_case(*case[1:])
    assert np.array_equal(codes, fx[f"{name}_codes"]) and np.array_equal(s16, fx[f"{name}_scales"])
    assert int(fx[f"{name}_roundtrip"]) == 1


@pytest.mark.parametrize("name", NAMES)
def test_stream_byte_identical_host(fx, name):
    codes, s16, levels = fx[f"{name}_codes"], fx[f"{name}_scales"], int(fx[f"{name}_levels"])
    sym, half, a = _symbols(codes, levels)
    counts = np.bincount(sym, minlength=a)
    blob = E.rans_pack_e8(sym, counts, half, levels, np.repeat(s16, codes.shape[1] // 8))
    assert blob == bytes(fx[f"{name}_stream"])
    dc, ds = E.rans_decode_e8(blob)
    assert np.array_equal(dc, codes.reshape(-1)) and np.array_equal(ds, np.repeat(s16, codes.shape[1] // 8))


@pytest.mark.parametrize("name", NAMES)
def test_entropy_stats_match_reference(fx, name):
    """measure_e8_entropy's statistics (the reference's own values) from symbol counts."""
    codes, levels = fx[f"{name}_codes"], int(fx[f"{name}_levels"])
    sym, half, a = _symbols(codes, levels)
    st = E.measure_entropy_counts(np.bincount(sym, minlength=a), a)
    ref = fx[f"{name}_entropy"]
    got = np.array([st["entropy_bps"], st["uniform_bps"], st["compression_ratio"], st["n_symbols"],
                    st["n_unique"]], np.float64)
    assert np.array_equal(got, ref), (got, ref)


def test_freq_table_edge_cases():
    # all counts zero: uniform table with the remainder on symbol 0
    f = E.rans_freq_table(np.zeros(9, np.int64))
    assert f.sum() == 4096 and f[0] == 4096 // 9 + 4096 % 9 and (f[1:] == 4096 // 9).all()
    # one symbol holds everything
    f = E.rans_freq_table(np.array([0, 0, 5, 0]))
    assert f.tolist() == [0, 0, 4096, 0]
    # a rare symbol keeps frequency 1
    f = E.rans_freq_table(np.array([10 ** 9, 1, 0]))
    assert f[1] >= 1 and f.sum() == 4096


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_rans_roundtrip_random(seed):
    rng = np.random.default_rng(seed)
    a = int(rng.integers(2, 34))
    p = rng.dirichlet(np.full(a, 0.3))
    sym = rng.choice(a, size=int(rng.integers(1, 50000)), p=p).astype(np.uint8)
    f = E.rans_freq_table(np.bincount(sym, minlength=a))
    w = E.rans_encode(sym, f)
    assert w.size <= sym.size + 2
    assert np.array_equal(E.rans_decode(w, sym.size, f), sym)


def test_rans_empty_stream():
    f = E.rans_freq_table(np.zeros(5, np.int64))
    w = E.rans_encode(np.zeros(0, np.uint8), f)
    assert w.tolist() == [1, 0]        # the initial state 2^16, high word first
    assert E.rans_decode(w, 0, f).size == 0


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_stream_byte_identical_device(fx, orc, name):
    """Histogram and symbols on the GPU from packed codes; the stream equals the reference's."""
    import torch
    from nexusquant_b200 import kernels as K
    codes, s16, levels = fx[f"{name}_codes"], fx[f"{name}_scales"], int(fx[f"{name}_levels"])
    packed = torch.from_numpy(orc.pack(codes, levels)).cuda()
    hist = K.code_histogram(packed, 128, levels).cpu().numpy()
    c = codes.astype(np.int64).reshape(-1)
    assert np.array_equal(hist, np.bincount(np.clip(c + levels, 0, 2 * levels), minlength=2 * levels + 1))
    sym, half, _ = _symbols(codes, levels)
    assert np.array_equal(K.code_symbols(packed, 128, levels, half).cpu().numpy().reshape(-1), sym)
    blob = E.rans_encode_e8(packed, torch.from_numpy(s16).cuda(), 128, levels)
    assert blob == bytes(fx[f"{name}_stream"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_entropy_stats_device(fx, orc, name):
    import torch
    codes, levels = fx[f"{name}_codes"], int(fx[f"{name}_levels"])
    packed = torch.from_numpy(orc.pack(codes, levels)).cuda()
    st = E.e8_entropy_stats(packed, 128, levels)
    ref = fx[f"{name}_entropy"]
    assert [st["entropy_bps"], st["uniform_bps"], st["compression_ratio"], st["n_symbols"], st["n_unique"]] == \
        ref.tolist()


@pytest.mark.gpu
def test_histogram_large_accumulates(orc):
    """Many CTAs (grid capped at 8 per SM, grid-stride) and accumulation into given counts."""
    import torch
    from nexusquant_b200 import kernels as K
    rng = np.random.default_rng(5)
    codes = (rng.integers(-2, 3, size=(300000, 128)) * 1).astype(np.int8)
    packed = torch.from_numpy(orc.pack(codes, 4)).cuda()
    cnt = torch.zeros(9, dtype=torch.int32, device="cuda")
    K.code_histogram(packed, 128, 4, cnt)
    K.code_histogram(packed, 128, 4, cnt)
    ref = 2 * np.bincount(codes.reshape(-1).astype(np.int64) + 4, minlength=9)
    assert np.array_equal(cnt.cpu().numpy(), ref)
