"""The entropy-coding host post-step (nexusquant_b200/entropy.py) against the reference's
temporal_codec.compress_indices output (tests/golden/entropy.npz).  No GPU needed."""
import os

import numpy as np
import pytest

from nexusquant_b200 import entropy as E
from tests.golden.make_golden import entropy_coords
from tests.parity import sha

FIX = os.path.join(os.path.dirname(__file__), "golden", "entropy.npz")


@pytest.fixture(scope="module")
def fx():
    return np.load(FIX)


def test_inputs_regenerate(fx):
    coords, n_tokens = entropy_coords()
    assert sha(coords) == bytes(fx["coords_sha"]).decode() and n_tokens == int(fx["n_tokens"])


@pytest.mark.parametrize("use_delta", [True, False])
def test_zlib_stream_byte_identical_to_reference(fx, use_delta):
    """Without the zstandard module the reference writes zlib streams; ours match byte for byte."""
    assert int(fx["has_zstd"]) == 0
    coords, n_tokens = entropy_coords()
    ours = E.compress_indices(coords, n_tokens, use_delta=use_delta, codec="zlib")
    ref = bytes(fx[f"stream_delta{int(use_delta)}"])
    assert ours == ref
    assert np.array_equal(E.decompress_indices(ref), coords)


def test_delta_matches_reference_layout(fx):
    """Our temporal delta equals the reference's: decompressing the reference's delta stream's
    payload gives exactly our temporal_delta_encode bytes."""
    import zlib
    coords, n_tokens = entropy_coords()
    raw = zlib.decompress(bytes(fx["stream_delta1"])[E.HEADER_BYTES:])
    assert raw == E.temporal_delta_encode(coords, n_tokens).tobytes()
    assert np.array_equal(E.temporal_delta_decode(E.temporal_delta_encode(coords, n_tokens), n_tokens), coords)


@pytest.mark.skipif(E.zstd() is None, reason="libzstd not on this system")
@pytest.mark.parametrize("level", [3, 22])
def test_zstd_roundtrip_and_header(level):
    coords, n_tokens = entropy_coords()
    blob = E.compress_indices(coords, n_tokens, level=level)
    n_el, nt, ud, comp = __import__("struct").unpack_from("<IIBB", blob)
    assert (n_el, nt, ud, comp) == (coords.size, n_tokens, 1, E.COMPRESSOR_ZSTD)
    assert np.array_equal(E.decompress_indices(blob), coords)
    # delta coding helps on temporally correlated codes, as the reference reports
    assert len(blob) < len(E.compress_indices(coords, n_tokens, use_delta=False, level=level))


def test_unreshapeable_input_is_left_as_is():
    x = np.arange(-5, 5, dtype=np.int8)
    assert np.array_equal(E.temporal_delta_encode(x, 3), x)
    assert np.array_equal(E.decompress_indices(E.compress_indices(x, 3, codec="zlib")), x)
