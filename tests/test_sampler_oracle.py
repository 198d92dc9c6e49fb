"""CPU checks of the fused sampler's contract (no kernel is launched):
the oracle's Philox4x32-10 against the generator's published known-answer
vectors (Salmon et al., SC 2011; the Random123 distribution's test vectors),
the Gumbel noise's range and moments, and the C-ABI validation of
gsp_row_sparse_sample."""
import ctypes

import numpy as np

from gsp import _native
from oracle import gsp_oracle as O


def test_philox_known_answers():
    cases = [
        ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
         (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF),
         (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, want in cases:
        got = O.philox4x32_10(np.array([ctr], dtype=np.uint32), *key)[0]
        assert tuple(int(x) for x in got) == want


def test_gumbel_noise_moments():
    g = O.gumbel_noise(2026, 3, np.arange(200000))
    assert g.dtype == np.float32 and np.isfinite(g).all()
    # standard Gumbel: mean = Euler-Mascheroni constant, variance = pi^2 / 6
    assert abs(g.mean() - 0.5772157) < 0.01
    assert abs(g.var() - np.pi ** 2 / 6) < 0.02
    # keyed: another seed or step gives other noise, the same ones the same noise
    assert not np.array_equal(g[:100], O.gumbel_noise(2027, 3, np.arange(100)))
    assert not np.array_equal(g[:100], O.gumbel_noise(2026, 4, np.arange(100)))
    assert np.array_equal(g[:100], O.gumbel_noise(2026, 3, np.arange(100)))


FAKE = ctypes.c_void_p(4096)  # never dereferenced: every call below fails validation first


def _sample_call(temperature=1.0, seeds=FAKE, sample=FAKE, ws=FAKE, wsb=1 << 30):
    lib = _native.load()
    return lib.gsp_row_sparse_sample(FAKE, 8, FAKE, 8, None, 0, 1, 64, 8, 0, 0, None, 64, temperature, seeds, 0,
                                     sample, None, None, None, None, None, ws, wsb, None)


def test_sample_entry_validation():
    lib = _native.load()
    assert _sample_call(temperature=0.0) == _native.GSP_ERR_INVALID_ARGUMENT
    assert b"temperature" in lib.gsp_last_error()
    assert _sample_call(temperature=float("inf")) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _sample_call(temperature=float("nan")) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _sample_call(seeds=None) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _sample_call(sample=None) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _sample_call(ws=None) == _native.GSP_ERR_WORKSPACE
    assert _sample_call(wsb=256) == _native.GSP_ERR_WORKSPACE
