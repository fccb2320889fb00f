"""The device draw (pb_row_params.rng = PB_RNG_PHILOX | step) on the CPU.

Philox4x32-10 is checked against the published known-answer vectors of the algorithm (Salmon,
Moraes, Dror and Shaw, SC 2011; the Random123 distribution's test vectors), in the oracle's own
restatement and in the library's host copy of the device function, and the two U53 derivations
are compared on many (seed, step) pairs. The library is loaded but no kernel is launched.
"""

import ctypes

import numpy as np
import pytest

import oracle
from pagedbatch_b200 import _lib, ops

# (counter[4], key[2], output[4]) for Philox4x32 with 10 rounds
KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", KAT)
def test_oracle_philox_known_answers(ctr, key, want):
    assert tuple(oracle.philox4x32_10(ctr, key)) == want


@pytest.mark.parametrize("ctr,key,want", KAT)
def test_library_philox_known_answers(ctr, key, want):
    L = _lib.load()
    c = np.array(ctr, dtype=np.uint32)
    k = np.array(key, dtype=np.uint32)
    o = np.zeros(4, dtype=np.uint32)
    L.pb_philox4x32_10(ctypes.c_void_p(c.ctypes.data), ctypes.c_void_p(k.ctypes.data), ctypes.c_void_p(o.ctypes.data))
    assert tuple(int(v) for v in o) == want


def test_u53_library_matches_oracle():
    L = _lib.load()
    rng = np.random.default_rng(0)
    seeds = rng.integers(0, 1 << 63, 200, dtype=np.int64)
    steps = rng.integers(0, 1 << 31, 200, dtype=np.int64)
    steps[:3] = [0, 1, (1 << 31) - 1]
    rec = oracle.make_device_rng_params([1.0] * 200, [1.0] * 200, [0] * 200, seeds, steps)
    for i in range(200):
        want = oracle.row_u53(rec[i])
        assert want is not None and 0 <= want < (1 << 53)
        assert L.pb_philox_u53(int(seeds[i]), int(steps[i])) == want


def test_u53_is_uniform_and_step_sensitive():
    """Device draws of one seed over consecutive steps: distinct, and spread over [0, 2^53)."""
    L = _lib.load()
    u = np.array([L.pb_philox_u53(12345, s) for s in range(20000)], dtype=np.float64) / 2.0**53
    assert len(np.unique(u)) == len(u)
    hist, _ = np.histogram(u, bins=20, range=(0, 1))
    expected = len(u) / 20
    chi2 = float(((hist - expected) ** 2 / expected).sum())
    assert chi2 < 50.0  # 19 degrees of freedom: p ~ 1e-4


def test_pack_params_device_draws_and_host_uniforms():
    rec = ops.pack_params([0.7, 1.0], [0.9, 1.0], [50, 0], [0.25, 0.5], seeds=[7, 2**62], steps=[3, 0])
    assert rec["rng"][0] == _lib.RNG_PHILOX | 3 and rec["rng"][1] == _lib.RNG_PHILOX
    assert rec["uniform"].view(np.uint64).tolist() == [7, 2**62]
    host = ops.pack_params([0.7], [0.9], [50], [0.25])
    assert host["rng"][0] == 0 and host["uniform"][0] == 0.25
    with pytest.raises(ValueError, match="steps"):
        ops.pack_params([0.7], [0.9], [50], [0.0], seeds=[1], steps=[-1])
