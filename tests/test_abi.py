"""The C-ABI library: it loads, exports every entry point include/*.h declares, and its host helpers
agree with the oracle. No kernel runs here (no GPU needed)."""

import glob
import os
import re

import numpy as np
import pytest

import oracle
from pagedbatch_b200 import _lib, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        txt = open(h).read()
        names |= set(re.findall(r"PB_API\s+[\w\s\*]+?\b(pb_\w+)\s*\(", txt))
    return names


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert {"pb_sample", "pb_key_of", "pb_exp", "pb_strerror", "pb_version"} <= names
    for n in names:
        assert hasattr(lib, n), n
    assert set(_lib.EXPORTS) <= names


def test_structs_match_header():
    txt = open(os.path.join(REPO, "include", "pagedbatch_b200.h")).read()
    assert "typedef struct pb_row_params" in txt and "typedef struct pb_row_info" in txt
    assert _lib.ROW_PARAMS == oracle.ROW_PARAMS
    assert _lib.ROW_INFO == oracle.ROW_INFO


def test_host_exp_matches_oracle(lib):
    L = oracle.lib()
    rng = np.random.default_rng(0)
    d = np.concatenate([-rng.exponential(5.0, 4000), -np.linspace(0, 88, 4001), [0.0, -0.0, -87.0, -87.0001]])
    for v in d.astype(np.float32):
        assert lib.pb_exp(float(v)) == L.pbo_exp(float(v)), v


def test_key_order(lib):
    vals = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf, np.nan], dtype=np.float32)
    keys = [lib.pb_key_of(float(v)) for v in vals]
    assert keys == sorted(keys)
    assert keys[3] == keys[4]  # -0 == +0
    assert keys[-1] == 0xFFFFFFFF
    assert keys == [oracle.lib().pbo_key(float(v)) for v in vals]
    assert (oracle.key_of(vals) == np.array(keys, np.uint32)).all()


def test_argument_errors(lib):
    # validated before any device work: no GPU is touched
    p = np.zeros(1, dtype=_lib.ROW_PARAMS)
    tok = np.zeros(1, np.int64)
    buf = np.zeros(8, np.float32)
    vp = lambda a: a.ctypes.data  # noqa: E731
    assert lib.pb_sample(vp(buf), 0, 1, 0, 8, None, vp(p), vp(tok), None, None, None) == -1  # vocab 0
    assert lib.pb_sample(vp(buf), 0, 1, 8, 4, None, vp(p), vp(tok), None, None, None) == -1  # stride < vocab
    assert lib.pb_sample(vp(buf), 7, 1, 8, 8, None, vp(p), vp(tok), None, None, None) == -1  # dtype
    assert lib.pb_sample(vp(buf), 0, 1, 1 << 24, 1 << 24, None, vp(p), vp(tok), None, None, None) == -2
    assert lib.pb_sample(None, 0, 1, 8, 8, None, vp(p), vp(tok), None, None, None) == -1
    assert lib.pb_sample(vp(buf), 0, 0, 8, 8, None, vp(p), vp(tok), None, None, None) == 0  # nothing to do
    assert lib.pb_strerror(-2).decode().startswith("vocabulary")
    assert lib.pb_version() >= 100


def test_launch_plan(lib, monkeypatch):
    """pb_sample_launches (host only): the streaming kernel joins in for batches with several rows
    per SM, never when probabilities are asked for; PB_PATH forces either path."""
    monkeypatch.delenv("PB_PATH", raising=False)
    sms = 148  # without a GPU the library assumes a B200's 148 SMs
    assert lib.pb_sample_launches(256, 128256, 0, 0) == 1
    assert lib.pb_sample_launches(3 * sms, 128256, 1, 0) == 2
    assert lib.pb_sample_launches(1024, 64128, 1, 1) == 1
    assert lib.pb_sample_launches(8, 49152, 7, 0) == -1
    assert lib.pb_sample_launches(0, 49152, 0, 0) == 0
    monkeypatch.setenv("PB_PATH", "stream")
    assert lib.pb_sample_launches(8, 49152, 0, 0) == 2
    monkeypatch.setenv("PB_PATH", "cluster")
    assert lib.pb_sample_launches(4096, 49152, 0, 0) == 1
