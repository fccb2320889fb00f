"""ctypes binding of the C ABI in ``include/pagedbatch_b200.h`` (library ``_pb_sample.so``).

The library is the product's only compute path. Loading fails loudly when it is missing or was
built without the expected symbols; there is no CPU fallback anywhere in this package.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "_pb_sample.so")

PB_DTYPE = {"float32": 0, "bfloat16": 1, "float16": 2}
PB_OK = 0
ERRORS = {-1: "invalid argument", -2: "vocabulary too large", -3: "kernel launch failed", -4: "device configuration failed",
          -5: "batch too large for the fixed scratch of pb_sample_noalloc"}

ROW_OK, ROW_NONFINITE, ROW_BAD_UNIFORM, ROW_TIMEOUT, ROW_INTERNAL, ROW_BAD_PARAMS = 0, 1, 2, 4, 8, 16
ROW_FALLBACK = 32
CAND_FALLBACK, CAND_GREEDY, CAND_MAX_CAP = 0x100, 0x200, 2048
PATH_GREEDY, PATH_SMALL, PATH_LARGE, PATH_STREAM = 1, 2, 4, 8
FINISH_NONE, FINISH_STOP, FINISH_LENGTH = 0, 1, 2
MAX_VOCAB = 1 << 24

# struct pb_row_params / pb_row_info (include/pagedbatch_b200.h)
ROW_PARAMS = np.dtype(
    [("temperature", "<f8"), ("top_p", "<f8"), ("uniform", "<f8"), ("top_k", "<i4"), ("rng", "<u4")]
)
RNG_PHILOX = 0x80000000  # pb_row_params.rng: the draw is made on the device (Philox, seed and step)
ROW_INFO = np.dtype(
    [
        ("thr_key", "<u4"),
        ("n_tie_kept", "<i4"),
        ("kept_count", "<i4"),
        ("status", "<i4"),
        ("max_key", "<f4"),
        ("flags", "<i4"),
        ("z_q", "<u8"),
        ("kept_q", "<u8"),
    ]
)
# struct pb_cand_header (a vocabulary-parallel record starts with it; uint64 entries follow)
CAND_HEADER = np.dtype([("count", "<i4"), ("flags", "<i4"), ("max_key", "<f4"), ("reserved", "<i4")])
assert ROW_PARAMS.itemsize == 32 and ROW_INFO.itemsize == 40 and CAND_HEADER.itemsize == 16


def record_bytes(cap: int) -> int:
    """Bytes of one row's candidate record (pb_record_bytes)."""
    return CAND_HEADER.itemsize + 8 * int(cap)

EXPORTS = (
    "pb_sample",
    "pb_sample_ws",
    "pb_sample_ws_bytes",
    "pb_sample_ws_launches",
    "pb_candidates_ws",
    "pb_candidates_ws_bytes",
    "pb_sample_noalloc",
    "pb_sample_noalloc_max_bytes",
    "pb_candidates",
    "pb_merge",
    "pb_record_bytes",
    "pb_sample_launches",
    "pb_key_of",
    "pb_exp",
    "pb_philox_u53",
    "pb_stop_check",
    "pb_philox4x32_10",
    "pb_strerror",
    "pb_version",
)

_lib: ctypes.CDLL | None = None


class SamplerUnavailable(RuntimeError):
    """The compiled sm_100a library is missing or unusable."""


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once (import torch first so the shared CUDA runtime is torch's)."""
    global _lib
    if _lib is not None:
        return _lib
    import torch  # noqa: F401  (loads libcudart before the library resolves it)

    if not os.path.exists(path):
        raise SamplerUnavailable(
            f"{path} is missing: build it with `python -m pagedbatch_b200.build` (nvcc, sm_100a)"
        )
    L = ctypes.CDLL(path)
    for name in EXPORTS:
        if not hasattr(L, name):
            raise SamplerUnavailable(f"{path} does not export {name}")
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.pb_sample.argtypes = [vp, i32, i64, i64, i64, vp, vp, vp, vp, vp, vp]
    L.pb_sample.restype = i32
    L.pb_sample_ws.argtypes = [vp, i32, i64, i64, i64, vp, vp, vp, vp, vp, vp, i64, vp]
    L.pb_sample_ws.restype = i32
    L.pb_sample_noalloc.argtypes = [vp, i32, i64, i64, i64, vp, vp, vp, vp, vp]
    L.pb_sample_noalloc.restype = i32
    L.pb_sample_noalloc_max_bytes.argtypes = []
    L.pb_sample_noalloc_max_bytes.restype = i64
    L.pb_sample_ws_bytes.argtypes = [i64, i64, i32]
    L.pb_sample_ws_bytes.restype = i64
    L.pb_sample_ws_launches.argtypes = [vp, i64, i64, i64, i32]
    L.pb_sample_ws_launches.restype = i32
    L.pb_candidates_ws.argtypes = [vp, i32, i64, i64, i64, vp, vp, i64, i32, vp, vp, i64, vp]
    L.pb_candidates_ws.restype = i32
    L.pb_candidates_ws_bytes.argtypes = [i64, i64, i32]
    L.pb_candidates_ws_bytes.restype = i64
    L.pb_candidates.argtypes = [vp, i32, i64, i64, i64, vp, vp, i64, i32, vp, vp]
    L.pb_candidates.restype = i32
    L.pb_merge.argtypes = [vp, i32, i64, i32, vp, vp, vp, vp]
    L.pb_merge.restype = i32
    L.pb_sample_launches.argtypes = [i64, i64, i32, i32]
    L.pb_sample_launches.restype = i32
    L.pb_record_bytes.argtypes = [i32]
    L.pb_record_bytes.restype = i64
    L.pb_key_of.argtypes = [ctypes.c_float]
    L.pb_key_of.restype = ctypes.c_uint32
    L.pb_exp.argtypes = [ctypes.c_float]
    L.pb_exp.restype = ctypes.c_float
    L.pb_stop_check.argtypes = [vp, i64, vp, vp, vp, i32, i32, vp, vp]
    L.pb_stop_check.restype = i32
    L.pb_philox_u53.argtypes = [ctypes.c_uint64, ctypes.c_uint32]
    L.pb_philox_u53.restype = ctypes.c_uint64
    L.pb_philox4x32_10.argtypes = [vp, vp, vp]
    L.pb_philox4x32_10.restype = None
    L.pb_strerror.argtypes = [i32]
    L.pb_strerror.restype = ctypes.c_char_p
    L.pb_version.argtypes = []
    L.pb_version.restype = i32
    _lib = L
    return L


def check(rc: int, what: str) -> None:
    if rc != PB_OK:
        msg = load().pb_strerror(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} ({rc})")
