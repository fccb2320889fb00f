"""TEST INFRASTRUCTURE — the CPU oracle for pagedbatch's sampling path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
package. It holds two checkers:

* ``libpb_oracle.so`` (``pb_oracle.c``): the exact restatement of ``pagedbatch/sampling.py:10-27``
  in the arithmetic the B200 kernels implement, loaded here through ctypes;
* ``torch_port``: ``sampling.py``'s own torch operations restated row by row, used to read the
  reference's kept sets and probabilities and as the timed CPU baseline.

The structured numpy dtypes below restate ``include/pagedbatch_b200.h`` independently of the
product package, so a layout mistake on either side shows up in the tests.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpb_oracle.so")

ROW_PARAMS = np.dtype(
    [("temperature", "<f8"), ("top_p", "<f8"), ("uniform", "<f8"), ("top_k", "<i4"), ("rng", "<u4")]
)
RNG_PHILOX = 0x80000000
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
assert ROW_PARAMS.itemsize == 32 and ROW_INFO.itemsize == 40

DTYPE_CODES = {"float32": 0, "bfloat16": 1, "float16": 2}

_lib = None


def build(force: bool = False) -> str:
    """Compile pb_oracle.c with its Makefile (gcc) and return the library path."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
        os.path.join(HERE, "pb_oracle.c")
    ):
        subprocess.run(["make", "-s", "-C", HERE, "libpb_oracle.so"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.pbo_sample.argtypes = [vp, i32, i64, i64, i64, vp, vp, vp, vp, vp]
        L.pbo_sample.restype = i32
        L.pbo_exp.argtypes = [ctypes.c_float]
        L.pbo_exp.restype = ctypes.c_float
        L.pbo_key.argtypes = [ctypes.c_float]
        L.pbo_key.restype = ctypes.c_uint32
        L.pbo_key_value.argtypes = [ctypes.c_uint32]
        L.pbo_key_value.restype = ctypes.c_float
        L.pbo_philox4x32_10.argtypes = [vp, vp, vp]
        L.pbo_philox4x32_10.restype = None
        L.pbo_row_u53.argtypes = [vp, vp]
        L.pbo_row_u53.restype = i32
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def logits_as_numpy(logits) -> tuple[np.ndarray, int]:
    """A 2-D CPU tensor / array as (contiguous raw numpy array, dtype code). bf16 is kept as uint16 bits."""
    import torch

    if isinstance(logits, torch.Tensor):
        t = logits.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).numpy().view(np.uint16), 1
        if t.dtype == torch.float16:
            return t.numpy().view(np.uint16), 2
        return t.float().numpy(), 0
    a = np.ascontiguousarray(logits)
    if a.dtype == np.float16:
        return a.view(np.uint16), 2
    return a.astype(np.float32, copy=False), 0


def philox4x32_10(ctr, key) -> list[int]:
    """The oracle's Philox4x32-10 (four counter words, two key words) -> four output words."""
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    o = np.zeros(4, dtype=np.uint32)
    lib().pbo_philox4x32_10(_ptr(c), _ptr(k), _ptr(o))
    return [int(v) for v in o]


def row_u53(rec: np.ndarray) -> int | None:
    """The oracle's U53 of one pb_row_params record (None: an unusable host uniform)."""
    r = np.ascontiguousarray(np.asarray(rec, dtype=ROW_PARAMS).reshape(1))
    u = np.zeros(1, dtype=np.uint64)
    return int(u[0]) if lib().pbo_row_u53(_ptr(r), _ptr(u)) else None


def make_device_rng_params(temperature, top_p, top_k, seeds, steps) -> np.ndarray:
    """Records whose draws are made on the device: Philox keyed by each row's 64-bit seed, at `step`."""
    p = make_params(temperature, top_p, top_k, np.zeros(len(temperature)))
    p["uniform"] = np.asarray(seeds, dtype=np.uint64).view(np.float64)
    p["rng"] = RNG_PHILOX | np.asarray(steps, dtype=np.uint32)
    return p


def make_params(temperature, top_p, top_k, uniform) -> np.ndarray:
    n = len(temperature)
    p = np.zeros(n, dtype=ROW_PARAMS)
    p["temperature"] = temperature
    p["top_p"] = top_p
    p["top_k"] = top_k
    p["uniform"] = uniform
    return p


def sample(logits, params: np.ndarray, row_index=None, want_probs: bool = False):
    """Run the C oracle over a [B, V] batch. Returns (tokens int64[n], info ROW_INFO[n], probs or None)."""
    raw, code = logits_as_numpy(logits)
    assert raw.ndim == 2
    B, V = raw.shape
    ri = None if row_index is None else np.ascontiguousarray(row_index, dtype=np.int32)
    n = len(params) if ri is None else len(ri)
    params = np.ascontiguousarray(params, dtype=ROW_PARAMS)
    assert len(params) == n
    tok = np.zeros(n, dtype=np.int64)
    info = np.zeros(n, dtype=ROW_INFO)
    probs = np.zeros((n, V), dtype=np.float32) if want_probs else None
    rc = lib().pbo_sample(_ptr(raw), code, n, V, V, _ptr(ri), _ptr(params), _ptr(tok), _ptr(info), _ptr(probs))
    if rc != 0:
        raise RuntimeError(f"pbo_sample failed: {rc}")
    return tok, info, probs


def key_of(x: np.ndarray) -> np.ndarray:
    """Vectorised order-preserving key (same mapping as pbo_key): NaN on top, -0 folded onto +0."""
    x = np.asarray(x, dtype=np.float32)
    b = x.view(np.uint32).copy()
    b[x == 0] = 0
    k = np.where(b & 0x80000000, ~b, b | 0x80000000).astype(np.uint32)
    k[np.isnan(x)] = 0xFFFFFFFF
    return k


def scaled_keys(raw_f32: np.ndarray, temperature: float) -> np.ndarray:
    """fp32 logits / fp32(temperature), IEEE division (sampling.py:14)."""
    return (raw_f32.astype(np.float32) / np.float32(temperature)).astype(np.float32)


def kept_mask(raw_f32_row: np.ndarray, temperature: float, info) -> np.ndarray:
    """Kept positions of one row from its ROW_INFO: key > thr, or key == thr among the first n_tie_kept indices.

    Like the reference's ``torch.isfinite(masked)``, -inf keys never count as kept.
    """
    y = raw_f32_row.astype(np.float32) if temperature == 0 else scaled_keys(raw_f32_row, temperature)
    k = key_of(y)
    thr = np.uint32(info["thr_key"])
    keep = k > thr
    tie = np.flatnonzero(k == thr)
    keep[tie[: int(info["n_tie_kept"])]] = True
    keep &= np.isfinite(y) | np.isnan(y)
    return keep


def to_f32(raw: np.ndarray, code: int) -> np.ndarray:
    """Raw numpy logits (as returned by logits_as_numpy) upcast exactly to float32."""
    if code == 0:
        return raw.astype(np.float32, copy=False)
    if code == 1:
        return (raw.astype(np.uint32) << 16).view(np.float32)
    return raw.view(np.float16).astype(np.float32)
