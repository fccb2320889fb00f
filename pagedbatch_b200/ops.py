"""The ``pagedbatch_b200::sample`` custom op: torch tensors in, one C-ABI launch, tensors out.

``sample(logits, params, row_index=None, with_info=False, with_probs=False)``

* ``logits``: CUDA tensor ``[B, V]`` (float32 / bfloat16 / float16), last dim contiguous;
* ``params``: CUDA ``uint8`` tensor holding ``n`` packed ``pb_row_params`` records (``pack_params``);
* ``row_index``: optional CUDA ``int32[n]`` selecting the logits row of each work item.

Returns ``tokens int64[n]`` (``-1`` where a row failed), plus ``info uint8[n, 40]``
(``pb_row_info`` records) and ``probs float32[n, V]`` when asked for. The launch goes on the
current CUDA stream of the logits' device, with no synchronisation.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from . import _lib

_DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def pack_params(temperature, top_p, top_k, uniform, seeds=None, steps=None) -> np.ndarray:
    """Per-row parameter records (struct pb_row_params) as a numpy structured array.

    With ``seeds`` and ``steps`` the rows' draws are made on the device (Philox keyed by the
    64-bit seed at that step, ``PB_RNG_PHILOX``) and ``uniform`` is ignored."""
    n = len(temperature)
    rec = np.zeros(n, dtype=_lib.ROW_PARAMS)
    rec["temperature"] = temperature
    rec["top_p"] = top_p
    # any top_k at or above the vocabulary switches the filter off (sampling.py:15), so values past
    # the int32 field saturate instead of failing
    rec["top_k"] = np.minimum(np.asarray(top_k, dtype=np.int64), np.iinfo(np.int32).max)
    if seeds is None:
        rec["uniform"] = uniform
    else:
        st = np.asarray(steps, dtype=np.int64)
        if st.shape != (n,) or (n and (st.min() < 0 or st.max() >= 1 << 31)):
            raise ValueError("steps must hold one value in [0, 2^31) per row")
        rec["uniform"] = (np.asarray(seeds, dtype=np.int64).astype(np.uint64)).view(np.float64)
        rec["rng"] = _lib.RNG_PHILOX | st.astype(np.uint32)
    return rec


GROUP_KMAX = 128  # largest top_k the two-pass launch of pb_sample_ws settles


def group_rows(rec: np.ndarray) -> tuple[bool, int]:
    """Whether every row is one the two-pass launch of pb_sample_ws settles itself (valid parameters,
    greedy or 0 < top_k <= 128, a usable draw), and the largest top_k among them (which must also
    stay below the vocabulary). Rows of other kinds go to the cluster kernel after both passes, so
    a batch holding them runs faster through pb_sample."""
    if rec.size == 0:
        return False, 0
    t, p, k = rec["temperature"], rec["top_p"], rec["top_k"]
    valid = (t >= 0.0) & (p > 0.0) & (p <= 1.0) & (k >= 0)
    greedy = t == 0.0
    draw = ((rec["rng"] & _lib.RNG_PHILOX) != 0) | ((rec["uniform"] >= 0.0) & (rec["uniform"] < 1.0))
    small = (k > 0) & (k <= GROUP_KMAX) & draw
    ok = bool(np.all(valid & (greedy | small)))
    kmax = int(k[~greedy].max()) if np.any(~greedy) else 0
    return ok, kmax


def mark_rows(params: torch.Tensor, rec: np.ndarray) -> torch.Tensor:
    """Record on the device params tensor which launch suits its rows (read by the path choice)."""
    params._pb_group_rows = group_rows(rec)
    return params


def params_tensor(rec: np.ndarray, device, pinned: bool = True) -> torch.Tensor:
    """Upload packed records: one pinned host buffer, one non-blocking H2D copy."""
    host = torch.from_numpy(rec.view(np.uint8).copy())
    if pinned:
        host = host.pin_memory()
    return mark_rows(host.to(device, non_blocking=True), rec)


_WS: dict = {}


def _ws_path(params: torch.Tensor | None = None, vocab: int = 0) -> bool:
    """Whether tokens without probabilities go through pb_sample_ws (over a workspace) rather than
    pb_sample. PB_PATH=ws / full (or cluster, stream: pb_sample's own choices) force one. By default
    pb_sample_ws runs when the params tensor's rows all suit its two-pass launch (see group_rows;
    measured on B200: [256, 128256] fp32 top-k rows 38 us against 41 us, [1024, 128256] bf16 85 us
    against 100 us), and pb_sample otherwise (a batch with temperature-only or top-p-only rows: 137
    us against 169 us)."""
    env = os.environ.get("PB_PATH", "auto")
    if env != "auto":
        return env == "ws"
    ok, kmax = getattr(params, "_pb_group_rows", (False, 0))
    return ok and kmax < vocab


def _workspace(dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Scratch for pb_sample_ws, one buffer per (device, stream), grown on demand (torch allocations
    are 256-byte aligned; the launches need no cleared memory). Calls on one stream are ordered, so
    they share its buffer; calls on different streams get different buffers."""
    if nbytes < 0:
        raise ValueError("bad workspace request")
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WS[key] = ws
    return ws


def _launch(logits: torch.Tensor, params: torch.Tensor, row_index, with_info: bool, with_probs: bool,
            check_rows: bool = True):
    if not logits.is_cuda:
        raise ValueError("pagedbatch_b200.sample needs CUDA logits; move the tensor with .cuda() first")
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a [B, V] tensor with a contiguous last dimension")
    if logits.dtype not in _DTYPE_CODE:
        raise ValueError(f"unsupported logits dtype {logits.dtype}")
    if params.dtype != torch.uint8 or params.numel() % _lib.ROW_PARAMS.itemsize:
        raise ValueError("params must be packed pb_row_params records (uint8)")
    n = params.numel() // _lib.ROW_PARAMS.itemsize
    B, V = logits.shape
    if row_index is not None:
        if row_index.dtype != torch.int32 or row_index.numel() != n or not row_index.is_cuda:
            raise ValueError("row_index must be a CUDA int32 tensor with one entry per params record")
        if check_rows and n and (int(row_index.min()) < 0 or int(row_index.max()) >= B):
            raise IndexError("row_index out of range")
    elif n != B:
        raise ValueError(f"{n} params records for {B} logits rows")
    dev = logits.device
    tokens = torch.empty(n, dtype=torch.int64, device=dev)
    info = torch.empty((n, _lib.ROW_INFO.itemsize), dtype=torch.uint8, device=dev) if with_info else None
    probs = torch.empty((n, V), dtype=torch.float32, device=dev) if with_probs else None
    L = _lib.load()
    if not with_probs and _ws_path(params, V):
        with torch.cuda.device(dev):
            need = L.pb_sample_ws_bytes(n, V, _DTYPE_CODE[logits.dtype])
            stream = torch.cuda.current_stream(dev).cuda_stream
            ws = _workspace(dev, stream, need)
            rc = L.pb_sample_ws(
                ctypes.c_void_p(logits.data_ptr()), _DTYPE_CODE[logits.dtype], n, V, logits.stride(0),
                ctypes.c_void_p(row_index.data_ptr()) if row_index is not None else None,
                ctypes.c_void_p(params.data_ptr()), ctypes.c_void_p(tokens.data_ptr()),
                ctypes.c_void_p(info.data_ptr()) if info is not None else None, None,
                ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(stream))
        _lib.check(rc, "pb_sample_ws")
        return tokens, info, probs
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = L.pb_sample(
            ctypes.c_void_p(logits.data_ptr()),
            _DTYPE_CODE[logits.dtype],
            n,
            V,
            logits.stride(0),
            ctypes.c_void_p(row_index.data_ptr()) if row_index is not None else None,
            ctypes.c_void_p(params.data_ptr()),
            ctypes.c_void_p(tokens.data_ptr()),
            ctypes.c_void_p(info.data_ptr()) if info is not None else None,
            ctypes.c_void_p(probs.data_ptr()) if probs is not None else None,
            ctypes.c_void_p(stream),
        )
    _lib.check(rc, "pb_sample")
    return tokens, info, probs


@torch.library.custom_op("pagedbatch_b200::sample", mutates_args=())
def sample_op(logits: torch.Tensor, params: torch.Tensor, row_index: torch.Tensor | None = None) -> torch.Tensor:
    """Tokens only (the engine's path)."""
    tokens, _, _ = _launch(logits, params, row_index, False, False)
    return tokens


@sample_op.register_fake
def _(logits, params, row_index=None):
    n = params.numel() // _lib.ROW_PARAMS.itemsize
    return logits.new_empty((n,), dtype=torch.int64)


def sample(logits: torch.Tensor, params: torch.Tensor, row_index=None, with_info: bool = False,
           with_probs: bool = False):
    """Tokens, and optionally the per-row info records and the final probabilities."""
    if not with_info and not with_probs:
        return sample_op(logits, params, row_index)
    return _launch(logits, params, row_index, with_info, with_probs)


def info_records(info: torch.Tensor) -> np.ndarray:
    """Device ``uint8[n, 40]`` info -> numpy structured ``pb_row_info`` records."""
    return info.cpu().numpy().reshape(-1).view(_lib.ROW_INFO)
