"""Finish reasons on the device: the per-row check of pagedbatch/engine.py:173-182.

``LLMEngine._finish_reason`` decides, after a request's token is appended, whether it stops (the
end-of-sequence id or one of its stop ids, unless it ignores EOS) or hits a length limit (its
``max_tokens``, or the engine's ``max_model_len``). ``stop_reasons`` runs that check for every
sampled row in one launch right after the sampler (``pb_stop_check``), on the tokens still on the
device, so the engine reads tokens and reasons back together.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import numpy as np
import torch

from . import _lib

__all__ = ["stop_reasons", "REASONS"]

REASONS = {_lib.FINISH_NONE: None, _lib.FINISH_STOP: "stop", _lib.FINISH_LENGTH: "length"}


def stop_reasons(tokens: torch.Tensor, ignore_eos: Sequence[bool], out_lens: Sequence[int],
                 max_tokens: Sequence[int], total_lens: Sequence[int], stop_ids: Sequence[Sequence[int]],
                 eos_id: int | None, max_model_len: int) -> torch.Tensor:
    """Device int8[n] finish codes (0 none, 1 stop, 2 length) for the sampled ``tokens`` (device
    int64[n]). Per row: whether it ignores EOS, its output length and total length counting the
    new token, its max_tokens and its stop ids. Launched on the tokens' current stream."""
    n = tokens.numel()
    if not tokens.is_cuda or tokens.dtype != torch.int64:
        raise ValueError("tokens must be a CUDA int64 tensor")
    if not (len(ignore_eos) == len(out_lens) == len(max_tokens) == len(total_lens) == len(stop_ids) == n):
        raise ValueError("one entry per row is needed in every per-row argument")
    counts = np.fromiter((len(s) for s in stop_ids), dtype=np.int64, count=n)
    total_ids = int(counts.sum())
    # one pinned buffer: row state (16-byte aligned), stop offsets, stop ids
    state = np.zeros((n, 4), dtype=np.int32)
    state[:, 0] = np.asarray(ignore_eos, dtype=bool)
    state[:, 1] = out_lens
    state[:, 2] = max_tokens
    state[:, 3] = total_lens
    offs = np.zeros(n + 1, dtype=np.int32)
    np.cumsum(counts, out=offs[1:])
    ids = np.fromiter((int(t) for s in stop_ids for t in s), dtype=np.int32, count=total_ids)
    nbytes = state.nbytes + offs.nbytes + ids.nbytes
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    h = host.numpy()
    h[: state.nbytes] = state.view(np.uint8).reshape(-1)
    h[state.nbytes : state.nbytes + offs.nbytes] = offs.view(np.uint8)
    h[state.nbytes + offs.nbytes :] = ids.view(np.uint8)
    dev = host.to(tokens.device, non_blocking=True)
    out = torch.empty(n, dtype=torch.int8, device=tokens.device)
    L = _lib.load()
    base = dev.data_ptr()
    with torch.cuda.device(tokens.device):
        rc = L.pb_stop_check(
            ctypes.c_void_p(tokens.data_ptr()), n, ctypes.c_void_p(base), ctypes.c_void_p(base + state.nbytes),
            ctypes.c_void_p(base + state.nbytes + offs.nbytes) if total_ids else ctypes.c_void_p(base),
            -1 if eos_id is None else int(eos_id), int(max_model_len), ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream(tokens.device).cuda_stream))
    _lib.check(rc, "pb_stop_check")
    return out
