"""Next-token sampling on B200: the drop-in for ``pagedbatch/sampling.py``.

``sample_token(logits, params, generator) -> int`` keeps the reference's signature and meaning
(pagedbatch/sampling.py:10): greedy when ``params.temperature == 0``, else temperature, top-k
and top-p filtering and a draw from the request's ``torch.Generator``. ``sample_tokens`` is the
batched entry the engine calls once per step instead of looping over rows
(pagedbatch/engine.py:133-139): one kernel launch for every sampled row, whatever mix of modes.

Randomness: each non-greedy row takes ONE float64 draw, ``torch.rand((), dtype=torch.float64,
generator=g)``, from its request generator (the per-request seeded generator or the engine's
shared one, pagedbatch/engine.py:58,84), and the kernel turns it into an inverse-CDF pick over
the kept set ordered by probability (key) descending, index ascending. Same seed, same tokens;
the stream differs from ``torch.multinomial``'s, which consumes vocab-many draws per row.

With ``steps=`` the draws are made on the device instead: Philox4x32-10 keyed by each row's
64-bit seed (``seeds=``, else ``params[i].seed``) with the request's step as the counter, so a
step costs no host random numbers and a request's draw depends only on (seed, step).
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from . import _lib, ops
from .config import SamplingParams

__all__ = ["sample_token", "sample_tokens", "launch_rows", "draw_uniforms", "pack_rows"]

_INVALID_DISTRIBUTION = "probability tensor contains either `inf`, `nan` or element < 0"


def _validate(p) -> None:
    # same checks and messages as SamplingParams.__post_init__ (pagedbatch/config.py:146-155)
    if p.temperature < 0:
        raise ValueError("temperature must be >= 0")
    if not 0 < p.top_p <= 1:
        raise ValueError("top_p must be in (0, 1]")
    if p.top_k < 0:
        raise ValueError("top_k must be >= 0")


def draw_uniforms(params: Sequence, generators: Sequence[torch.Generator]) -> np.ndarray:
    """One float64 draw per non-greedy row from its generator, in row order (0 for greedy rows)."""
    u = np.zeros(len(params), dtype=np.float64)
    for i, (p, g) in enumerate(zip(params, generators, strict=True)):
        if p.temperature != 0:
            u[i] = float(torch.rand((), dtype=torch.float64, generator=g))
    return u


def pack_rows(params: Sequence, uniforms: np.ndarray, seeds=None, steps=None) -> np.ndarray:
    """pb_row_params records for the rows (device draws when ``seeds`` and ``steps`` are given)."""
    for p in params:
        _validate(p)
    return ops.pack_params(
        [float(p.temperature) for p in params],
        [float(p.top_p) for p in params],
        [int(p.top_k) for p in params],
        uniforms,
        seeds=seeds,
        steps=steps,
    )


def _upload(rec: np.ndarray, rows: np.ndarray | None, device) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Params (+ row indices) in one pinned buffer and one non-blocking H2D copy."""
    pb = rec.view(np.uint8).reshape(-1)
    if rows is None:
        host = torch.empty(pb.size, dtype=torch.uint8, pin_memory=True)
        host.numpy()[:] = pb
        dev = host.to(device, non_blocking=True)
        return ops.mark_rows(dev, rec), None
    ri = rows.astype(np.int32).view(np.uint8)
    host = torch.empty(pb.size + ri.size, dtype=torch.uint8, pin_memory=True)
    host.numpy()[: pb.size] = pb
    host.numpy()[pb.size :] = ri
    dev = host.to(device, non_blocking=True)
    return ops.mark_rows(dev[: pb.size], rec), dev[pb.size :].view(torch.int32)


def launch_rows(
    logits: torch.Tensor,
    params: Sequence,
    generators: Sequence[torch.Generator] | None,
    rows: Sequence[int] | None = None,
    *,
    steps: Sequence[int] | None = None,
    seeds: Sequence[int] | None = None,
):
    """The launch of ``sample_tokens`` without the host read: (device tokens, logits, device
    params, device row indices), or None when there is no row. Arguments as ``sample_tokens``."""
    if logits.dim() == 1:
        logits = logits.unsqueeze(0)
    if logits.dim() != 2:
        raise ValueError("logits must be [vocab] or [rows, vocab]")
    B = logits.shape[0]
    n = len(params)
    if steps is None and (generators is None or len(generators) != n):
        raise ValueError(f"{0 if generators is None else len(generators)} generators for {n} params")
    if steps is not None:
        if len(steps) != n:
            raise ValueError(f"{len(steps)} steps for {n} params")
        if seeds is None:
            if any(getattr(p, "seed", None) is None for p in params):
                raise ValueError("device draws need a seed per row: pass seeds= or set params[i].seed")
            seeds = [int(p.seed) for p in params]
        elif len(seeds) != n:
            raise ValueError(f"{len(seeds)} seeds for {n} params")
    if rows is None:
        if n != B:
            raise ValueError(f"{n} params for {B} logits rows; pass rows= to sample a subset")
        ri = None
    else:
        ri = np.asarray(rows, dtype=np.int64)
        if ri.shape != (n,) or (n and (ri.min() < 0 or ri.max() >= B)):
            raise IndexError("rows must hold one in-range logits row index per params entry")
    if n == 0:
        return None
    if not logits.is_cuda:
        if not torch.cuda.is_available():
            raise RuntimeError("pagedbatch_b200 samples on a CUDA device and none is available")
        logits = logits.to(torch.cuda.current_device(), non_blocking=logits.is_pinned())
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    if steps is None:
        rec = pack_rows(params, draw_uniforms(params, generators))
    else:
        rec = pack_rows(params, np.zeros(n), seeds=seeds, steps=steps)
    dparams, drows = _upload(rec, ri, logits.device)
    tokens, _, _ = ops._launch(logits, dparams, drows, False, False, check_rows=False)
    return tokens, logits, dparams, drows


def sample_tokens(
    logits: torch.Tensor,
    params: Sequence,
    generators: Sequence[torch.Generator] | None,
    rows: Sequence[int] | None = None,
    *,
    steps: Sequence[int] | None = None,
    seeds: Sequence[int] | None = None,
) -> list[int]:
    """Sample one token per selected row of ``logits [B, V]`` in one launch.

    ``params[i]`` / ``generators[i]`` belong to logits row ``rows[i]`` (default: row i, and then
    ``len(params) == B``). ``params`` are ``SamplingParams`` (this package's or the reference's).
    CPU logits are copied to the current CUDA device first (the kernels are the only compute path).
    With ``steps`` the draws are made on the device (see the module docstring) and ``generators``
    are not used.
    """
    got = launch_rows(logits, params, generators, rows, steps=steps, seeds=seeds)
    if got is None:
        return []
    tokens, logits, dparams, drows = got
    out = tokens.tolist()
    if any(t < 0 for t in out):
        _raise_row_errors(logits, dparams, drows)
    return out


def _raise_row_errors(logits, dparams, drows) -> None:
    _, info, _ = ops._launch(logits, dparams, drows, True, False, check_rows=False)
    rec = ops.info_records(info)
    bad = np.flatnonzero(rec["status"] != _lib.ROW_OK)
    st = int(rec["status"][bad[0]]) if bad.size else -1
    if st == _lib.ROW_NONFINITE:
        raise RuntimeError(_INVALID_DISTRIBUTION)
    raise RuntimeError(f"sampling failed on row {int(bad[0]) if bad.size else -1} (status {st})")


def sample_token(logits: torch.Tensor, params: SamplingParams, generator: torch.Generator) -> int:
    """Pick one token from a ``[vocab]`` logits row."""
    return sample_tokens(logits.reshape(1, -1), [params], [generator])[0]
