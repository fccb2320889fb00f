"""Vocabulary-parallel sampling: each rank holds a column slice of every logits row.

This is the sampling step behind a tensor-parallel LM head, where rank ``g`` of a process group
computes ``logits[:, lo_g:hi_g]`` and nobody holds whole rows. The reference samples whole rows
(pagedbatch/sampling.py:10-27, per row from pagedbatch/engine.py:133-139); the result here is the
same token, bit for bit, as ``sample_tokens`` on the full rows:

1. every rank runs the sampler in shard mode (``pb_candidates``): per row it publishes a fixed-size
   record with its top-k survivors (every value >= the shard's k-th, ties kept; scaled keys and
   global indices), or its first maximum for greedy rows;
2. one all-gather (NCCL over NVLink on GPUs) gives every rank every shard's records;
3. every rank merges (``pb_merge``): the union of the survivors holds the row's top-k set and its
   maximum, so the exact k-th key, the weights, the top-p cut and the inverse-CDF draw with the
   row's uniform give the full-row answer, identical on all ranks without a broadcast.

Rows the records cannot settle (top-k off, k at least a shard's width, or a tie group larger than
the record) come back as ``PB_ROW_FALLBACK``; their column slices are all-gathered and sampled as
full rows. All ranks take the same collective steps in the same order.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import numpy as np
import torch
import torch.distributed as dist

from . import _lib, ops
from .sampling import _INVALID_DISTRIBUTION, _upload, draw_uniforms, pack_rows

__all__ = ["sample_tokens_vocab_parallel", "record_cap", "CudaKernels"]


def record_cap(params: Sequence) -> int:
    """Entries per record: twice the largest active top_k plus a margin for ties (same on all ranks)."""
    ks = [int(p.top_k) for p in params if p.temperature != 0 and p.top_k > 0]
    k = max(ks) if ks else 1
    return int(min(_lib.CAND_MAX_CAP, max(64, 2 * k + 32)))


class CudaKernels:
    """The sm_100a library: shard candidates, merge, and full-row sampling for fallback rows."""

    def candidates(self, logits: torch.Tensor, dparams: torch.Tensor, vocab_offset: int, cap: int) -> torch.Tensor:
        if not logits.is_cuda:
            raise ValueError("vocabulary-parallel sampling needs CUDA logits")
        if logits.dim() != 2 or logits.stride(1) != 1:
            raise ValueError("logits must be a [B, V] tensor with a contiguous last dimension")
        L = _lib.load()
        B, V = logits.shape
        rec = torch.empty((B, _lib.record_bytes(cap)), dtype=torch.uint8, device=logits.device)
        code = ops._DTYPE_CODE[logits.dtype]
        with torch.cuda.device(logits.device):
            stream = torch.cuda.current_stream(logits.device).cuda_stream
            if ops._ws_path(dparams, V):
                # every row suits the two passes (see ops.group_rows): pb_candidates over a workspace
                need = L.pb_candidates_ws_bytes(B, V, code)
                ws = ops._workspace(logits.device, stream, need)
                rc = L.pb_candidates_ws(
                    ctypes.c_void_p(logits.data_ptr()), code, B, V, logits.stride(0), None,
                    ctypes.c_void_p(dparams.data_ptr()), int(vocab_offset), int(cap), ctypes.c_void_p(rec.data_ptr()),
                    ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(stream))
                _lib.check(rc, "pb_candidates_ws")
                return rec
            rc = L.pb_candidates(
                ctypes.c_void_p(logits.data_ptr()), code, B, V, logits.stride(0), None,
                ctypes.c_void_p(dparams.data_ptr()), int(vocab_offset), int(cap), ctypes.c_void_p(rec.data_ptr()),
                ctypes.c_void_p(stream))
        _lib.check(rc, "pb_candidates")
        return rec

    def merge(self, records: torch.Tensor, dparams: torch.Tensor, cap: int) -> tuple[torch.Tensor, torch.Tensor]:
        n_shards, B, _ = records.shape
        L = _lib.load()
        tokens = torch.empty(B, dtype=torch.int64, device=records.device)
        info = torch.empty((B, _lib.ROW_INFO.itemsize), dtype=torch.uint8, device=records.device)
        with torch.cuda.device(records.device):
            rc = L.pb_merge(
                ctypes.c_void_p(records.data_ptr()), n_shards, B, int(cap), ctypes.c_void_p(dparams.data_ptr()),
                ctypes.c_void_p(tokens.data_ptr()), ctypes.c_void_p(info.data_ptr()),
                ctypes.c_void_p(torch.cuda.current_stream(records.device).cuda_stream))
        _lib.check(rc, "pb_merge")
        return tokens, info

    def sample_full(self, logits: torch.Tensor, dparams: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        tokens, info, _ = ops._launch(logits, dparams, None, True, False, check_rows=False)
        return tokens, info


def _gather_cat(t: torch.Tensor, world: int, group, nccl: bool) -> torch.Tensor:
    """All-gather equally shaped tensors into one [world, *t.shape] tensor (rank order)."""
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    if nccl:
        dist.all_gather_into_tensor(out.view(world * t.shape[0], *t.shape[1:]), t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out


def sample_tokens_vocab_parallel(
    local_logits: torch.Tensor,
    params: Sequence,
    generators: Sequence[torch.Generator],
    group=None,
    kernels=None,
) -> list[int]:
    """Sample one token per row when this rank holds only columns of the rows.

    ``local_logits [B, V_rank]`` is this rank's contiguous column slice; slices follow rank order
    and may differ in width. ``params`` / ``generators`` describe all B rows and must be the same on
    every rank (replicated request state), so every rank draws the same uniforms and returns the
    same tokens. ``kernels`` defaults to the CUDA library.
    """
    kernels = kernels or CudaKernels()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    nccl = dist.get_backend(group) == "nccl"
    if local_logits.dim() != 2:
        raise ValueError("local_logits must be [rows, vocab_slice]")
    B, v_local = local_logits.shape
    if len(params) != B or len(generators) != B:
        raise ValueError(f"{len(params)} params and {len(generators)} generators for {B} rows")
    if B == 0:
        return []
    dev = local_logits.device
    widths = _gather_cat(torch.tensor([v_local], dtype=torch.int64, device=dev), world, group, nccl)
    widths = [int(w) for w in widths.view(-1).tolist()]
    offset = sum(widths[:rank])
    cap = record_cap(params)
    rec = pack_rows(params, draw_uniforms(params, generators))
    dparams = _upload(rec, None, dev)[0] if dev.type == "cuda" else torch.from_numpy(rec.view(np.uint8).copy())

    mine = kernels.candidates(local_logits, dparams, offset, cap)
    records = _gather_cat(mine, world, group, nccl)
    tokens, info = kernels.merge(records, dparams, cap)
    out = tokens.tolist()
    status = np.frombuffer(info.cpu().numpy().tobytes(), dtype=_lib.ROW_INFO)["status"].copy()

    fb = np.flatnonzero(status == _lib.ROW_FALLBACK)
    if fb.size:
        # the same rows on every rank: gather their slices (padded to the widest) into full rows
        wmax = max(widths)
        part = torch.zeros((fb.size, wmax), dtype=local_logits.dtype, device=dev)
        part[:, :v_local] = local_logits[torch.as_tensor(fb, device=dev)]
        parts = _gather_cat(part, world, group, nccl)
        full = torch.cat([parts[r, :, : widths[r]] for r in range(world)], dim=1).contiguous()
        sub = rec[fb]
        dsub = _upload(sub, None, dev)[0] if dev.type == "cuda" else torch.from_numpy(sub.view(np.uint8).copy())
        t2, info2 = kernels.sample_full(full, dsub)
        st2 = np.frombuffer(info2.cpu().numpy().tobytes(), dtype=_lib.ROW_INFO)["status"]
        t2 = t2.tolist()
        for j, r in enumerate(fb.tolist()):
            out[r] = int(t2[j])
            status[r] = st2[j]
    bad = np.flatnonzero(status != _lib.ROW_OK)
    if bad.size:
        st = int(status[bad[0]])
        if st == _lib.ROW_NONFINITE:
            raise RuntimeError(_INVALID_DISTRIBUTION)
        raise RuntimeError(f"sampling failed on row {int(bad[0])} (status {st})")
    return out
