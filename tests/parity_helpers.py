"""Shared GPU-parity helpers: run a batch through the C ABI and compare with the CPU oracle."""

import os

import numpy as np
import torch

import oracle
from pagedbatch_b200 import ops

INFO_FIELDS = ("thr_key", "n_tie_kept", "kept_count", "status", "z_q", "kept_q")


def run_gpu(logits_dev, rec, row_index=None, probs=True):
    params = ops.params_tensor(rec, logits_dev.device)
    ri = None if row_index is None else torch.as_tensor(np.asarray(row_index, np.int32), device=logits_dev.device)
    tok, info, pr = ops.sample(logits_dev, params, ri, with_info=True, with_probs=probs)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), ops.info_records(info), (pr.cpu().numpy() if probs else None)


def _check(g_tok, g_info, o_tok, o_info, label):
    bad = np.flatnonzero(g_tok != o_tok)
    assert bad.size == 0, f"{label}: tokens differ at rows {bad[:10]}: gpu {g_tok[bad[:10]]} oracle {o_tok[bad[:10]]}"
    for f in INFO_FIELDS:
        d = np.flatnonzero(g_info[f] != o_info[f])
        assert d.size == 0, f"{label}: info.{f} differs at rows {d[:10]}: gpu {g_info[f][d[:10]]} oracle {o_info[f][d[:10]]}"
    assert np.array_equal(g_info["max_key"], o_info["max_key"], equal_nan=True), label


def _run_with_path(dev, rec, row_index, path, ws=None):
    """Tokens and info through one launch path (PB_PATH as the ops layer and the library read it;
    PB_WS=balanced makes pb_sample_ws take its balanced streaming launch)."""
    saved = {k: os.environ.get(k) for k in ("PB_PATH", "PB_WS")}
    os.environ["PB_PATH"] = path
    if ws is None:
        os.environ.pop("PB_WS", None)
    else:
        os.environ["PB_WS"] = ws
    try:
        return run_gpu(dev, rec, row_index, False)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def padded(logits_cpu, pad_to, device="cuda"):
    """The logits on the device with a row stride of pad_to elements (rows padded with NaN)."""
    B, V = logits_cpu.shape
    buf = torch.full((B, pad_to), float("nan"), dtype=logits_cpu.dtype, device=device)
    view = buf[:, :V]
    view.copy_(logits_cpu)
    return view


def compare(logits_cpu, rec, row_index=None, probs=True, device="cuda", label="", pad_to=None):
    """GPU against the oracle. With probs: the launch that writes probabilities (the cluster kernel
    alone), then the same rows without probabilities through pb_sample's streaming kernel (whole
    rows per CTA) and through both launches of pb_sample_ws (the two passes over 128-byte group
    keys when rows are 16-byte aligned; the balanced streaming launch, rows cut into pieces), each
    followed by the cluster kernel on the rows it leaves. Without probs: the path PB_PATH and PB_WS
    select. pad_to: the rows pass with that stride (in elements)."""
    dev = logits_cpu.to(device) if pad_to is None else padded(logits_cpu, pad_to, device)
    g_tok, g_info, g_pr = run_gpu(dev, rec, row_index, probs)
    o_tok, o_info, o_pr = oracle.sample(logits_cpu, rec, row_index, want_probs=probs)
    _check(g_tok, g_info, o_tok, o_info, label)
    if probs:
        ok = g_info["status"] == 0
        same = g_pr[ok].view(np.uint32) == o_pr[ok].view(np.uint32)
        rows_bad = np.flatnonzero(~same.all(axis=1))
        assert rows_bad.size == 0, f"{label}: probs differ on rows {rows_bad[:10]}"
        for path, ws in (("stream", None), ("ws", None), ("ws", "balanced")):
            s_tok, s_info, _ = _run_with_path(dev, rec, row_index, path, ws)
            _check(s_tok, s_info, o_tok, o_info, f"{label} ({path} path{', ' + ws if ws else ''})")
    return g_tok, g_info


def rec_for(params, uniforms):
    return oracle.make_params(
        [p.temperature for p in params], [p.top_p for p in params], [p.top_k for p in params], uniforms
    )


