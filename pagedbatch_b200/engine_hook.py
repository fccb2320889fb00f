"""One sampling launch per step inside pagedbatch's own ``LLMEngine``.

The reference engine samples row by row: ``LLMEngine._postprocess`` (pagedbatch/engine.py:130-171)
calls ``sample_token(logits[i], seq.sampling, state.generator)`` (engine.py:139) for every
scheduled sequence whose ``samples_token`` is set (engine.py:136-137), through the name
``sample_token`` it imported at engine.py:17.

``install(engine)`` keeps that method and everything it does around the call (finish reasons,
detokenisation, metrics, preemption bookkeeping) and changes only where the tokens come from:

* the engine module's ``sample_token`` becomes a dispatcher. Inside a batched step it hands out
  the step's tokens in order. Anywhere else it samples the one row with
  ``pagedbatch_b200.sample_token``.
* the engine's ``_postprocess`` first samples every row of the step with one ``sample_tokens``
  launch (``rows=`` selects the logits rows, so mid-prompt prefill rows are skipped without a
  copy), then runs the original method.

Each non-greedy row draws one float64 from its request generator, in row order, as the per-row
path does. So an engine with the hook and an engine calling ``pagedbatch_b200.sample_token`` per
row produce the same tokens. ``stats`` accumulates the device-synchronised time of the batched
calls (for the sampling share of a step).

Two more things of the step move to the device with ``install`` (both optional):

* the finish-reason check of every sampled row (engine.py:173-182, ``_finish_reason``) runs as one
  launch right after the sampler (``pagedbatch_b200.finish``), and the engine's ``_finish_reason``
  hands out those results in order, so tokens and reasons come back in one host read;
* the engine's metrics gain a ``pagedbatch_sampling_seconds`` histogram (the time of each step's
  batched sampling, read-back included) in their Prometheus rendering (metrics.py:38-79).
"""

from __future__ import annotations

import hashlib
import sys
import threading
import time

import torch

from .finish import REASONS, stop_reasons
from .sampling import _raise_row_errors, launch_rows
from .sampling import sample_token as _sample_one

__all__ = ["install", "uninstall", "stats", "dispatch_sample_token"]


class _Local(threading.local):
    tokens = None  # iterator over the current batched step's tokens (None outside one)
    reasons = None  # iterator over their finish reasons, when the device computed them


_LOCAL = _Local()


class SamplingStats:
    """Batched sampling calls and the time they took (host clock around the call, which ends with
    the device-to-host read of the tokens)."""

    def __init__(self) -> None:
        self.calls = 0
        self.rows = 0
        self.seconds = 0.0

    def reset(self) -> None:
        self.calls, self.rows, self.seconds = 0, 0, 0.0


stats = SamplingStats()


def dispatch_sample_token(logits, params, generator) -> int:
    """Stands in for the engine module's ``sample_token``: the next token of the batched step in
    progress, or one row sampled on the GPU outside a batched step."""
    it = _LOCAL.tokens
    if it is None:
        return _sample_one(logits, params, generator)
    try:
        return next(it)
    except StopIteration:
        raise RuntimeError("the engine asked for more tokens than rows it marked to sample") from None


def _engine_module(engine):
    mod = sys.modules.get(type(engine).__module__)
    if mod is None or not hasattr(mod, "sample_token"):
        raise TypeError("engine does not come from a module that samples through a `sample_token` name")
    return mod


def request_seed(request_id: str, seed: int | None) -> int:
    """The 63-bit key of a request's device draws: its own seed, else one derived from its id."""
    if seed is not None:
        return int(seed) & ((1 << 63) - 1)
    return int.from_bytes(hashlib.blake2b(request_id.encode(), digest_size=8).digest(), "little") >> 1


def _read_back(tok_dev, why):
    """Tokens (and finish codes) to the host together: copies into pinned buffers, one wait."""
    if not tok_dev.is_cuda:
        return tok_dev, why
    host_tok = torch.empty(tok_dev.numel(), dtype=torch.int64, pin_memory=True)
    host_tok.copy_(tok_dev, non_blocking=True)
    host_why = None
    if why is not None:
        host_why = torch.empty(why.numel(), dtype=torch.int8, pin_memory=True)
        host_why.copy_(why, non_blocking=True)
    torch.cuda.current_stream(tok_dev.device).synchronize()
    return host_tok, host_why


# sampling takes tens of microseconds to a few milliseconds: finer buckets than the step's
SAMPLING_BUCKETS = (1e-5, 2.5e-5, 5e-5, 1e-4, 2.5e-4, 5e-4, 1e-3, 2.5e-3, 5e-3, 1e-2, 2.5e-2)


def _add_sampling_histogram(engine):
    metrics = engine.metrics
    if hasattr(metrics, "sampling_seconds"):
        return metrics.sampling_seconds
    hist = type(metrics.step_seconds)(buckets=SAMPLING_BUCKETS)
    metrics.sampling_seconds = hist
    render = metrics.render

    def render_with_sampling() -> str:
        return render() + hist.render("pagedbatch_sampling_seconds",
                                      "Batched token sampling of one step, read-back included.") + "\n"

    metrics.render = render_with_sampling
    return hist


def install(engine, device_rng: bool = False, device_stop: bool = True, histogram: bool = True) -> None:
    """Make ``engine`` sample each step in one launch (see the module docstring). With
    ``device_rng`` the draws are made on the device, keyed by (request seed, request step): the
    request's step is the number of tokens it has generated, and a request without a seed is keyed
    by its id; no host random numbers are drawn and the request generators are left untouched.
    ``device_stop`` checks finish reasons on the device; ``histogram`` adds the sampling-time
    histogram to the engine's metrics."""
    mod = _engine_module(engine)
    if getattr(engine, "_pb_batched", False):
        return
    if mod.sample_token is not dispatch_sample_token:
        mod._pb_original_sample_token = mod.sample_token
        mod.sample_token = dispatch_sample_token
    original = engine._postprocess
    original_finish = engine._finish_reason
    hist = _add_sampling_histogram(engine) if histogram else None
    eos = engine.model_config.eos_token_id
    max_len = engine.config.max_model_len

    def _postprocess(sched, logits, step_start):
        picked = [i for i, s in enumerate(sched.scheduled) if s.samples_token]
        seqs = [sched.scheduled[i].seq for i in picked]
        tokens: list[int] = []
        reasons = None
        if picked:
            t0 = time.perf_counter()
            ps = [q.sampling for q in seqs]
            if device_rng:
                got = launch_rows(logits, ps, None, rows=picked, steps=[len(q.output_token_ids) for q in seqs],
                                  seeds=[request_seed(q.request_id, q.sampling.seed) for q in seqs])
            else:
                got = launch_rows(logits, ps, [engine._requests[q.request_id].generator for q in seqs], rows=picked)
            tok_dev, logits_dev, dparams, drows = got
            why = None
            if device_stop:
                why = stop_reasons(tok_dev, [p.ignore_eos for p in ps], [len(q.output_token_ids) + 1 for q in seqs],
                                   [p.max_tokens for p in ps], [q.num_tokens + 1 for q in seqs],
                                   [tuple(p.stop_token_ids) for p in ps], eos, max_len)
            host_tok, host_why = _read_back(tok_dev, why)  # the step's one host read
            tokens = host_tok.tolist()
            if any(t < 0 for t in tokens):
                _raise_row_errors(logits_dev, dparams, drows)
            if device_stop:
                reasons = [REASONS[int(c)] for c in host_why.tolist()]
            dt = time.perf_counter() - t0
            stats.seconds += dt
            stats.calls += 1
            stats.rows += len(picked)
            if hist is not None:
                hist.observe(dt)
        _LOCAL.tokens = iter(tokens)
        _LOCAL.reasons = iter(reasons) if reasons is not None else None
        try:
            return original(sched, logits, step_start)
        finally:
            _LOCAL.tokens = None
            _LOCAL.reasons = None

    def _finish_reason(seq, token):
        it = _LOCAL.reasons
        return original_finish(seq, token) if it is None else next(it)

    engine._postprocess = _postprocess
    engine._finish_reason = _finish_reason
    engine._pb_batched = True
    engine._pb_original_postprocess = original
    engine._pb_original_finish = original_finish


def uninstall(engine) -> None:
    """Undo ``install`` on this engine (the module keeps the dispatcher, which samples per row with
    pagedbatch_b200 outside a batched step; ``restore_module`` puts the reference's function back)."""
    if getattr(engine, "_pb_batched", False):
        engine._postprocess = engine._pb_original_postprocess
        engine._finish_reason = engine._pb_original_finish
        engine._pb_batched = False


def restore_module(engine_module) -> None:
    """Put the engine module's own ``sample_token`` back."""
    orig = getattr(engine_module, "_pb_original_sample_token", None)
    if orig is not None:
        engine_module.sample_token = orig
