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
"""

from __future__ import annotations

import sys
import threading
import time

from .sampling import sample_token as _sample_one
from .sampling import sample_tokens

__all__ = ["install", "uninstall", "stats", "dispatch_sample_token"]


class _Local(threading.local):
    tokens = None  # iterator over the current batched step's tokens (None outside one)


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


def install(engine) -> None:
    """Make ``engine`` sample each step in one launch (see the module docstring)."""
    mod = _engine_module(engine)
    if getattr(engine, "_pb_batched", False):
        return
    if mod.sample_token is not dispatch_sample_token:
        mod._pb_original_sample_token = mod.sample_token
        mod.sample_token = dispatch_sample_token
    original = engine._postprocess

    def _postprocess(sched, logits, step_start):
        picked = [i for i, s in enumerate(sched.scheduled) if s.samples_token]
        seqs = [sched.scheduled[i].seq for i in picked]
        tokens: list[int] = []
        if picked:
            t0 = time.perf_counter()
            tokens = sample_tokens(logits, [q.sampling for q in seqs],
                                   [engine._requests[q.request_id].generator for q in seqs], rows=picked)
            stats.seconds += time.perf_counter() - t0
            stats.calls += 1
            stats.rows += len(picked)
        _LOCAL.tokens = iter(tokens)
        try:
            return original(sched, logits, step_start)
        finally:
            _LOCAL.tokens = None

    engine._postprocess = _postprocess
    engine._pb_batched = True
    engine._pb_original_postprocess = original


def uninstall(engine) -> None:
    """Undo ``install`` on this engine (the module keeps the dispatcher, which samples per row with
    pagedbatch_b200 outside a batched step; ``restore_module`` puts the reference's function back)."""
    if getattr(engine, "_pb_batched", False):
        engine._postprocess = engine._pb_original_postprocess
        engine._pb_batched = False


def restore_module(engine_module) -> None:
    """Put the engine module's own ``sample_token`` back."""
    orig = getattr(engine_module, "_pb_original_sample_token", None)
    if orig is not None:
        engine_module.sample_token = orig
