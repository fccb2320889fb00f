"""The engine drop-in (pagedbatch_b200.engine_hook) inside the reference's own LLMEngine.

CPU part: the hook's plumbing with the sampler replaced by a CPU stand-in that follows the same
draw discipline (one float64 from the row's generator for each non-greedy row, in row order). An
engine with the hook (one batched call per step) and an engine calling the stand-in per row
(pagedbatch/engine.py:139) must produce the same tokens for every request, through the
reference's own scheduling, finish-reason and detokenisation code (engine.py:130-182).

GPU part (tests/test_engine_gpu.py) runs the real kernels.
"""

import numpy as np
import pytest
import torch

import ref_engine as R

ref = R.import_reference()
pytestmark = pytest.mark.skipif(ref is None, reason="reference package not found (PAGEDBATCH_REF or baseline/_ref)")


def _stand_in_row(logits, params, generator):
    """One row: greedy argmax, else one float64 draw mapped onto the vocabulary (a stand-in rule)."""
    x = logits.float().reshape(-1)
    if params.temperature == 0:
        return int(torch.argmax(x))
    u = float(torch.rand((), dtype=torch.float64, generator=generator))
    return min(int(u * x.numel()), x.numel() - 1)


def _stand_in_launch(logits, params, generators, rows=None, *, steps=None, seeds=None):
    rows = range(logits.shape[0]) if rows is None else rows
    toks = [_stand_in_row(logits[r], p, g) for r, p, g in zip(rows, params, generators, strict=True)]
    return torch.tensor(toks, dtype=torch.int64), logits, None, None


def _stand_in_stop(tokens, ignore_eos, out_lens, max_tokens, total_lens, stop_ids, eos, max_model_len):
    """The finish rule of pagedbatch/engine.py:173-182 per row (0 none, 1 stop, 2 length)."""
    out = []
    for t, ig, ol, mt, tl, st in zip(tokens.tolist(), ignore_eos, out_lens, max_tokens, total_lens, stop_ids,
                                     strict=True):
        if not ig and ((eos is not None and t == eos) or t in st):
            out.append(1)
        elif ol >= mt or tl >= max_model_len:
            out.append(2)
        else:
            out.append(0)
    return torch.tensor(out, dtype=torch.int8)


@pytest.fixture
def stand_in(monkeypatch):
    from pagedbatch_b200 import engine_hook

    monkeypatch.setattr(engine_hook, "launch_rows", _stand_in_launch)
    monkeypatch.setattr(engine_hook, "stop_reasons", _stand_in_stop)
    monkeypatch.setattr(engine_hook, "_sample_one", _stand_in_row)
    yield engine_hook
    engine_hook.restore_module(ref[1])


def test_batched_step_matches_per_row_calls(stand_in):
    hook = stand_in
    reqs = R.mixed_requests()
    # per row: the engine module's sample_token is the stand-in, called once per sampled row
    em = ref[1]
    saved = em.sample_token
    em.sample_token = _stand_in_row
    try:
        per_row = R.run_to_completion(R.build_tiny_engine("cpu"), reqs)
    finally:
        em.sample_token = saved
    # batched: one call per step through the hook
    hook.stats.reset()
    eng = R.build_tiny_engine("cpu")
    hook.install(eng)
    batched = R.run_to_completion(eng, reqs)
    assert batched == per_row
    assert hook.stats.calls > 0 and hook.stats.rows == sum(len(v) for v in batched.values())
    # an engine without the hook still works (the module's dispatcher samples per row)
    plain = R.run_to_completion(R.build_tiny_engine("cpu"), reqs)
    assert plain == per_row


def test_same_seed_same_tokens(stand_in):
    hook = stand_in
    reqs = [(p, sp) for p, sp in R.mixed_requests() if sp.seed is not None or sp.temperature == 0]
    outs = []
    for _ in range(2):
        eng = R.build_tiny_engine("cpu")
        hook.install(eng)
        outs.append(R.run_to_completion(eng, reqs))
    assert outs[0] == outs[1]
    assert all(len(v) == 9 for v in outs[0].values())


def test_dispatcher_refuses_extra_tokens(stand_in):
    hook = stand_in
    hook._LOCAL.tokens = iter([1])
    try:
        assert hook.dispatch_sample_token(None, None, None) == 1
        with pytest.raises(RuntimeError, match="more tokens"):
            hook.dispatch_sample_token(None, None, None)
    finally:
        hook._LOCAL.tokens = None


def test_finish_reasons_and_histogram(stand_in):
    """Finish reasons served from the (stand-in) device check equal the engine's own: requests that
    stop on a stop id or EOS, and ones that hit max_tokens; the sampling histogram is rendered."""
    from pagedbatch.config import SamplingParams

    hook = stand_in
    reqs = [([5, 6, 7], SamplingParams(temperature=0.0, max_tokens=4)),
            ([9, 9], SamplingParams(temperature=0.0, max_tokens=50, stop_token_ids=tuple(range(258)))),
            ([1, 2, 3, 4], SamplingParams(temperature=0.9, max_tokens=6, seed=3, stop_token_ids=(11, 12))),
            ([3], SamplingParams(temperature=0.0, max_tokens=7, ignore_eos=True))]

    def finals(eng):
        for i, (p, sp) in enumerate(reqs):
            eng.add_request(prompt_token_ids=p, sampling=sp, request_id=f"q{i}")
        out = {}
        while eng.has_unfinished_requests:
            for o in eng.step():
                if o.finished:
                    out[o.request_id] = (o.finish_reason, list(o.output_token_ids))
        return out

    em = ref[1]
    saved = em.sample_token
    em.sample_token = _stand_in_row  # the same per-row sampler, with the engine's own finish check
    try:
        plain = finals(R.build_tiny_engine("cpu"))
    finally:
        em.sample_token = saved
    eng = R.build_tiny_engine("cpu")
    hook.install(eng)
    batched = finals(eng)
    assert batched == plain
    assert batched["q1"][0] == "stop" and batched["q0"][0] == "length"
    text = eng.metrics.render()
    assert "pagedbatch_sampling_seconds_count" in text and "pagedbatch_step_seconds_count" in text
    assert eng.metrics.sampling_seconds.count > 0
