"""Locating and driving the reference engine (pagedbatch) in tests.

The reference package is imported from ``$PAGEDBATCH_REF`` (a checkout holding ``pagedbatch/``)
or from ``baseline/_ref`` (the offline install beside this repository); tests that need it skip
when neither is there.
"""

from __future__ import annotations

import importlib
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_root() -> str | None:
    for cand in (os.environ.get("PAGEDBATCH_REF"), os.path.join(REPO, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "pagedbatch")):
            return cand
    return None


def import_reference():
    """(pagedbatch package, its engine module, where it came from) or None."""
    root = reference_root()
    if root is None:
        return None
    if root not in sys.path:
        sys.path.insert(0, root)
    pkg = importlib.import_module("pagedbatch")
    return pkg, importlib.import_module("pagedbatch.engine"), root


def build_tiny_engine(device: str, max_num_seqs: int = 8, seed: int = 0):
    """The reference's two-layer random model ('tiny', pagedbatch/config.py ModelConfig.tiny) in an
    engine on `device`."""
    from pagedbatch.config import EngineConfig
    from pagedbatch.engine import LLMEngine
    from pagedbatch.loader import load_model

    model, mcfg, tok = load_model("tiny", device=device, dtype="float32", seed=seed)
    cfg = EngineConfig(device=device, dtype="float32", max_num_seqs=max_num_seqs, max_num_batched_tokens=64,
                       num_blocks=256, block_size=16, seed=seed)
    return LLMEngine(model, mcfg, tok, cfg)


def mixed_requests(n: int = 12, vocab: int = 258):
    """Prompts (token ids) and reference SamplingParams mixing greedy, temperature-only, top-k and
    top-p rows, seeded and unseeded (the unseeded ones share the engine generator)."""
    import numpy as np
    from pagedbatch.config import SamplingParams

    rng = np.random.default_rng(7)
    reqs = []
    for i in range(n):
        prompt = rng.integers(0, 256, size=int(rng.integers(3, 40))).tolist()
        mode = i % 4
        if mode == 0:
            sp = SamplingParams(temperature=0.0, max_tokens=9, ignore_eos=True)
        elif mode == 1:
            sp = SamplingParams(temperature=0.8, max_tokens=9, seed=100 + i, ignore_eos=True)
        elif mode == 2:
            sp = SamplingParams(temperature=1.0, top_k=20, top_p=0.95, max_tokens=9, seed=200 + i, ignore_eos=True)
        else:
            sp = SamplingParams(temperature=0.7, top_p=0.9, max_tokens=9, seed=None if i % 8 == 3 else 300 + i,
                                ignore_eos=True)
        reqs.append((prompt, sp))
    return reqs


def run_to_completion(engine, reqs):
    """Every request's output token ids, by request id (ids are the request order)."""
    for i, (prompt, sp) in enumerate(reqs):
        engine.add_request(prompt_token_ids=prompt, sampling=sp, request_id=f"r{i}")
    out = {}
    steps = 0
    while engine.has_unfinished_requests:
        for o in engine.step():
            if o.finished:
                out[o.request_id] = list(o.output_token_ids)
        steps += 1
        assert steps < 10_000
    return out
