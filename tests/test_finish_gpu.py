"""pb_stop_check on a B200 against the reference's own finish rule.

Random rows (tokens, EOS, stop ids, ignore_eos, lengths near max_tokens and max_model_len) go
through ``pagedbatch_b200.finish.stop_reasons``; each row's reason must equal what
``LLMEngine._finish_reason`` (pagedbatch/engine.py:173-182) returns for the same sequence and token.
"""

import types

import numpy as np
import pytest
import torch

import ref_engine as R
from pagedbatch_b200.finish import REASONS, stop_reasons

pytestmark = pytest.mark.gpu
ref = R.import_reference()


def test_stop_reasons_match_the_reference(cuda):
    if ref is None:
        pytest.skip("reference package not found (PAGEDBATCH_REF or baseline/_ref)")
    from pagedbatch.config import SamplingParams
    from pagedbatch.engine import LLMEngine
    from pagedbatch.sequence import Sequence

    rng = np.random.default_rng(4)
    n, eos, max_model_len = 5000, 257, 300
    toks, seqs = [], []
    for i in range(n):
        prompt = [1] * int(rng.integers(1, 200))
        max_tokens = int(rng.integers(1, 120))
        out_len = int(rng.integers(0, max_tokens + 3))
        stops = tuple(int(t) for t in rng.integers(0, 300, int(rng.integers(0, 4))))
        sp = SamplingParams(max_tokens=max_tokens, ignore_eos=bool(rng.random() < 0.3), stop_token_ids=stops)
        seq = Sequence(request_id=f"s{i}", prompt_token_ids=prompt, sampling=sp)
        seq.output_token_ids = [7] * out_len
        tok = int(rng.choice([eos, *stops, int(rng.integers(0, 300))])) if rng.random() < 0.5 else int(rng.integers(0, 300))
        seq.output_token_ids.append(tok)  # as the engine does before it asks
        toks.append(tok)
        seqs.append(seq)
    me = types.SimpleNamespace(model_config=types.SimpleNamespace(eos_token_id=eos),
                               config=types.SimpleNamespace(max_model_len=max_model_len))
    want = [LLMEngine._finish_reason(me, s, t) for s, t in zip(seqs, toks)]
    got_dev = stop_reasons(torch.tensor(toks, dtype=torch.int64, device=cuda),
                           [s.sampling.ignore_eos for s in seqs], [len(s.output_token_ids) for s in seqs],
                           [s.sampling.max_tokens for s in seqs], [s.num_tokens for s in seqs],
                           [s.sampling.stop_token_ids for s in seqs], eos, max_model_len)
    got = [REASONS[int(c)] for c in got_dev.cpu().tolist()]
    assert got == want
    assert {"stop", "length", None} <= set(want)
