"""The engine drop-in on a B200: the reference's own LLMEngine (pagedbatch/engine.py) with its
'tiny' random model on CUDA, sampling through the kernels.

* one batched launch per step (pagedbatch_b200.engine_hook.install, the replacement of the per-row
  call at engine.py:139) gives the same tokens as calling pagedbatch_b200.sample_token per row;
* the same seeds give the same tokens on a second engine;
* greedy requests match the reference's own greedy sampler (sampling.py:12-13, an argmax), which
  the kernels reproduce exactly.
The reference package comes from $PAGEDBATCH_REF or baseline/_ref; the test prints which.
"""

import pytest
import torch

import ref_engine as R

pytestmark = pytest.mark.gpu
ref = R.import_reference()


@pytest.fixture
def engine_module(cuda):
    if ref is None:
        pytest.skip("reference package not found (PAGEDBATCH_REF or baseline/_ref)")
    print(f"reference engine imported from {ref[2]}")
    from pagedbatch_b200 import engine_hook

    yield ref[1], engine_hook
    engine_hook.restore_module(ref[1])


def test_batched_engine_matches_per_row_kernel_calls(engine_module):
    em, hook = engine_module
    import pagedbatch_b200

    reqs = R.mixed_requests()
    saved = em.sample_token
    em.sample_token = pagedbatch_b200.sample_token  # the level-1 drop-in: same call, per row
    try:
        per_row = R.run_to_completion(R.build_tiny_engine("cuda"), reqs)
    finally:
        em.sample_token = saved
    hook.stats.reset()
    eng = R.build_tiny_engine("cuda")
    hook.install(eng)
    batched = R.run_to_completion(eng, reqs)
    assert batched == per_row
    assert hook.stats.calls > 0 and hook.stats.rows == sum(len(v) for v in batched.values())


def test_same_seed_same_tokens_and_greedy_matches_reference(engine_module):
    em, hook = engine_module
    reqs = [(p, sp) for p, sp in R.mixed_requests() if sp.seed is not None or sp.temperature == 0]
    outs = []
    for _ in range(2):
        eng = R.build_tiny_engine("cuda")
        hook.install(eng)
        outs.append(R.run_to_completion(eng, reqs))
    assert outs[0] == outs[1]
    # greedy requests alone, the reference's own sampler against the hooked engine
    greedy = [(p, sp) for p, sp in reqs if sp.temperature == 0]
    hook.restore_module(em)  # the reference's own sample_token (sampling.py:10-27)
    theirs = R.run_to_completion(R.build_tiny_engine("cuda"), greedy)
    eng = R.build_tiny_engine("cuda")
    hook.install(eng)  # (puts the dispatcher back)
    ours = R.run_to_completion(eng, greedy)
    assert ours == theirs
    assert torch.cuda.is_available()
