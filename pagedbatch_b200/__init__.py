"""pagedbatch_b200 — B200-native (sm_100a) batched token sampling for pagedbatch.

Drop-in for ``pagedbatch.sampling.sample_token`` plus the batched ``sample_tokens`` the engine
calls once per step. The compute path is the C-ABI library ``_pb_sample.so`` built from
``csrc/`` (see ``include/pagedbatch_b200.h``); importing this package does not load it, the
first sampling call does, and fails loudly if it is missing.
"""

from .config import SamplingParams
from .sampling import draw_uniforms, pack_rows, sample_token, sample_tokens

__version__ = "0.1.0"

__all__ = ["SamplingParams", "sample_token", "sample_tokens", "draw_uniforms", "pack_rows", "__version__"]
