"""Per-request sampling parameters — the same dataclass as pagedbatch/config.py:134-158.

Field names, defaults, validation messages and the ``greedy`` property are kept identical so
that code written against ``pagedbatch.config.SamplingParams`` (the engine, the HTTP server's
``CompletionRequest.sampling()`` at pagedbatch/server.py:116-126) can construct either class.
The sampler itself accepts any object with these attributes, including the reference's own.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class SamplingParams:
    """What one request asks of the sampler and the decode loop: how many tokens, the sampling
    knobs (temperature 0 means greedy; top_k 0 and top_p 1 switch those filters off), whether to
    ignore the end-of-sequence token, a seed for the request's own generator, and extra stop ids."""

    max_tokens: int = 64
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    ignore_eos: bool = False
    seed: int | None = None
    stop_token_ids: tuple[int, ...] = ()

    def __post_init__(self) -> None:
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0")

    @property
    def greedy(self) -> bool:
        return self.temperature == 0
