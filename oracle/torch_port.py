"""TEST INFRASTRUCTURE — pagedbatch's ``sample_token`` restated with the same torch operations.

``pagedbatch/sampling.py:10-27`` runs, per row: argmax (greedy), ``logits.float() / T``,
``topk`` + ``masked_fill`` (top-k), ``sort`` + ``softmax`` + ``cumsum`` + ``masked_fill`` +
``scatter`` (top-p), a final ``softmax`` and ``torch.multinomial`` with the request's generator.
This module performs the same calls in the same order, so that

* ``filtered_logits`` exposes the masked row the reference builds (its finite entries are the
  reference's kept set, its softmax the reference's final distribution), and
* ``sample_row`` draws exactly as the reference does — the golden-fixture script checks it
  token for token against the reference — and serves as the timed CPU baseline
  (``bench.py --impl reference`` and the ``cpu_baseline`` field), called once per row as
  ``pagedbatch/engine.py:133-139`` does.
"""

from __future__ import annotations

import torch


def filtered_logits(logits: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """The masked fp32 row of sampling.py:14-25 (non-greedy rows)."""
    x = logits.float() / temperature  # sampling.py:14
    if top_k > 0 and top_k < x.shape[-1]:  # sampling.py:15-17
        kth = torch.topk(x, top_k).values[-1]
        x = x.masked_fill(x < kth, float("-inf"))
    if top_p < 1.0:  # sampling.py:18-25
        vals, order = torch.sort(x, descending=True)
        p = torch.softmax(vals, dim=-1)
        before = torch.cumsum(p, dim=-1) - p
        vals = vals.masked_fill(before > top_p, float("-inf"))
        x = torch.full_like(x, float("-inf")).scatter(0, order, vals)
    return x


def final_probs(logits: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """sampling.py:26: softmax over the masked row."""
    return torch.softmax(filtered_logits(logits, temperature, top_k, top_p), dim=-1)


def sample_row(logits: torch.Tensor, temperature: float, top_k: int, top_p: float, generator: torch.Generator) -> int:
    """One draw exactly as sampling.py:12-27 makes it."""
    if temperature == 0:
        return int(torch.argmax(logits))
    probs = final_probs(logits, temperature, top_k, top_p)
    return int(torch.multinomial(probs, 1, generator=generator))


def sample_batch(logits: torch.Tensor, params, generators) -> list[int]:
    """The engine's per-row loop (engine.py:133-139) over a [B, V] CPU batch.

    ``params`` is a sequence of (temperature, top_k, top_p); ``generators`` one torch.Generator per row.
    """
    return [sample_row(logits[i], t, k, p, g) for i, ((t, k, p), g) in enumerate(zip(params, generators))]
