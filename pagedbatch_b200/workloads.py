"""Seeded synthetic inputs shaped like the sampling benchmark configurations.

The reference publishes no sampling benchmark data; these generators stand in for logits a
Llama-style LM head would produce (pagedbatch/model.py:280-283 returns ``[B, vocab]`` logits):

* ``head_boosted``: ``3*N(0,1)`` plus ``8*r^-0.7`` on a seeded random permutation of the token
  ids (rank r = 1..V), so each row has a Zipf-like head over a Gaussian floor;
* ``flat``: ``0.05*N(0,1)``, the worst case for top-p (the kept set approaches the vocabulary).

Everything is generated on the CPU from ``torch.Generator`` seeds, so tests, the oracle and the
benchmark see the same bits on any machine with the same torch build.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .config import SamplingParams

SMOLLM2_VOCAB = 49152  # pagedbatch/config.py:59-75 (smollm2_135m)
LLAMA3_VOCAB = 128256


def head_boosted(rows: int, vocab: int, seed: int = 0, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, vocab, generator=g) * 3.0
    boost = 8.0 * torch.arange(1, vocab + 1, dtype=torch.float64).pow(-0.7)
    boost = boost.float()
    for r in range(rows):
        perm = torch.randperm(vocab, generator=g)
        x[r, perm] += boost
    return x.to(dtype)


def flat(rows: int, vocab: int, seed: int = 0, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(rows, vocab, generator=g) * 0.05).to(dtype)


def plant_duplicate_maxima(x: torch.Tensor, rows, seed: int = 0) -> torch.Tensor:
    """Copy each listed row's maximum to 1-3 other random positions (greedy tie cases)."""
    g = torch.Generator().manual_seed(seed + 1)
    V = x.shape[1]
    for r in rows:
        m = x[r].max()
        n = int(torch.randint(1, 4, (), generator=g))
        pos = torch.randint(0, V, (n,), generator=g)
        x[r, pos] = m
    return x


def first_uniform(seed: int) -> float:
    """The first draw ``sample_tokens`` takes from a request generator seeded with ``seed``."""
    g = torch.Generator().manual_seed(seed)
    return float(torch.rand((), dtype=torch.float64, generator=g))


@dataclass
class Workload:
    name: str
    logits: torch.Tensor  # CPU, [B, V]
    params: list[SamplingParams]
    seeds: list[int]

    @property
    def rows(self) -> int:
        return self.logits.shape[0]

    @property
    def vocab(self) -> int:
        return self.logits.shape[1]

    def uniforms(self) -> list[float]:
        return [first_uniform(s) for s in self.seeds]

    def generators(self) -> list[torch.Generator]:
        return [torch.Generator().manual_seed(s) for s in self.seeds]


def config0(seed: int = 0) -> Workload:
    """[8, 49152] fp32, T 0.8, top_k 50, top_p 0.9, seeds 0..7."""
    x = head_boosted(8, SMOLLM2_VOCAB, seed)
    p = [SamplingParams(temperature=0.8, top_k=50, top_p=0.9, seed=i) for i in range(8)]
    return Workload("cfg0_8x49152_f32", x, p, list(range(8)))


def config1(seed: int = 0, rows: int = 256) -> Workload:
    """[256, 49152] bf16, four blocks of 64 rows: greedy (planted ties), temperature-only, top-k, top-p."""
    assert rows % 4 == 0
    q = rows // 4
    x = head_boosted(rows, SMOLLM2_VOCAB, seed)
    x = plant_duplicate_maxima(x, range(q), seed)
    x = x.to(torch.bfloat16)
    ps: list[SamplingParams] = []
    for i in range(rows):
        blk, j = divmod(i, q)
        if blk == 0:
            ps.append(SamplingParams(temperature=0.0, seed=i))
        elif blk == 1:
            ps.append(SamplingParams(temperature=(0.5, 1.0, 1.5)[j % 3], seed=i))
        elif blk == 2:
            ps.append(SamplingParams(temperature=1.0, top_k=(1, 20, 100, 1000)[j % 4], seed=i))
        else:
            ps.append(SamplingParams(temperature=1.0, top_p=(0.5, 0.9, 0.99)[j % 3], seed=i))
    return Workload(f"cfg1_{rows}x49152_bf16_mixed", x, ps, list(range(rows)))


def config2(seed: int = 0, rows: int = 256, vocab: int = LLAMA3_VOCAB) -> Workload:
    """[256, 128256] fp32, T 0.7, top_k 50, top_p 0.95 (the headline sampling step)."""
    x = head_boosted(rows, vocab, seed)
    p = [SamplingParams(temperature=0.7, top_k=50, top_p=0.95, seed=i) for i in range(rows)]
    return Workload(f"cfg2_{rows}x{vocab}_f32_k50_p095", x, p, list(range(rows)))


def config2_flat(seed: int = 0, rows: int = 256, vocab: int = LLAMA3_VOCAB) -> Workload:
    """Worst case of config 2: flat 0.05*N(0,1) logits, top_k off, top_p 0.999."""
    x = flat(rows, vocab, seed)
    p = [SamplingParams(temperature=0.7, top_k=0, top_p=0.999, seed=i) for i in range(rows)]
    return Workload(f"cfg2flat_{rows}x{vocab}_f32_p0999", x, p, list(range(rows)))


def config3(seed: int = 0, rows: int = 1024, vocab: int = LLAMA3_VOCAB) -> Workload:
    """[1024, 128256] bf16, T 1.0, top_k 64, top_p 0.9 (vocab-parallel case)."""
    x = head_boosted(rows, vocab, seed).to(torch.bfloat16)
    p = [SamplingParams(temperature=1.0, top_k=64, top_p=0.9, seed=i) for i in range(rows)]
    return Workload(f"cfg3_{rows}x{vocab}_bf16_k64_p09", x, p, list(range(rows)))
