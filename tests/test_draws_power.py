"""The chi-square check of tests/test_draws_gpu.py can fail: its power, on the CPU.

Draws are simulated from the reference's final distribution (``oracle/torch_port.py``) with a
multinomial, once as they should be and once with a planted mistake (5 % of the top token's mass
moved to the second token, or a kept token never drawn). The unbiased draws must pass the same
pooled chi-square bound, the biased ones must fail it. (At 10^6 draws a 1 % shift of the top
token's mass is not reliably detected: that is the resolution of this check.)
"""

import numpy as np
import pytest
from scipy import stats

from oracle import torch_port
from pagedbatch_b200 import workloads

from test_draws_gpu import CASES, N_DRAWS, P_MIN, _pooled


def _pvalue(counts: np.ndarray, expected: np.ndarray) -> float:
    kept = expected > 0
    o, e = _pooled(counts[kept].astype(np.float64), expected[kept] * N_DRAWS)
    return float(stats.chisquare(o, e * (o.sum() / e.sum())).pvalue)


@pytest.mark.parametrize("label,V,dtype,T,k,p", CASES, ids=[c[0] for c in CASES])
def test_chi_square_rejects_planted_bias(label, V, dtype, T, k, p):
    row = workloads.head_boosted(1, V, seed=V, dtype=dtype)
    expected = torch_port.final_probs(row[0], T, k, p).double().numpy()
    expected /= expected.sum()
    rng = np.random.default_rng(V)
    assert _pvalue(rng.multinomial(N_DRAWS, expected), expected) > P_MIN, f"{label}: unbiased draws rejected"

    order = np.argsort(-expected)
    moved = expected.copy()
    shift = 0.05 * expected[order[0]]  # 5 % of the top token's mass goes to the second
    moved[order[0]] -= shift
    moved[order[1]] += shift
    assert _pvalue(rng.multinomial(N_DRAWS, moved), expected) < P_MIN, f"{label}: a 5 % mass shift passed"

    dropped = expected.copy()
    dropped[order[2]] = 0.0  # a kept token that is never drawn
    dropped /= dropped.sum()
    assert _pvalue(rng.multinomial(N_DRAWS, dropped), expected) < P_MIN, f"{label}: a dropped token passed"
