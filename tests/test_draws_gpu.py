"""Free-running draws: 10^6 draws per row against the reference's distribution (chi-square).

The sampler turns each row's uniform into a token by the inverse CDF of the kept set. Here the
uniforms are 10^6 consecutive float64 draws of one seeded torch generator (what a request's
generator yields step after step), fed through the product path (``ops.sample_op`` over the C
ABI) in batches of 8192 parameter records that all point at the same logits row (``row_index``).
The token counts must stay inside the reference's kept set and match the reference's final
distribution, ``softmax`` over the masked row of ``pagedbatch/sampling.py:14-26``
(restated in ``oracle/torch_port.py``), by a chi-square test; expected counts below 5 are pooled.
"""

import numpy as np
import pytest
import torch
from scipy import stats

import oracle
from oracle import torch_port
from pagedbatch_b200 import ops, workloads

pytestmark = pytest.mark.gpu

N_DRAWS = 1_000_000
BATCH = 8192
P_MIN = 1e-3  # the seeded draws are fixed, so the statistic is too: this is a pass/fail bound, not a flaky test

CASES = [
    # label, vocabulary, dtype, temperature, top_k, top_p
    ("k50_p095_llama3", 128256, torch.float32, 0.7, 50, 0.95),
    ("temperature_only", 1000, torch.float32, 1.0, 0, 1.0),
    ("top_p_only", 5000, torch.float32, 1.3, 0, 0.9),
    ("top_k20_bf16", 49152, torch.bfloat16, 1.0, 20, 1.0),
    ("k1000_p099", 49152, torch.float32, 1.5, 1000, 0.99),
]


def _pooled(observed: np.ndarray, expected: np.ndarray):
    """Merge the bins with the smallest expected counts until every bin expects at least 5."""
    order = np.argsort(expected)
    e, o = expected[order], observed[order]
    m = int(np.searchsorted(e, 5.0))  # bins expecting fewer than 5
    while m < e.size and 0.0 < e[:m].sum() < 5.0:
        m += 1
    if m == 0:
        return o, e
    return np.concatenate([[o[:m].sum()], o[m:]]), np.concatenate([[e[:m].sum()], e[m:]])


@pytest.mark.parametrize("label,V,dtype,T,k,p", CASES, ids=[c[0] for c in CASES])
def test_free_running_draws_chi_square(label, V, dtype, T, k, p):
    dev = torch.device("cuda", 0)
    row = workloads.head_boosted(1, V, seed=V, dtype=dtype)
    x = row.to(dev)
    expected = torch_port.final_probs(row[0], T, k, p).double().numpy()
    kept = expected > 0

    gen = torch.Generator().manual_seed(1234 + V)
    u = torch.rand(N_DRAWS, dtype=torch.float64, generator=gen).to(dev)
    params = ops.params_tensor(oracle.make_params([T] * BATCH, [p] * BATCH, [k] * BATCH, [0.0] * BATCH), dev)
    fields = params.view(torch.float64).view(BATCH, 4)  # temperature, top_p, uniform, (top_k, reserved)
    same_row = torch.zeros(BATCH, dtype=torch.int32, device=dev)
    counts = torch.zeros(V, dtype=torch.int64, device=dev)
    for i0 in range(0, N_DRAWS, BATCH):
        n = min(BATCH, N_DRAWS - i0)
        fields[:n, 2].copy_(u[i0 : i0 + n])
        tok = ops.sample_op(x, params[: n * 32], same_row[:n])
        assert int(tok.min()) >= 0, f"{label}: a draw failed"
        counts += torch.bincount(tok, minlength=V)
    counts = counts.cpu().numpy()

    assert counts.sum() == N_DRAWS
    assert counts[~kept].sum() == 0, f"{label}: tokens outside the reference's kept set were drawn"
    o, e = _pooled(counts[kept].astype(np.float64), expected[kept] * N_DRAWS)
    chi2, pval = stats.chisquare(o, e * (o.sum() / e.sum()))
    assert pval > P_MIN, f"{label}: chi-square {chi2:.1f} on {o.size - 1} dof, p = {pval:.2e}"
