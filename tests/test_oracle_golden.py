"""The CPU oracle against golden vectors produced by the reference itself (tests/golden/make_golden.py).

Pins: greedy tokens exact; top-k kept sets exact; top-p kept sets exact except (a) cuts that fall
inside a group of equal keys, where the reference's unstable sort picks arbitrary members and
only the count is defined, and (b) cuts whose float64 margin to top_p is below the reference's
own fp32 softmax rounding (counted, and bounded); renormalised probabilities within 1e-6 relative
of the reference's softmax wherever the kept sets agree.
"""

import hashlib

import numpy as np
import pytest
import torch

import oracle
from pagedbatch_b200 import workloads

NEAR_CUT = 2e-5  # float64 mass distance to top_p within which the reference's fp32 softmax can flip a cut
PROB_RTOL = 1e-6


def _cases(golden, prefix):
    n = len(golden[f"{prefix}_temp"])
    kept = np.unpackbits(golden[f"{prefix}_kept"], axis=1).astype(bool)
    off = golden[f"{prefix}_probs_off"]
    for i in range(n):
        yield dict(
            i=i,
            row=int(golden[f"{prefix}_row"][i]),
            t=float(golden[f"{prefix}_temp"][i]),
            k=int(golden[f"{prefix}_topk"][i]),
            p=float(golden[f"{prefix}_topp"][i]),
            ref_token=int(golden[f"{prefix}_ref_token"][i]),
            margin=float(golden[f"{prefix}_margin"][i]),
            tie_cut=bool(golden[f"{prefix}_tie_cut"][i]),
            kept=kept[i],
            probs=golden[f"{prefix}_probs"][off[i] : off[i + 1]],
        )


def _check(rows, cases):
    stats = dict(exact=0, tie_cut=0, near_cut=0, greedy=0)
    worst = 0.0
    for c in cases:
        x = rows[c["row"]]
        V = x.shape[0]
        prm = oracle.make_params([c["t"]], [c["p"]], [c["k"]], [0.5])
        tok, info, probs = oracle.sample(x[None, :], prm, want_probs=True)
        assert info["status"][0] == 0
        if c["t"] == 0:
            assert tok[0] == c["ref_token"], c
            stats["greedy"] += 1
            continue
        mine = oracle.kept_mask(x, c["t"], info[0])
        ref = c["kept"][:V]
        if np.array_equal(mine, ref):
            stats["exact"] += 1
            rp = c["probs"]
            mp = probs[0][ref]
            big = rp > 1e-30
            rel = np.abs(mp[big].astype(np.float64) - rp[big]) / rp[big]
            worst = max(worst, float(rel.max(initial=0)))
            assert rel.max(initial=0) <= PROB_RTOL, (c["i"], float(rel.max()))
            continue
        # top-p only: the sets may differ at the boundary of the cut and nowhere else
        assert c["p"] < 1.0, c["i"]
        same_count = int(mine.sum()) == int(ref.sum())
        near = not (c["tie_cut"] and same_count)
        if near:  # the cut itself moved: only allowed within the reference's own rounding of the mass
            assert c["margin"] < NEAR_CUT, (c["i"], c["t"], c["k"], c["p"], c["margin"])
            assert abs(int(mine.sum()) - int(ref.sum())) <= 1, c["i"]
        y = x.astype(np.float32) / np.float32(c["t"])
        boundary = {float(y[mine].min()), float(y[ref].min())}
        diff = np.flatnonzero(mine != ref)
        assert set(y[diff].tolist()) <= boundary, "kept sets may differ only at the cut"
        stats["near_cut" if near else "tie_cut"] += 1
    return stats, worst


def test_small_rows_match_reference(golden):
    rows = [golden["small_logits"][i, : golden["small_vocab"][i]] for i in range(len(golden["small_vocab"]))]
    stats, worst = _check(rows, _cases(golden, "small"))
    total = sum(stats.values())
    assert stats["greedy"] > 20 and stats["exact"] > 800
    assert stats["near_cut"] <= 0.01 * total, stats
    assert worst <= PROB_RTOL


def test_config0_rows_match_reference(golden):
    w = workloads.config0(seed=0)
    digest = np.frombuffer(hashlib.sha256(w.logits.numpy().tobytes()).digest(), np.uint8)
    assert np.array_equal(digest, golden["cfg0_sha256"]), "synthetic logits drifted from the fixtures"
    rows = [w.logits[r].numpy() for r in range(w.rows)]
    stats, _ = _check(rows, _cases(golden, "cfg0"))
    assert stats["exact"] == 8 and stats["greedy"] == 8, stats


def test_reference_primitives(golden):
    """tests/test_engine.py:86-93 of the reference, through the oracle."""
    x = np.array([[0.1, 3.0, 0.2, 2.9]], dtype=np.float32)
    for t, k, p in [(0.0, 0, 1.0), (1.0, 1, 1.0), (1.0, 0, 1e-6)]:
        tok, _, _ = oracle.sample(x, oracle.make_params([t], [p], [k], [0.999]))
        assert tok[0] == 1
    g = torch.Generator().manual_seed(0)
    us = [float(torch.rand((), dtype=torch.float64, generator=g)) for _ in range(50)]
    tok, _, _ = oracle.sample(np.repeat(x, 50, 0), oracle.make_params([1.0] * 50, [1.0] * 50, [2] * 50, us))
    assert set(tok.tolist()) <= {1, 3}


def test_fixed_exp_accuracy():
    """The weights' exp: within 1 ulp of libm on a dense sample of [-87, 0], exactly 1 at 0."""
    L = oracle.lib()
    assert L.pbo_exp(0.0) == 1.0
    assert L.pbo_exp(-88.0) == 0.0
    d = -np.linspace(0, 87, 20001).astype(np.float32)
    got = np.array([L.pbo_exp(float(v)) for v in d], dtype=np.float32)
    ref = np.exp(d.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got - ref) / ulp) < 1.0


def test_inverse_cdf_order():
    """The draw walks keys descending, indices ascending: u just below a boundary picks the earlier token."""
    x = np.array([[1.0, 2.0, 2.0, 0.5]], dtype=np.float32)  # order: 1, 2, 0, 3
    _, info, probs = oracle.sample(x, oracle.make_params([1.0], [1.0], [0], [0.0]), want_probs=True)
    p = probs[0].astype(np.float64)
    order = [1, 2, 0, 3]
    cum = np.cumsum(p[order])
    for j, tok in enumerate(order):
        lo = 0.0 if j == 0 else cum[j - 1]
        u = (lo + (cum[j] - lo) / 2)
        t, _, _ = oracle.sample(x, oracle.make_params([1.0], [1.0], [0], [u]))
        assert t[0] == tok


@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_nonfinite_rows_report_status(bad):
    x = np.array([[0.0, bad, 1.0]], dtype=np.float32)
    tok, info, _ = oracle.sample(x, oracle.make_params([1.0], [1.0], [0], [0.5]))
    assert tok[0] == -1 and info["status"][0] == 1
    tok, info, _ = oracle.sample(x, oracle.make_params([0.0], [1.0], [0], [0.5]))
    assert tok[0] == 1  # greedy: NaN counts as the largest value, +inf is the largest
