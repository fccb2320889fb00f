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


# ---- the benchmark configurations at full vocabulary (tests/golden/golden_big.npz) ----------------

PROB_RTOL_BF16 = 1e-3  # the kept-probability tolerance for bf16 logits
PROB_RTOL_FP64 = 1e-6  # temperature-only full-vocabulary rows: against a float64 softmax
# The reference's own fp32 softmax drifts up to ~5e-6 relative on full-vocabulary rows (argument
# rounding of x - max far below the max); against it those rows get this bound.
PROB_RTOL_REF_FULL = 1e-5


@pytest.fixture(scope="module")
def golden_big():
    import os

    return np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_big.npz"))


def _digest(x: torch.Tensor) -> np.ndarray:
    t = x.contiguous()
    raw = t.view(torch.int16).numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.numpy()
    return np.frombuffer(hashlib.sha256(raw.tobytes()).digest(), np.uint8)


def _check_big(gb, prefix, logits: torch.Tensor):
    """Oracle against the reference's recorded outputs on rows of a regenerated workload.

    Returns per-class counts and the worst relative probability errors (against the reference, and
    against a float64 softmax of the oracle's own kept set on temperature-only full rows)."""
    assert np.array_equal(_digest(logits), gb[f"{prefix}_sha256"]), f"{prefix}: synthetic logits drifted"
    bf16 = logits.dtype == torch.bfloat16
    x32 = logits.float().numpy()
    V = x32.shape[1]
    kept_all = np.unpackbits(gb[f"{prefix}_kept"], axis=1, count=V).astype(bool)
    off, pidx, pval = gb[f"{prefix}_probs_off"], gb[f"{prefix}_probs_idx"], gb[f"{prefix}_probs"]
    n = len(gb[f"{prefix}_temp"])
    rows = gb[f"{prefix}_row"]
    prm = oracle.make_params(gb[f"{prefix}_temp"], gb[f"{prefix}_topp"], gb[f"{prefix}_topk"], np.full(n, 0.5))
    tok, info, probs = oracle.sample(logits, prm, rows, want_probs=True)
    stats = dict(exact=0, tie_cut=0, near_cut=0, greedy=0)
    worst = dict(ref=0.0, ref_full=0.0, fp64_full=0.0)
    assert np.array_equal(gb[f"{prefix}_ref_token"], gb[f"{prefix}_port_token"])
    for i in range(n):
        t, k, p = float(gb[f"{prefix}_temp"][i]), int(gb[f"{prefix}_topk"][i]), float(gb[f"{prefix}_topp"][i])
        x = x32[rows[i]]
        assert info["status"][i] == 0, (prefix, i)
        if t == 0:
            assert tok[i] == gb[f"{prefix}_ref_token"][i], (prefix, i)
            stats["greedy"] += 1
            continue
        mine = oracle.kept_mask(x, t, info[i])
        ref = kept_all[i]
        if np.array_equal(mine, ref):
            stats["exact"] += 1
            idx = pidx[off[i] : off[i + 1]]
            rp = pval[off[i] : off[i + 1]].astype(np.float64)
            mp = probs[i][idx].astype(np.float64)
            big = rp > 1e-30
            rel = float((np.abs(mp[big] - rp[big]) / rp[big]).max(initial=0))
            full = not (0 < k < V) and not (p < 1.0 and np.float32(p) < 1.0)
            if full:
                # float64 softmax over the same kept set (here: every finite key)
                y = (x.astype(np.float32) / np.float32(t)).astype(np.float64)
                e = np.exp(y - y.max())
                q = e[idx] / e.sum()
                ok = q > 1e-30
                rel64 = float((np.abs(mp[ok] - q[ok]) / q[ok]).max(initial=0))
                worst["fp64_full"] = max(worst["fp64_full"], rel64)
                worst["ref_full"] = max(worst["ref_full"], rel)
                assert rel64 <= PROB_RTOL_FP64, (prefix, i, rel64)
                assert rel <= PROB_RTOL_REF_FULL, (prefix, i, rel)
            else:
                worst["ref"] = max(worst["ref"], rel)
                assert rel <= (PROB_RTOL_BF16 if bf16 else PROB_RTOL), (prefix, i, rel)
            continue
        assert p < 1.0, (prefix, i)
        # Top-p only: the sets may differ at the cut and nowhere else. Position j of the order
        # (key descending) is kept iff the mass before it is <= fp32(top_p); the reference's fp32
        # softmax and cumsum can move the cut only across positions whose exact (float64) mass
        # before them lies within its rounding of top_p, and its unstable sort may pick other
        # members of the tie group at the cut (then only the count is defined).
        ys, excl = _sorted_mass64(x, t, k)
        c_mine, c_ref = int(mine.sum()), int(ref.sum())
        lo, hi = min(c_mine, c_ref), max(c_mine, c_ref)
        assert lo >= 1
        if hi > lo:
            band = np.abs(excl[lo:hi] - float(np.float32(p)))
            assert band.max() < NEAR_CUT, (prefix, i, float(band.max()))
        y = (x.astype(np.float32) / np.float32(t)).astype(np.float32)
        diff = np.flatnonzero(mine != ref)
        assert y[diff].min() >= ys[hi - 1] and y[diff].max() <= ys[lo - 1], (prefix, i, "sets differ away from the cut")
        stats["near_cut" if hi > lo else "tie_cut"] += 1
    return stats, worst


def _sorted_mass64(x: np.ndarray, t: float, k: int):
    """The top-k-filtered keys in descending order, and before each position the exact (float64)
    softmax mass of the positions ahead of it."""
    y = (x.astype(np.float32) / np.float32(t)).astype(np.float32)
    y = y[np.isfinite(y)]
    ys = np.sort(y)[::-1]
    if 0 < k < x.size:
        ys = ys[ys >= ys[k - 1]]
    yy = ys.astype(np.float64)
    e = np.exp(yy - yy.max())
    pr = e / e.sum()
    return ys, np.cumsum(pr) - pr


def test_config2_rows_match_reference(golden_big):
    """32 rows of the headline configuration ([256, 128256] fp32, T 0.7, k 50, p 0.95)."""
    stats, worst = _check_big(golden_big, "cfg2", workloads.config2(seed=0).logits)
    print("cfg2", stats, worst)
    assert stats["exact"] == 32, stats
    assert worst["ref"] <= PROB_RTOL


def test_config2_flat_rows_match_reference(golden_big):
    """16 flat rows (0.05 N(0,1), top_k off, top_p 0.999): kept sets of nearly the whole vocabulary,
    where the reference's fp32 cumulative sum is most exposed to rounding."""
    stats, worst = _check_big(golden_big, "cfg2flat", workloads.config2_flat(seed=0).logits)
    print("cfg2flat", stats, worst)
    assert stats["exact"] + stats["tie_cut"] + stats["near_cut"] == 16


def test_config1_rows_match_reference(golden_big):
    """All 256 rows of the mixed bf16 batch: greedy with planted duplicate maxima, temperature-only
    full-vocabulary rows (checked against float64 too), top-k and top-p rows."""
    stats, worst = _check_big(golden_big, "cfg1", workloads.config1(seed=0).logits)
    print("cfg1", stats, worst)
    assert stats["greedy"] == 64
    # bf16 rows hold large tie groups, and at 49152 entries the reference's fp32 cumsum rounding
    # reaches ~1e-5 of the mass: top-p 0.9 / 0.99 cuts often land in that band (every differing
    # position is checked against it above); top-k and temperature-only rows must be exact
    assert stats["exact"] + stats["tie_cut"] + stats["near_cut"] == 192
    assert stats["near_cut"] + stats["tie_cut"] <= 64, stats


def test_top_p_rounding_to_one(golden_big):
    """top_p just below 1.0 in float64 (three values that round to 1.0 in fp32, and the largest fp32
    below 1.0). The reference still runs its top-p branch (sampling.py:18, a float64 compare) and
    compares the fp32 cumulative mass against fp32(top_p): where its fp32 cumsum overshoots 1.0 it
    drops tail positions whose exact mass before them is within its rounding of 1.0. The sampler
    skips top-p when fp32(top_p) == 1.0. Every difference must sit in that band (checked per
    position); rows whose kept set ends far from the total mass (top_k 50) are exact."""
    gb = golden_big
    stats, worst = _check_big(gb, "p1", workloads.config0(seed=0).logits)
    print("p1", stats, worst)
    assert stats["exact"] + stats["near_cut"] + stats["tie_cut"] == len(gb["p1_temp"])
    x = workloads.config0(seed=0).logits.numpy()
    k50 = np.flatnonzero(gb["p1_topk"] == 50)
    prm = oracle.make_params(gb["p1_temp"][k50], gb["p1_topp"][k50], gb["p1_topk"][k50], np.full(k50.size, 0.5))
    _, info, _ = oracle.sample(x, prm, gb["p1_row"][k50])
    kept = np.unpackbits(gb["p1_kept"], axis=1, count=x.shape[1]).astype(bool)
    for j, i in enumerate(k50):
        assert np.array_equal(oracle.kept_mask(x[gb["p1_row"][i]], float(gb["p1_temp"][i]), info[j]), kept[i]), i
