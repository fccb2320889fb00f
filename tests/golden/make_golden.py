"""Generate the golden fixtures that pin the CPU oracle to the reference implementation.

Run where the reference package can be imported: set ``PAGEDBATCH_REF`` to a checkout of
pagedbatch (the directory holding ``pagedbatch/``), or install it into ``baseline/_ref``. Then
``python tests/golden/make_golden.py [small|big|all]`` writes ``tests/golden/golden.npz`` (small rows
and config 0) and/or ``tests/golden/golden_big.npz`` (the benchmark configurations at full
vocabulary: config 2, config 2-flat, config 1, and top_p values that round to 1.0 in fp32).

For every case row it records what the reference itself produces:

* ``ref_token``   — ``pagedbatch.sampling.sample_token(row, SamplingParams(...), Generator(seed))``;
* ``port_token``  — ``oracle.torch_port.sample_row`` with an identically seeded generator (must equal
                    ``ref_token``: this pins the torch restatement to the reference, draw for draw);
* ``kept``        — the finite entries of the masked row of sampling.py:14-25 (via the torch port);
* ``probs``       — sampling.py:26's softmax of that masked row (fp32), stored at the kept positions;
* ``margin``      — for top-p rows, the float64 distance between fp32(top_p) and the nearest exclusive
                    cumulative mass on either side of the cut (rows whose margin is within the
                    reference's own softmax rounding can legitimately differ);
* ``tie_cut``     — the top-p cut falls inside a group of equal keys, where the reference's unstable
                    sort picks arbitrary members (only the count is determined).

Small rows are stored verbatim; the benchmark rows are stored as their generator seed plus a
checksum of the regenerated logits. For rows whose kept set is large, the probabilities are
stored at a subset of the kept positions (the 64 largest and a seeded sample of the rest).
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def _reference_path() -> str:
    """Where the reference package is imported from: $PAGEDBATCH_REF, else baseline/_ref."""
    for cand in (os.environ.get("PAGEDBATCH_REF"), os.path.join(REPO, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "pagedbatch")):
            return cand
    raise SystemExit("set PAGEDBATCH_REF to a pagedbatch checkout (the directory holding pagedbatch/)")


sys.path.insert(0, _reference_path())

from pagedbatch.config import SamplingParams as RefParams  # noqa: E402  (the reference)
from pagedbatch.sampling import sample_token as ref_sample_token  # noqa: E402

from oracle import torch_port  # noqa: E402
from pagedbatch_b200 import workloads  # noqa: E402


def masked_info(row: torch.Tensor, t: float, k: int, p: float):
    """(kept mask, fp32 probs, cut margin, tie_cut) of one case as the reference computes them."""
    if t == 0:
        kept = np.zeros(row.numel(), dtype=bool)
        kept[int(torch.argmax(row))] = True
        return kept, kept.astype(np.float32), np.nan, False
    masked = torch_port.filtered_logits(row, t, k, p)
    kept = torch.isfinite(masked).numpy()
    probs = torch.softmax(masked, -1).numpy()
    margin, tie_cut = np.nan, False
    if p < 1.0:
        keys = (row.float() / t).double()
        if 0 < k < row.numel():
            kth = torch.topk(row.float() / t, k).values[-1].double()
            keys = keys.masked_fill(keys < kth, float("-inf"))
        vals, _ = torch.sort(keys, descending=True)
        pr = torch.softmax(vals, -1)
        excl = torch.cumsum(pr, -1) - pr
        pf = float(np.float32(p))
        cut = int((excl <= pf).sum())  # positions kept under exact float64 arithmetic
        lo = pf - float(excl[cut - 1]) if cut >= 1 else np.inf
        hi = float(excl[cut]) - pf if cut < excl.numel() else np.inf
        margin = min(lo, hi)
        if 1 <= cut < vals.numel():
            tie_cut = bool(vals[cut - 1] == vals[cut])
    return kept, probs, margin, tie_cut


def small_cases():
    """(row id, temperature, top_k, top_p, seed) over a set of unique rows."""
    g = torch.Generator().manual_seed(1234)
    rows = [torch.tensor([0.1, 3.0, 0.2, 2.9])]  # tests/test_engine.py:86-93 of the reference
    cases = [(0, t, k, p, 0) for t, k, p in
             [(0.0, 0, 1.0), (1.0, 1, 1.0), (1.0, 0, 1e-6), (1.0, 2, 1.0), (0.7, 0, 0.9), (1.0, 3, 1.0)]]
    grid_kp = [(0, 1.0), (0, 0.9), (20, 1.0), (50, 0.95), (1, 1.0), (2, 0.5), (1000, 0.99), (0, 0.5),
               (0, 0.99), (20, 0.9)]
    for V in (10, 258, 1000, 4099):
        for rep in range(6):
            row = torch.randn(V, generator=g) * (3.0 if rep % 2 == 0 else 0.3)
            if rep == 2:  # integer-valued row: heavy ties for argmax / kth / top-p cuts
                row = torch.randint(-4, 5, (V,), generator=g).float()
            if rep == 3:  # bf16 row: ties from the 8-bit mantissa
                row = (torch.randn(V, generator=g) * 3.0).to(torch.bfloat16)
            if rep == 4:  # masked vocabulary and signed zeros
                row[torch.randint(0, V, (V // 5,), generator=g)] = float("-inf")
                row[: min(4, V)] = torch.tensor([0.0, -0.0, 0.0, -0.0][: min(4, V)])
            rows.append(row)
            rid = len(rows) - 1
            cases.append((rid, 0.0, 0, 1.0, 0))
            for t in (0.5, 0.7, 1.0, 1.5):
                for k, p in grid_kp:
                    cases.append((rid, t, k, p, int(torch.randint(0, 2**31 - 1, (), generator=g))))
    return rows, cases


def pack_cases(rows, cases, prefix):
    V_max = max(r.numel() for r in rows)
    R, n = len(rows), len(cases)
    logits = np.full((R, V_max), np.nan, dtype=np.float32)
    vocab = np.zeros(R, np.int32)
    is_bf16 = np.zeros(R, bool)
    for i, r in enumerate(rows):
        logits[i, : r.numel()] = r.float().numpy()
        vocab[i] = r.numel()
        is_bf16[i] = r.dtype == torch.bfloat16
    cols = {c: np.zeros(n, dt) for c, dt in [("row", np.int32), ("temp", np.float64), ("topk", np.int32),
                                             ("topp", np.float64), ("seed", np.int64), ("ref_token", np.int64),
                                             ("margin", np.float64), ("tie_cut", bool)]}
    kept = np.zeros((n, V_max), bool)
    pvals, poff = [], [0]
    for i, (rid, t, k, p, seed) in enumerate(cases):
        row = rows[rid]
        params = RefParams(temperature=t, top_k=k, top_p=p)
        ref = ref_sample_token(row, params, torch.Generator().manual_seed(seed))
        port = torch_port.sample_row(row, t, k, p, torch.Generator().manual_seed(seed))
        assert ref == port, f"torch port disagrees with the reference on case {i}"
        kp, pr, mg, tc = masked_info(row, t, k, p)
        V = row.numel()
        kept[i, :V] = kp
        pvals.append(pr[kp].astype(np.float32))
        poff.append(poff[-1] + int(kp.sum()))
        for c, v in [("row", rid), ("temp", t), ("topk", k), ("topp", p), ("seed", seed), ("ref_token", ref),
                     ("margin", mg), ("tie_cut", tc)]:
            cols[c][i] = v
    out = {f"{prefix}_logits": logits, f"{prefix}_vocab": vocab, f"{prefix}_bf16": is_bf16,
           f"{prefix}_kept": np.packbits(kept, axis=1), f"{prefix}_probs": np.concatenate(pvals),
           f"{prefix}_probs_off": np.array(poff, np.int64)}
    out.update({f"{prefix}_{c}": v for c, v in cols.items()})
    return out


def _digest(x: torch.Tensor) -> np.ndarray:
    """sha256 of a CPU tensor's raw bytes (bf16 / fp16 as their 16-bit patterns)."""
    t = x.contiguous()
    raw = t.view(torch.int16).numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.numpy()
    return np.frombuffer(hashlib.sha256(raw.tobytes()).digest(), np.uint8)


PROB_ALL = 512  # kept sets up to this size store every probability; larger ones a subset
PROB_TOP = 64


def pack_big(logits: torch.Tensor, cases, prefix: str, seed: int = 99):
    """Cases over rows of a regenerated workload: kept sets in full (bit-packed), probabilities at
    every kept position of small kept sets and at the PROB_TOP largest plus a seeded sample of the
    other kept positions of large ones."""
    rng = np.random.default_rng(seed)
    V = logits.shape[1]
    n = len(cases)
    cols = {c: np.zeros(n, dt) for c, dt in [("row", np.int32), ("temp", np.float64), ("topk", np.int32),
                                             ("topp", np.float64), ("seed", np.int64), ("ref_token", np.int64),
                                             ("port_token", np.int64), ("margin", np.float64),
                                             ("tie_cut", bool), ("kept_n", np.int64)]}
    kept = np.zeros((n, V), bool)
    pidx, pval, poff = [], [], [0]
    for i, (rid, t, k, p, seed_i) in enumerate(cases):
        row = logits[rid]
        ref = ref_sample_token(row, RefParams(temperature=t, top_k=k, top_p=p), torch.Generator().manual_seed(seed_i))
        port = torch_port.sample_row(row, t, k, p, torch.Generator().manual_seed(seed_i))
        assert ref == port, f"torch port disagrees with the reference on {prefix} case {i}"
        kp, pr, mg, tc = masked_info(row, t, k, p)
        kept[i] = kp
        pos = np.flatnonzero(kp)
        if pos.size > PROB_ALL:
            top = pos[np.argsort(-pr[pos], kind="stable")[:PROB_TOP]]
            rest = np.setdiff1d(pos, top)
            pos = np.sort(np.concatenate([top, rng.choice(rest, PROB_ALL - PROB_TOP, replace=False)]))
        pidx.append(pos.astype(np.int32))
        pval.append(pr[pos].astype(np.float32))
        poff.append(poff[-1] + pos.size)
        for c, v in [("row", rid), ("temp", t), ("topk", k), ("topp", p), ("seed", seed_i), ("ref_token", ref),
                     ("port_token", port), ("margin", mg), ("tie_cut", tc), ("kept_n", int(kp.sum()))]:
            cols[c][i] = v
    out = {f"{prefix}_kept": np.packbits(kept, axis=1), f"{prefix}_probs_idx": np.concatenate(pidx),
           f"{prefix}_probs": np.concatenate(pval), f"{prefix}_probs_off": np.array(poff, np.int64)}
    out.update({f"{prefix}_{c}": v for c, v in cols.items()})
    return out


# top_p values just below 1.0 in float64: the first three round to 1.0 in fp32 (the reference
# still takes its top-p branch, sampling.py:18, since the Python compare is in float64), the last
# is the largest fp32 below 1.0
P_NEAR_ONE = (1.0 - 2.0**-30, 1.0 - 2.0**-25, 0.99999999, 1.0 - 2.0**-24)


def big_fixtures() -> dict:
    out = {}
    w2 = workloads.config2(seed=0)
    out["cfg2_sha256"] = _digest(w2.logits)
    cases = [(r, w2.params[r].temperature, w2.params[r].top_k, w2.params[r].top_p, w2.seeds[r]) for r in range(32)]
    out.update(pack_big(w2.logits, cases, "cfg2"))
    del w2
    wf = workloads.config2_flat(seed=0)
    out["cfg2flat_sha256"] = _digest(wf.logits)
    cases = [(r, wf.params[r].temperature, wf.params[r].top_k, wf.params[r].top_p, wf.seeds[r]) for r in range(16)]
    out.update(pack_big(wf.logits, cases, "cfg2flat"))
    del wf
    w1 = workloads.config1(seed=0)
    out["cfg1_sha256"] = _digest(w1.logits)
    cases = [(r, sp.temperature, sp.top_k, sp.top_p, w1.seeds[r]) for r, sp in enumerate(w1.params)]
    out.update(pack_big(w1.logits, cases, "cfg1"))
    del w1
    w0 = workloads.config0(seed=0)
    cases = []
    for j, p in enumerate(P_NEAR_ONE):
        for r in range(w0.rows):
            t, k = ((1.0, 0), (0.8, 50), (1.0, 0), (1.3, 1000))[(j + r) % 4]
            cases.append((r, t, k, p, 1000 + 8 * j + r))
    out["p1_sha256"] = _digest(w0.logits)
    out.update(pack_big(w0.logits, cases, "p1"))
    return out


def main(which: str = "all"):
    if which in ("small", "all"):
        out = {}
        rows, cases = small_cases()
        out.update(pack_cases(rows, cases, "small"))
        w = workloads.config0(seed=0)
        out["cfg0_sha256"] = np.frombuffer(hashlib.sha256(w.logits.numpy().tobytes()).digest(), np.uint8)
        cfg_rows = [w.logits[r] for r in range(w.rows)]
        cfg_cases = [(r, sp.temperature, sp.top_k, sp.top_p, w.seeds[r]) for r, sp in enumerate(w.params)]
        cfg_cases += [(r, 0.0, 0, 1.0, 0) for r in range(w.rows)]
        packed = pack_cases(cfg_rows, cfg_cases, "cfg0")
        del packed["cfg0_logits"]  # regenerated from the seed by the tests
        out.update(packed)
        path = os.path.join(HERE, "golden.npz")
        np.savez_compressed(path, **out)
        print(f"wrote {path}: {len(cases)} small cases over {len(rows)} rows, {len(cfg_cases)} config-0 cases, "
              f"{os.path.getsize(path)/1e6:.2f} MB")
    if which in ("big", "all"):
        out = big_fixtures()
        path = os.path.join(HERE, "golden_big.npz")
        np.savez_compressed(path, **out)
        n = {g: len(out[f"{g}_temp"]) for g in ("cfg2", "cfg2flat", "cfg1", "p1")}
        print(f"wrote {path}: {n}, {os.path.getsize(path)/1e6:.2f} MB")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "all")
