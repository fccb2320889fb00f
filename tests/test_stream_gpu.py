"""The persistent streaming kernel (greedy rows and top-k rows with top_k <= 128) on a B200.

pb_sample runs it first and the cluster kernel after it, on the rows it does not take or could not
settle. These tests check, against the CPU oracle bit for bit, that the rows it takes are settled by
it (info flag PB_PATH_STREAM) and that the rows it hands back come out right: many rows per CTA,
mixed modes in one batch, unaligned and short rows, NaN rows, candidate overflow, tie groups larger
than the finisher orders, the shard records of the vocabulary-parallel mode, and the bounded-wait
path (every wait on a staged chunk made to give up, which must end in PB_ROW_TIMEOUT and leave the
device usable).
"""

import os

import numpy as np
import pytest
import torch

import oracle
from pagedbatch_b200 import _lib, ops, workloads

from parity_helpers import _check, rec_for, run_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _env(cuda):
    os.environ["PB_PATH"] = "stream"  # whatever the batch size, the streaming kernel goes first
    yield
    for k in ("PB_PATH", "PB_WS", "PB_TEST_STAGE_POLLS", "PB_NO_PDL"):
        os.environ.pop(k, None)


def _eligible(rec, V):
    t, k, p, u = rec["temperature"], rec["top_k"], rec["top_p"], rec["uniform"]
    good = (t >= 0) & (p > 0) & (p <= 1) & (k >= 0)
    return good & ((t == 0) | ((k > 0) & (k <= 128) & (k < V) & (u >= 0) & (u < 1)))


def _run(x_cpu, rec, row_index=None, label=""):
    dev = x_cpu.cuda()
    g_tok, g_info, _ = run_gpu(dev, rec, row_index, probs=False)
    o_tok, o_info, _ = oracle.sample(x_cpu, rec, row_index)
    _check(g_tok, g_info, o_tok, o_info, label)
    return g_tok, g_info


def test_headline_rows_are_settled_by_the_streaming_kernel():
    w = workloads.config2()
    rec = rec_for(w.params, w.uniforms())
    _, info = _run(w.logits, rec, label="cfg2 stream")
    assert np.all(info["flags"] & _lib.PATH_STREAM), "every config-2 row belongs to the streaming kernel"


@pytest.mark.parametrize("pdl", [True, False])
def test_mixed_batch_many_rows_per_cta(pdl):
    if not pdl:
        os.environ["PB_NO_PDL"] = "1"
    rng = np.random.default_rng(3)
    B, V = 700, 20011  # ~5 rows per CTA, odd vocabulary (a scalar tail)
    x = workloads.head_boosted(B, V, seed=9)
    t = rng.choice([0.0, 0.5, 0.7, 1.0, 1.3], B)
    k = rng.choice([0, 1, 2, 20, 50, 64, 100, 128, 129, 1000], B)
    p = rng.choice([1.0, 0.5, 0.9, 0.95, 1e-6], B)
    rec = oracle.make_params(t, p, k, rng.random(B))
    _, info = _run(x, rec, label="mixed 700")
    el = _eligible(rec, V)
    assert np.all((info["flags"][el] & _lib.PATH_STREAM) != 0)
    assert not np.any(info["flags"][~el] & _lib.PATH_STREAM)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_short_unaligned_rows_and_row_index(dtype):
    rng = np.random.default_rng(11)
    for V in (2, 5, 17, 130, 1001, 8193, 32769):
        B = 40
        base = workloads.head_boosted(B, V + 7, seed=V).to(dtype)
        x = base[:, 3 : 3 + V]  # row starts off the 16-byte grid; stride V + 7
        k = rng.choice([1, 2, min(V - 1, 50), min(V - 1, 128)], B)
        t = rng.choice([0.0, 0.8, 1.0], B)
        rec = oracle.make_params(t, rng.choice([1.0, 0.9], B), k, rng.random(B))
        dev = base.cuda()[:, 3 : 3 + V]
        g_tok, g_info, _ = run_gpu(dev, rec, probs=False)
        o_tok, o_info, _ = oracle.sample(x.contiguous(), rec)
        _check(g_tok, g_info, o_tok, o_info, f"unaligned V={V} {dtype}")
        sel = rng.integers(0, B, 25).astype(np.int32)
        g_tok, g_info, _ = run_gpu(dev, rec[:25], sel, probs=False)
        o_tok, o_info, _ = oracle.sample(x.contiguous(), rec[:25], sel)
        _check(g_tok, g_info, o_tok, o_info, f"row_index V={V} {dtype}")


def test_rows_it_hands_back():
    """NaN / inf / all -inf rows, rising rows (candidate overflow), tie groups beyond what the
    finisher orders: marked by the streaming kernel, settled by the cluster kernel."""
    V = 50000
    x = workloads.head_boosted(10, V, seed=4)
    x[0, 77] = float("nan")  # greedy row with a NaN: the first NaN wins
    x[0, 99] = float("nan")
    x[1, 5] = float("nan")
    x[2, 9] = float("inf")
    x[3, :] = float("-inf")
    x[4] = torch.arange(V, dtype=torch.float32)  # rising: every chunk passes the threshold
    x[5, :] = 2.0  # one value: the tie group is the whole row
    x[6, :1000] = 7.0  # 1000 ties above everything else
    x[7, 40000:] = float("-inf")
    rec = oracle.make_params([0.0, 0.7, 0.7, 0.7, 1.0, 1.0, 1.0, 1.0, 0.0, 1.0], [1.0, 0.9, 1.0, 1.0, 0.9, 1.0, 0.5, 0.9, 1.0, 0.95],
                             [0, 50, 50, 50, 50, 128, 100, 20, 0, 128], np.linspace(0.05, 0.95, 10))
    tok, info = _run(x, rec, label="handed back")
    assert list(info["status"][:4]) == [0, 1, 1, 1]
    assert tok[0] == 77


def test_shard_records_match_the_cluster_kernel():
    """pb_candidates through the streaming kernel writes the same records (header, and the same set
    of entries) as the cluster kernel alone."""
    from pagedbatch_b200.vocab_parallel import CudaKernels, record_cap

    w = workloads.config3(rows=300)
    x = w.logits.cuda()
    rec = rec_for(w.params, w.uniforms())
    rec["temperature"][::7] = 0.0
    params = [type(w.params[0])(temperature=float(t), top_k=int(k), top_p=float(p))
              for t, k, p in zip(rec["temperature"], rec["top_k"], rec["top_p"])]
    dparams = ops.params_tensor(rec, x.device)
    cap = record_cap(params)
    kern = CudaKernels()
    V = x.shape[1]
    for lo, hi in ((0, V // 2), (V // 2, V), (V // 8, V // 8 + V // 8)):
        a = kern.candidates(x[:, lo:hi], dparams, lo, cap).cpu().numpy()
        os.environ["PB_PATH"] = "cluster"
        b = kern.candidates(x[:, lo:hi], dparams, lo, cap).cpu().numpy()
        os.environ["PB_PATH"] = "stream"
        rb = _lib.record_bytes(cap)
        for r in range(a.shape[0]):
            ha = a[r, :16].view(_lib.CAND_HEADER)[0]
            hb = b[r, :16].view(_lib.CAND_HEADER)[0]
            assert tuple(ha) == tuple(hb), (r, ha, hb)
            n = int(ha["count"])
            ea = np.sort(a[r, 16 : 16 + 8 * n].view(np.uint64))
            eb = np.sort(b[r, 16 : 16 + 8 * n].view(np.uint64))
            assert np.array_equal(ea, eb), r
        assert a.shape[1] == rb


def test_bounded_wait_gives_up_and_reports_timeout():
    """Every consumer wait on a staged chunk gives up at once (PB_TEST_STAGE_POLLS=0): the CTAs stop,
    let their issued copies land and report PB_ROW_TIMEOUT for their rows; rows the streaming kernel
    does not take are still sampled; the next call (normal waits) is correct."""
    w = workloads.config1(rows=64)
    rec = rec_for(w.params, w.uniforms())
    x = w.logits.cuda()
    os.environ["PB_TEST_STAGE_POLLS"] = "0"
    tok, info, _ = run_gpu(x, rec, probs=False)
    el = _eligible(rec, x.shape[1])
    assert np.all(info["status"][el] == _lib.ROW_TIMEOUT) and np.all(tok[el] == -1)
    o_tok, o_info, _ = oracle.sample(w.logits, rec)
    assert np.array_equal(tok[~el], o_tok[~el])
    os.environ.pop("PB_TEST_STAGE_POLLS")
    torch.cuda.synchronize()
    tok, info, _ = run_gpu(x, rec, probs=False)
    _check(tok, info, o_tok, o_info, "after timeout")


def test_balanced_bounded_wait_gives_up_and_reports_timeout():
    """The same with pb_sample_ws, whose rows are cut into pieces over neighbouring CTAs: a piece whose
    CTA gave up still arrives (with a timed-out record), so every split row reports PB_ROW_TIMEOUT,
    its arrival counter completes, and the next call (normal waits) over the same workspace is right."""
    os.environ["PB_PATH"] = "ws"
    os.environ["PB_WS"] = "balanced"  # the balanced streaming launch (the two-pass launch never waits)
    w = workloads.config1(rows=64)
    rec = rec_for(w.params, w.uniforms())
    x = w.logits.cuda()
    os.environ["PB_TEST_STAGE_POLLS"] = "0"
    tok, info, _ = run_gpu(x, rec, probs=False)
    el = _eligible(rec, x.shape[1])
    assert np.all(info["status"][el] == _lib.ROW_TIMEOUT) and np.all(tok[el] == -1)
    o_tok, o_info, _ = oracle.sample(w.logits, rec)
    assert np.array_equal(tok[~el], o_tok[~el])
    os.environ.pop("PB_TEST_STAGE_POLLS")
    torch.cuda.synchronize()
    for _ in range(2):
        tok, info, _ = run_gpu(x, rec, probs=False)
        _check(tok, info, o_tok, o_info, "balanced, after timeout")
