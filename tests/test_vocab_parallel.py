"""Vocabulary-parallel sampling, host side: the record layout and the exchange protocol.

Two gloo ranks on the CPU each hold a column slice (uneven widths) of the same rows and run
``sample_tokens_vocab_parallel`` with stand-in kernels built on the oracle: shard candidates as
the C ABI specifies them, a merge that rebuilds each row from the exchanged candidates only, and
full-row sampling for fallback rows. Both ranks must return the oracle's full-row tokens. The
CUDA kernels themselves are checked against the full-row sampler in test_parity_gpu.py.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from pagedbatch_b200 import SamplingParams, _lib
from pagedbatch_b200.vocab_parallel import record_cap, sample_tokens_vocab_parallel

B, V, SPLIT = 12, 1001, 437  # rank 0 holds columns [0, 437), rank 1 [437, 1001)


def _keys(x: np.ndarray, t: float) -> np.ndarray:
    return oracle.key_of(oracle.scaled_keys(x, t) if t != 0 else x)


def _compose(key: int, idx: int) -> int:
    return (int(key) << 32) | (0xFFFFFFFF - int(idx))


class OracleKernels:
    """Stand-ins with the C ABI's record semantics, on the CPU."""

    def __init__(self, full: np.ndarray):
        self.full = full  # the whole rows, used only to rebuild rows from exchanged candidates

    def candidates(self, logits, dparams, vocab_offset, cap):
        prm = dparams.numpy().view(_lib.ROW_PARAMS)
        x = logits.numpy()
        rb = _lib.record_bytes(cap)
        out = np.zeros((x.shape[0], rb), np.uint8)
        for r in range(x.shape[0]):
            t, k = float(prm["temperature"][r]), int(prm["top_k"][r])
            hdr = out[r, :16].view(_lib.CAND_HEADER)
            ent = out[r, 16:].view(np.uint64)
            keys = _keys(x[r], t)
            if t == 0:
                i = int(np.argmax(keys))
                hdr["count"], hdr["flags"], hdr["max_key"] = 1, _lib.CAND_GREEDY, x[r, i]
                ent[0] = _compose(keys[i], i + vocab_offset)
                continue
            hdr["max_key"] = np.float32(np.float32(x[r].max()) / np.float32(t))
            if not 0 < k < x.shape[1]:
                hdr["flags"] = _lib.CAND_FALLBACK
                continue
            kth = np.sort(keys)[::-1][k - 1]
            sel = np.flatnonzero(keys >= kth)
            if sel.size > cap:
                hdr["flags"] = _lib.CAND_FALLBACK
                continue
            hdr["count"] = sel.size
            for j, i in enumerate(sel):
                ent[j] = _compose(keys[i], i + vocab_offset)
        return torch.from_numpy(out)

    def merge(self, records, dparams, cap):
        recs = records.numpy()
        prm = dparams.numpy().view(_lib.ROW_PARAMS)
        n, b = recs.shape[0], recs.shape[1]
        tokens = np.full(b, -1, np.int64)
        info = np.zeros(b, _lib.ROW_INFO)
        for r in range(b):
            hdrs = [recs[s, r, :16].view(_lib.CAND_HEADER)[0] for s in range(n)]
            ents = [recs[s, r, 16:].view(np.uint64)[: hdrs[s]["count"]] for s in range(n)]
            if any(h["flags"] & _lib.CAND_FALLBACK for h in hdrs):
                info["status"][r] = _lib.ROW_FALLBACK
                continue
            if prm["temperature"][r] == 0:
                best = max(int(e[0]) for e in ents)
                tokens[r] = 0xFFFFFFFF - (best & 0xFFFFFFFF)
                continue
            # rebuild the row from the exchanged candidates alone
            row = np.full(self.full.shape[1], -np.inf, np.float32)
            for e in ents:
                idx = 0xFFFFFFFF - (e.astype(np.int64) & 0xFFFFFFFF)
                row[idx] = self.full[r, idx]
            tok, inf, _ = oracle.sample(torch.from_numpy(row[None]), prm[r : r + 1])
            tokens[r], info[r] = tok[0], inf[0]
        return torch.from_numpy(tokens), torch.from_numpy(info.view(np.uint8).reshape(b, -1).copy())

    def sample_full(self, logits, dparams):
        tok, inf, _ = oracle.sample(logits, dparams.numpy().view(_lib.ROW_PARAMS))
        return torch.from_numpy(tok), torch.from_numpy(inf.view(np.uint8).reshape(len(tok), -1).copy())


def _rows():
    x = torch.randn(B, V, generator=torch.Generator().manual_seed(3)) * 3.0
    x[:, 700] += 9.0  # a clear leader on rank 1's side
    params = [
        SamplingParams(temperature=0.0),
        SamplingParams(temperature=0.0),
        SamplingParams(temperature=0.7, top_k=50, top_p=0.95),
        SamplingParams(temperature=1.0, top_k=5),
        SamplingParams(temperature=1.3, top_k=64, top_p=0.5),
        SamplingParams(temperature=1.0, top_k=1),
        SamplingParams(temperature=1.0),  # top-k off: full-row fallback
        SamplingParams(temperature=0.8, top_p=0.9),  # top-k off: full-row fallback
        SamplingParams(temperature=1.0, top_k=500),  # k above rank 0's width: fallback
        SamplingParams(temperature=0.5, top_k=20, top_p=0.99),
        SamplingParams(temperature=2.0, top_k=200),
        SamplingParams(temperature=1.0, top_k=10, top_p=1e-6),
    ]
    x[1, 5] = x[1].max() + 1.0  # greedy leader on rank 0's side
    return x, params


def _worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        x, params = _rows()
        local = (x[:, :SPLIT] if rank == 0 else x[:, SPLIT:]).contiguous()
        gens = [torch.Generator().manual_seed(i) for i in range(B)]
        toks = sample_tokens_vocab_parallel(local, params, gens, kernels=OracleKernels(x.numpy()))
        q.put((rank, toks))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_two_gloo_ranks_match_full_rows():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, params = _rows()
    gens = [torch.Generator().manual_seed(i) for i in range(B)]
    u = [float(torch.rand((), dtype=torch.float64, generator=g)) if p.temperature else 0.0
         for p, g in zip(params, gens)]
    rec = oracle.make_params([p.temperature for p in params], [p.top_p for p in params],
                             [p.top_k for p in params], u)
    want, _, _ = oracle.sample(x, rec)
    assert got[0] == got[1] == want.tolist()


def test_record_layout_and_cap():
    assert _lib.record_bytes(64) == 16 + 8 * 64
    assert record_cap([SamplingParams(temperature=1.0, top_k=64)]) == 160
    assert record_cap([SamplingParams(temperature=0.0, top_k=4000)]) == 64
    assert record_cap([SamplingParams(temperature=1.0, top_k=5000)]) == _lib.CAND_MAX_CAP


@pytest.mark.parametrize("bad", [0, _lib.CAND_MAX_CAP + 1])
def test_candidates_rejects_bad_cap(bad):
    L = _lib.load()
    rc = L.pb_candidates(None, 0, 1, 10, 10, None, None, 0, bad, None, None)
    assert rc == -1  # PB_E_INVALID, returned before any device work


def _worker_fail(rank, port, q, mode):
    """Two steps; between them rank 1 leaves ("exit") or stalls past the group's timeout ("stall").
    Rank 0's second step must end with an error, not hang."""
    import datetime
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=4))
    x, params = _rows()
    local = (x[:, :SPLIT] if rank == 0 else x[:, SPLIT:]).contiguous()
    kern = OracleKernels(x.numpy())
    gens = [torch.Generator().manual_seed(i) for i in range(B)]
    sample_tokens_vocab_parallel(local, params, gens, kernels=kern)  # step 1, every rank
    if rank == 1:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()  # (os._exit below skips the queue's flush)
        if mode == "stall":
            time.sleep(12)  # (longer than the group's timeout; no collective in flight)
        os._exit(0)  # between steps: nothing of this rank is in flight
    t0 = time.monotonic()
    try:
        sample_tokens_vocab_parallel(local, params, gens, kernels=kern)
        q.put((rank, "returned", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - any error ends the step; the test reads its kind
        q.put((rank, f"raised {type(e).__name__}", time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_surviving_rank_raises_when_a_peer_leaves(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_fail, args=(r, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1][0] == "left"
    what, dt = got[0]
    assert what.startswith("raised"), what
    assert dt < 60.0
