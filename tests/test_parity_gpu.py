"""Kernel parity: the sm_100a sampler (through the C ABI) against the CPU oracle, bit for bit.

Every comparison is exact: tokens, the kept-set description (threshold key, tie count, kept
count), the fixed-point masses, the status, and the float32 probabilities (same operations on both
sides, so the same bits). Covers the golden rows, the benchmark configurations at full size,
odd vocabularies, unaligned rows, row selection, every dtype, every cluster size, tie groups
larger than the gather buffer, k above the streamed-candidate limit, and non-finite rows.
"""

import os

import numpy as np
import pytest
import torch

import oracle
from pagedbatch_b200 import _lib, ops, workloads
from parity_helpers import INFO_FIELDS, _check, compare, rec_for, run_gpu  # noqa: F401

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda(cuda):
    yield
    os.environ.pop("PB_CLUSTER", None)
    os.environ.pop("PB_BALANCED_GRID", None)
    os.environ.pop("PB_PATH", None)
    os.environ.pop("PB_WS", None)


def test_golden_rows(golden):
    rows = golden["small_logits"]
    vocab = golden["small_vocab"]
    n = len(golden["small_temp"])
    rng = np.random.default_rng(1)
    for V in np.unique(vocab):
        idx = np.flatnonzero(vocab[golden["small_row"]] == V)
        x = torch.from_numpy(np.ascontiguousarray(rows[:, :V]))
        rec = oracle.make_params(golden["small_temp"][idx], golden["small_topp"][idx], golden["small_topk"][idx],
                                 rng.random(idx.size))
        for bf in (False, True):
            xx = x.to(torch.bfloat16) if bf else x
            compare(xx, rec, golden["small_row"][idx], label=f"golden V={V} bf16={bf}")
    assert n > 900


@pytest.mark.parametrize("cluster", ["1", "2", "4", "8"])
def test_cluster_sizes_and_modes(cluster):
    os.environ["PB_CLUSTER"] = cluster
    rng = np.random.default_rng(int(cluster))
    for V in (1, 3, 17, 258, 4099, 49152):
        B = 24
        x = workloads.head_boosted(B, V, seed=V)
        t = rng.choice([0.0, 0.5, 0.7, 1.0, 1.5], B)
        k = rng.choice([0, 1, 2, 20, 50, 1000, 2000, max(1, V - 1), V], B)
        p = rng.choice([1.0, 0.5, 0.9, 0.99, 0.999, 1e-6], B)
        u = rng.random(B)
        u[:2] = [0.0, np.nextafter(1.0, 0.0)]
        compare(x, oracle.make_params(t, p, k, u), label=f"C={cluster} V={V}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_unaligned_rows_and_row_index(dtype):
    rng = np.random.default_rng(7)
    V, B = 1001, 16
    base = workloads.head_boosted(B, V + 5, seed=3).to(dtype)
    x = base[:, 3 : 3 + V]  # row starts not 16-byte aligned, stride V+5
    rec = oracle.make_params(rng.choice([0.0, 1.0], B), rng.choice([1.0, 0.9], B), rng.choice([0, 20], B), rng.random(B))
    dev = base.cuda()[:, 3 : 3 + V]
    g_tok, _, g_pr = run_gpu(dev, rec)
    o_tok, _, o_pr = oracle.sample(x.contiguous(), rec, want_probs=True)
    assert np.array_equal(g_tok, o_tok)
    assert np.array_equal(g_pr.view(np.uint32), o_pr.view(np.uint32))
    sel = np.array([5, 5, 0, 15, 2], np.int32)
    rec2 = rec[: len(sel)]
    g_tok, _, _ = run_gpu(dev, rec2, sel, probs=False)
    o_tok, _, _ = oracle.sample(x.contiguous(), rec2, sel)
    assert np.array_equal(g_tok, o_tok)


def test_config0():
    w = workloads.config0()
    compare(w.logits, rec_for(w.params, w.uniforms()), label="cfg0")


def test_config1_mixed_bf16():
    w = workloads.config1()
    tok, info = compare(w.logits, rec_for(w.params, w.uniforms()), label="cfg1")
    # greedy rows with planted duplicate maxima: lowest index wins
    x = w.logits.float().numpy()
    for r in range(64):
        assert tok[r] == int(np.flatnonzero(x[r] == x[r].max())[0])


def test_config2_headline():
    w = workloads.config2()
    compare(w.logits, rec_for(w.params, w.uniforms()), probs=False, label="cfg2")


def test_config2_flat_worst_case():
    w = workloads.config2_flat()
    compare(w.logits, rec_for(w.params, w.uniforms()), probs=False, label="cfg2flat")


@pytest.mark.parametrize("cluster", ["1", "2"])
def test_long_rows(cluster):
    """Rows far longer than the TMA ring, bf16 and fp32, k up to the small-path limit."""
    os.environ["PB_CLUSTER"] = cluster
    rng = np.random.default_rng(11)
    for V, dtype in ((300_001, torch.float32), (600_000, torch.bfloat16)):
        x = workloads.head_boosted(4, V, seed=V).to(dtype)
        rec = oracle.make_params([0.7, 1.0, 1.0, 1.3], [0.95, 1.0, 0.9, 1.0], [50, 1000, 7, 1024], rng.random(4))
        compare(x, rec, label=f"long V={V} C={cluster}")


@pytest.mark.parametrize("cluster", ["1", "8"])
def test_rows_with_fewer_finite_values_than_k(cluster):
    """The k-th value is -inf: every -inf element is kept (weight 0) and none is ever drawn."""
    os.environ["PB_CLUSTER"] = cluster
    rng = np.random.default_rng(5)
    V = 4099
    x = torch.full((4, V), float("-inf"))
    for r, n in enumerate((1, 37, 500, 999)):
        cols = torch.from_numpy(rng.choice(V, n, replace=False))
        x[r, cols] = torch.randn(n, generator=torch.Generator().manual_seed(r)) * 2.0
    rec = oracle.make_params([1.0, 0.7, 1.0, 1.3], [1.0, 0.9, 1.0, 0.5], [1000, 1000, 1000, 1000], rng.random(4))
    tok, info = compare(x, rec, label=f"sparse-finite C={cluster}")
    assert np.all(np.isfinite(x.numpy()[np.arange(4), tok]))


def test_large_tie_groups():
    """Rows with one repeated value (tie groups far above the gather buffer) and few distinct values."""
    V = 20000
    x = torch.zeros(6, V)
    x[1, ::3] = 1.0
    x[2] = torch.randint(0, 3, (V,), generator=torch.Generator().manual_seed(0)).float()
    x[3, 100] = 5.0
    x[4] = (torch.arange(V) % 7).float()
    x[5, :] = -1.0
    rng = np.random.default_rng(3)
    for t, k, p in [(1.0, 0, 1.0), (1.0, 0, 0.5), (0.5, 5000, 1.0), (1.0, 10000, 0.3), (0.0, 0, 1.0), (1.0, 7, 0.99)]:
        rec = oracle.make_params([t] * 6, [p] * 6, [k] * 6, rng.random(6))
        for c in ("1", "4"):
            os.environ["PB_CLUSTER"] = c
            compare(x, rec, label=f"ties t={t} k={k} p={p} C={c}")


def test_nonfinite_and_bad_uniform_rows():
    x = torch.randn(6, 300)
    x[0, 5] = float("nan")
    x[1, 7] = float("inf")
    x[2, :] = float("-inf")
    x[3, 10] = float("-inf")
    rec = oracle.make_params([1.0, 1.0, 1.0, 1.0, 1.0, 0.0], [1.0] * 6, [0, 0, 0, 10, 0, 0], [0.5] * 6)
    rec["uniform"][4] = 1.0  # outside [0, 1)
    tok, info = compare(x, rec, label="nonfinite")
    assert list(info["status"]) == [1, 1, 1, 0, 2, 0]
    # greedy with NaN: the first NaN wins, like torch.argmax; an all -inf row picks index 0
    x2 = torch.tensor([[1.0, float("nan"), 3.0, float("nan")], [float("-inf")] * 4, [-0.0, 0.0, -1.0, 0.0]])
    tok, _ = compare(x2, oracle.make_params([0.0] * 3, [1.0] * 3, [0] * 3, [0.0] * 3), label="greedy edge")
    assert list(tok) == [1, 0, 0]


def test_rejected_parameters_report_status():
    x = torch.randn(4, 100)
    rec = oracle.make_params([-1.0, 1.0, 1.0, float("nan")], [1.0, 0.0, 1.5, 1.0], [0, 0, 0, 0], [0.5] * 4)
    tok, info = compare(x, rec, label="bad params")
    assert list(info["status"]) == [16, 16, 16, 16] and list(tok) == [-1] * 4
    rec = oracle.make_params([1.0], [1.0], [-3], [0.5])
    tok, info = compare(x[:1], rec, label="bad top_k")
    assert info["status"][0] == 16


def test_reference_primitives_through_dropin():
    """pagedbatch tests/test_engine.py:86-93, unchanged in substance, on the B200 path."""
    from pagedbatch_b200 import SamplingParams, sample_token

    g = torch.Generator().manual_seed(0)
    logits = torch.tensor([0.1, 3.0, 0.2, 2.9])
    assert sample_token(logits, SamplingParams(temperature=0.0), g) == 1
    assert sample_token(logits, SamplingParams(temperature=1.0, top_k=1), g) == 1
    assert sample_token(logits, SamplingParams(temperature=1.0, top_p=1e-6), g) == 1
    picks = {sample_token(logits, SamplingParams(temperature=1.0, top_k=2), g) for _ in range(50)}
    assert picks <= {1, 3}


def test_seeded_sampling_is_reproducible():
    from pagedbatch_b200 import SamplingParams, sample_tokens

    w = workloads.config1(rows=32)
    x = w.logits.cuda()
    p = [SamplingParams(temperature=1.0, top_p=0.9, seed=7)] * 32
    a = sample_tokens(x, p, [torch.Generator().manual_seed(7) for _ in range(32)])
    b = sample_tokens(x, p, [torch.Generator().manual_seed(7) for _ in range(32)])
    assert a == b
    with pytest.raises(RuntimeError, match="nan"):
        sample_tokens(torch.full((1, 8), float("nan"), device="cuda"), [SamplingParams()], [torch.Generator()])


@pytest.mark.parametrize("n_shards", [2, 4, 8])
def test_vocab_parallel_shards_match_full_rows(n_shards):
    """Shard candidates + merge (one GPU standing in for N shards) equal the full-row sampler."""
    from pagedbatch_b200 import SamplingParams
    from pagedbatch_b200.vocab_parallel import CudaKernels, record_cap

    kern = CudaKernels()
    cases = []
    w3 = workloads.config3(rows=128)
    cases.append((w3.logits, w3.params, w3.uniforms()))
    w1 = workloads.config1(rows=64)
    cases.append((w1.logits, w1.params, w1.uniforms()))
    x = workloads.head_boosted(8, 9001, seed=9)
    x[3, ::5] = 2.5  # a large tie group
    ps = [SamplingParams(temperature=t, top_k=k, top_p=p) for t, k, p in
          [(0.7, 50, 0.95), (1.0, 1, 1.0), (0.0, 0, 1.0), (1.0, 64, 0.9), (1.3, 200, 0.5), (0.5, 20, 1e-6),
           (1.0, 0, 0.9), (2.0, 7, 1.0)]]
    cases.append((x, ps, list(np.random.default_rng(4).random(8))))
    for logits, params, u in cases:
        dev = logits.cuda()
        B, V = dev.shape
        rec = oracle.make_params([p.temperature for p in params], [p.top_p for p in params],
                                 [p.top_k for p in params], u)
        dparams = ops.params_tensor(rec, dev.device)
        cap = record_cap(params)
        bounds = [V * s // n_shards for s in range(n_shards + 1)]
        recs = [kern.candidates(dev[:, bounds[s]:bounds[s + 1]], dparams, bounds[s], cap) for s in range(n_shards)]
        tok, info = kern.merge(torch.stack(recs), dparams, cap)
        g_tok = tok.cpu().numpy()
        g_info = ops.info_records(info)
        f_tok, f_info, _ = ops.sample(dev, dparams, None, with_info=True)
        f_tok = f_tok.cpu().numpy()
        f_info = ops.info_records(f_info)
        fb = g_info["status"] == _lib.ROW_FALLBACK
        ks = np.array([p.top_k for p in params])
        greedy = np.array([p.temperature == 0 for p in params])
        assert not fb[greedy].any()
        assert fb[(ks == 0) & ~greedy].all()
        ok = ~fb
        assert np.array_equal(g_tok[ok], f_tok[ok]), (np.flatnonzero(g_tok[ok] != f_tok[ok]))
        for f in INFO_FIELDS:
            assert np.array_equal(g_info[f][ok], f_info[f][ok]), f
        assert np.array_equal(g_info["max_key"][ok], f_info["max_key"][ok], equal_nan=True)
        if logits is w3.logits:
            assert not fb.any()  # config 3 (top_k 64) never needs full rows


def test_vocab_parallel_api_one_rank_nccl():
    """The public entry through a real (one-rank) NCCL group, against sample_tokens."""
    import socket

    import torch.distributed as dist

    from pagedbatch_b200 import sample_tokens
    from pagedbatch_b200.vocab_parallel import sample_tokens_vocab_parallel

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        w = workloads.config1(rows=32)
        x = w.logits.cuda()
        a = sample_tokens_vocab_parallel(x, w.params, w.generators())
        b = sample_tokens(x, w.params, w.generators())
        assert a == b
    finally:
        dist.destroy_process_group()


def _ws_kernel(ws):
    """pb_sample_ws's launch: "groups" (the two passes over group keys; its default for 16-byte
    aligned rows) or "balanced" (the balanced streaming launch)."""
    os.environ["PB_PATH"] = "ws"
    if ws == "balanced":
        os.environ["PB_WS"] = "balanced"
    else:
        os.environ.pop("PB_WS", None)


WS_KERNELS = ["groups", "balanced"]


@pytest.mark.parametrize("ws,grid", [("balanced", "1"), ("balanced", "3"), ("balanced", "16"), ("balanced", "148"),
                                     ("groups", "148")])
def test_balanced_path_modes_and_edges(ws, grid):
    """pb_sample_ws (either launch, then the cluster kernel on the rest) against the oracle; for the
    balanced launch with the grid capped so rows are cut into different numbers of pieces. Rows
    whose bytes are not a multiple of 16 take the balanced launch in any case (the two passes read
    whole 16-byte vectors from each row's start)."""
    _ws_kernel(ws)
    os.environ["PB_BALANCED_GRID"] = grid
    rng = np.random.default_rng(20 + int(grid))
    for V in (1, 3, 17, 258, 4099, 49152, 128256):
        B = 24
        x = workloads.head_boosted(B, V, seed=V)
        t = rng.choice([0.0, 0.5, 0.7, 1.0, 1.5], B)
        k = rng.choice([0, 1, 2, 20, 50, 128, 129, 512, 1000, max(1, V - 1), V], B)
        p = rng.choice([1.0, 0.5, 0.9, 0.99, 1e-6], B)
        u = rng.random(B)
        u[:2] = [0.0, np.nextafter(1.0, 0.0)]
        compare(x, oracle.make_params(t, p, k, u), probs=False, label=f"balanced grid={grid} V={V}")
    x = torch.randn(7, 60000)
    x[0, 5] = float("nan")
    x[1, 40007] = float("inf")
    x[2, :] = float("-inf")
    x[3, 300:] = float("-inf")
    x[4, :] = 1.0
    x[6, 100:] = float("-inf")
    x[6, 59000] = float("nan")
    rec = oracle.make_params([1.0, 1.0, 1.0, 1.0, 0.0, 1.0, 0.0], [1.0] * 7, [10, 10, 10, 10, 0, 10, 0], [0.5] * 7)
    rec["uniform"][5] = 1.0
    compare(x, rec, probs=False, label=f"balanced nonfinite grid={grid}")
    x2 = torch.full((4, 40000), float("-inf"))
    x2[0, 1] = float("nan")
    x2[0, 30000] = float("nan")
    x2[2] = 0.0
    x2[2, ::2] = -0.0
    x2[3, 39999] = 2.0
    x2[3, 20000] = 2.0
    compare(x2, oracle.make_params([0.0] * 4, [1.0] * 4, [0] * 4, [0.0] * 4), probs=False,
            label=f"balanced greedy edge grid={grid}")
    rec = oracle.make_params([-1.0, 1.0, 1.0, float("nan")], [1.0, 0.0, 1.5, 1.0], [0, 0, 0, 0], [0.5] * 4)
    compare(torch.randn(4, 100), rec, probs=False, label="balanced bad params")


@pytest.mark.parametrize("ws", WS_KERNELS)
def test_balanced_path_configs_and_row_index(ws):
    _ws_kernel(ws)
    for w in (workloads.config0(), workloads.config1(), workloads.config2(), workloads.config3(rows=300)):
        compare(w.logits, rec_for(w.params, w.uniforms()), probs=False, label=f"balanced {w.name}")
    # many rows per CTA, and rows cut into many pieces
    for B, V in ((400, 128256), (3000, 4099), (2, 128256), (1, 1 << 20)):
        rng = np.random.default_rng(B)
        x = workloads.head_boosted(B, V, seed=B)
        t = rng.choice([0.0, 0.7, 1.0], B)
        k = rng.choice([1, 20, 50, 128, 129], B)
        p = rng.choice([1.0, 0.9, 0.95], B)
        compare(x, oracle.make_params(t, p, k, rng.random(B)), probs=False, label=f"balanced B={B} V={V}")
    # rising values: the first chunk's threshold admits every later value, pieces overflow and the
    # rows fall back to the cluster kernel
    x = torch.arange(6 * 70000, dtype=torch.float32).reshape(6, 70000) % 70001
    compare(x, oracle.make_params([1.0] * 6, [0.9] * 6, [50] * 6, [0.3] * 6), probs=False, label="balanced rising")
    w = workloads.config1(rows=32)
    sel = np.array([31, 0, 5, 5, 17, 2, 30], np.int32)
    rec = rec_for([w.params[i] for i in sel], [w.uniforms()[i] for i in sel])
    compare(w.logits, rec, sel, probs=False, label="balanced row_index")
    os.environ["PB_PATH"] = "full"
    compare(w.logits, rec, sel, probs=False, label="full row_index")
    os.environ.pop("PB_PATH")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_group_passes_padded_rows(dtype):
    """The two-pass launch on rows padded to a 16-byte stride: vocabularies whose last vector is
    partial (read element by element), one-group and sub-group rows, rows read as coarse groups
    (more than 4096 groups), row_index, every mode, and rows with non-finite values; each against
    the oracle and, through compare's probabilities run, every other path."""
    _ws_kernel("groups")
    es = torch.finfo(dtype).bits // 8
    epv = 16 // es
    rng = np.random.default_rng(es)
    for V in (1, 3, 17, 63, 65, 258, 4099, 49155, 128257, (1 << 20) + 5):
        B = 12 if V < (1 << 20) else 3
        x = workloads.head_boosted(B, V, seed=V).to(dtype)
        t = rng.choice([0.0, 0.7, 1.0, 1.5], B)
        k = rng.choice([0, 1, 2, 20, 50, 128, 129, max(1, V - 1), V], B)
        p = rng.choice([1.0, 0.9, 0.99, 1e-6], B)
        pad = (V + epv - 1) // epv * epv + epv
        compare(x, oracle.make_params(t, p, k, rng.random(B)), probs=(V <= 4099), pad_to=pad,
                label=f"groups padded {dtype} V={V}")
    V = 40990
    x = torch.full((6, V), float("-inf"))
    for r, n in enumerate((1, 37, 500, 999, 3, 60)):
        cols = torch.from_numpy(rng.choice(V, n, replace=False))
        x[r, cols] = torch.randn(n, generator=torch.Generator().manual_seed(r)) * 2.0
    x[4, 7] = float("nan")
    x[5, 40989] = float("inf")
    x = x.to(dtype)
    rec = oracle.make_params([1.0, 0.7, 1.0, 1.3, 0.0, 1.0], [1.0, 0.9, 1.0, 0.5, 1.0, 1.0], [100, 100, 128, 100, 0, 5],
                             rng.random(6))
    compare(x, rec, probs=False, pad_to=V + 2 * epv, label=f"groups sparse-finite {dtype}")
    sel = np.array([5, 0, 3, 3, 1], np.int32)
    rec2 = oracle.make_params([0.0, 1.0, 0.7, 0.7, 1.0], [1.0] * 5, [0, 50, 50, 2, 128], rng.random(5))
    compare(x, rec2, sel, probs=False, pad_to=V + epv, label=f"groups row_index {dtype}")


@pytest.mark.parametrize("ws", WS_KERNELS)
def test_balanced_path_ties_and_sparse_rows(ws):
    _ws_kernel(ws)
    V = 20000
    x = torch.zeros(6, V)
    x[1, ::3] = 1.0
    x[2] = torch.randint(0, 3, (V,), generator=torch.Generator().manual_seed(0)).float()
    x[3, 100] = 5.0
    x[4] = (torch.arange(V) % 7).float()
    x[5, :] = -1.0
    rng = np.random.default_rng(13)
    for t, k, p in [(0.5, 500, 1.0), (1.0, 7, 0.99), (0.0, 0, 1.0), (1.0, 1, 1.0), (1.0, 100, 0.3)]:
        for grid in ("1", "4"):
            os.environ["PB_BALANCED_GRID"] = grid
            compare(x, oracle.make_params([t] * 6, [p] * 6, [k] * 6, rng.random(6)), probs=False,
                    label=f"balanced ties t={t} k={k} grid={grid}")
    V = 40990
    x = torch.full((4, V), float("-inf"))
    for r, n in enumerate((1, 37, 500, 999)):
        cols = torch.from_numpy(rng.choice(V, n, replace=False))
        x[r, cols] = torch.randn(n, generator=torch.Generator().manual_seed(r)) * 2.0
    rec = oracle.make_params([1.0, 0.7, 1.0, 1.3], [1.0, 0.9, 1.0, 0.5], [100, 100, 128, 100], rng.random(4))
    for grid in ("1", "8"):
        os.environ["PB_BALANCED_GRID"] = grid
        compare(x, rec, probs=False, label=f"balanced sparse-finite grid={grid}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_power_of_two_temperatures_cooperative_path(dtype):
    """Temperature-only and top-p rows (the cooperative path) at power-of-two temperatures, where the
    kernel scales by the exact reciprocal; includes rows whose scaled keys are subnormal."""
    B, V = 12, 6001
    x = workloads.head_boosted(B, V, seed=77, dtype=torch.float32)
    x[8:10] *= 1e-37  # x / 4 and x / 2 land among the subnormals
    x = x.to(dtype)
    t = [0.25, 0.5, 1.0, 2.0, 4.0, 0.125, 1.0, 2.0, 4.0, 2.0, 0.5, 8.0]
    p = [1.0, 0.9, 1.0, 0.95, 0.5, 1.0, 0.99, 1.0, 1.0, 0.9, 0.7, 0.8]
    u = np.random.default_rng(5).random(B)
    compare(x, oracle.make_params(t, p, [0] * B, u), label=f"pow2 T {dtype}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_shard_records_two_pass_launch(dtype):
    """Vocabulary-parallel records from the two-pass launch (pb_candidates_ws) on column slices of
    the same GPU, merged with pb_merge: the same tokens and row info as pb_sample on the full rows,
    for 2 and 4 slices, greedy and top-k rows (the path the ops layer takes when every row suits it),
    and rows it hands to the cluster kernel (NaN, +inf)."""
    from pagedbatch_b200.vocab_parallel import CudaKernels, record_cap

    w = workloads.config3(rows=96)
    x = w.logits.to(dtype)
    x[5, 1000] = float("nan")
    x[6, 70000] = float("inf")
    params = list(w.params)
    params[7] = type(params[7])(temperature=0.0, top_p=1.0, top_k=0)
    rec = rec_for(params, w.uniforms())
    dev = x.cuda()
    dparams = ops.params_tensor(rec, dev.device)
    B, V = x.shape
    assert ops._ws_path(dparams, V // 4)
    kern = CudaKernels()
    cap = record_cap(params)
    full_tok, full_info, _ = run_gpu(dev, rec, probs=False)
    for n in (2, 4):
        cuts = [V * r // n for r in range(n + 1)]
        assert all((c * x.element_size()) % 16 == 0 for c in cuts)
        recs = [kern.candidates(dev[:, cuts[r]:cuts[r + 1]].contiguous(), dparams, cuts[r], cap) for r in range(n)]
        tok, info = kern.merge(torch.stack(recs), dparams, cap)
        inf = ops.info_records(info)
        ok = inf["status"] != _lib.ROW_FALLBACK
        assert ok[:5].all() and ok[8:].all()
        t = tok.cpu().numpy()
        assert np.array_equal(t[ok], full_tok[ok]), f"{n} slices: tokens differ"
        for f in INFO_FIELDS:
            assert np.array_equal(inf[f][ok], full_info[f][ok]), f"{n} slices: info.{f} differs"
