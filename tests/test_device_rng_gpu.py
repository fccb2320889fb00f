"""Device draws (pb_row_params.rng = PB_RNG_PHILOX | step) on a B200.

* every launch path (the cluster kernel, the streaming kernel, the balanced workspace path) gives
  the oracle's tokens and kept-set description bit for bit on rows whose draws are made on the
  device, mixed with host-draw rows in one batch;
* a request's token depends only on (seed, step): the same records give the same tokens, and the
  engine hook with device draws repeats itself across engines;
* 10^6 device draws of one seed over consecutive steps follow the reference's final distribution
  (chi-square, as tests/test_draws_gpu.py does for host draws).
"""

import os

import numpy as np
import pytest
import torch
from scipy import stats

import oracle
from oracle import torch_port
from pagedbatch_b200 import _lib, ops, workloads
from parity_helpers import compare

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _env(cuda):
    yield
    os.environ.pop("PB_PATH", None)


def _mixed(B, V, seed, dtype=torch.float32):
    x = workloads.head_boosted(B, V, seed=seed, dtype=dtype)
    rng = np.random.default_rng(seed)
    t = rng.choice([0.0, 0.5, 0.7, 1.0, 1.3], B)
    k = rng.choice([0, 1, 20, 50, 128, 1000], B)
    p = rng.choice([1.0, 0.5, 0.9, 0.99], B)
    rec = oracle.make_device_rng_params(t, p, k, rng.integers(0, 1 << 62, B), rng.integers(0, 1 << 30, B))
    host = rng.random(B) < 0.25  # a quarter of the rows keep host draws
    rec["rng"][host] = 0
    rec["uniform"][host] = rng.random(int(host.sum()))
    return x, rec


@pytest.mark.parametrize("B,V,dtype", [(64, 49152, torch.bfloat16), (300, 4099, torch.float32),
                                       (48, 128256, torch.float32)])
def test_device_draws_match_the_oracle_on_every_path(B, V, dtype):
    x, rec = _mixed(B, V, seed=B + V, dtype=dtype)
    compare(x, rec, label=f"device rng B={B} V={V}")  # cluster kernel with probs, then stream and ws


def test_same_seed_and_step_same_token():
    x, rec = _mixed(256, 49152, seed=3)
    dev = x.cuda()
    params = ops.params_tensor(rec, dev.device)
    a = ops.sample_op(dev, params).cpu().numpy()
    b = ops.sample_op(dev, params).cpu().numpy()
    assert np.array_equal(a, b)
    rec2 = rec.copy()
    dev_rows = (rec2["rng"] & _lib.RNG_PHILOX) != 0
    rec2["rng"][dev_rows] += 1  # the next step (host-draw rows keep theirs)
    c = ops.sample_op(dev, ops.params_tensor(rec2, dev.device)).cpu().numpy()
    o, _, _ = oracle.sample(x, rec2)
    assert np.array_equal(c, o)


def test_device_draws_over_steps_chi_square():
    N, BATCH, V, T, k, p = 1_000_000, 8192, 49152, 1.0, 100, 0.95
    dev = torch.device("cuda", 0)
    row = workloads.head_boosted(1, V, seed=11)
    x = row.to(dev)
    expected = torch_port.final_probs(row[0], T, k, p).double().numpy()
    kept = expected > 0
    same_row = torch.zeros(BATCH, dtype=torch.int32, device=dev)
    counts = torch.zeros(V, dtype=torch.int64, device=dev)
    for i0 in range(0, N, BATCH):
        n = min(BATCH, N - i0)
        rec = oracle.make_device_rng_params([T] * n, [p] * n, [k] * n, [987654321] * n, np.arange(i0, i0 + n))
        tok = ops.sample_op(x, ops.params_tensor(rec, dev), same_row[:n])
        assert int(tok.min()) >= 0
        counts += torch.bincount(tok, minlength=V)
    counts = counts.cpu().numpy()
    assert counts[~kept].sum() == 0
    e = expected[kept] * N
    o = counts[kept].astype(np.float64)
    order = np.argsort(e)
    e, o = e[order], o[order]
    m = int(np.searchsorted(e, 5.0))
    if m:
        e = np.concatenate([[e[:m].sum()], e[m:]])
        o = np.concatenate([[o[:m].sum()], o[m:]])
    chi2, pval = stats.chisquare(o, e * (o.sum() / e.sum()))
    assert pval > 1e-3, f"chi-square {chi2:.1f} on {o.size - 1} dof, p = {pval:.2e}"


def test_engine_hook_with_device_draws_repeats():
    import ref_engine as R

    ref = R.import_reference()
    if ref is None:
        pytest.skip("reference package not found")
    from pagedbatch_b200 import engine_hook

    reqs = R.mixed_requests()
    outs = []
    try:
        for _ in range(2):
            eng = R.build_tiny_engine("cuda")
            engine_hook.install(eng, device_rng=True)
            outs.append(R.run_to_completion(eng, reqs))
    finally:
        engine_hook.restore_module(ref[1])
    assert outs[0] == outs[1]
    assert all(len(v) == 9 for v in outs[0].values())
