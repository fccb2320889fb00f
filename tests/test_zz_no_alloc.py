"""pb_sample_noalloc: the sampler for callers that cannot allocate device memory.

Such callers (a plugin inside an application that owns the whole GPU through its own allocator,
or plain C code without cudaMalloc) get an entry point whose scratch is an array compiled into the
library. These tests call it through the C ABI and check that it returns exactly what pb_sample
returns (tokens and the kept-set description, bit for bit, as every parity test here), on two
calls in a row, since the second call finds the first call's leftovers in the shared array. They
also check that a batch too large for the array is refused before any launch.

The file name makes pytest collect it last, so a run that stops at the first failure has run
every other test before this one.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from pagedbatch_b200 import _lib, ops, workloads

pytestmark = pytest.mark.gpu

INFO_FIELDS = ("thr_key", "n_tie_kept", "kept_count", "status", "max_key", "flags", "z_q", "kept_q")


def _call(name, x, params, with_info=True):
    L = _lib.load()
    n, V = x.shape
    tok = torch.empty(n, dtype=torch.int64, device=x.device)
    info = torch.empty((n, _lib.ROW_INFO.itemsize), dtype=torch.uint8, device=x.device) if with_info else None
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    args = [ctypes.c_void_p(x.data_ptr()), ops._DTYPE_CODE[x.dtype], n, V, x.stride(0), None,
            ctypes.c_void_p(params.data_ptr()), ctypes.c_void_p(tok.data_ptr()),
            ctypes.c_void_p(info.data_ptr()) if with_info else None]
    if name == "pb_sample":
        rc = L.pb_sample(*args, None, stream)
    else:
        rc = L.pb_sample_noalloc(*args, stream)
    assert rc == 0, (name, rc, L.pb_strerror(rc))
    torch.cuda.synchronize()
    return tok.cpu().numpy(), (ops.info_records(info) if with_info else None)


def test_noalloc_matches_pb_sample_on_two_calls_in_a_row(cuda):
    batches = [workloads.config1(rows=64), workloads.config2(rows=48)]
    for w in batches:
        x = w.logits.to(cuda)
        rec = oracle.make_params([p.temperature for p in w.params], [p.top_p for p in w.params],
                                 [p.top_k for p in w.params], w.uniforms())
        params = ops.params_tensor(rec, cuda)
        want_tok, want_info = _call("pb_sample", x, params)
        got_tok, got_info = _call("pb_sample_noalloc", x, params)
        assert np.array_equal(got_tok, want_tok), w.name
        for f in INFO_FIELDS:
            if f == "flags":  # which path settled a row may differ; the result may not
                continue
            if f == "max_key":
                assert np.array_equal(got_info[f], want_info[f], equal_nan=True), (w.name, f)
            else:
                assert np.array_equal(got_info[f], want_info[f]), (w.name, f)


def test_noalloc_refuses_a_batch_larger_than_its_scratch(cuda):
    L = _lib.load()
    limit = L.pb_sample_noalloc_max_bytes()
    assert limit == 32 << 20
    x = torch.zeros((1, 128256), dtype=torch.float32, device=cuda)
    params = torch.zeros(32, dtype=torch.uint8, device=cuda)
    tok = torch.empty(1, dtype=torch.int64, device=cuda)
    n_rows = 1 << 16  # needs far more than 32 MiB of records; refused before anything is read
    rc = L.pb_sample_noalloc(ctypes.c_void_p(x.data_ptr()), 0, n_rows, 128256, 128256, None,
                             ctypes.c_void_p(params.data_ptr()), ctypes.c_void_p(tok.data_ptr()), None, None)
    assert rc == -5, L.pb_strerror(rc)
    assert b"scratch" in L.pb_strerror(rc)


def test_noalloc_without_info_keeps_row_state_in_its_array(cuda):
    """Without out_info, what the streaming launch leaves for the cluster kernel that follows lives
    in the fixed array and the tokens themselves. Two calls in a row, the second on a different
    batch whose rows must reach the cluster kernel (a greedy row with a NaN, top_k above what the
    streaming kernel settles, temperature-only and top-p-only rows), so that it reads only what it
    wrote, never the first call's leftovers."""
    w = workloads.config2(rows=40)
    x = w.logits.to(cuda)
    rec = oracle.make_params([p.temperature for p in w.params], [p.top_p for p in w.params],
                             [p.top_k for p in w.params], w.uniforms())
    params = ops.params_tensor(rec, cuda)
    want, _ = _call("pb_sample", x, params, with_info=False)
    got, _ = _call("pb_sample_noalloc", x, params, with_info=False)
    assert np.array_equal(got, want)
    x2 = workloads.head_boosted(40, 128256, seed=5)
    x2[3, 1000] = float("nan")
    rng = np.random.default_rng(2)
    t = rng.choice([0.0, 0.7, 1.0], 40)
    t[3] = 0.0
    k = rng.choice([0, 50, 300, 2000], 40)
    p = rng.choice([1.0, 0.9], 40)
    rec2 = oracle.make_params(t, p, k, rng.random(40))
    params2 = ops.params_tensor(rec2, cuda)
    x2d = x2.to(cuda)
    want2, _ = _call("pb_sample", x2d, params2, with_info=False)
    got2, _ = _call("pb_sample_noalloc", x2d, params2, with_info=False)
    assert np.array_equal(got2, want2)
    o_tok, _, _ = oracle.sample(x2, rec2)
    assert np.array_equal(got2, o_tok)
    assert got2[3] == 1000
