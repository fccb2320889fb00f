"""Host-side logic of the drop-in API (CPU only): parameter validation and packing, the per-row
draws, and the refusal to compute anywhere but on the GPU."""

import numpy as np
import pytest
import torch

from pagedbatch_b200 import SamplingParams, _lib, draw_uniforms, pack_rows, sample_token, sample_tokens


def test_sampling_params_mirror_reference_validation():
    # pagedbatch/config.py:146-155
    with pytest.raises(ValueError, match="max_tokens must be >= 1"):
        SamplingParams(max_tokens=0)
    with pytest.raises(ValueError, match="temperature must be >= 0"):
        SamplingParams(temperature=-0.1)
    with pytest.raises(ValueError, match=r"top_p must be in \(0, 1\]"):
        SamplingParams(top_p=0.0)
    with pytest.raises(ValueError, match="top_k must be >= 0"):
        SamplingParams(top_k=-1)
    assert SamplingParams(temperature=0.0).greedy and not SamplingParams().greedy


def test_pack_rows_layout():
    ps = [SamplingParams(temperature=0.7, top_k=50, top_p=0.95), SamplingParams(temperature=0.0)]
    rec = pack_rows(ps, np.array([0.25, 0.0]))
    assert rec.dtype == _lib.ROW_PARAMS and rec.itemsize == 32
    raw = rec.view(np.uint8).reshape(2, 32)
    assert np.frombuffer(raw[0, 0:8].tobytes(), "<f8")[0] == 0.7
    assert np.frombuffer(raw[0, 8:16].tobytes(), "<f8")[0] == 0.95
    assert np.frombuffer(raw[0, 16:24].tobytes(), "<f8")[0] == 0.25
    assert np.frombuffer(raw[0, 24:28].tobytes(), "<i4")[0] == 50


def test_pack_rows_validates_duck_typed_params():
    class P:
        temperature, top_p, top_k = 1.0, 1.5, 0

    with pytest.raises(ValueError, match="top_p"):
        pack_rows([P()], np.zeros(1))


def test_uniform_draws_follow_generators():
    ps = [SamplingParams(temperature=1.0), SamplingParams(temperature=0.0), SamplingParams(temperature=0.5)]
    shared = torch.Generator().manual_seed(3)
    u = draw_uniforms(ps, [torch.Generator().manual_seed(7), shared, shared])
    assert u[1] == 0.0  # greedy rows do not consume their generator (sampling.py:12-13)
    assert u[0] == float(torch.rand((), dtype=torch.float64, generator=torch.Generator().manual_seed(7)))
    assert u[2] == float(torch.rand((), dtype=torch.float64, generator=torch.Generator().manual_seed(3)))
    assert all(0.0 <= x < 1.0 for x in u) and all((x * 2**53).is_integer() for x in u)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        sample_token(torch.tensor([0.1, 3.0, 0.2, 2.9]), SamplingParams(temperature=0.0), torch.Generator())
    with pytest.raises(RuntimeError, match="CUDA"):
        sample_tokens(torch.zeros(2, 4), [SamplingParams()] * 2, [torch.Generator()] * 2)


def test_row_selection_validation():
    with pytest.raises(ValueError, match="rows="):
        sample_tokens(torch.zeros(3, 4, device="meta"), [SamplingParams()] * 2, [torch.Generator()] * 2)


def test_huge_top_k_saturates():
    """The reference accepts any top_k >= 0 and treats top_k >= vocab as no filter (sampling.py:15):
    a top_k past int32 must pack (saturated), not raise."""
    rec = pack_rows([SamplingParams(temperature=1.0, top_k=2**40)], np.array([0.5]))
    assert rec["top_k"][0] == 2**31 - 1


def test_workspace_path_choice(monkeypatch):
    """The ops layer sends a batch to pb_sample_ws only when every row suits its two-pass launch
    (greedy, or 0 < top_k <= 128 below the vocabulary, valid parameters, a usable draw), unless
    PB_PATH forces a path."""
    import oracle
    from pagedbatch_b200 import ops

    monkeypatch.delenv("PB_PATH", raising=False)

    def choice(t, p, k, u, vocab=1000, rec=None):
        rec = oracle.make_params(t, p, k, u) if rec is None else rec
        return ops._ws_path(ops.mark_rows(torch.empty(0), rec), vocab)

    assert choice([0.7, 0.0, 1.0], [0.95, 1.0, 0.5], [50, 0, 128], [0.3, 0.1, 0.0])
    assert not choice([0.7, 1.0], [0.95, 1.0], [50, 0], [0.3, 0.1])  # temperature-only row
    assert not choice([0.7, 1.0], [0.95, 0.9], [50, 129], [0.3, 0.1])  # top_k above 128
    assert not choice([0.7], [0.95], [50], [0.3], vocab=50)  # top_k not below the vocabulary
    assert not choice([0.7], [0.95], [50], [1.0])  # a draw outside [0, 1)
    assert not choice([-1.0], [0.95], [50], [0.3])  # rejected parameters
    assert not choice([], [], [], [])
    dev_rec = oracle.make_device_rng_params([0.7, 0.0], [0.9, 1.0], [20, 0], [5, 6], [0, 3])
    assert choice(None, None, None, None, rec=dev_rec)
    assert not ops._ws_path(torch.empty(0), 1000)  # a params tensor made elsewhere: pb_sample
    monkeypatch.setenv("PB_PATH", "full")
    assert not choice([0.7], [0.95], [50], [0.3])
    monkeypatch.setenv("PB_PATH", "ws")
    assert choice([0.7, 1.0], [0.95, 1.0], [50, 0], [0.3, 0.1])
