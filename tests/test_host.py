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
