"""slm_grad_norm_noalloc: the gradient norm for callers that cannot allocate.

Callers running where cudaMalloc is off limits (another allocator owns the HBM
budget, or a latency-critical loop must not take cudaMalloc's device-wide
synchronisation) get the norm, clip scale and non-finite flag from a fixed,
library-owned device array instead of an optimizer handle's scratch.  This
test calls the entry point through the C ABI twice in a row -- a full
135,285,504-element bf16 gradient, then a small ragged fp32 gradient -- and
requires each result to equal, bit for bit, what an optimizer handle's norm
pass reports for the same gradients.  It also checks that sizes above the
fixed maximum are refused before anything runs.  Kept in its own file so it
runs last and alone works too.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from slmopt import B200Adamw, GqaDimensions, SlmError, StepOptions, TensorTable, _lib, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as _torch

    if not _torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    return _torch


def noalloc_norm(torch, grads, dtype: int, scale: float, max_norm: float) -> _lib.NormResult:
    lib = _lib.load()
    out = torch.zeros(ctypes.sizeof(_lib.NormResult), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    _lib.check(lib.slm_grad_norm_noalloc(grads.data_ptr(), dtype, grads.numel(), scale, max_norm,
                                         out.data_ptr(), stream.cuda_stream))
    torch.cuda.synchronize()
    return _lib.NormResult.from_buffer_copy(out.cpu().numpy().tobytes())


def handle_norm(table: TensorTable, grads, scale: float, max_norm: float) -> _lib.StepResult:
    with B200Adamw(table) as opt:
        opt.norm_pass(grads, StepOptions(static_loss_scale=scale, max_grad_norm=max_norm))
        return opt.read_result()


def test_noalloc_norm_equals_the_handle_norm_pass_on_two_calls(torch):
    cases = []
    big = TensorTable.from_dimensions(GqaDimensions.canonical())
    g1 = torch.from_numpy(synth.grads_bf16(big.parameter_count, 0)).cuda()
    cases.append((big, g1, _lib.DTYPE_BF16, 65536.0, 1.0))
    small = TensorTable.from_sizes([65536 * 3 + 5, 768, 1001], [True, False, True])
    g2 = torch.from_numpy(
        (synth.grads_f32(small.parameter_count, 4) * np.float32(3.0)).astype(np.float32)).cuda()
    cases.append((small, g2, _lib.DTYPE_F32, 1.0, 0.5))
    for table, grads, dtype, scale, max_norm in cases:  # two calls in a row
        got = noalloc_norm(torch, grads, dtype, scale, max_norm)
        want = handle_norm(table, grads, scale, max_norm)
        assert want.status == 0 and want.nonfinite == 0
        assert got.nonfinite == 0
        assert got.sum_squares == want.sum_squares
        assert got.grad_norm == want.grad_norm
        assert np.float32(got.clip_scale) == np.float32(want.clip_scale)
        assert got.clip_scale < 1.0


def test_noalloc_norm_refuses_oversized_input(torch):
    lib = _lib.load()
    g = torch.zeros(8, dtype=torch.float32, device="cuda")
    out = torch.zeros(ctypes.sizeof(_lib.NormResult), dtype=torch.uint8, device="cuda")
    st = lib.slm_grad_norm_noalloc(g.data_ptr(), _lib.DTYPE_F32, _lib.NOALLOC_MAX_ELEMENTS + 1,
                                   1.0, 1.0, out.data_ptr(), None)
    assert st == _lib.SLM_ERR_SIZE_LIMIT
    with pytest.raises(SlmError) as e:
        _lib.check(st)
    assert e.value.code == "SLM_SIZE_LIMIT"
