"""slm_grad_norm_noalloc: the gradient norm for callers that cannot allocate.

Callers running where cudaMalloc is off limits (another allocator owns the HBM
budget, or a latency-critical loop must not take cudaMalloc's device-wide
synchronisation) get the norm, clip scale and non-finite flag from a fixed,
library-owned device array instead of an optimizer handle's scratch.  These
tests call the entry point through the C ABI several times in a row:

* a full 135,285,504-element bf16 gradient, then a small ragged fp32 gradient:
  each result must equal, bit for bit, both the CPU oracle's fixed-tree norm
  and what an optimizer handle's norm pass reports for the same gradients;
* a small bf16 gradient carrying one +inf (non-finite flag set, clip 0),
  then the same gradient without it: the flag the bad call raised must not
  leak into the clean call, which again equals the oracle bit for bit.

Sizes above the fixed maximum are refused before anything runs.  Kept in its
own file so it runs last; it also passes when run alone.
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np
import pytest

import slm_oracle as oracle
from slmopt import B200Adamw, GqaDimensions, SlmError, StepOptions, TensorTable, _lib, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as _torch

    if not _torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    return _torch


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


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


def oracle_norm(host_grads: np.ndarray, scale: float, max_norm: float):
    """(sum of squares, clip scale, non-finite) from the oracle's fixed tree."""
    u = oracle.unscale(host_grads, scale, threads=8)
    partials, flags = oracle.chunk_partials(u, threads=8)
    s = oracle.tree_sum(partials)
    clip, bad = oracle.clip_from_sum(s, max_norm)
    return s, clip, bool(flags.any()) or bad


def test_noalloc_norm_equals_the_oracle_and_the_handle_on_two_calls(torch):
    big = TensorTable.from_dimensions(GqaDimensions.canonical())
    h1 = synth.grads_bf16(big.parameter_count, 0)
    small = TensorTable.from_sizes([65536 * 3 + 5, 768, 1001], [True, False, True])
    h2 = (synth.grads_f32(small.parameter_count, 4) * np.float32(3.0)).astype(np.float32)
    cases = [(big, h1, _lib.DTYPE_BF16, 65536.0, 1.0), (small, h2, _lib.DTYPE_F32, 1.0, 0.5)]
    for table, host, dtype, scale, max_norm in cases:  # two calls in a row
        grads = torch.from_numpy(host).cuda()
        got = noalloc_norm(torch, grads, dtype, scale, max_norm)
        want_s, want_clip, want_bad = oracle_norm(host, scale, max_norm)
        assert not want_bad and got.nonfinite == 0
        assert got.sum_squares == want_s
        assert got.grad_norm == float(np.sqrt(np.float64(want_s)))
        assert f32_bits(got.clip_scale) == f32_bits(want_clip)
        assert got.clip_scale < 1.0
        handle = handle_norm(table, grads, scale, max_norm)
        assert handle.status == 0 and handle.nonfinite == 0
        assert got.sum_squares == handle.sum_squares
        assert got.grad_norm == handle.grad_norm
        assert f32_bits(got.clip_scale) == f32_bits(handle.clip_scale)


def test_noalloc_norm_flags_an_inf_and_the_next_call_starts_clean(torch):
    table = TensorTable.from_sizes([65536 * 2 + 8, 768, 4096 + 3], [True, False, True])
    clean = synth.grads_bf16(table.parameter_count, 7)
    bad = clean.copy()
    synth.inject_nonfinite(bad, 3, table.offsets)
    got_bad = noalloc_norm(torch, torch.from_numpy(bad).cuda(), _lib.DTYPE_BF16, 65536.0, 1.0)
    assert got_bad.nonfinite == 1
    assert got_bad.clip_scale == 0.0
    assert oracle_norm(bad, 65536.0, 1.0)[2]  # the oracle flags it too
    got = noalloc_norm(torch, torch.from_numpy(clean).cuda(), _lib.DTYPE_BF16, 65536.0, 1.0)
    want_s, want_clip, want_bad = oracle_norm(clean, 65536.0, 1.0)
    assert not want_bad
    assert got.nonfinite == 0
    assert got.sum_squares == want_s
    assert f32_bits(got.clip_scale) == f32_bits(want_clip)


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
