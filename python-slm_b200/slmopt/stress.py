"""The 100-step ZeRO-1 stress run: its seeded inputs and schedule.

Every rank r draws, for update t = 1..100, gradients 1e-3 * Student-t(3)
(``synth.grads_student_t(P, 100 + r, t)``; about 5 % of steps exceed the clip),
multiplies them by the current dynamic loss scale in f32 and rounds to bf16;
at two seeded steps one rank's gradient carries an injected +inf
(``INJECT``), so those steps must be skipped and the scale halved.  The
learning rate warms up linearly for 20 updates, then follows the cosine to
3e-5 at update 100 (the reference's schedule form, ``trainer.rs:102-119``, with
these constants).  The tests, the oracle-side generator of the golden
trajectory and the benchmark's post-run check all build the inputs here.
"""
from __future__ import annotations

import numpy as np

from . import synth

STEPS = 100
INJECT = {17: 1, 63: 0}  # update -> rank whose gradient carries an inf
PEAK_LR, MIN_LR, WARMUP = 3e-4, 3e-5, 20
SEED_BASE = 100


def rank_gradient(P: int, offsets, rank: int, t: int, scale: float) -> np.ndarray:
    """bf16 bits of rank's gradient for update t under loss scale `scale`."""
    g = synth.grads_student_t(P, SEED_BASE + rank, t)
    bits = synth.bf16_rne_bits((g * np.float32(scale)).astype(np.float32))
    if INJECT.get(t) == rank:
        synth.inject_nonfinite(bits, t, offsets)
    return bits


def learning_rate(t: int) -> float:
    """The schedule through the library's host function (bit-equal to the oracle's)."""
    import ctypes

    from . import _lib

    out = ctypes.c_float()
    _lib.check(_lib.load().slm_schedule_learning_rate(t, PEAK_LR, MIN_LR, WARMUP, STEPS,
                                                      ctypes.byref(out)))
    return out.value
