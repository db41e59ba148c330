"""ctypes wrapper of the CPU oracle (oracle/libslmoracle.so).

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  See slm_oracle.h for the reference lines each function restates
and the known-answer tests that pin it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libslmoracle.so"

OK = 0
MODEL_GRADIENT_NONFINITE = 10
MODEL_GRADIENT_NORM_NONFINITE = 11
MODEL_OPTIMIZER_INPUT_INVALID = 12
MODEL_OPTIMIZER_RESULT_NONFINITE = 13
P12_OPTIMIZER_GRADIENT_INVALID = 20
P12_SCHEDULER_STATE_MISMATCH = 21
P12_OPTIMIZER_STATE_INVALID = 22
P12_UPDATE_INDEX_INVALID = 23
P12_SCHEDULE_INDEX_INVALID = 24
INVALID_ARGUMENT = 30

DTYPE_F32 = 0
DTYPE_BF16 = 1
CHUNK_ELEMS = 65536


class StepConfig(ctypes.Structure):
    _fields_ = [
        ("learning_rate", ctypes.c_float),
        ("one_based_update", ctypes.c_uint32),
        ("beta1", ctypes.c_float),
        ("beta2", ctypes.c_float),
        ("epsilon", ctypes.c_float),
        ("decay_weight", ctypes.c_float),
        ("no_decay_weight", ctypes.c_float),
        ("max_grad_norm", ctypes.c_float),
        ("apply_clip", ctypes.c_int32),
        ("min_clip_accept", ctypes.c_float),
        ("nonfinite_policy", ctypes.c_int32),
        ("loss_scale_mode", ctypes.c_int32),
        ("static_loss_scale", ctypes.c_float),
        ("growth_interval", ctypes.c_uint32),
    ]


class StepResult(ctypes.Structure):
    _fields_ = [
        ("sum_squares", ctypes.c_double),
        ("grad_norm", ctypes.c_double),
        ("clip_scale", ctypes.c_float),
        ("loss_scale_used", ctypes.c_float),
        ("next_loss_scale", ctypes.c_float),
        ("skipped", ctypes.c_uint32),
        ("nonfinite", ctypes.c_uint32),
        ("result_nonfinite", ctypes.c_uint32),
        ("rejected", ctypes.c_uint32),
        ("good_steps", ctypes.c_uint32),
        ("status", ctypes.c_int32),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class Scaler(ctypes.Structure):
    _fields_ = [("scale", ctypes.c_float), ("good_steps", ctypes.c_uint32)]


_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (the system gcc)."""
    env = dict(os.environ)
    env.pop("CC", None)
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    L = ctypes.CDLL(str(LIB_PATH))
    P, U64, U32, I32, F, D = (ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int32,
                              ctypes.c_float, ctypes.c_double)
    sig = {
        "slmo_f32_to_bf16_bits": (ctypes.c_uint16, [F]),
        "slmo_bf16_bits_to_f32": (F, [ctypes.c_uint16]),
        "slmo_powi": (F, [F, I32]),
        "slmo_gradient_clip_scale": (ctypes.c_int, [P, U64, ctypes.POINTER(F)]),
        "slmo_reference_sum_squares": (ctypes.c_int, [P, U64, ctypes.POINTER(F)]),
        "slmo_adamw_scalar_step": (ctypes.c_int, [F, F, F, F, F, U32, F, ctypes.POINTER(F),
                                                  ctypes.POINTER(F), ctypes.POINTER(F),
                                                  ctypes.POINTER(ctypes.c_uint16)]),
        "slmo_canonical_learning_rate": (ctypes.c_int, [U64, ctypes.POINTER(F)]),
        "slmo_schedule_learning_rate": (ctypes.c_int, [U64, F, F, U64, U64, ctypes.POINTER(F)]),
        "slmo_sha256": (None, [P, U64, P]),
        "slmo_chunk_count": (U64, [U64]),
        "slmo_chunk_partials_f32": (None, [P, U64, P, P, ctypes.c_int]),
        "slmo_tree_sum": (D, [P, U64]),
        "slmo_clip_from_sum": (F, [D, F, ctypes.POINTER(ctypes.c_int)]),
        "slmo_unscale_f32": (None, [P, U64, F, P, ctypes.c_int]),
        "slmo_unscale_bf16": (None, [P, U64, F, P, ctypes.c_int]),
        "slmo_rank_sum_bf16": (None, [P, U32, U64, P, ctypes.c_int]),
        "slmo_adamw_apply_range": (ctypes.c_int, [ctypes.POINTER(StepConfig), P, U64, U64, P, P,
                                                  U32, F, F, P, P, P, P, ctypes.c_int]),
        "slmo_step": (ctypes.c_int, [ctypes.POINTER(StepConfig), P, ctypes.c_int, U64, P, P, U32,
                                     P, P, P, P, ctypes.POINTER(Scaler),
                                     ctypes.POINTER(StepResult), ctypes.c_int]),
        "slmo_apply_normalized_clipped_gradients": (ctypes.c_int, [P, U64, F, U64, P, P, U32, P,
                                                                   P, P, P, ctypes.POINTER(F)]),
        "slmo_state_sha256": (ctypes.c_int, [P, P, P, U32, P, P, P, P, ctypes.c_char_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ---- scalar OPT-001 arithmetic -------------------------------------------------
def f32_to_bf16_bits(x: float) -> int:
    return int(lib().slmo_f32_to_bf16_bits(x))


def bf16_bits_to_f32(b: int) -> float:
    return float(lib().slmo_bf16_bits_to_f32(b))


def powi(base: float, exponent: int) -> float:
    return float(lib().slmo_powi(base, exponent))


def reference_sum_squares(g: np.ndarray) -> tuple[int, float]:
    """(status, the reference's sequential f32 sum of squares)."""
    g = np.ascontiguousarray(g, dtype=np.float32)
    out = ctypes.c_float()
    st = lib().slmo_reference_sum_squares(_ptr(g), g.size, ctypes.byref(out))
    return st, out.value


def gradient_clip_scale(g: np.ndarray) -> tuple[int, float]:
    g = np.ascontiguousarray(g, dtype=np.float32)
    out = ctypes.c_float()
    st = lib().slmo_gradient_clip_scale(_ptr(g), g.size, ctypes.byref(out))
    return st, out.value


def adamw_scalar_step(theta, gradient, moment, variance, lr, t, wd):
    m, mo, va, b = ctypes.c_float(), ctypes.c_float(), ctypes.c_float(), ctypes.c_uint16()
    st = lib().slmo_adamw_scalar_step(theta, gradient, moment, variance, lr, t, wd,
                                      ctypes.byref(m), ctypes.byref(mo), ctypes.byref(va),
                                      ctypes.byref(b))
    return st, (np.float32(m.value), np.float32(mo.value), np.float32(va.value), int(b.value))


def canonical_learning_rate(t: int) -> tuple[int, float]:
    out = ctypes.c_float()
    st = lib().slmo_canonical_learning_rate(t, ctypes.byref(out))
    return st, out.value


def schedule_learning_rate(t, peak, minimum, warmup, total) -> tuple[int, float]:
    out = ctypes.c_float()
    st = lib().slmo_schedule_learning_rate(t, peak, minimum, warmup, total, ctypes.byref(out))
    return st, out.value


def sha256(data: bytes) -> bytes:
    buf = np.frombuffer(data, dtype=np.uint8) if data else np.zeros(1, np.uint8)
    out = np.zeros(32, dtype=np.uint8)
    lib().slmo_sha256(_ptr(buf), len(data), _ptr(out))
    return out.tobytes()


# ---- norm tree -----------------------------------------------------------------------
def chunk_partials(g: np.ndarray, threads: int = 1) -> tuple[np.ndarray, np.ndarray]:
    g = np.ascontiguousarray(g, dtype=np.float32)
    c = int(lib().slmo_chunk_count(g.size))
    partials = np.zeros(c, dtype=np.float64)
    flags = np.zeros(c, dtype=np.uint8)
    lib().slmo_chunk_partials_f32(_ptr(g), g.size, _ptr(partials), _ptr(flags), threads)
    return partials, flags


def tree_sum(partials: np.ndarray) -> float:
    p = np.ascontiguousarray(partials, dtype=np.float64)
    return float(lib().slmo_tree_sum(_ptr(p), p.size))


def clip_from_sum(s: float, max_norm: float = 1.0) -> tuple[float, bool]:
    bad = ctypes.c_int()
    c = lib().slmo_clip_from_sum(s, max_norm, ctypes.byref(bad))
    return float(c), bool(bad.value)


def unscale(x: np.ndarray, scale: float, threads: int = 1) -> np.ndarray:
    out = np.empty(x.size, dtype=np.float32)
    if x.dtype == np.uint16:
        lib().slmo_unscale_bf16(_ptr(x), x.size, scale, _ptr(out), threads)
    else:
        xf = np.ascontiguousarray(x, dtype=np.float32)
        lib().slmo_unscale_f32(_ptr(xf), xf.size, scale, _ptr(out), threads)
    return out


def rank_sum_bf16(grads: list[np.ndarray], threads: int = 1) -> np.ndarray:
    arrs = [np.ascontiguousarray(g, dtype=np.uint16) for g in grads]
    n = arrs[0].size
    ptrs = (ctypes.c_void_p * len(arrs))(*[_ptr(a) for a in arrs])
    out = np.empty(n, dtype=np.float32)
    lib().slmo_rank_sum_bf16(ctypes.cast(ptrs, ctypes.c_void_p), len(arrs), n, _ptr(out), threads)
    return out


# ---- full step -------------------------------------------------------------------------
def make_config(lr=3e-4, t=1, beta1=0.9, beta2=0.95, eps=1e-8, decay=0.1, no_decay=0.0,
                max_norm=1.0, apply_clip=True, min_clip_accept=0.0, nonfinite_policy=0,
                dynamic=False, static_scale=1.0, growth_interval=2000) -> StepConfig:
    c = StepConfig()
    c.learning_rate = lr
    c.one_based_update = t
    c.beta1, c.beta2, c.epsilon = beta1, beta2, eps
    c.decay_weight, c.no_decay_weight = decay, no_decay
    c.max_grad_norm = max_norm
    c.apply_clip = 1 if apply_clip else 0
    c.min_clip_accept = min_clip_accept
    c.nonfinite_policy = nonfinite_policy
    c.loss_scale_mode = 1 if dynamic else 0
    c.static_loss_scale = static_scale
    c.growth_interval = growth_interval
    return c


def step(cfg: StepConfig, grads: np.ndarray, offsets: np.ndarray, decay, state: dict,
         scaler: Scaler | None = None, threads: int = 1) -> StepResult:
    """Run the fused step in place over state {master, moment, variance, bf16}."""
    dtype = DTYPE_BF16 if grads.dtype == np.uint16 else DTYPE_F32
    g = np.ascontiguousarray(grads)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    dec = np.ascontiguousarray(np.asarray(decay, dtype=np.uint8))
    res = StepResult()
    lib().slmo_step(ctypes.byref(cfg), _ptr(g), dtype, g.size, _ptr(off), _ptr(dec),
                    dec.size, _ptr(state["master"]), _ptr(state["moment"]),
                    _ptr(state["variance"]), _ptr(state["bf16"]),
                    ctypes.byref(scaler) if scaler is not None else None, ctypes.byref(res),
                    threads)
    return res


def adamw_apply_range(cfg: StepConfig, g_raw: np.ndarray, elem_base: int, offsets, decay,
                      scale: float, clip: float, state: dict, threads: int = 1) -> int:
    """AdamW over a slice of the flat buffer (global start elem_base) with a
    given clip; state holds the slice's master/moment/variance/bf16."""
    g = np.ascontiguousarray(g_raw, dtype=np.float32)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    dec = np.ascontiguousarray(np.asarray(decay, dtype=np.uint8))
    return int(lib().slmo_adamw_apply_range(
        ctypes.byref(cfg), _ptr(g), g.size, elem_base, _ptr(off), _ptr(dec), dec.size, scale, clip,
        _ptr(state["master"]), _ptr(state["moment"]), _ptr(state["variance"]),
        _ptr(state["bf16"]), threads))


def apply_normalized_clipped_gradients(grads: np.ndarray, lr: float, t: int, offsets, decay,
                                       state: dict) -> tuple[int, float]:
    g = np.ascontiguousarray(grads, dtype=np.float32)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    dec = np.ascontiguousarray(np.asarray(decay, dtype=np.uint8))
    clip = ctypes.c_float()
    st = lib().slmo_apply_normalized_clipped_gradients(
        _ptr(g), g.size, lr, t, _ptr(off), _ptr(dec), dec.size, _ptr(state["master"]),
        _ptr(state["moment"]), _ptr(state["variance"]), _ptr(state["bf16"]), ctypes.byref(clip))
    return st, clip.value


def state_sha256(names, offsets, decay, state: dict) -> tuple[int, str]:
    raw = [n.encode() for n in names]
    arr = (ctypes.c_char_p * len(raw))(*raw)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    dec = np.ascontiguousarray(np.asarray(decay, dtype=np.uint8))
    out = ctypes.create_string_buffer(65)
    st = lib().slmo_state_sha256(ctypes.cast(arr, ctypes.c_void_p), _ptr(off), _ptr(dec),
                                 len(raw), _ptr(state["master"]), _ptr(state["bf16"]),
                                 _ptr(state["moment"]), _ptr(state["variance"]), out)
    return st, out.value.decode()
