"""ctypes binding of libslmopt.so (include/slmopt.h).

This is the same binding a Rust host would declare with ``extern "C"``: plain
pointers, sizes and POD structs.  Loading fails loudly when the library is
missing -- there is no CPU fallback for the optimizer step.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

# slm_status values (include/slmopt.h) and the reference ProductError codes.
SLM_OK = 0
SLM_ERR_MODEL_GRADIENT_NONFINITE = 10
SLM_ERR_MODEL_GRADIENT_NORM_NONFINITE = 11
SLM_ERR_MODEL_OPTIMIZER_INPUT_INVALID = 12
SLM_ERR_MODEL_OPTIMIZER_RESULT_NONFINITE = 13
SLM_ERR_P12_OPTIMIZER_GRADIENT_INVALID = 20
SLM_ERR_P12_SCHEDULER_STATE_MISMATCH = 21
SLM_ERR_P12_OPTIMIZER_STATE_INVALID = 22
SLM_ERR_P12_UPDATE_INDEX_INVALID = 23
SLM_ERR_P12_SCHEDULE_INDEX_INVALID = 24
SLM_ERR_E1_PARAMETER_LAYOUT_MISMATCH = 25
SLM_ERR_E1_STATE_ARTIFACT_INVALID = 26
SLM_ERR_P12_OPTIMIZER_PARAMETER_DUPLICATE = 27
SLM_ERR_INVALID_ARGUMENT = 30
SLM_ERR_SIZE_LIMIT = 31
SLM_ERR_CUDA = 40
SLM_ERR_OUT_OF_MEMORY = 41
SLM_ERR_NCCL = 42
SLM_ERR_TIMEOUT = 43
SLM_ERR_NO_DEVICE = 44
SLM_ERR_INTERNAL = 50

ROLE_PARAMETERS_BF16 = 0
ROLE_MASTER_F32 = 1
ROLE_MOMENT1_F32 = 2
ROLE_MOMENT2_F32 = 3

DTYPE_F32 = 0
DTYPE_BF16 = 1
MEMORY_DEVICE = 0
MEMORY_HOST = 1
NONFINITE_SKIP = 0
NONFINITE_ERROR = 1
SCALE_STATIC = 0
SCALE_DYNAMIC = 1
ZERO1_NCCL = 0
ZERO1_PEER = 1


class TensorSpec(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("elements", ctypes.c_uint64),
        ("weight_decay", ctypes.c_uint32),
    ]


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


class NormResult(ctypes.Structure):
    """slm_norm_result (written to device memory by slm_grad_norm_noalloc)."""

    _fields_ = [
        ("sum_squares", ctypes.c_double),
        ("grad_norm", ctypes.c_double),
        ("clip_scale", ctypes.c_float),
        ("nonfinite", ctypes.c_uint32),
    ]


class ClipResult(ctypes.Structure):
    """slm_clip_result (written to device memory by slm_gradient_clip_scale)."""

    _fields_ = [
        ("sum_squares", ctypes.c_float),
        ("clip_scale", ctypes.c_float),
        ("status", ctypes.c_int32),
        ("kernel_error", ctypes.c_uint32),
    ]


NOALLOC_MAX_ELEMENTS = 268435456

_P = ctypes.c_void_p
_U64 = ctypes.c_uint64
_U32 = ctypes.c_uint32
_I = ctypes.c_int
_F = ctypes.c_float

# (name, restype, argtypes) of every entry point declared in include/slmopt.h.
SIGNATURES = [
    ("slm_abi_version", _I, []),
    ("slm_status_code_string", ctypes.c_char_p, [_I]),
    ("slm_status_category", _I, [_I]),
    ("slm_last_error_message", ctypes.c_char_p, []),
    ("slm_step_config_default", None, [ctypes.POINTER(StepConfig)]),
    ("slm_opt_create", _I, [ctypes.POINTER(TensorSpec), _U32, _I, ctypes.POINTER(_P)]),
    ("slm_opt_destroy", _I, [_P]),
    ("slm_opt_parameter_count", _U64, [_P]),
    ("slm_opt_last_error", ctypes.c_char_p, [_P]),
    ("slm_opt_init_master", _I, [_P, _P, _P]),
    ("slm_opt_snapshot", _I, [_P, _I, _P, _U64]),
    ("slm_opt_restore", _I, [_P, _I, _P, _U64]),
    ("slm_opt_validate_state", _I, [_P]),
    ("slm_opt_device_buffer", _I, [_P, _I, ctypes.POINTER(_P)]),
    ("slm_opt_state_sha256", _I, [_P, ctypes.c_char_p]),
    ("slm_opt_step", _I, [_P, _P, _I, _I, ctypes.POINTER(StepConfig), ctypes.POINTER(StepResult), _P]),
    ("slm_opt_read_result", _I, [_P, ctypes.POINTER(StepResult)]),
    ("slm_opt_upload_gradients", _I, [_P, _P, _I, ctypes.POINTER(_I)]),
    ("slm_opt_step_uploaded", _I, [_P, _I, ctypes.POINTER(StepConfig),
                                   ctypes.POINTER(StepResult), _P]),
    ("slm_opt_export_weights_f32", _I, [_P, _P, _U64, _P]),
    ("slm_opt_phase_timing", _I, [_P, _I]),
    ("slm_opt_phase_times", _I, [_P, ctypes.POINTER(ctypes.c_double), _U32,
                                 ctypes.POINTER(_U32), ctypes.POINTER(_U64)]),
    ("slm_opt_phase_name", ctypes.c_char_p, [_P, _U32]),
    ("slm_opt_norm_pass", _I, [_P, _P, _I, _I, ctypes.POINTER(StepConfig), _P]),
    ("slm_opt_update_pass", _I, [_P, ctypes.POINTER(StepConfig), _P]),
    ("slm_grad_accumulate", _I, [_P, _P, _I, _U64, _I, _P]),
    ("slm_opt_norm_pass_accumulate", _I, [_P, _P, _P, _I, _I, _I, ctypes.POINTER(StepConfig),
                                          _P]),
    ("slm_opt_apply_update", _I, [_P, _P, _U64, _F, _U64, _U64, ctypes.c_char_p]),
    ("slm_zero1_unique_id", _I, [_P]),
    ("slm_opt_create_zero1", _I, [ctypes.POINTER(TensorSpec), _U32, _I, _I, _I, _P, _U32,
                                  ctypes.POINTER(_P)]),
    ("slm_opt_shard_range", _I, [_P, ctypes.POINTER(_U64), ctypes.POINTER(_U64)]),
    ("slm_opt_zero1_set_exchange", _I, [_P, _I]),
    ("slm_opt_zero1_exchange", _I, [_P]),
    ("slm_opt_gradient_buffer", _I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_U64)]),
    ("slm_grad_norm_noalloc", _I, [_P, _I, _U64, _F, _F, _P, _P]),
    ("slm_gradient_clip_scale", _I, [_P, _U64, _P, _P]),
    ("slm_gradient_clip_workspace_bytes", _U64, [_U64]),
    ("slm_gradient_clip_scale_ws", _I, [_P, _U64, _P, _U64, _P, _P]),
    ("slm_opt_set_loss_scale", _I, [_P, _F, _U32]),
    ("slm_opt_get_loss_scale", _I, [_P, ctypes.POINTER(_F), ctypes.POINTER(_U32)]),
    ("slm_canonical_learning_rate", _I, [_U64, ctypes.POINTER(_F)]),
    ("slm_schedule_learning_rate", _I, [_U64, _F, _F, _U64, _U64, ctypes.POINTER(_F)]),
]


def library_path() -> Path:
    return _build.LIB_PATH


def load(build_if_missing: bool = False) -> ctypes.CDLL:
    """Load libslmopt.so (the in-tree build).  Raises if it is absent."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if not path.exists():
            if not build_if_missing:
                raise RuntimeError(
                    f"{path} is missing: build it with `python python-slm_b200/slmopt/build.py` "
                    "(the optimizer step has no CPU fallback)"
                )
            _build.build()
        lib = ctypes.CDLL(str(path))
        for name, restype, argtypes in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = lib
        return lib


class SlmError(RuntimeError):
    """A failed C-ABI call, shaped like the reference's ProductError
    (src/error.rs:16-22): ``code`` string, ``category`` exit code, message."""

    def __init__(self, status: int, message: str):
        lib = load()
        self.status = int(status)
        self.code = lib.slm_status_code_string(status).decode()
        self.category = int(lib.slm_status_category(status))
        self.message = message
        super().__init__(f"[{self.code}] {message}")


def check(status: int, handle=None) -> None:
    if status == SLM_OK:
        return
    lib = load()
    msg = (lib.slm_opt_last_error(handle) if handle else lib.slm_last_error_message()).decode()
    raise SlmError(status, msg)


def default_config() -> StepConfig:
    cfg = StepConfig()
    load().slm_step_config_default(ctypes.byref(cfg))
    return cfg
