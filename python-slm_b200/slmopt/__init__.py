"""slmopt -- B200-native optimizer step for python-slm's gqa-135m-v1.

The numeric work lives in libslmopt.so (CUDA for sm_100a behind the C ABI of
include/slmopt.h); this package is the host-side mirror of the reference's
optimizer interface (CanonicalAdamw / TrainerBackend) plus the PARAM-001
tensor table, seeded synthetic inputs and the ZeRO-1 data-parallel driver.
"""
from . import _lib
from ._lib import SlmError, StepResult, load
from .layout import GqaDimensions, TensorTable, weight_decay_for
from .optimizer import ARTIFACTS, B200Adamw, B200TrainerBackend, StepOptions

__all__ = [
    "_lib",
    "ARTIFACTS",
    "B200Adamw",
    "B200TrainerBackend",
    "GqaDimensions",
    "SlmError",
    "StepOptions",
    "StepResult",
    "TensorTable",
    "load",
    "weight_decay_for",
]
