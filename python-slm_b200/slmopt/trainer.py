"""Update bookkeeping of the reference's trainer around the optimizer step.

``DeterministicTrainer::process_batch`` (src/train/trainer.rs:808-955) wraps
every optimizer update in exact target accounting: the batch must start at
the training cursor, must not cross the update's target boundary, the update
fires when exactly ``canonical_update_target_count(t)`` targets have been
accumulated, the backend's state hash must be a lowercase SHA-256, and the
update is reported as an ``UpdateEvent`` (consumed targets, the normalised
loss and the learning rate as little-endian hex, the state hash, whether an
evaluation / checkpoint boundary was crossed and whether training is done).

``UpdateAccounting`` restates that bookkeeping on the host (it is scalar
integer work; nothing here touches a gradient).  ``B200Trainer`` drives the
device path with it: micro-batch gradients are summed on the GPU
(``slm_grad_accumulate``), the last micro-batch of an update goes through the
fused accumulate + norm pass, normalised by the update's target count, then
the update pass and the state hash.  Evaluation and the forward/backward graph
are not part of this path: ``checkpoint_due`` reports the boundary the
reference evaluates and checkpoints at.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass

# src/train/trainer.rs:12-19
TOTAL_TARGETS = 2_000_000_000
TARGETS_PER_FULL_UPDATE = 65_536
FULL_UPDATES = 30_517
FINAL_UPDATE_TARGETS = 37_888
TOTAL_UPDATES = 30_518
EVENT_INTERVAL_TARGETS = 100_000_000
_U64_MAX = (1 << 64) - 1

# ProductError categories (src/error.rs:85-93): exit codes.
INTEGRITY = 3
GATE = 5


class TrainerError(RuntimeError):
    """A trainer-level failure shaped like the reference's ProductError:
    ``code`` string, ``category`` exit code, message."""

    def __init__(self, code: str, category: int, message: str):
        self.code = code
        self.category = category
        self.message = message
        super().__init__(f"[{code}] {message}")


def canonical_update_target_count(one_based_update: int) -> int:
    """src/train/trainer.rs:91-99: 65,536 targets per update, 37,888 in the last."""
    if 1 <= one_based_update <= FULL_UPDATES:
        return TARGETS_PER_FULL_UPDATE
    if one_based_update == TOTAL_UPDATES:
        return FINAL_UPDATE_TARGETS
    raise TrainerError("P12_UPDATE_INDEX_INVALID", INTEGRITY,
                       "the optimizer update index is outside the canonical 30,518-update run")


def is_sha256(value: str) -> bool:
    """src/train/trainer.rs:371-375: 64 lowercase hexadecimal characters."""
    return len(value) == 64 and all(c in "0123456789abcdef" for c in value)


def event_boundary_crossed(previous: int, current: int) -> bool:
    """src/train/trainer.rs:1049-1051: the run ended, or a 100M-target
    evaluation boundary was crossed."""
    return current == TOTAL_TARGETS or \
        previous // EVENT_INTERVAL_TARGETS < current // EVENT_INTERVAL_TARGETS


def f32_le_hex(value: float) -> str:
    return struct.pack("<f", value).hex()


def f64_le_hex(value: float) -> str:
    return struct.pack("<d", value).hex()


@dataclass(frozen=True)
class UpdateEvent:
    """src/train/trainer.rs:697-708 without the evaluation result."""

    one_based_update: int
    consumed_targets: int
    valid_targets: int
    normalized_loss_f64_le_hex: str
    learning_rate_f32_le_hex: str
    update_state_sha256: str
    checkpoint_due: bool
    training_complete: bool


class UpdateAccounting:
    """Target accounting of one trainer (src/train/trainer.rs:808-955).

    ``add_batch`` admits a micro-batch (cursor, boundary and loss checks) and
    says whether the update is now due; ``complete_update`` records the
    applied update and returns its event.  Nothing advances when a check
    fails."""

    def __init__(self, consumed_targets: int = 0, completed_updates: int = 0):
        self.consumed_targets = int(consumed_targets)
        self.completed_updates = int(completed_updates)
        self.accumulated_targets = 0
        self.accumulated_loss = 0.0
        self.last_learning_rate: float | None = None
        self.last_update_state_sha256: str | None = None

    @property
    def one_based_update(self) -> int:
        return self.completed_updates + 1

    def required_targets(self) -> int:
        return canonical_update_target_count(self.one_based_update)

    def check_batch(self, first_target: int, valid_targets: int) -> int:
        """The checks before a batch's gradients are touched
        (trainer.rs:810-837); returns the update's required target count."""
        if valid_targets <= 0:  # the target-count part of TrainingBatch::validate (:469-483)
            raise TrainerError("P12_BATCH_SHAPE_INVALID", INTEGRITY,
                               "a training batch must contribute at least one valid target")
        if self.consumed_targets == TOTAL_TARGETS:
            raise TrainerError("P12_TARGET_OVERSHOOT", GATE,
                               "training received another batch after exactly two billion targets")
        first = self.consumed_targets + self.accumulated_targets
        if first > _U64_MAX:
            raise TrainerError("P12_TARGET_ACCOUNTING_OVERFLOW", INTEGRITY,
                               "trainer target accounting overflowed")
        if first_target != first:
            raise TrainerError("P12_TRAINING_CURSOR_MISMATCH", INTEGRITY,
                               "the batch does not begin at the exact deterministic training cursor")
        required = self.required_targets()
        if self.accumulated_targets + valid_targets > required:
            raise TrainerError("P12_UPDATE_TARGET_OVERSHOOT", GATE,
                               "a batch would cross the exact optimizer-update target boundary")
        return required

    def add_batch(self, first_target: int, valid_targets: int, loss_sum: float) -> bool:
        """Admit one micro-batch's loss and targets; True when the update is due."""
        required = self.check_batch(first_target, valid_targets)
        if not math.isfinite(loss_sum):
            raise TrainerError("P12_GRADIENT_NONFINITE", GATE,
                               "a batch returned empty or nonfinite loss or gradients")
        self.accumulated_loss += float(loss_sum)
        self.accumulated_targets += int(valid_targets)
        return self.accumulated_targets == required

    def normalized_loss(self) -> float:
        """trainer.rs:884-890: the f64 loss sum over the update's target count."""
        loss = self.accumulated_loss / float(self.required_targets())
        if not math.isfinite(loss):
            raise TrainerError("P12_LOSS_NONFINITE", GATE,
                               "valid-target-normalized training loss became nonfinite")
        return loss

    def complete_update(self, learning_rate: float, update_state_sha256: str) -> UpdateEvent:
        """trainer.rs:905-955: validate the state identity, advance the
        cursor, reset the accumulators, report the event."""
        required = self.required_targets()
        if self.accumulated_targets != required:
            raise TrainerError("P12_UPDATE_INDEX_INVALID", INTEGRITY,
                               "an update was recorded before its targets were accumulated")
        loss = self.normalized_loss()
        if not isinstance(update_state_sha256, str) or not is_sha256(update_state_sha256):
            raise TrainerError("P12_UPDATE_STATE_INVALID", GATE,
                               "the backend update did not return a lowercase SHA-256 state "
                               "identity")
        previous = self.consumed_targets
        consumed = previous + required
        if consumed > _U64_MAX:
            raise TrainerError("P12_TARGET_ACCOUNTING_OVERFLOW", INTEGRITY,
                               "trainer target accounting overflowed")
        t = self.one_based_update
        self.consumed_targets = consumed
        self.completed_updates = t
        self.accumulated_targets = 0
        self.accumulated_loss = 0.0
        self.last_learning_rate = learning_rate
        self.last_update_state_sha256 = update_state_sha256
        due = event_boundary_crossed(previous, consumed)
        return UpdateEvent(one_based_update=t, consumed_targets=consumed, valid_targets=required,
                           normalized_loss_f64_le_hex=f64_le_hex(loss),
                           learning_rate_f32_le_hex=f32_le_hex(learning_rate),
                           update_state_sha256=update_state_sha256, checkpoint_due=due,
                           training_complete=consumed == TOTAL_TARGETS)


def canonical_learning_rate(one_based_update: int) -> float:
    """trainer.rs:102-119 through the C ABI (bit-exact f32)."""
    import ctypes

    from . import _lib

    out = ctypes.c_float()
    _lib.check(_lib.load().slm_canonical_learning_rate(one_based_update, ctypes.byref(out)))
    return out.value


class B200Trainer:
    """``process_batch`` around the device optimizer: micro-batch gradients
    summed on the GPU in arrival order, the update's last micro-batch fused
    with the norm pass (normalised by the target count, fixed-tree norm,
    clip 1.0), the AdamW update pass, then the state hash, all under
    ``UpdateAccounting``.  ``optimizer`` is a ``B200Adamw``; gradients are
    device tensors of P f32 or bf16 values (the backward pass's output)."""

    def __init__(self, optimizer, accounting: UpdateAccounting | None = None):
        import torch

        self.optimizer = optimizer
        self.accounting = accounting or UpdateAccounting()
        self._acc = torch.empty(optimizer.P, dtype=torch.float32,
                                device=f"cuda:{optimizer.device}")
        self._first = True

    def process_batch(self, first_target: int, valid_targets: int, loss_sum: float,
                      gradients, stream=None) -> UpdateEvent | None:
        from . import _lib
        from .optimizer import StepOptions

        acct = self.accounting
        required = acct.check_batch(first_target, valid_targets)
        due = acct.accumulated_targets + valid_targets == required
        if not due:
            self.optimizer.accumulate(self._acc, gradients, overwrite=self._first, stream=stream)
            acct.add_batch(first_target, valid_targets, loss_sum)
            self._first = False
            return None
        lr = canonical_learning_rate(acct.one_based_update)
        opts = StepOptions(learning_rate=lr, one_based_update=acct.one_based_update,
                           static_loss_scale=float(required),
                           nonfinite_policy=_lib.NONFINITE_ERROR)
        saved = (acct.accumulated_targets, acct.accumulated_loss)
        acct.add_batch(first_target, valid_targets, loss_sum)
        try:
            acct.normalized_loss()  # trainer.rs:885-890 checks it before the update
        except TrainerError:
            acct.accumulated_targets, acct.accumulated_loss = saved
            raise
        keep = self.optimizer.norm_pass_accumulate(self._acc, gradients, opts,
                                                   overwrite=self._first, stream=stream)
        self.optimizer.update_pass(opts, stream=stream)
        try:
            self.optimizer.read_result()
        except _lib.SlmError as e:
            # Like the reference, nothing is counted for a batch that failed.
            acct.accumulated_targets, acct.accumulated_loss = saved
            if e.status in (_lib.SLM_ERR_MODEL_GRADIENT_NONFINITE,
                            _lib.SLM_ERR_MODEL_GRADIENT_NORM_NONFINITE):
                raise TrainerError("P12_GRADIENT_NONFINITE", GATE,
                                   "gradient accumulation became nonfinite") from e
            raise
        finally:
            del keep
        self._first = True
        return acct.complete_update(lr, self.optimizer.state_sha256())
