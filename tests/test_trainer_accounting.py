"""Update bookkeeping around the optimizer step (src/train/trainer.rs:808-955):
target accounting, update events and their failure codes, on the host.

The expected values are the reference's own: the canonical plan's arithmetic
(trainer.rs:12-19, 91-99), the event boundaries (trainer.rs:1049-1051), the
first update (p12_trainer.rs:221-231: update 1, no checkpoint due) and the
final partial update (p12_trainer.rs:283-309: 37,888 targets, exactly two
billion consumed, checkpoint due, training complete, a further batch refused
with P12_TARGET_OVERSHOOT); learning-rate bits come from the oracle."""
from __future__ import annotations

import math
import struct

import pytest

import slm_oracle as oracle
from slmopt import trainer as tr


def sha(i: int) -> str:
    return f"{i:064x}"


def test_canonical_plan_arithmetic():
    assert tr.canonical_update_target_count(1) == 65_536
    assert tr.canonical_update_target_count(tr.FULL_UPDATES) == 65_536
    assert tr.canonical_update_target_count(tr.TOTAL_UPDATES) == 37_888
    for bad in (0, tr.TOTAL_UPDATES + 1):
        with pytest.raises(tr.TrainerError) as e:
            tr.canonical_update_target_count(bad)
        assert e.value.code == "P12_UPDATE_INDEX_INVALID" and e.value.category == 3
    assert tr.FULL_UPDATES * tr.TARGETS_PER_FULL_UPDATE + tr.FINAL_UPDATE_TARGETS == \
        tr.TOTAL_TARGETS


def test_first_update_event_and_micro_batch_accounting():
    acct = tr.UpdateAccounting()
    # four micro-batches of 16,384 targets make the first update
    losses = [1.5, 2.25, 0.75, 3.0]
    for k, loss in enumerate(losses):
        due = acct.add_batch(k * 16_384, 16_384, loss * 16_384)
        assert due == (k == 3)
    status, lr = oracle.canonical_learning_rate(1)
    assert status == 0
    lr_bits = struct.unpack("<I", struct.pack("<f", lr))[0]
    ev = acct.complete_update(lr, sha(7))
    assert ev.one_based_update == 1
    assert ev.consumed_targets == 65_536 and ev.valid_targets == 65_536
    assert not ev.checkpoint_due and not ev.training_complete
    assert ev.learning_rate_f32_le_hex == struct.pack("<I", lr_bits).hex()
    want_loss = sum(x * 16_384 for x in losses) / 65_536.0
    assert ev.normalized_loss_f64_le_hex == struct.pack("<d", want_loss).hex()
    assert ev.update_state_sha256 == sha(7)
    assert acct.accumulated_targets == 0 and acct.accumulated_loss == 0.0
    assert acct.last_learning_rate == lr and acct.last_update_state_sha256 == sha(7)


def test_checkpoint_boundary_every_hundred_million_targets():
    # update 1,526 is the first whose targets cross 100,000,000
    acct = tr.UpdateAccounting(consumed_targets=1_524 * 65_536, completed_updates=1_524)
    for t in (1_525, 1_526):
        acct.add_batch(acct.consumed_targets, 65_536, 1.0)
        ev = acct.complete_update(oracle.canonical_learning_rate(t)[1], sha(t))
        assert ev.one_based_update == t
        assert ev.checkpoint_due == (t == 1_526)
    assert tr.event_boundary_crossed(99_942_400, 100_007_936)
    assert not tr.event_boundary_crossed(0, 65_536)


def test_final_partial_update_reaches_exact_target_and_rejects_overshoot():
    first = tr.FULL_UPDATES * tr.TARGETS_PER_FULL_UPDATE
    acct = tr.UpdateAccounting(consumed_targets=first, completed_updates=tr.FULL_UPDATES)
    assert acct.add_batch(first, tr.FINAL_UPDATE_TARGETS, 10.0)
    ev = acct.complete_update(oracle.canonical_learning_rate(tr.TOTAL_UPDATES)[1], sha(1))
    assert ev.one_based_update == tr.TOTAL_UPDATES
    assert ev.consumed_targets == tr.TOTAL_TARGETS
    assert ev.valid_targets == tr.FINAL_UPDATE_TARGETS
    assert ev.checkpoint_due and ev.training_complete
    with pytest.raises(tr.TrainerError) as e:
        acct.add_batch(tr.TOTAL_TARGETS, 1, 0.0)
    assert e.value.code == "P12_TARGET_OVERSHOOT" and e.value.category == 5


def test_failed_checks_leave_the_accounting_unchanged():
    acct = tr.UpdateAccounting()
    acct.add_batch(0, 60_000, 1.0)
    cases = [
        ((60_000, 6_000, 1.0), "P12_UPDATE_TARGET_OVERSHOOT", 5),
        ((59_999, 10, 1.0), "P12_TRAINING_CURSOR_MISMATCH", 3),
        ((60_000, 0, 1.0), "P12_BATCH_SHAPE_INVALID", 3),
        ((60_000, 10, math.inf), "P12_GRADIENT_NONFINITE", 5),
    ]
    for args, code, category in cases:
        with pytest.raises(tr.TrainerError) as e:
            acct.add_batch(*args)
        assert (e.value.code, e.value.category) == (code, category)
        assert acct.accumulated_targets == 60_000 and acct.accumulated_loss == 1.0
    with pytest.raises(tr.TrainerError) as e:  # recorded before the boundary
        acct.complete_update(1e-4, sha(1))
    assert e.value.code == "P12_UPDATE_INDEX_INVALID"
    assert acct.add_batch(60_000, 5_536, 2.0)
    for bad in ("A" * 64, sha(3)[:63], "g" * 64, None):
        with pytest.raises(tr.TrainerError) as e:
            acct.complete_update(1e-4, bad)
        assert e.value.code == "P12_UPDATE_STATE_INVALID" and e.value.category == 5
        assert acct.completed_updates == 0 and acct.consumed_targets == 0
    acct.accumulated_loss = math.inf
    with pytest.raises(tr.TrainerError) as e:
        acct.complete_update(1e-4, sha(3))
    assert e.value.code == "P12_LOSS_NONFINITE"
    assert acct.completed_updates == 0


def test_learning_rate_through_the_c_abi_matches_the_oracle():
    for t in (1, 999, 1_000, 1_001, 15_000, tr.TOTAL_UPDATES):
        status, want = oracle.canonical_learning_rate(t)
        assert status == 0
        got = tr.canonical_learning_rate(t)
        assert struct.pack("<f", got) == struct.pack("<f", want)
