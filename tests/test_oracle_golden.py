"""Pin the CPU oracle against the reference's own known-answer tests.

The values come from tests/golden/reference_kats.json, extracted from the
reference's test sources by tests/golden/make_kats.py (file:line recorded per
value).  A failure here means the oracle no longer restates the reference.
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

import slm_oracle as oracle
from slmopt.layout import GqaDimensions, TensorTable


def f32_from_bits(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


def bits_of(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def test_bf16_round_to_nearest_even(kats):
    # src/model/oracle.rs:1388-1394
    for case in kats["bf16_rne"]:
        x = f32_from_bits(int(case["f32_bits"], 16))
        assert oracle.f32_to_bf16_bits(x) == int(case["bf16"], 16), case["at"]
    assert oracle.bf16_bits_to_f32(0x3F80) == 1.0


def test_gradient_clip_scale_kats(kats):
    # src/model/oracle.rs:1466-1474
    st, c = oracle.gradient_clip_scale(np.array(kats["clip_3_4"]["input"], np.float32))
    assert st == oracle.OK
    assert bits_of(c) == bits_of(np.float32(kats["clip_3_4"]["expected_f32"]))
    st, c = oracle.gradient_clip_scale(np.array(kats["clip_zero"]["input"], np.float32))
    assert st == oracle.OK and c == kats["clip_zero"]["expected_f32"]
    st, _ = oracle.gradient_clip_scale(np.array([np.nan], np.float32))
    assert kats["clip_nan"]["expected_code"] == "MODEL_GRADIENT_NONFINITE"
    assert st == oracle.MODEL_GRADIENT_NONFINITE
    st, _ = oracle.gradient_clip_scale(np.array([3e38, 3e38], np.float32))
    assert st == oracle.MODEL_GRADIENT_NORM_NONFINITE


def test_adamw_scalar_step_kat(kats):
    # src/model/oracle.rs:1475-1480
    k = kats["adamw_step"]
    st, (master, moment, variance, storage) = oracle.adamw_scalar_step(
        k["theta"], k["gradient"], k["moment"], k["variance"], k["learning_rate"], k["t"],
        k["weight_decay"])
    assert st == oracle.OK
    assert bits_of(moment) == k["moment_bits"]
    assert bits_of(variance) == k["variance_bits"]
    assert master < k["master_below"]
    assert storage == oracle.f32_to_bf16_bits(float(master))


def test_adamw_scalar_step_rejects_invalid_input():
    # src/model/oracle.rs:518-531 and :544-552
    assert oracle.adamw_scalar_step(1.0, 0.5, 0.0, 0.0, 1e-3, 0, 0.1)[0] == \
        oracle.MODEL_OPTIMIZER_INPUT_INVALID
    assert oracle.adamw_scalar_step(float("inf"), 0.5, 0.0, 0.0, 1e-3, 1, 0.1)[0] == \
        oracle.MODEL_OPTIMIZER_INPUT_INVALID
    assert oracle.adamw_scalar_step(1.0, 0.5, 0.0, 0.0, float("nan"), 1, 0.1)[0] == \
        oracle.MODEL_OPTIMIZER_INPUT_INVALID
    assert oracle.adamw_scalar_step(3e38, 0.5, 0.0, 0.0, -3e38, 1, 0.1)[0] == \
        oracle.MODEL_OPTIMIZER_RESULT_NONFINITE


def test_optimizer_rules_bits(kats):
    # tests/p9b_model_oracle.rs:40-47 -- the constants the oracle and the
    # product's default config both use.
    from slmopt import _lib

    cfg = _lib.default_config()
    r = kats["optimizer_rules"]
    assert r["algorithm"]["value"] == "adamw-opt-001"
    for field, key in (("beta1", "beta1"), ("beta2", "beta2"), ("epsilon", "epsilon"),
                       ("decay_weight", "decay_weight"), ("no_decay_weight", "no_decay_weight"),
                       ("max_grad_norm", "global_l2_clip")):
        assert bits_of(getattr(cfg, field)) == bits_of(np.float32(r[key]["value_f32"])), key


def test_param001_layout(kats):
    # src/model/oracle.rs:1344-1372, tests/p9b_model_oracle.rs:8-37,
    # tests/e1_full_model_backend.rs:35-75
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    assert len(table) == kats["tensor_count"]["value"] == 111
    assert table.parameter_count == kats["canonical_parameter_count"]["value"]
    assert table.layout_sha256() == kats["layout_sha256"]["value"]
    for idx, name in kats["tensor_names"]["value"].items():
        assert table.names[int(idx)] == name
    for idx, shape in kats["tensor_shapes"]["value"].items():
        assert list(table.shapes[int(idx)]) == shape
    no_decay = [n for n, d in zip(table.names, table.decay) if not d]
    assert len(no_decay) == kats["no_decay_tensor_count"]["value"]
    assert all(n.endswith("norm.weight") for n in no_decay)
    assert sum(e for e, d in zip(table.elements, table.decay) if not d) == 19_200
    ref = TensorTable.from_dimensions(GqaDimensions.reference_124m())
    assert ref.parameter_count == kats["reference_parameter_count"]["value"]


def test_canonical_learning_rate(kats):
    # src/train/trainer.rs:102-119 with the constants of :13-22
    c = kats["trainer_constants"]
    peak = np.float32(c["PEAK_LEARNING_RATE"]["value_f32"])
    minimum = np.float32(c["MINIMUM_LEARNING_RATE"]["value_f32"])
    warm = c["WARMUP_UPDATES"]["value"]
    total = c["TOTAL_UPDATES"]["value"]
    assert oracle.canonical_learning_rate(0)[0] == oracle.P12_SCHEDULE_INDEX_INVALID
    assert oracle.canonical_learning_rate(total + 1)[0] == oracle.P12_SCHEDULE_INDEX_INVALID
    for t in (1, 2, 500, warm):
        st, lr = oracle.canonical_learning_rate(t)
        assert st == oracle.OK
        assert bits_of(lr) == bits_of(np.float32(peak * np.float32(t)) / np.float32(warm))
    import math

    for t in (warm + 1, 5000, 20000, total):
        st, lr = oracle.canonical_learning_rate(t)
        progress = (t - warm) / (total - warm)
        expect = float(minimum) + 0.5 * float(np.float32(peak - minimum)) * (
            1.0 + math.cos(math.pi * progress))
        assert bits_of(lr) == bits_of(np.float32(expect))


@pytest.mark.parametrize("count_index", [0, 1, 2, 3])
def test_clip_probe_at_production_width(kats, count_index):
    # tests/p12_trainer.rs:406-446: a clipped gradient still verifies within
    # CLIP_VERIFICATION_TOLERANCE, up to the canonical parameter count.
    probe = kats["clip_probe"]
    count = probe["counts"][count_index]
    if count == "CANONICAL":
        count = kats["canonical_parameter_count"]["value"]
    idx = np.arange(count, dtype=np.int64)
    g = ((idx % probe["modulus"]).astype(np.float32) - np.float32(probe["offset"])) * \
        np.float32(probe["scale"])
    st, scale = oracle.gradient_clip_scale(g)
    assert st == oracle.OK and scale < 1.0
    g *= np.float32(scale)
    st, verified = oracle.gradient_clip_scale(g)
    tol = np.float32(kats["trainer_constants"]["CLIP_VERIFICATION_TOLERANCE"]["value_f32"])
    assert st == oracle.OK and verified >= np.float32(1.0) - tol


def _two_parameter_state():
    # tests/p12_trainer.rs:331-362
    names = ["matrix.weight", "norm.weight"]
    offsets = np.array([0, 1, 2], np.uint64)
    decay = [1, 0]
    state = {"master": np.ones(2, np.float32), "moment": np.zeros(2, np.float32),
             "variance": np.zeros(2, np.float32), "bf16": np.full(2, 0x3F80, np.uint16)}
    return names, offsets, decay, state


def test_canonical_adamw_decay_group_and_moments():
    names, offsets, decay, state = _two_parameter_state()
    st, before = oracle.state_sha256(names, offsets, decay, state)
    assert st == oracle.OK
    lr = oracle.canonical_learning_rate(1)[1]
    st, _ = oracle.apply_normalized_clipped_gradients(
        np.array([0.5, 0.5], np.float32), lr, 1, offsets, decay, state)
    assert st == oracle.OK
    st, after = oracle.state_sha256(names, offsets, decay, state)
    assert before != after
    assert state["master"][0] < state["master"][1]
    assert state["moment"][0] != 0.0 and state["variance"][0] != 0.0


def test_state_rejects_bf16_that_is_not_rne_of_master():
    # tests/p12_trainer.rs:364-383
    st, _ = oracle.state_sha256(["weight"], np.array([0, 1], np.uint64), [1],
                                {"master": np.ones(1, np.float32),
                                 "moment": np.zeros(1, np.float32),
                                 "variance": np.zeros(1, np.float32),
                                 "bf16": np.zeros(1, np.uint16)})
    assert st == oracle.P12_OPTIMIZER_STATE_INVALID


def test_strict_apply_update_error_order():
    # src/train/trainer.rs:235-273: length, clip, u32 index, schedule, lr bits.
    names, offsets, decay, state = _two_parameter_state()
    lr1 = oracle.canonical_learning_rate(1)[1]
    g = np.array([0.5, 0.5], np.float32)
    assert oracle.apply_normalized_clipped_gradients(
        np.array([np.nan, 0.5], np.float32), 1e9, 1, offsets, decay, state)[0] == \
        oracle.MODEL_GRADIENT_NONFINITE
    assert oracle.apply_normalized_clipped_gradients(
        np.array([3.0, 4.0], np.float32), lr1, 1, offsets, decay, state)[0] == \
        oracle.P12_OPTIMIZER_GRADIENT_INVALID
    assert oracle.apply_normalized_clipped_gradients(g, lr1, 1 << 33, offsets, decay, state)[0] \
        == oracle.P12_UPDATE_INDEX_INVALID
    assert oracle.apply_normalized_clipped_gradients(g, lr1, 0, offsets, decay, state)[0] == \
        oracle.P12_SCHEDULE_INDEX_INVALID
    assert oracle.apply_normalized_clipped_gradients(g, 3e-4, 1, offsets, decay, state)[0] == \
        oracle.P12_SCHEDULER_STATE_MISMATCH
    assert np.all(state["master"] == 1.0)  # nothing written before the checks pass


def test_e1_codec_round_trip_after_one_update(kats):
    # tests/e1_full_model_backend.rs:99-149 on the 140-parameter fixture shape:
    # one canonical update, byte snapshot, restore, identical state hash.
    from slmopt import synth

    k = kats["e1_codec"]
    table = TensorTable.from_dimensions(GqaDimensions.oracle_fixture())
    assert table.parameter_count == k["elements"]
    n = table.parameter_count
    master = synth.bf16_bits_to_f32(synth.bf16_rne_bits(synth.normal_f32(n, 0.02, 7, 1)))
    state = {"master": master.copy(), "moment": np.zeros(n, np.float32),
             "variance": np.zeros(n, np.float32), "bf16": synth.bf16_rne_bits(master)}
    g = np.where(np.arange(n) % k["modulus"] == 0, np.float32(k["hit"]),
                 np.float32(k["miss"])).astype(np.float32)
    lr = oracle.canonical_learning_rate(1)[1]
    st, _ = oracle.apply_normalized_clipped_gradients(g, lr, 1, table.offsets, table.decay, state)
    assert st == oracle.OK
    st, updated = oracle.state_sha256(table.names, table.offsets, table.decay, state)
    blobs = {key: state[key].tobytes() for key in state}
    restored = {"master": np.frombuffer(blobs["master"], np.float32).copy(),
                "moment": np.frombuffer(blobs["moment"], np.float32).copy(),
                "variance": np.frombuffer(blobs["variance"], np.float32).copy(),
                "bf16": np.frombuffer(blobs["bf16"], np.uint16).copy()}
    st2, again = oracle.state_sha256(table.names, table.offsets, table.decay, restored)
    assert st == st2 == oracle.OK and again == updated
