"""CUDA path vs the CPU oracle, through the C ABI (libslmopt.so).

Bar: bit-exact master / m / v / bf16 and bit-equal f64 norm, clip and skip
decision on identical seeded inputs, from tiny ragged tables to the full
135,285,504-parameter gqa-135m-v1 step (fp32 and bf16 gradients).
"""
from __future__ import annotations

import numpy as np
import pytest

import slm_oracle as oracle
from slmopt import B200Adamw, SlmError, StepOptions, TensorTable, _lib, synth
from slmopt.layout import GqaDimensions

pytestmark = pytest.mark.gpu

THREADS = 8


@pytest.fixture(scope="module")
def torch():
    import torch as _torch

    if not _torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    return _torch


def assert_same_bits(got: np.ndarray, want: np.ndarray, what: str):
    g = got.view(np.uint16 if got.dtype == np.uint16 else np.uint32)
    w = want.view(np.uint16 if want.dtype == np.uint16 else np.uint32)
    bad = np.flatnonzero(g != w)
    assert bad.size == 0, (f"{what}: {bad.size} of {g.size} differ; first at {bad[0]}: "
                           f"got {got[bad[0]]!r} want {want[bad[0]]!r}")


def to_device(torch, grads: np.ndarray):
    t = torch.from_numpy(grads)
    return t.cuda()


def oracle_config(opts: StepOptions):
    return oracle.make_config(
        lr=opts.learning_rate, t=opts.one_based_update, beta1=opts.beta1, beta2=opts.beta2,
        eps=opts.epsilon, decay=opts.decay_weight, no_decay=opts.no_decay_weight,
        max_norm=opts.max_grad_norm, apply_clip=opts.apply_clip,
        min_clip_accept=opts.min_clip_accept, nonfinite_policy=opts.nonfinite_policy,
        dynamic=opts.loss_scale_mode == _lib.SCALE_DYNAMIC,
        static_scale=opts.static_loss_scale, growth_interval=opts.growth_interval)


def run_both(torch, table: TensorTable, grads: np.ndarray, opts: StepOptions, seed: int = 0,
             state: dict | None = None, host_grads: bool = False):
    n = table.parameter_count
    state = state if state is not None else synth.optimizer_state(n, seed)
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        g = grads if host_grads else to_device(torch, grads)
        res = opt.step(g, opts)
        got = opt.read_state()
    ost = {k: v.copy() for k, v in state.items()}
    ores = oracle.step(oracle_config(opts), grads, table.offsets, table.decay, ost,
                       threads=THREADS)
    return res, got, ores, ost


def check_equal(res, got, ores, ost):
    assert res.skipped == ores.skipped
    assert res.nonfinite == ores.nonfinite
    assert res.status == ores.status
    if not ores.nonfinite:
        assert res.sum_squares == ores.sum_squares
        assert res.grad_norm == ores.grad_norm
        assert np.float32(res.clip_scale) == np.float32(ores.clip_scale)
    assert res.loss_scale_used == ores.loss_scale_used
    assert res.next_loss_scale == ores.next_loss_scale
    for key in ("master", "moment", "variance", "bf16"):
        assert_same_bits(got[key], ost[key], key)


SMALL = [[1], [3, 5], [7, 9, 11, 4095], [65536, 5, 70000], [768] * 7 + [131075],
         [2048 * 3 + 1, 13, 65536 * 2 + 8]]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("sizes", SMALL, ids=lambda s: f"{len(s)}t{sum(s)}")
def test_small_tables_bit_exact(torch, dtype, sizes):
    rng = np.random.default_rng(len(sizes))
    table = TensorTable.from_sizes(sizes, rng.integers(0, 2, len(sizes)).astype(bool))
    n = table.parameter_count
    scale = 65536.0 if dtype == "bf16" else 1.0
    grads = synth.grads_bf16(n, 5) if dtype == "bf16" else synth.grads_f32(n, 5)
    opts = StepOptions(learning_rate=3e-4, one_based_update=10, static_loss_scale=scale)
    check_equal(*run_both(torch, table, grads, opts, seed=5))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_clipped_step_bit_exact(torch, dtype):
    table = TensorTable.from_sizes([300_001, 77, 5000], [True, False, True])
    n = table.parameter_count
    if dtype == "bf16":
        grads = synth.grads_bf16(n, 8, loss_scale=65536.0 * 40)
        opts = StepOptions(one_based_update=3, static_loss_scale=65536.0)
    else:
        grads = (synth.grads_f32(n, 8) * np.float32(40.0)).astype(np.float32)
        opts = StepOptions(one_based_update=3)
    res, got, ores, ost = run_both(torch, table, grads, opts, seed=8)
    assert ores.clip_scale < 1.0
    check_equal(res, got, ores, ost)


def test_non_power_of_two_scale_uses_true_division(torch):
    # The reference's final update normalises by 37,888 targets (trainer.rs:15).
    table = TensorTable.from_sizes([100_003])
    n = table.parameter_count
    grads = synth.grads_f32(n, 9) * np.float32(37888.0)
    opts = StepOptions(one_based_update=30518, static_loss_scale=37888.0)
    check_equal(*run_both(torch, table, grads.astype(np.float32), opts, seed=9))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_smoke_model_step_bit_exact(torch, dtype):
    # config 0's tensor list (model-smoke.example.json, tied: 20 tensors) on the GPU
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    n = table.parameter_count
    assert n == 4_489_856
    scale = 65536.0 if dtype == "bf16" else 1.0
    grads = synth.grads_bf16(n, 0) if dtype == "bf16" else synth.grads_f32(n, 0)
    opts = StepOptions(learning_rate=3e-4, one_based_update=10, static_loss_scale=scale)
    check_equal(*run_both(torch, table, grads, opts, seed=0))


def test_135m_fp32_step_bit_exact(torch):
    # config 1: gqa-135m-v1, fp32 gradients, t = 10
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    n = table.parameter_count
    grads = synth.grads_f32(n, 0)
    opts = StepOptions(learning_rate=3e-4, one_based_update=10)
    res, got, ores, ost = run_both(torch, table, grads, opts, seed=0)
    check_equal(res, got, ores, ost)
    # the fixed tree is within 1e-6 relative of an f64 sequential sum
    g = grads.astype(np.float64)
    seq = float(np.dot(g, g))
    assert abs(res.sum_squares - seq) <= 1e-6 * seq


def test_135m_bf16_step_and_inf_skip(torch):
    # config 2: bf16 gradients * 65536, dynamic scale; then one injected +inf
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    n = table.parameter_count
    state = synth.optimizer_state(n, 0)
    grads = synth.grads_bf16(n, 0)
    opts = StepOptions(learning_rate=3e-4, one_based_update=10,
                       loss_scale_mode=_lib.SCALE_DYNAMIC)
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        opt.set_loss_scale(65536.0)
        res = opt.step(to_device(torch, grads), opts)
        got = opt.read_state()
        ost = {k: v.copy() for k, v in state.items()}
        scaler = oracle.Scaler(65536.0, 0)
        ores = oracle.step(oracle_config(opts), grads, table.offsets, table.decay, ost, scaler,
                           threads=THREADS)
        check_equal(res, got, ores, ost)
        assert res.skipped == 0 and opt.loss_scale() == (65536.0, 1)

        bad = grads.copy()
        k, i = synth.inject_nonfinite(bad, 1, table.offsets)
        res2 = opt.step(to_device(torch, bad), StepOptions(
            learning_rate=3e-4, one_based_update=11, loss_scale_mode=_lib.SCALE_DYNAMIC))
        after = opt.read_state()
        assert res2.skipped == 1 and res2.nonfinite == 1 and res2.status == 0
        assert res2.loss_scale_used == 65536.0 and res2.next_loss_scale == 32768.0
        assert opt.loss_scale() == (32768.0, 0)
        for key in got:
            assert_same_bits(after[key], got[key], key + " after skip")


def test_runs_are_bit_identical(torch):
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    n = table.parameter_count
    grads = synth.grads_bf16(n, 2)
    opts = StepOptions(one_based_update=10, static_loss_scale=65536.0)
    outs = []
    for _ in range(2):
        res, got, _, _ = run_both(torch, table, grads, opts, seed=2)
        outs.append((res.sum_squares, got))
    assert outs[0][0] == outs[1][0]
    for key in outs[0][1]:
        assert_same_bits(outs[0][1][key], outs[1][1][key], key)


def test_host_gradients_equal_device_gradients(torch):
    table = TensorTable.from_sizes([70_000, 33])
    n = table.parameter_count
    grads = synth.grads_bf16(n, 4)
    opts = StepOptions(one_based_update=2, static_loss_scale=65536.0)
    r1, g1, _, _ = run_both(torch, table, grads, opts, seed=4)
    r2, g2, _, _ = run_both(torch, table, grads, opts, seed=4, host_grads=True)
    assert r1.sum_squares == r2.sum_squares
    for key in g1:
        assert_same_bits(g1[key], g2[key], key)


def test_async_step_on_a_stream_then_read_result(torch):
    table = TensorTable.from_sizes([123_457])
    n = table.parameter_count
    state = synth.optimizer_state(n, 6)
    grads = synth.grads_f32(n, 6)
    s = torch.cuda.Stream()
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        with torch.cuda.stream(s):
            dev = to_device(torch, grads)
        assert opt.step(dev, StepOptions(one_based_update=4), stream=s, wait=False) is None
        res = opt.read_result()
        got = opt.read_state()
    ost = {k: v.copy() for k, v in state.items()}
    ores = oracle.step(oracle.make_config(t=4), grads, table.offsets, table.decay, ost)
    check_equal(res, got, ores, ost)


def test_phase_timing_leaves_results_unchanged(torch):
    table = TensorTable.from_sizes([200_003, 768])
    n = table.parameter_count
    grads = synth.grads_bf16(n, 8)
    state = synth.optimizer_state(n, 8)
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        opt.phase_timing(True)
        dev = to_device(torch, grads)
        for t in range(1, 5):
            res = opt.step(dev, StepOptions(one_based_update=t, static_loss_scale=65536.0))
        times, steps = opt.phase_times()
        got = opt.read_state()
        opt.phase_timing(False)
        assert opt.phase_times() == ({}, 0)
    assert steps == 4 and list(times) == ["norm pass", "update"]
    assert all(ms > 0.0 for ms in times.values())
    ost = {k: v.copy() for k, v in state.items()}
    for t in range(1, 5):
        ores = oracle.step(oracle.make_config(t=t, static_scale=65536.0), grads, table.offsets,
                           table.decay, ost)
    check_equal(res, got, ores, ost)


def test_export_weights_f32_is_the_graph_reload_values(torch):
    # after a step, the f32 export equals bf16_bits_to_f32 of the bf16 copy,
    # which the oracle's step produced bit-exactly
    table = TensorTable.from_sizes([65536 * 2 + 24, 768, 13])
    n = table.parameter_count
    grads = synth.grads_bf16(n, 9)
    state = synth.optimizer_state(n, 9)
    opts = StepOptions(one_based_update=5, static_loss_scale=65536.0)
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        opt.step(to_device(torch, grads), opts)
        w = opt.export_weights_f32().cpu().numpy()
        with pytest.raises(ValueError):
            opt.export_weights_f32(torch.empty(n - 1, dtype=torch.float32, device="cuda"))
    ost = {k: v.copy() for k, v in state.items()}
    oracle.step(oracle_config(opts), grads, table.offsets, table.decay, ost)
    assert_same_bits(w, synth.bf16_bits_to_f32(ost["bf16"]), "f32 weights")


@pytest.mark.parametrize("t", [1, 3, 10, 200, 1000])
def test_wide_exponent_moments_bit_exact(torch, t):
    # m and v spread over (almost) every f32 exponent, with zeros, -0.0 and
    # subnormals (kept: the library builds with -ftz=false): the divisions,
    # the square root and the bf16 rounding must equal the oracle's bit for
    # bit at the edges of the range too, for small and large t.
    table = TensorTable.from_sizes([70_000, 4101], [True, False])
    n = table.parameter_count
    rng = np.random.default_rng(t)
    state = synth.optimizer_state(n, 12)
    sign = np.where(rng.random(n) < 0.5, -1.0, 1.0)
    m = (sign * np.exp2(rng.uniform(-149, 20, n))).astype(np.float32)
    v = np.exp2(rng.uniform(-149, 40, n)).astype(np.float32)
    m[:64] = 0.0
    m[64:128] = -0.0
    v[:32] = 0.0
    m[128:192] = (np.arange(64) * np.float32(2.0**-149)).astype(np.float32)  # subnormals
    state["moment"], state["variance"] = m, v
    grads = synth.grads_f32(n, 12)
    grads[200:264] = 0.0
    opts = StepOptions(one_based_update=t)
    res, got, ores, ost = run_both(torch, table, grads, opts, state=state)
    check_equal(res, got, ores, ost)


def test_pipelined_uploads_match_oracle(torch):
    # the next update's gradients are uploaded before stepping on the current
    # ones (copy on the handle's stream, step on the caller's): same results
    # as the oracle's sequential steps; misuse is rejected
    table = TensorTable.from_sizes([65536 * 3 + 5, 768], [True, False])
    n = table.parameter_count
    steps = 5
    grads = [synth.grads_bf16(n, 100 + t) for t in range(steps)]
    pinned = [torch.from_numpy(g.view(np.int16)).pin_memory() for g in grads]
    state = synth.optimizer_state(n, 14)
    s = torch.cuda.Stream()
    res = []
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        opt.set_loss_scale(65536.0)
        slot = opt.upload(pinned[0])
        for t in range(1, steps + 1):
            nxt = opt.upload(pinned[t]) if t < steps else None
            if t == 1:
                with pytest.raises(SlmError) as e:
                    opt.upload(pinned[0])  # both slots hold gradients not yet stepped on
                assert e.value.status == _lib.SLM_ERR_INVALID_ARGUMENT
            res.append(opt.step_uploaded(slot, StepOptions(
                one_based_update=t, loss_scale_mode=_lib.SCALE_DYNAMIC), stream=s))
            slot = nxt
        with pytest.raises(SlmError):
            opt.step_uploaded(0, StepOptions(one_based_update=9))  # nothing uploaded there
        got = opt.read_state()
    ost = {k: v.copy() for k, v in state.items()}
    scaler = oracle.Scaler(65536.0, 0)
    for t in range(1, steps + 1):
        ores = oracle.step(oracle.make_config(t=t, dynamic=True), grads[t - 1], table.offsets,
                           table.decay, ost, scaler)
        assert res[t - 1].sum_squares == ores.sum_squares, t
        assert np.float32(res[t - 1].clip_scale) == np.float32(ores.clip_scale), t
    for key in ("master", "moment", "variance", "bf16"):
        assert_same_bits(got[key], ost[key], key)


def test_misaligned_device_gradients_are_rejected(torch):
    table = TensorTable.from_sizes([64])
    buf = torch.zeros(65, dtype=torch.float32, device="cuda")
    with B200Adamw(table) as opt:
        with pytest.raises(SlmError) as e:
            opt.step(buf[1:], StepOptions())
        assert e.value.code == "SLM_INVALID_ARGUMENT"


def test_error_policy_leaves_state_unchanged(torch):
    table = TensorTable.from_sizes([5000, 100], [True, False])
    n = table.parameter_count
    state = synth.optimizer_state(n, 3)
    grads = synth.grads_f32(n, 3)
    grads[4321] = np.nan
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        with pytest.raises(SlmError) as e:
            opt.step(to_device(torch, grads), StepOptions(nonfinite_policy=_lib.NONFINITE_ERROR))
        assert e.value.code == "MODEL_GRADIENT_NONFINITE" and e.value.category == 5
        got = opt.read_state()
    for key in got:
        assert_same_bits(got[key], state[key], key)


# ---- strict TrainerBackend::apply_update drop-in ------------------------------------
def test_apply_update_two_parameter_canonical_adamw(torch):
    # tests/p12_trainer.rs:331-362 through the C ABI, hashed like trainer.rs:297-320
    table = TensorTable(names=("matrix.weight", "norm.weight"), shapes=((1,), (1,)),
                        elements=(1, 1), decay=(True, False))
    st0 = {"master": np.ones(2, np.float32), "moment": np.zeros(2, np.float32),
           "variance": np.zeros(2, np.float32), "bf16": np.full(2, 0x3F80, np.uint16)}
    lr = oracle.canonical_learning_rate(1)[1]
    with B200Adamw(table) as opt:
        opt.load_state(st0["master"], st0["moment"], st0["variance"], st0["bf16"])
        before = opt.state_sha256()
        after = opt.apply_normalized_clipped_gradients(np.array([0.5, 0.5], np.float32), lr, 1)
        got = opt.read_state()
    ost = {k: v.copy() for k, v in st0.items()}
    assert oracle.apply_normalized_clipped_gradients(
        np.array([0.5, 0.5], np.float32), lr, 1, table.offsets, table.decay, ost)[0] == 0
    assert oracle.state_sha256(table.names, table.offsets, table.decay, st0)[1] == before
    assert oracle.state_sha256(table.names, table.offsets, table.decay, ost)[1] == after
    assert before != after
    assert got["master"][0] < got["master"][1]
    for key in got:
        assert_same_bits(got[key], ost[key], key)


def test_apply_update_rejections_match_reference(torch):
    table = TensorTable.from_sizes([1000, 24], [True, False])
    n = table.parameter_count
    state = synth.optimizer_state(n, 1)
    lr1 = oracle.canonical_learning_rate(1)[1]
    small = (synth.grads_f32(n, 1) * np.float32(0.01)).astype(np.float32)
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        cases = [
            (small[:-1], lr1, 1, "P12_OPTIMIZER_GRADIENT_INVALID"),
            (np.where(np.arange(n) == 7, np.float32(np.inf), small).astype(np.float32), lr1, 1,
             "MODEL_GRADIENT_NONFINITE"),
            ((small * np.float32(1e4)).astype(np.float32), lr1, 1, "P12_OPTIMIZER_GRADIENT_INVALID"),
            (small, lr1, 1 << 33, "P12_UPDATE_INDEX_INVALID"),
            (small, lr1, 0, "P12_SCHEDULE_INDEX_INVALID"),
            (small, 3e-4, 1, "P12_SCHEDULER_STATE_MISMATCH"),
        ]
        for g, lr, t, code in cases:
            with pytest.raises(SlmError) as e:
                opt.apply_normalized_clipped_gradients(g, lr, t, with_sha=False)
            assert e.value.code == code
            if len(g) == n:
                ost = {k: v.copy() for k, v in state.items()}
                assert oracle.apply_normalized_clipped_gradients(
                    g, lr, t, table.offsets, table.decay, ost)[0] == getattr(oracle, code)
        got = opt.read_state()
    for key in got:
        assert_same_bits(got[key], state[key], key)


def test_reference_known_answers_on_the_device(torch):
    # The reference's own optimizer KATs (src/model/oracle.rs:1464-1481, read as
    # text into tests/golden/reference_kats.json), reproduced by the CUDA path:
    # the AdamW step's moment / variance bits through the fused step, and the
    # clip of [3, 4] / [0, 0] / NaN through the strict apply_update check.
    import json
    from pathlib import Path

    kats = json.loads((Path(__file__).resolve().parent / "golden" /
                       "reference_kats.json").read_text())["values"]
    k = kats["adamw_step"]
    table = TensorTable(names=("w.weight",), shapes=((1,),), elements=(1,), decay=(True,))
    with B200Adamw(table) as opt:
        th = np.array([k["theta"]], np.float32)
        opt.load_state(th, np.array([k["moment"]], np.float32),
                       np.array([k["variance"]], np.float32), synth.bf16_rne_bits(th))
        opt.step(to_device(torch, np.array([k["gradient"]], np.float32)),
                 StepOptions(learning_rate=k["learning_rate"], one_based_update=k["t"],
                             decay_weight=k["weight_decay"], apply_clip=False))
        got = opt.read_state()
    assert int(got["moment"].view(np.uint32)[0]) == k["moment_bits"]
    assert int(got["variance"].view(np.uint32)[0]) == k["variance_bits"]
    assert got["master"][0] < k["master_below"]
    assert int(got["bf16"][0]) == int(synth.bf16_rne_bits(got["master"])[0])

    two = TensorTable(names=("a.weight", "b.weight"), shapes=((1,), (1,)), elements=(1, 1),
                      decay=(True, True))
    st = synth.optimizer_state(2, 0)
    lr1 = oracle.canonical_learning_rate(1)[1]
    with B200Adamw(two) as opt:
        opt.load_state(st["master"], st["moment"], st["variance"], st["bf16"])
        with pytest.raises(SlmError) as e:  # clip [3, 4] = 0.2: rejected, 0.2 reported
            opt.apply_normalized_clipped_gradients(
                np.array(kats["clip_3_4"]["input"], np.float32), lr1, 1, with_sha=False)
        assert e.value.code == "P12_OPTIMIZER_GRADIENT_INVALID"
        assert f"{float(np.float32(kats['clip_3_4']['expected_f32'])):e}" in e.value.message
        with pytest.raises(SlmError) as e:
            opt.apply_normalized_clipped_gradients(
                np.array([np.nan, 1.0], np.float32), lr1, 1, with_sha=False)
        assert e.value.code == kats["clip_nan"]["expected_code"]
        # [0, 0] re-verifies at exactly 1.0 and is applied
        opt.apply_normalized_clipped_gradients(
            np.array(kats["clip_zero"]["input"], np.float32), lr1, 1, with_sha=False)


def test_apply_update_accepts_the_production_width_clip_probe(torch):
    # tests/p12_trainer.rs:406-446 at the canonical width: g_i = ((i % 977) - 488)
    # * 1e-3, clipped once with the reference's own sequential f32 clip scale
    # (oracle.rs:486-507).  The strict apply_update re-verifies the clip over
    # the fixed tree, must accept it (tolerance 0.05), and update exactly like
    # the oracle's strict apply.
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    n = table.parameter_count
    g = ((np.arange(n) % 977).astype(np.float32) - np.float32(488.0)) * np.float32(1e-3)
    st, scale = oracle.gradient_clip_scale(g)
    assert st == oracle.OK and 0.0 < scale < 1.0
    g = (g * np.float32(scale)).astype(np.float32)
    state = synth.optimizer_state(n, 3)
    lr = oracle.canonical_learning_rate(1)[1]
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        opt.apply_normalized_clipped_gradients(g, lr, 1, with_sha=False)
        got = opt.read_state()
    ost = {k: v.copy() for k, v in state.items()}
    assert oracle.apply_normalized_clipped_gradients(g, lr, 1, table.offsets, table.decay,
                                                     ost)[0] == oracle.OK
    for key in ("master", "moment", "variance", "bf16"):
        assert_same_bits(got[key], ost[key], key)


def test_apply_update_matches_oracle_over_steps(torch):
    table = TensorTable.from_dimensions(GqaDimensions.oracle_fixture())
    n = table.parameter_count
    master = synth.bf16_bits_to_f32(synth.bf16_rne_bits(synth.normal_f32(n, 0.02, 7, 1)))
    st = {"master": master.copy(), "moment": np.zeros(n, np.float32),
          "variance": np.zeros(n, np.float32), "bf16": synth.bf16_rne_bits(master)}
    ost = {k: v.copy() for k, v in st.items()}
    with B200Adamw(table) as opt:
        opt.load_state(st["master"], st["moment"], st["variance"], st["bf16"])
        for t in range(1, 6):
            g = np.where(np.arange(n) % 3 == 0, np.float32(0.01 * t),
                         np.float32(-0.004)).astype(np.float32)
            lr = oracle.canonical_learning_rate(t)[1]
            sha = opt.apply_normalized_clipped_gradients(g, lr, t)
            assert oracle.apply_normalized_clipped_gradients(
                g, lr, t, table.offsets, table.decay, ost)[0] == 0
            assert sha == oracle.state_sha256(table.names, table.offsets, table.decay, ost)[1]


# ---- codec ------------------------------------------------------------------------------
def test_snapshot_restore_round_trip(torch):
    from slmopt import B200TrainerBackend

    dims = GqaDimensions.oracle_fixture()
    be = B200TrainerBackend(dims)
    n = be.optimizer.P
    master = synth.normal_f32(n, 0.02, 1, 1)
    be.optimizer.init_master(master)
    lr = oracle.canonical_learning_rate(1)[1]
    g = np.where(np.arange(n) % 3 == 0, np.float32(0.01), np.float32(-0.004)).astype(np.float32)
    updated = be.apply_update(g, lr, 1, 65536)
    arts = be.snapshot()
    assert [a[0] for a in arts] == ["parameters_bf16", "master_parameters_fp32",
                                    "adamw_first_moments_fp32", "adamw_second_moments_fp32"]
    assert len(arts[0][2]) == 2 * n and all(len(a[2]) == 4 * n for a in arts[1:])
    be2 = B200TrainerBackend(dims)
    be2.restore(arts)
    assert be2.state_sha256() == updated
    assert be2.snapshot() == arts
    bad = [(r, p, b) for r, p, b in arts if r != "adamw_first_moments_fp32"]
    with pytest.raises(SlmError) as e:
        be2.restore(bad)
    assert e.value.code == "E1_STATE_ARTIFACT_INVALID"
    truncated = [(r, p, b[:-4] if r == "master_parameters_fp32" else b) for r, p, b in arts]
    with pytest.raises(SlmError) as e:
        be2.restore(truncated)
    assert e.value.code == "E1_STATE_ARTIFACT_INVALID"


def test_validate_rejects_inconsistent_state(torch):
    table = TensorTable.from_sizes([100])
    st = synth.optimizer_state(100, 1)
    bf = st["bf16"].copy()
    bf[50] ^= 1
    with B200Adamw(table) as opt:
        with pytest.raises(SlmError) as e:
            opt.load_state(st["master"], st["moment"], st["variance"], bf)
        assert e.value.code == "P12_OPTIMIZER_STATE_INVALID"
        m = st["moment"].copy()
        m[3] = np.inf
        with pytest.raises(SlmError):
            opt.load_state(st["master"], m, st["variance"], st["bf16"])


# ---- 100-step trajectory (config 4 at the smoke tensor list) ------------------------------
def test_stress_trajectory_bit_exact_and_repeatable(torch):
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    n = table.parameter_count
    steps = 100
    inject = {17, 63}

    def run_gpu():
        st = synth.optimizer_state(n, 0)
        results = []
        with B200Adamw(table) as opt:
            opt.load_state(st["master"], st["moment"], st["variance"], st["bf16"])
            opt.set_loss_scale(65536.0)
            scale = 65536.0
            for t in range(1, steps + 1):
                g = synth.grads_student_t(n, 0, t)
                bits = synth.bf16_rne_bits((g * np.float32(scale)).astype(np.float32))
                if t in inject:
                    synth.inject_nonfinite(bits, t, table.offsets)
                lr = oracle.schedule_learning_rate(t, 3e-4, 3e-5, 20, 100)[1]
                r = opt.step(to_device(torch, bits), StepOptions(
                    learning_rate=lr, one_based_update=t, loss_scale_mode=_lib.SCALE_DYNAMIC))
                results.append((r.skipped, r.sum_squares, r.clip_scale, r.next_loss_scale))
                scale = r.next_loss_scale
            return results, opt.read_state()

    res_a, state_a = run_gpu()
    res_b, state_b = run_gpu()
    assert res_a == res_b
    for key in state_a:
        assert_same_bits(state_a[key], state_b[key], key)

    ost = synth.optimizer_state(n, 0)
    scaler = oracle.Scaler(65536.0, 0)
    for t in range(1, steps + 1):
        g = synth.grads_student_t(n, 0, t)
        bits = synth.bf16_rne_bits((g * np.float32(scaler.scale)).astype(np.float32))
        if t in inject:
            synth.inject_nonfinite(bits, t, table.offsets)
        lr = oracle.schedule_learning_rate(t, 3e-4, 3e-5, 20, 100)[1]
        r = oracle.step(oracle.make_config(lr=lr, t=t, dynamic=True), bits, table.offsets,
                        table.decay, ost, scaler, threads=THREADS)
        skipped, s, c, nxt = res_a[t - 1]
        assert skipped == r.skipped, t
        if not r.skipped:
            assert s == r.sum_squares and np.float32(c) == np.float32(r.clip_scale), t
        assert nxt == r.next_loss_scale
    assert sum(x[0] for x in res_a) == len(inject)
    for key in state_a:
        assert_same_bits(state_a[key], ost[key], key)


# ---- micro-batch accumulation (src/train/trainer.rs:856-904) ------------------------------
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_accumulated_micro_batches_then_fused_norm_and_update(torch, dtype):
    # Four micro-batch gradient sums accumulated in f32 on the device, the last
    # one fused with the norm pass, normalised by the update's 65,536 targets;
    # equal, bit for bit, to the oracle step on the host-accumulated gradient.
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    n = table.parameter_count
    micro = []
    for i in range(4):
        g = (synth.grads_f32(n, 20 + i) * np.float32(16384.0)).astype(np.float32)
        micro.append(synth.bf16_rne_bits(g) if dtype == "bf16" else g)
    as_f32 = [synth.bf16_bits_to_f32(m) if dtype == "bf16" else m for m in micro]
    want_acc = as_f32[0].copy()
    for m in as_f32[1:]:
        want_acc = (want_acc + m).astype(np.float32)
    opts = StepOptions(learning_rate=3e-4, one_based_update=7, static_loss_scale=65536.0)
    state = synth.optimizer_state(n, 21)
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        acc = torch.empty(n, dtype=torch.float32, device="cuda")
        dev = [to_device(torch, m) for m in micro]
        opt.accumulate(acc, dev[0], overwrite=True)
        opt.accumulate(acc, dev[1])
        opt.accumulate(acc, dev[2])
        keep = opt.norm_pass_accumulate(acc, dev[3], opts)
        opt.update_pass(opts)
        res = opt.read_result()
        del keep
        got = opt.read_state()
        got_acc = acc.cpu().numpy()
    assert_same_bits(got_acc, want_acc, "accumulator")
    ost = {k: v.copy() for k, v in state.items()}
    ores = oracle.step(oracle.make_config(lr=3e-4, t=7, static_scale=65536.0), want_acc,
                       table.offsets, table.decay, ost, threads=THREADS)
    check_equal(res, got, ores, ost)


# ---- the trainer's update bookkeeping around the device step (trainer.rs:808-955) ------
def test_trainer_process_batch_drives_the_device_step(torch):
    # Two updates of four micro-batches each through B200Trainer: gradients
    # summed on the device, the last micro-batch fused with the norm pass
    # (normalised by 65,536 targets), the canonical learning rate, the update
    # pass and the state hash; the state after each update equals the oracle's
    # step on the host-summed gradient, and the events carry the reference's
    # accounting.
    from slmopt import trainer as tr

    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    n = table.parameter_count
    state = synth.optimizer_state(n, 31)
    ost = {k: v.copy() for k, v in state.items()}
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        run = tr.B200Trainer(opt)
        cursor = 0
        for t in (1, 2):
            micro = [(synth.grads_f32(n, 40 + 4 * t + i) * np.float32(16384.0)).astype(np.float32)
                     for i in range(4)]
            events = []
            for i, m in enumerate(micro):
                events.append(run.process_batch(cursor, 16_384, 2.0 * (i + 1),
                                                to_device(torch, m)))
                cursor += 16_384
            assert events[:3] == [None, None, None]
            ev = events[3]
            acc = micro[0].copy()
            for m in micro[1:]:
                acc = (acc + m).astype(np.float32)
            status, lr = oracle.canonical_learning_rate(t)
            assert status == 0
            ores = oracle.step(oracle.make_config(lr=lr, t=t, static_scale=65536.0,
                                                  nonfinite_policy=1),
                               acc, table.offsets, table.decay, ost, threads=THREADS)
            assert ores.status == 0 and not ores.skipped
            want_sha = oracle.state_sha256(table.names, table.offsets, table.decay, ost)[1]
            assert ev.one_based_update == t and ev.consumed_targets == 65_536 * t
            assert ev.valid_targets == 65_536 and not ev.checkpoint_due
            assert ev.update_state_sha256 == want_sha
            assert ev.learning_rate_f32_le_hex == tr.f32_le_hex(lr)
            assert ev.normalized_loss_f64_le_hex == tr.f64_le_hex(20.0 / 65_536.0)
        # a non-finite micro-batch fails the update and counts nothing
        clean = (synth.grads_f32(n, 99) * np.float32(16384.0)).astype(np.float32)
        bad = clean.copy()
        synth.inject_nonfinite(bad, 2, table.offsets)
        for _ in range(3):
            run.process_batch(cursor, 16_384, 1.0, to_device(torch, clean))
            cursor += 16_384
        with pytest.raises(tr.TrainerError) as e:
            run.process_batch(cursor, 16_384, 1.0, to_device(torch, bad))
        assert e.value.code == "P12_GRADIENT_NONFINITE"
        assert run.accounting.accumulated_targets == 3 * 16_384
        assert run.accounting.completed_updates == 2


# ---- gradient_clip_scale: the reference's sequential f32 sum (oracle.rs:486-507) -------
def _clip_cases():
    rng = np.random.default_rng(5)
    cases = {
        "kat_3_4": np.array([3.0, 4.0], np.float32),
        "zeros": np.zeros(10_000, np.float32),
        "one": np.array([0.5], np.float32),
        "empty": np.zeros(0, np.float32),
    }
    for n in (7, 8191, 8192, 8193, 65_537, 1_000_003):
        cases[f"normal_{n}"] = rng.standard_normal(n).astype(np.float32)
    # exact ties: powers of two whose squares land on half an ulp of the sum
    cases["powers_of_two"] = (2.0 ** rng.integers(-70, 8, 300_000)).astype(np.float32)
    cases["subnormal_squares"] = (rng.standard_normal(200_000) * 1e-22).astype(np.float32)
    cases["leading_zeros"] = np.concatenate(
        [np.zeros(50_000, np.float32), rng.standard_normal(90_000).astype(np.float32) * 1e-3])
    cases["drifting"] = (rng.standard_normal(3_000_000) * 1e-3).astype(np.float32)
    cases["overflow"] = (rng.standard_normal(20_000) * 1e18).astype(np.float32)
    inf = rng.standard_normal(50_000).astype(np.float32)
    inf[31_337] = np.inf
    cases["inf"] = inf
    nan = rng.standard_normal(50_000).astype(np.float32)
    nan[9_000] = np.nan
    cases["nan"] = nan
    # the sum crosses a binade every few hundred terms, inside windows
    cases["crossings"] = np.geomspace(1e-6, 1e3, 400_000).astype(np.float32)
    # large squares early, then small ones: the running f32 sum stops moving
    # for long stretches while the exact prefix keeps growing
    stall = np.full(2_000_000, np.float32(np.sqrt(0.9) * 2.0**-12), np.float32)
    stall[:3] = 1.0
    cases["stalled"] = stall
    late = (rng.standard_normal(100_000) * 1e18).astype(np.float32)
    late[77_777] = np.nan  # after the sum overflowed: still a non-finite gradient
    cases["overflow_then_nan"] = late
    return cases


CLIP_CASES = _clip_cases()


@pytest.mark.parametrize("parallel", [True, False], ids=["all_sms", "one_cta"])
@pytest.mark.parametrize("name", sorted(CLIP_CASES))
def test_gradient_clip_scale_is_the_reference_sequential_sum(torch, name, parallel):
    from slmopt.optimizer import gradient_clip_scale

    g = CLIP_CASES[name]
    dev = torch.from_numpy(g).cuda() if g.size else torch.zeros(0, dtype=torch.float32,
                                                                 device="cuda")
    status, got_sum, got_clip = gradient_clip_scale(dev, parallel=parallel)
    want_status, want_clip = oracle.gradient_clip_scale(g)
    sum_status, want_sum = oracle.reference_sum_squares(g)
    assert status == want_status, (status, want_status)
    if want_status == 0:
        assert np.float32(got_sum).view(np.uint32) == np.float32(want_sum).view(np.uint32)
        assert np.float32(got_clip).view(np.uint32) == np.float32(want_clip).view(np.uint32)
    elif want_status == oracle.MODEL_GRADIENT_NORM_NONFINITE:
        assert sum_status == 0 and not np.isfinite(want_sum) and not np.isfinite(got_sum)


@pytest.mark.parametrize("parallel", [True, False], ids=["all_sms", "one_cta"])
def test_gradient_clip_scale_at_production_width(torch, parallel):
    # the reference's 135,285,504-element probe shape: a clipped gradient whose
    # sequential f32 sum drifts ~35 % below the exact one
    from slmopt.optimizer import gradient_clip_scale

    n = 135_285_504
    g = synth.grads_f32(n, 1)
    g *= np.float32(0.9 / float(np.sqrt(np.sum(g.astype(np.float64) ** 2))))
    status, got_sum, got_clip = gradient_clip_scale(torch.from_numpy(g).cuda(), parallel=parallel)
    st, want_sum = oracle.reference_sum_squares(g)
    assert status == 0 and st == 0
    assert np.float32(got_sum).view(np.uint32) == np.float32(want_sum).view(np.uint32)
    assert got_clip == 1.0
    assert got_sum < 0.7 * 0.81  # the drift the exact sum would not show


# ---- pageable host gradients through the pinned ring (several 32 MB slices) --------------
def test_pageable_host_gradients_at_135m_equal_device_gradients(torch):
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    n = table.parameter_count
    grads = synth.grads_bf16(n, 6)  # numpy: pageable, 270 MB = 9 slices
    opts = StepOptions(one_based_update=4, static_loss_scale=65536.0)
    r1, g1, _, _ = run_both(torch, table, grads, opts, seed=6)
    r2, g2, ores, ost = run_both(torch, table, grads, opts, seed=6, host_grads=True)
    check_equal(r2, g2, ores, ost)
    assert r1.sum_squares == r2.sum_squares
    for key in g1:
        assert_same_bits(g1[key], g2[key], key)


def test_apply_update_rejects_late_slices_like_the_reference(torch):
    # The strict path checks slice by slice as the upload lands: a non-finite
    # value in slice 15 of 17, or a gradient too large for the 0.95 clip
    # tolerance, must still be refused with nothing written.
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    n = table.parameter_count
    g = synth.grads_f32(n, 9)
    g *= np.float32(0.5 / float(np.sqrt(np.sum(g.astype(np.float64) ** 2))))
    state = synth.optimizer_state(n, 9)
    lr = oracle.canonical_learning_rate(1)[1]
    bad = g.copy()
    bad[125_000_003] = np.inf
    big = (g * np.float32(30.0)).astype(np.float32)
    with B200Adamw(table) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
        for grads, want in ((bad, oracle.MODEL_GRADIENT_NONFINITE),
                            (big, oracle.P12_OPTIMIZER_GRADIENT_INVALID)):
            assert oracle.apply_normalized_clipped_gradients(
                grads, lr, 1, table.offsets, table.decay,
                {k: v.copy() for k, v in state.items()})[0] == want
            with pytest.raises(SlmError) as e:
                opt.apply_normalized_clipped_gradients(grads, lr, 1, with_sha=False)
            assert e.value.status == want
        got = opt.read_state()
        for key in ("master", "moment", "variance", "bf16"):
            assert_same_bits(got[key], state[key], key)
        # and a good one afterwards still matches the oracle bit for bit
        opt.apply_normalized_clipped_gradients(g, lr, 1, with_sha=False)
        got = opt.read_state()
    ost = {k: v.copy() for k, v in state.items()}
    assert oracle.apply_normalized_clipped_gradients(g, lr, 1, table.offsets, table.decay,
                                                     ost)[0] == oracle.OK
    for key in ("master", "moment", "variance", "bf16"):
        assert_same_bits(got[key], ost[key], key)
