"""The committed golden outcomes that bench.py and the GPU tests check against
are reproducible from their generators: the first updates of the stress
trajectory (tests/golden/make_stress_golden.py) and the structure of the
one-step records (tests/golden/make_step_golden.py; the 135M steps themselves
take minutes on the CPU and are re-derived only by the generator)."""
from __future__ import annotations

import json
import struct
from pathlib import Path

import slm_oracle as oracle
from slmopt import GqaDimensions, TensorTable, stress, synth

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_stress_golden_first_updates_match_the_oracle():
    g = json.loads((GOLDEN / "stress_golden.json").read_text())
    assert g["steps"] == stress.STEPS
    assert {int(k): v for k, v in g["inject"].items()} == stress.INJECT
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    P = table.parameter_count
    assert g["params"] == P
    world = 2
    state = synth.optimizer_state(P, 0)
    scaler = oracle.Scaler(65536.0, 0)
    for t in (1, 2, 3):
        st, lr = oracle.schedule_learning_rate(t, stress.PEAK_LR, stress.MIN_LR, stress.WARMUP,
                                               stress.STEPS)
        grads = [stress.rank_gradient(P, table.offsets, r, t, scaler.scale) for r in range(world)]
        res = oracle.step(oracle.make_config(lr=lr, t=t, dynamic=True),
                          oracle.rank_sum_bf16(grads, threads=8), table.offsets, table.decay,
                          state, scaler, threads=8)
        got = [int(res.skipped), float(res.sum_squares).hex(),
               struct.unpack("<I", struct.pack("<f", res.clip_scale))[0],
               float(res.next_loss_scale)]
        assert got == g["worlds"][str(world)]["trace"][t - 1], t
    for w in ("2", "4", "8"):
        rec = g["worlds"][w]
        assert rec["skipped_updates"] == sorted(stress.INJECT)
        assert len(rec["trace"]) == stress.STEPS and len(rec["final_sha256"]) == 64


def test_step_golden_records_are_complete():
    g = json.loads((GOLDEN / "step_golden.json").read_text())
    assert g["params"] == TensorTable.from_dimensions(GqaDimensions.canonical()).parameter_count
    keys = {"sha256", "sum_squares_hex", "clip_scale_bits", "skipped", "nonfinite",
            "next_loss_scale"}
    for rec in [g["mixed"], g["fp32"], *g["zero1"].values(), *g["skip"].values()]:
        assert keys <= set(rec)
    for n, rec in g["skip"].items():
        assert rec["skipped"] == 1 and rec["sha256"] == g["initial_sha256"]
        assert rec["next_loss_scale"] == 32768.0
    assert set(g["zero1"]) == {"2", "4", "8"}
    assert len({g["mixed"]["sha256"], *(r["sha256"] for r in g["zero1"].values())}) == 4
