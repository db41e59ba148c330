"""The oracle's trajectory of the 100-step ZeRO-1 stress run, for 2, 4 and 8 ranks.

The inputs are ``slmopt.stress`` (Student-t(3) x 1e-3 bf16 gradients per rank
and update, dynamic loss scale from 65,536, +inf injected at two seeded
updates, warmup 20 then cosine from 3e-4 to 3e-5) on the smoke tensor list
(4,489,856 parameters) from the seeded state ``synth.optimizer_state(P, 0)``.
For each rank count the expected trajectory is the single replica's step on
the rank-ordered f32 sum of the ranks' bf16 gradients (oracle.rank_sum_bf16),
update after update.  Recorded per update: skipped, the f64 sum of squares
(hex), the clip scale's f32 bits and the next loss scale; and the final
state's SHA-256 (the reference's state_sha256 framing, trainer.rs:297-320).
``bench.py``'s ZeRO-1 arm and ``tests/test_gpu_zero1.py`` compare against it.

    python tests/golden/make_stress_golden.py
"""
from __future__ import annotations

import json
import os
import struct
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
for sub in ("python-slm_b200", "oracle"):
    sys.path.insert(0, str(ROOT / sub))

import slm_oracle as oracle  # noqa: E402
from slmopt import GqaDimensions, TensorTable, stress, synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "stress_golden.json"
WORLDS = (2, 4, 8)


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def trajectory(world: int, threads: int) -> dict:
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    P = table.parameter_count
    state = synth.optimizer_state(P, 0)
    scaler = oracle.Scaler(65536.0, 0)
    trace = []
    for t in range(1, stress.STEPS + 1):
        st, lr = oracle.schedule_learning_rate(t, stress.PEAK_LR, stress.MIN_LR, stress.WARMUP,
                                               stress.STEPS)
        assert st == 0
        grads = [stress.rank_gradient(P, table.offsets, r, t, scaler.scale) for r in range(world)]
        g = oracle.rank_sum_bf16(grads, threads=threads)
        res = oracle.step(oracle.make_config(lr=lr, t=t, dynamic=True), g, table.offsets,
                          table.decay, state, scaler, threads=threads)
        trace.append([int(res.skipped), float(res.sum_squares).hex(), f32_bits(res.clip_scale),
                      float(res.next_loss_scale)])
    st, sha = oracle.state_sha256(table.names, table.offsets, table.decay, state)
    assert st == 0
    assert sum(x[0] for x in trace) == len(stress.INJECT)
    return {"trace": trace, "final_sha256": sha, "skipped_updates": [
        t for t, x in enumerate(trace, 1) if x[0]]}


def main() -> None:
    t0 = time.time()
    threads = os.cpu_count() or 1
    out = {"what": "oracle trajectory of the 100-step ZeRO-1 stress run (smoke tensor list)",
           "generator": "tests/golden/make_stress_golden.py",
           "params": TensorTable.from_dimensions(GqaDimensions.smoke()).parameter_count,
           "steps": stress.STEPS, "inject": {str(k): v for k, v in stress.INJECT.items()},
           "worlds": {str(w): trajectory(w, threads) for w in WORLDS}}
    OUT.write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(f"wrote {OUT} in {time.time() - t0:.0f} s")


if __name__ == "__main__":
    main()
