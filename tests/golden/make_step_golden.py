"""Expected outcome of one optimizer step of the 135M benchmark workload, from the oracle.

bench.py checks the state its GPU run produces against these values after its
timed region (it reads this file; it never runs the oracle), and the GPU tests
can use them too.  Every case starts from the benchmark's seeded state
(``synth.optimizer_state(P, 0)``, dynamic loss scale 65,536) and takes one step
with lr 3e-4, betas (0.9, 0.95), eps 1e-8, decay 0.1 / 0.0, clip 1.0, t = 10:

* ``mixed``  -- bf16 gradients ``synth.grads_bf16(P, 0)`` (N(0,1e-3) x 65,536),
  dynamic scale (the single-GPU bench workload);
* ``fp32``   -- fp32 gradients ``synth.grads_f32(P, 0)``, static scale 1;
* ``zero1/<N>`` -- N ranks, rank r holding ``synth.grads_bf16(P, r)``; the
  expected state is the single replica's step on the rank-ordered f32 sum of
  the N bf16 gradients (oracle.rank_sum_bf16), dynamic scale;
* ``skip/<N>`` -- the same with one +inf written into the last rank's gradient
  by ``synth.inject_nonfinite(bits, 5, offsets)``: the step is skipped, the
  state keeps ``initial_sha256`` and the scale halves to 32,768.

State hashes are the reference's state_sha256 framing (src/train/trainer.rs:297-320).
Run from the repository root (takes a few minutes on 8 cores):

    python tests/golden/make_step_golden.py
"""
from __future__ import annotations

import json
import os
import struct
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
for sub in ("python-slm_b200", "oracle"):
    sys.path.insert(0, str(ROOT / sub))

import numpy as np  # noqa: E402

import slm_oracle as oracle  # noqa: E402
from slmopt import GqaDimensions, TensorTable, synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "step_golden.json"
WORLDS = (2, 4, 8)
LR, T, SCALE = 3e-4, 10, 65536.0
INF_SEED = 5


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def result_record(res, sha: str) -> dict:
    return {"sha256": sha, "sum_squares_hex": float(res.sum_squares).hex(),
            "clip_scale_bits": f32_bits(res.clip_scale), "skipped": int(res.skipped),
            "nonfinite": int(res.nonfinite), "next_loss_scale": float(res.next_loss_scale)}


def main() -> None:
    t0 = time.time()
    threads = os.cpu_count() or 1
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    P = table.parameter_count
    base = synth.optimizer_state(P, 0)

    def sha(state: dict) -> str:
        st, h = oracle.state_sha256(table.names, table.offsets, table.decay, state)
        assert st == 0, st
        return h

    def one_step(grads: np.ndarray, dynamic: bool, static_scale: float = 1.0):
        state = {k: v.copy() for k, v in base.items()}
        scaler = oracle.Scaler(SCALE, 0)
        cfg = oracle.make_config(lr=LR, t=T, dynamic=dynamic, static_scale=static_scale)
        res = oracle.step(cfg, grads, table.offsets, table.decay, state,
                          scaler if dynamic else None, threads=threads)
        return result_record(res, sha(state))

    out = {"what": "one optimizer step of the 135M benchmark workload from the seeded state",
           "generator": "tests/golden/make_step_golden.py",
           "params": P, "tensors": len(table), "lr": LR, "t": T, "initial_loss_scale": SCALE,
           "initial_sha256": sha(base)}
    out["mixed"] = one_step(synth.grads_bf16(P, 0), dynamic=True)
    out["fp32"] = one_step(synth.grads_f32(P, 0), dynamic=False, static_scale=1.0)
    with ThreadPoolExecutor(max_workers=min(8, threads)) as ex:
        grads = list(ex.map(lambda r: synth.grads_bf16(P, r), range(max(WORLDS))))
    out["zero1"], out["skip"] = {}, {}
    for n in WORLDS:
        out["zero1"][str(n)] = one_step(oracle.rank_sum_bf16(grads[:n], threads=threads),
                                        dynamic=True)
    for n in (1,) + WORLDS:
        bad = [g if r < n - 1 else g.copy() for r, g in enumerate(grads[:n])]
        k, i = synth.inject_nonfinite(bad[n - 1], INF_SEED, table.offsets)
        rec = one_step(oracle.rank_sum_bf16(bad, threads=threads) if n > 1 else bad[0],
                       dynamic=True)
        assert rec["skipped"] == 1 and rec["sha256"] == out["initial_sha256"], rec
        rec["inf_at"] = {"rank": n - 1, "tensor": k, "index": i}
        out["skip"][str(n)] = rec
    OUT.write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(f"wrote {OUT} in {time.time() - t0:.0f} s")


if __name__ == "__main__":
    main()
