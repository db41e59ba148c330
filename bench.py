#!/usr/bin/env python
"""Benchmark of the gqa-135m-v1 optimizer step on B200.

One step = one pass of the optimizer hot path over one batch of synthetic
gradients for all 135,285,504 parameters (111 PARAM-001 tensors):

* N = 1, workload "mixed" (default): bf16 gradients x 65,536 -> unscale ->
  non-finite check -> fixed-tree f64 norm -> clip 1.0 -> AdamW over fp32
  master/m/v (lr 3e-4, betas 0.9/0.95, eps 1e-8, decay 0.1 on matrices,
  t = 10) -> bf16 weight copy, dynamic loss scale.  ``--workload fp32`` runs
  the fp32-gradient step instead.
* N > 1: the ZeRO-1 step -- fixed-order reduce-scatter of every rank's bf16
  gradient fused with the unscale and norm partials, all-gather of the
  partials, AdamW on the rank's 1/N shard, all-gather of the bf16 weights.
  The total work (one step over P) is fixed, so scaling is "strong".

``value`` is params/s of the whole job (P / step time, max over ranks); the
state and gradients are resident in HBM when timing starts and each step
touches 4.06 GB, far more than the 126 MB L2.  ``e2e`` repeats the step through
the public C ABI with the gradients in pinned host memory (H2D copy and the
D2H result read inside the timed region).  ``--impl reference`` times the CPU
oracle -- the restatement of the reference's Rust scalar step (the reference
itself cannot be built here) -- on all host cores.

After the timed region every arm re-runs one step from the seeded state and
compares the resulting state hash, norm, clip and loss scale with the values
the oracle produced for the same inputs (``tests/golden/step_golden.json``,
written by ``tests/golden/make_step_golden.py``), plus one step with an
injected +inf that must be skipped; the line carries the outcome as
``parity`` and the run exits non-zero on a mismatch.

For N > 1 the line also replays the 100-update dynamic-loss-scale stress run
against the oracle's trajectory (``stress``).  For N = 1 at full size it also
times the reference's own drop-in, ``slm_opt_apply_update`` (pageable host
f32 gradients, the reference's sequential clip re-check reproduced on the
device, AdamW), and that clip check alone in both device forms
(``apply_update``).

``--nvlink-peak`` (one process, ``--gpus N`` devices) measures the peer-copy
bandwidth the ZeRO-1 roofline is quoted against instead of benchmarking.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "python-slm_b200"))

METRIC = "AdamW step ms and params/s at 135M; achieved HBM GB/s vs peak; 1/2/4/8 GPU"
UNIT = "params/s"
FALLBACK_HBM_GBS = 6650.0
# Algorithmic HBM bytes per parameter of the update kernel (the dominant one):
# read g (2 or 4) + master/m/v (12), write master/m/v (12) + bf16 (2).
UPDATE_BYTES = {"mixed": 28, "fp32": 30}
STEP_BYTES = {"mixed": 30, "fp32": 34}  # + the norm pass's read of g
# dram__bytes_read.sum + dram__bytes_write.sum of one full-size update-kernel
# launch (135,285,504 params, one-pass ncu capture, cold cache), one capture
# per workload; the summaries of those captures are kept under profiles/.
UPDATE_TRAFFIC_BYTES = {"mixed": 3.725e9, "fp32": 3.996e9}
# ... and of the whole step (the norm pass's launch added).
STEP_TRAFFIC_BYTES = {"mixed": 3.9998e9, "fp32": 4.5408e9}
GOLDEN = ROOT / "tests" / "golden" / "step_golden.json"
INF_SEED = 5  # seed of the injected +inf in the skip check (make_step_golden.py)


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["mixed", "fp32"], default="mixed")
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="ZeRO-1 data movement: peer-memory kernels (default) or NCCL")
    ap.add_argument("--params", type=int, default=0,
                    help="profiling only: run on the first N parameters (whole 65,536-element "
                         "chunks) of the 135M layout instead of all of it")
    ap.add_argument("--no-parity", action="store_true",
                    help="profiling only: skip the post-run check against the golden step")
    ap.add_argument("--nvlink-peak", action="store_true",
                    help="measure peer-copy bandwidth over --gpus devices and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.steps < 1:
        ap.error("--steps must be at least 1")
    return args


def dist_env() -> tuple[int, int, int]:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def workload_config(args, world: int, P: int, tensors: int) -> dict:
    if world == 1:
        desc = ("gqa-135m-v1 optimizer step, " +
                ("mixed precision: bf16 grads x65536, dynamic loss scale"
                 if args.workload == "mixed" else "fp32 grads") +
                ", fp32 master/m/v, clip 1.0, AdamW t=10, bf16 weight copy")
    else:
        desc = ("gqa-135m-v1 ZeRO-1 optimizer step: per-rank bf16 grads x65536, fixed-order "
                "reduce-scatter + unscale + norm partials, AdamW on 1/N shard, bf16 all-gather")
    return {
        "workload": desc,
        "params": P,
        "tensors": tensors,
        "seed": 0,
        "parallelism": "single-gpu" if world == 1 else f"zero1-dp{world}",
        "l2": "inputs larger than L2 (4.06 GB touched per step vs 126 MB L2); no flush",
    }


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.15)

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        max_sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(max_sm) if max_sm else None,
                "reasons": reasons, "samples": len(rows)}


def prefix_table(table, n: int):
    """The first n parameters (rounded down to whole chunks) of a tensor table."""
    import numpy as np

    from slmopt import TensorTable

    n = max(65536, n // 65536 * 65536)
    names, shapes, elems, decay = [], [], [], []
    for name, shape, e, d, lo in zip(table.names, table.shapes, table.elements, table.decay,
                                     table.offsets[:-1]):
        if lo >= n:
            break
        take = int(min(e, n - lo))
        names.append(name)
        shapes.append(shape if take == e else (take,))
        elems.append(take)
        decay.append(d)
    return TensorTable(tuple(names), tuple(shapes), tuple(elems), tuple(decay))


def gpu_smi_id(device: int) -> str:
    """nvidia-smi --id for a torch device (its UUID, independent of masking)."""
    import torch

    try:
        u = str(torch.cuda.get_device_properties(device).uuid)
        return u if u.startswith("GPU-") else f"GPU-{u}"
    except Exception:
        return str(device)


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for every CPU number."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def load_golden() -> dict | None:
    try:
        return json.loads(GOLDEN.read_text())
    except Exception:
        return None


def f32_bits(x: float) -> int:
    import struct

    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def compare_step(res, sha: str, want: dict) -> dict:
    """One step's outcome against a golden record (bit-level comparisons)."""
    out = {"state_bit_exact": sha == want["sha256"],
           "sum_squares_equal": float(res.sum_squares).hex() == want["sum_squares_hex"],
           "clip_equal": f32_bits(res.clip_scale) == want["clip_scale_bits"],
           "skipped_equal": int(res.skipped) == want["skipped"],
           "next_loss_scale_equal": float(res.next_loss_scale) == want["next_loss_scale"]}
    out["ok"] = all(out.values())
    return out


def single_parity(opt, table, state, host_grads, dev_grads, opts, workload: str) -> dict:
    """Post-run check of the single-GPU step: from the seeded state, one step
    on the benchmark's gradients and one on a copy carrying an injected +inf,
    each compared with the oracle's outcome in tests/golden/step_golden.json."""
    import torch

    from slmopt import synth

    g = load_golden()
    P = table.parameter_count
    if g is None or g.get("params") != P:
        return {"checked": False, "reason": "no golden record for this parameter count"}
    opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"],
                   validate=False)
    opt.set_loss_scale(65536.0)
    res = opt.step(dev_grads, opts)
    out = {"checked": True, "case": workload, "against": "tests/golden/step_golden.json"}
    out["step"] = compare_step(res, opt.state_sha256(), g[workload])
    ok = out["step"]["ok"]
    if workload == "mixed":
        bad = host_grads.copy()
        synth.inject_nonfinite(bad, INF_SEED, table.offsets)
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"],
                       validate=False)
        opt.set_loss_scale(65536.0)
        res = opt.step(torch.from_numpy(bad).cuda(), opts)
        out["skip"] = compare_step(res, opt.state_sha256(), g["skip"]["1"])
        ok = ok and out["skip"]["ok"]
    out["bit_exact"] = ok
    return out


def time_apply_update(table, state, calls: int = 2) -> dict:
    """The strict drop-in (slm_opt_apply_update, the reference's apply_update
    contract) at full size: host f32 gradients already clipped (norm 0.9),
    the reference's sequential clip re-check on the device, AdamW, no hash.
    Wall clock per call (the call is synchronous) and the device time of its
    three phases (upload, sequential clip check, update) from the handle's
    phase timer."""
    import numpy as np
    import torch

    from slmopt import B200Adamw, _lib, synth

    P = table.parameter_count
    g = synth.grads_f32(P, 0)
    g *= np.float32(0.9 / float(np.sqrt(np.sum(g.astype(np.float64) ** 2))))
    lib = _lib.load()
    times = []
    with B200Adamw(table, device=0) as opt:
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"],
                       validate=False)
        for t in range(1, calls + 2):
            if t == 2:
                opt.phase_timing(True)  # after the first call, which allocates staging
            lr = ctypes_lr(lib, t)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            opt.apply_normalized_clipped_gradients(g, lr, t, 0, with_sha=False)
            times.append((time.perf_counter() - t0) * 1e3)
        phases, n = opt.phase_times()
        opt.phase_timing(False)
    times = times[1:]
    # The sequential clip check alone on a device-resident gradient, in both
    # forms: one CTA streaming the terms (slm_gradient_clip_scale) and the
    # window summaries on every SM chained by one CTA (slm_gradient_clip_scale_ws).
    # CUDA events on the launching stream.
    import ctypes

    dev = torch.from_numpy(g).cuda()
    out = torch.zeros(ctypes.sizeof(_lib.ClipResult), dtype=torch.uint8, device="cuda")
    ws_bytes = int(lib.slm_gradient_clip_workspace_bytes(P))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def one_cta():
        _lib.check(lib.slm_gradient_clip_scale(dev.data_ptr(), P, out.data_ptr(),
                                               stream.cuda_stream))

    def all_sms():
        _lib.check(lib.slm_gradient_clip_scale_ws(dev.data_ptr(), P, ws.data_ptr(), ws_bytes,
                                                  out.data_ptr(), stream.cuda_stream))

    clip_ms = {}
    results = {}
    for name, fn, reps in (("one_cta", one_cta, 3), ("all_sms", all_sms, 10)):
        fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        clip_ms[name] = e0.elapsed_time(e1) / reps
        results[name] = bytes(out.cpu().numpy().tobytes())
    clip_ms["same_bits"] = results["one_cta"] == results["all_sms"]
    return {"api": "slm_opt_apply_update", "params": P, "calls": len(times),
            "ms_per_call": statistics.median(times),
            "phases_ms": phases, "phase_calls": n,
            "clip_scale_alone_ms": clip_ms,
            "note": "synchronous wall clock; host f32 gradients (pageable), the reference's "
                    "sequential f32 clip re-verification on the device, AdamW; state hash off"}


def ctypes_lr(lib, t: int) -> float:
    import ctypes

    out = ctypes.c_float()
    lib.slm_canonical_learning_rate(ctypes.c_uint64(t), ctypes.byref(out))
    return out.value


def run_nvlink_peak(args) -> None:
    """Peer-copy bandwidth between this machine's GPUs: cudaMemcpyPeerAsync on
    copy engines, one non-blocking stream per (source, destination) pair
    created on the destination device, peer access enabled both ways.

    * one direction: 1 GiB from GPU 0 to GPU 1, 10 copies back to back;
    * both directions at once: the same between GPU 0 and GPU 1 in both
      directions concurrently (GB/s per direction);
    * all-to-all over N GPUs: every GPU receives a 256 MiB slice from each of
      the other N-1 concurrently, 5 rounds (the ZeRO-1 gradient exchange's
      pattern; GB/s inbound per GPU).
    Wall clock between full synchronisations over many back-to-back copies;
    GB/s = 1e9 bytes/s."""
    from cuda.bindings import runtime as rt

    def ok(ret):
        err = ret[0] if isinstance(ret, tuple) else ret
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"CUDA error {err}")
        return ret[1] if isinstance(ret, tuple) and len(ret) > 1 else None

    n = min(args.gpus, ok(rt.cudaGetDeviceCount()))
    if n < 2:
        raise SystemExit("--nvlink-peak needs --gpus >= 2 and as many visible GPUs")
    for a in range(n):
        ok(rt.cudaSetDevice(a))
        for b in range(n):
            if a != b:
                if not ok(rt.cudaDeviceCanAccessPeer(a, b)):
                    raise SystemExit(f"GPU {a} cannot access GPU {b}")
                err = rt.cudaDeviceEnablePeerAccess(b, 0)[0]
                if err not in (rt.cudaError_t.cudaSuccess,
                               rt.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
                    raise RuntimeError(f"enable peer access {a}->{b}: {err}")

    def run(pairs, nbytes, reps):
        bufs = []
        for src, dst in pairs:
            ok(rt.cudaSetDevice(src))
            a = ok(rt.cudaMalloc(nbytes))
            ok(rt.cudaSetDevice(dst))
            b = ok(rt.cudaMalloc(nbytes))
            st = ok(rt.cudaStreamCreateWithFlags(rt.cudaStreamNonBlocking))
            bufs.append((src, dst, a, b, st))

        def go(r):
            for src, dst, a, b, st in bufs:
                for _ in range(r):
                    ok(rt.cudaMemcpyPeerAsync(b, dst, a, src, nbytes, st))
            for src, dst, a, b, st in bufs:
                ok(rt.cudaStreamSynchronize(st))

        go(1)  # warm up
        t0 = time.perf_counter()
        go(reps)
        dt = time.perf_counter() - t0
        for src, dst, a, b, st in bufs:
            ok(rt.cudaStreamDestroy(st))
            ok(rt.cudaSetDevice(src))
            ok(rt.cudaFree(a))
            ok(rt.cudaSetDevice(dst))
            ok(rt.cudaFree(b))
        return dt

    gib = 1 << 30
    one = run([(0, 1)], gib, 10)
    both = run([(0, 1), (1, 0)], gib, 10)
    out = {"what": "peer copy bandwidth (cudaMemcpyPeerAsync, copy engines, wall clock over "
                   "back-to-back copies)", "gpus": n,
           "one_direction_gbs": 10 * gib / one / 1e9,
           "both_directions_gbs_per_direction": 10 * gib / both / 1e9}
    if n > 2:
        sl = 256 << 20
        pairs = [(q, d) for d in range(n) for q in range(n) if q != d]
        dt = run(pairs, sl, 5)
        out["all_to_all_inbound_gbs_per_gpu"] = 5 * (n - 1) * sl / dt / 1e9
        out["all_to_all_slice_bytes"] = sl
    print(json.dumps(out), flush=True)


def cpu_baseline_sample(table, state, grads, workload: str, seconds: float = 12.0) -> dict:
    """The oracle (CPU port of the reference's step) on the host cores."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import slm_oracle as oracle

    cores = os.cpu_count() or 1
    P = table.parameter_count
    cfg = oracle.make_config(lr=3e-4, t=10, static_scale=65536.0 if workload == "mixed" else 1.0)
    st = {k: v.copy() for k, v in state.items()}
    oracle.step(cfg, grads, table.offsets, table.decay, st, threads=cores)  # warm
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        oracle.step(cfg, grads, table.offsets, table.decay, st, threads=cores)
        times.append(time.perf_counter() - t0)
    t0 = time.perf_counter()
    oracle.step(cfg, grads, table.offsets, table.decay, st, threads=1)
    single = time.perf_counter() - t0
    med = statistics.median(times)
    return {"value": P / med, "unit": UNIT, "cores": cores, "cpu_model": cpu_model(),
            "kind": "port",
            "sample": f"{len(times)} full {P:,}-param steps ({workload}) with {cores} threads, "
                      f"median {med * 1e3:.1f} ms",
            "ms_per_step": med * 1e3,
            "single_thread_value": P / single, "single_thread_ms_per_step": single * 1e3,
            "smoke_step": smoke_cpu_step(oracle, cores)}


def smoke_cpu_step(oracle, cores: int) -> dict:
    """The CPU oracle step over the smoke tensor list (4,489,856 params, fp32
    gradients, clip 1.0, t = 10): single-threaded like the reference's loop,
    and on every host core; median of 10 each."""
    from slmopt import GqaDimensions, TensorTable, synth

    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    P = table.parameter_count
    state = synth.optimizer_state(P, 0)
    grads = synth.grads_f32(P, 0)
    cfg = oracle.make_config(lr=3e-4, t=10)
    out = {"params": P, "tensors": len(table)}
    for key, threads in (("single_thread_ms", 1), ("all_cores_ms", cores)):
        st = {k: v.copy() for k, v in state.items()}
        times = []
        for _ in range(11):
            t0 = time.perf_counter()
            oracle.step(cfg, grads, table.offsets, table.decay, st, threads=threads)
            times.append((time.perf_counter() - t0) * 1e3)
        out[key] = statistics.median(times[1:])
    return out


def run_reference(args) -> None:
    """CPU reference arm: the oracle port on every host core, rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import slm_oracle as oracle
    from slmopt import GqaDimensions, TensorTable, synth

    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    P = table.parameter_count
    cores = os.cpu_count() or 1
    # Bounded sample: a chunk-aligned prefix of the flat PARAM-001 buffer sized
    # so the whole --warmup + --steps run takes about 90 s of CPU time.
    probe = 64 * 65536
    st = synth.optimizer_state(probe, 0)
    g = synth.grads_bf16(probe, 0) if args.workload == "mixed" else synth.grads_f32(probe, 0)
    scale = 65536.0 if args.workload == "mixed" else 1.0
    cfg = oracle.make_config(lr=3e-4, t=10, static_scale=scale)
    off = np.array([0, probe], np.uint64)
    oracle.step(cfg, g, off, [1], st, threads=cores)
    t0 = time.perf_counter()
    oracle.step(cfg, g, off, [1], st, threads=cores)
    rate = probe / (time.perf_counter() - t0)
    per_step = 90.0 / (args.steps + args.warmup)
    if rate * per_step >= P:  # the whole step fits the time budget
        n = P
        off = np.asarray(table.offsets, dtype=np.uint64)
        decay = list(table.decay)
    else:
        n = int(max(16 * 65536, rate * per_step) // 65536 * 65536)
        offsets = table.offsets
        k_end = int(np.searchsorted(offsets, n, side="right"))
        off = np.unique(np.concatenate([offsets[:k_end], [n]]).astype(np.uint64))
        decay = list(table.decay[: len(off) - 1])
    st = synth.optimizer_state(n, 0)
    g = synth.grads_bf16(n, 0) if args.workload == "mixed" else synth.grads_f32(n, 0)
    for _ in range(args.warmup):
        oracle.step(cfg, g, off, decay, st, threads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.step(cfg, g, off, decay, st, threads=cores)
    dt = time.perf_counter() - t0
    value = n * args.steps / dt
    sample = (f"all {P:,} params per step, {cores} threads" if n == P else
              f"first {n:,} of {P:,} params (whole 65,536-element chunks of the PARAM-001 "
              f"flat buffer) per step, {cores} threads")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": P / value * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy Philox normals)",
        "config": workload_config(args, world, P, len(table)),
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "cpu_model": cpu_model(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_single(args) -> None:
    import numpy as np
    import torch

    from slmopt import B200Adamw, GqaDimensions, StepOptions, TensorTable, _lib, synth

    torch.cuda.set_device(0)
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    if args.params:
        table = prefix_table(table, args.params)
    P = table.parameter_count
    state = synth.optimizer_state(P, 0)
    mixed = args.workload == "mixed"
    grads = synth.grads_bf16(P, 0) if mixed else synth.grads_f32(P, 0)
    opts = StepOptions(learning_rate=3e-4, one_based_update=10,
                       loss_scale_mode=_lib.SCALE_DYNAMIC if mixed else _lib.SCALE_STATIC,
                       static_loss_scale=1.0)
    opt = B200Adamw(table, device=0)
    opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"])
    opt.set_loss_scale(65536.0)
    dev_grads = torch.from_numpy(grads).cuda()
    stream = torch.cuda.current_stream()

    def one_step():
        opt.step(dev_grads, opts, stream=stream, wait=False)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    first = opt.read_result()
    if first.status != 0 or first.skipped:
        raise RuntimeError(f"warm-up step failed: {first.as_dict()}")

    # Timed region: K whole steps back to back (slm_opt_step, enqueue only),
    # CUDA events on the launching stream at its two ends.  Inside a step the
    # update is launched programmatically dependent on the norm pass, so the
    # two kernels overlap; nothing is recorded between them here.
    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(gpu_smi_id(0))
    clocks.start()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(K):
        one_step()
    end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = start.elapsed_time(end) / K
    res = opt.read_result()
    if res.status != 0 or res.skipped:
        raise RuntimeError(f"timed step failed: {res.as_dict()}")

    # Per-kernel split, outside the timed region: events between the two
    # passes (which may serialise them).
    S = min(K, 200)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(S)]
    for i in range(S):
        ev[i][0].record(stream)
        opt.norm_pass(dev_grads, opts, stream)
        ev[i][1].record(stream)
        opt.update_pass(opts, stream)
        ev[i][2].record(stream)
    torch.cuda.synchronize()
    norm_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    upd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)

    peak, peak_kind = hbm_peak()
    step_bytes = STEP_BYTES[args.workload] * P
    achieved = step_bytes / (ms * 1e-3) / 1e9
    upd_gbs = UPDATE_BYTES[args.workload] * P / (upd_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": STEP_TRAFFIC_BYTES[args.workload],
                "kernel": "one step = norm_bulk_kernel + adamw_update_bulk_kernel (the update "
                          "launched programmatically dependent on the norm pass)",
                "peak_source": peak_kind, "algorithmic_bytes_per_launch": step_bytes,
                "step_ms": ms,
                "kernels": {"norm_pass_ms": norm_ms, "update_ms": upd_ms,
                            "update_algorithmic_bytes": UPDATE_BYTES[args.workload] * P,
                            "update_gbs": upd_gbs, "update_frac": upd_gbs / peak,
                            "update_traffic": UPDATE_TRAFFIC_BYTES[args.workload],
                            "split": "separate loop with events between the passes"}}

    # End to end through the public API: pinned host gradients in, result out.
    host = torch.from_numpy(grads).pin_memory()
    E = max(3, args.e2e_steps)
    # (a) serial: slm_opt_step on host memory (H2D copy, both passes, D2H
    # result, one after the other on one stream).
    opt.step(host, opts)  # warm the staging buffer
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(E):
        r = opt.step(host, opts, stream=stream)
        if r.status != 0:
            raise RuntimeError(f"e2e step failed: {r.as_dict()}")
    e1.record(stream)
    torch.cuda.synchronize()
    serial_ms = e0.elapsed_time(e1) / E
    # (b) pipelined: each update's gradients are uploaded (handle's copy
    # stream) before stepping on the previous ones, so the PCIe copy overlaps
    # the step; every step still copies its P gradients in and reads its
    # result back.  Wall clock between device synchronisations.
    slot = opt.upload(host)
    opt.step_uploaded(slot, opts, stream=stream)  # warm both slots
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    slot = opt.upload(host)
    for i in range(E):
        nxt = opt.upload(host) if i + 1 < E else None
        r = opt.step_uploaded(slot, opts, stream=stream)
        if r.status != 0:
            raise RuntimeError(f"e2e step failed: {r.as_dict()}")
        slot = nxt
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / E
    # Both are the public API with every step's gradients copied in and its
    # result read back; the line reports the faster (which one wins depends on
    # the machine's PCIe and host-memory behaviour) and keeps both.
    pipelined = e2e_ms <= serial_ms
    best_ms = e2e_ms if pipelined else serial_ms
    e2e = {"value": P / (best_ms * 1e-3), "unit": UNIT,
           "h2d_bytes_per_step": int(grads.nbytes), "d2h_bytes_per_step": 80,
           "ms_per_step": best_ms,
           "api": ("slm_opt_upload_gradients + slm_opt_step_uploaded" if pipelined else
                   "slm_opt_step on pinned host gradients"),
           "pipelined_ms_per_step": e2e_ms, "serial_ms_per_step": serial_ms,
           "h2d_gbs": grads.nbytes / (best_ms * 1e-3) / 1e9}

    line = {
        "metric": METRIC, "value": P / (ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy Philox normals)",
        "config": workload_config(args, 1, P, len(table)),
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": 2 * K,
        "clocks": clk,
        "result": {"sum_squares": res.sum_squares, "clip_scale": res.clip_scale,
                   "loss_scale": res.loss_scale_used},
    }
    full = P == TensorTable.from_dimensions(GqaDimensions.canonical()).parameter_count
    if not args.no_parity:
        line["parity"] = single_parity(opt, table, state, grads, dev_grads, opts, args.workload)
    opt.close()
    if full and not args.no_parity:
        line["apply_update"] = time_apply_update(table, state)
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(table, state, grads, args.workload)
    print(json.dumps(line), flush=True)
    if "parity" in line and line["parity"].get("checked") and not line["parity"]["bit_exact"]:
        raise SystemExit("parity check against the oracle's golden step FAILED")


def main():
    args = parse_args()
    rank, world, _ = dist_env()
    if args.nvlink_peak:
        run_nvlink_peak(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    if world > 1 or args.gpus > 1:
        from slmopt import zero1

        zero1.bench_main(args, METRIC, UNIT, workload_config, ClockSampler, hbm_peak)
        return
    run_single(args)


if __name__ == "__main__":
    main()
