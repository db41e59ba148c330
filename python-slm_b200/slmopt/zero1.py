"""ZeRO-1 data-parallel optimizer step: partition math, the per-rank handle,
and the multi-GPU benchmark driver.

The reference runs one device per process and has no collective
(src/train/cuda_backend.rs:56-73); this path is new.  Every rank holds the
master/m/v of one chunk-aligned shard of the flat PARAM-001 buffer plus the
full bf16 weights; one step exchanges gradient slices, sums them in rank order,
agrees on one norm, updates its shard and all-gathers the bf16 weights (the
collectives run inside libslmopt.so over NCCL).  The result is bit-identical to
a single replica's step on the rank-ordered f32 sum of all ranks' gradients.
"""
from __future__ import annotations

import ctypes
import os
import statistics
import time
from dataclasses import dataclass

from . import _lib
from .layout import TensorTable
from .optimizer import B200Adamw

CHUNK = 65536
# Peer-copy bandwidth per direction between two B200s over NVLink 5 /
# NVSwitch, measured with cudaMemcpyPeerAsync (bench.py --nvlink-peak).
NVLINK_PEAK_GBS = 770.0


@dataclass(frozen=True)
class Partition:
    """Chunk-aligned shards of a P-element flat buffer over `world` ranks."""

    P: int
    world: int
    chunks: int
    chunks_per_rank: int

    @property
    def stride(self) -> int:
        """Padded elements per rank (a whole number of chunks)."""
        return self.chunks_per_rank * CHUNK

    def shard(self, rank: int) -> tuple[int, int]:
        """(begin, length) of rank's elements; length may be 0 for tiny P."""
        begin = rank * self.stride
        return begin, max(0, min(self.stride, self.P - begin))

    def padded_chunks(self) -> int:
        return self.chunks_per_rank * self.world


def partition(P: int, world: int) -> Partition:
    if P <= 0 or world <= 0:
        raise ValueError("P and world must be positive")
    chunks = (P + CHUNK - 1) // CHUNK
    return Partition(P, world, chunks, (chunks + world - 1) // world)


def unique_id() -> bytes:
    """A fresh NCCL unique id for rank 0 to broadcast."""
    buf = (ctypes.c_uint8 * 128)()
    _lib.check(_lib.load().slm_zero1_unique_id(buf))
    return bytes(buf)


class Zero1Adamw(B200Adamw):
    """One rank's ZeRO-1 optimizer handle (collective calls: construction,
    step, init_master, read_state, state_sha256 -- every rank in the same order)."""

    def __init__(self, table: TensorTable, rank: int, world: int, uid: bytes, device: int = 0,
                 timeout_ms: int = 0):
        self.lib = _lib.load()
        self.table = table
        self.device = device
        self.rank = rank
        self.world = world
        specs = (_lib.TensorSpec * len(table))()
        self._names = [n.encode() for n in table.names]
        for i, (name, n, dec) in enumerate(zip(self._names, table.elements, table.decay)):
            specs[i].name = name
            specs[i].elements = n
            specs[i].weight_decay = 1 if dec else 0
        if len(uid) != 128:
            raise ValueError("the NCCL unique id is 128 bytes")
        idbuf = (ctypes.c_uint8 * 128)(*uid)
        h = ctypes.c_void_p()
        _lib.check(self.lib.slm_opt_create_zero1(specs, len(table), device, rank, world, idbuf,
                                                 timeout_ms, ctypes.byref(h)))
        self._h = h
        self.P = int(self.lib.slm_opt_parameter_count(h))

    def shard_range(self) -> tuple[int, int]:
        b, n = ctypes.c_uint64(), ctypes.c_uint64()
        self._check(self.lib.slm_opt_shard_range(self._h, ctypes.byref(b), ctypes.byref(n)))
        return int(b.value), int(n.value)

    @property
    def exchange(self) -> int:
        """_lib.ZERO1_PEER (peer-memory kernels) or _lib.ZERO1_NCCL."""
        return int(self.lib.slm_opt_zero1_exchange(self._h))

    def set_exchange(self, exchange: int) -> None:
        """Collective: every rank selects the same exchange before its next step."""
        self._check(self.lib.slm_opt_zero1_set_exchange(self._h, exchange))

    def gradient_buffer(self, dtype: str = "bf16"):
        """The registered gradient buffer as a CUDA tensor of P elements (bf16
        bits as int16, or float32); a step given it reads it in place."""
        import torch

        ptr, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
        self._check(self.lib.slm_opt_gradient_buffer(self._h, ctypes.byref(ptr),
                                                     ctypes.byref(nbytes)))
        typestr = "<i2" if dtype == "bf16" else "<f4"

        class _View:
            __cuda_array_interface__ = {"shape": (self.P,), "typestr": typestr,
                                        "data": (int(ptr.value), False), "version": 3}

        t = torch.as_tensor(_View(), device=f"cuda:{self.device}")
        return t.view(torch.bfloat16) if dtype == "bf16" else t


# ---- multi-GPU benchmark (bench.py --gpus N under torchrun) ----------------------------
class _stdout_to_stderr:
    """Points file descriptor 1 at stderr for the duration of a block."""

    def __enter__(self):
        import sys

        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)

    def __exit__(self, *exc):
        import sys

        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)



def _zero1_parity(opt, table, state, grads, dev, opts, rank, world, args) -> dict:
    """Post-run check of the ZeRO-1 step (collective: every rank runs it).

    From the seeded state, one step on every rank's seeded gradient must give
    the state hash, norm, clip and loss scale the oracle computed for a single
    replica stepping on the rank-ordered f32 sum of all ranks' gradients
    (tests/golden/step_golden.json, key zero1/<N>); then one step in which the
    last rank's gradient carries an injected +inf must be skipped by every
    rank (key skip/<N>).  The outcome is AND-ed over the ranks."""
    import json as _json
    from pathlib import Path

    import torch
    import torch.distributed as dist

    from . import synth

    golden_path = Path(__file__).resolve().parents[2] / "tests" / "golden" / "step_golden.json"
    try:
        g = _json.loads(golden_path.read_text())
    except Exception:
        g = None
    P = table.parameter_count
    if g is None or g.get("params") != P or str(world) not in g.get("zero1", {}):
        return {"checked": False, "reason": f"no golden record for {world} ranks at P={P}"}

    def compare(res, sha, want):
        import struct

        bits = struct.unpack("<I", struct.pack("<f", float(res.clip_scale)))[0]
        out = {"state_bit_exact": sha == want["sha256"],
               "sum_squares_equal": float(res.sum_squares).hex() == want["sum_squares_hex"],
               "clip_equal": bits == want["clip_scale_bits"],
               "skipped_equal": int(res.skipped) == want["skipped"],
               "next_loss_scale_equal": float(res.next_loss_scale) == want["next_loss_scale"]}
        out["ok"] = all(out.values())
        return out

    def reload():
        opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"],
                       validate=False)
        opt.set_loss_scale(65536.0)

    with _stdout_to_stderr():
        reload()
        res = opt.step(dev, opts)
        step = compare(res, opt.state_sha256(), g["zero1"][str(world)])
        bad = grads.copy()
        if rank == world - 1:
            synth.inject_nonfinite(bad, 5, table.offsets)
        reload()
        res = opt.step(bad, opts)  # host gradients, copied into the exchange buffer
        skip = compare(res, opt.state_sha256(), g["skip"][str(world)])
    ok = torch.tensor([1 if (step["ok"] and skip["ok"]) else 0], dtype=torch.int32)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    return {"checked": True, "against": "tests/golden/step_golden.json",
            "case": f"zero1/{world} and skip/{world}", "step": step, "skip": skip,
            "bit_exact": bool(ok.item()), "all_ranks": True}


def _zero1_stress(rank: int, world: int) -> dict:
    """The 100-update dynamic-loss-scale stress run (collective), checked against the
    oracle's trajectory for this rank count (tests/golden/stress_golden.json):
    per update the skip decision, the f64 norm's bits, the clip's bits and the
    next loss scale, and the final state's SHA-256.  Smoke tensor list, inputs
    from slmopt.stress; the outcome is AND-ed over the ranks."""
    import json as _json
    import struct
    from pathlib import Path

    import torch
    import torch.distributed as dist

    from . import stress
    from .layout import GqaDimensions
    from .optimizer import StepOptions

    golden_path = Path(__file__).resolve().parents[2] / "tests" / "golden" / "stress_golden.json"
    try:
        g = _json.loads(golden_path.read_text())["worlds"][str(world)]
    except Exception:
        return {"checked": False, "reason": f"no golden trajectory for {world} ranks"}
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    P = table.parameter_count
    ids = [unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    from . import synth

    with _stdout_to_stderr():
        opt = Zero1Adamw(table, rank, world, ids[0], device=torch.cuda.current_device(),
                         timeout_ms=120000)
        st = synth.optimizer_state(P, 0)
        opt.load_state(st["master"], st["moment"], st["variance"], st["bf16"], validate=False)
        opt.set_loss_scale(65536.0)
        scale, mismatches = 65536.0, []
        for t in range(1, stress.STEPS + 1):
            bits = stress.rank_gradient(P, table.offsets, rank, t, scale)
            r = opt.step(bits, StepOptions(learning_rate=stress.learning_rate(t),
                                           one_based_update=t,
                                           loss_scale_mode=_lib.SCALE_DYNAMIC))
            got = [int(r.skipped), float(r.sum_squares).hex(),
                   struct.unpack("<I", struct.pack("<f", float(r.clip_scale)))[0],
                   float(r.next_loss_scale)]
            if got != g["trace"][t - 1]:
                mismatches.append(t)
            scale = r.next_loss_scale
        sha = opt.state_sha256()
        opt.close()
    ok = not mismatches and sha == g["final_sha256"]
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return {"checked": True, "against": "tests/golden/stress_golden.json", "updates": stress.STEPS,
            "params": P, "skipped_updates": g["skipped_updates"],
            "trajectory_equal": not mismatches, "mismatched_updates": mismatches[:10],
            "final_state_equal": sha == g["final_sha256"], "bit_exact": bool(flag.item()),
            "all_ranks": True}


def bench_main(args, metric, unit, workload_config, clock_sampler, hbm_peak) -> None:
    """ZeRO-1 step on N GPUs: every rank holds its own seeded bf16 gradient
    (seed = rank) x 65,536; value = P / (max over ranks of the step time)."""
    import json
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from . import synth
    from .layout import GqaDimensions
    from .optimizer import StepOptions

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world < 2:
        raise SystemExit("the ZeRO-1 bench needs torchrun with WORLD_SIZE >= 2")
    torch.cuda.set_device(local)
    # Host-side plumbing only (barriers, the id broadcast, the max over ranks);
    # the step's collectives run on libslmopt's own NCCL communicator.
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    table = TensorTable.from_dimensions(GqaDimensions.canonical())
    P = table.parameter_count
    ids = [unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    # Native libraries may print banners on stdout while the communicator is
    # set up; rank 0's stdout must carry exactly one JSON line.
    with _stdout_to_stderr():
        opt = Zero1Adamw(table, rank, world, ids[0], device=local, timeout_ms=120000)
    if getattr(args, "exchange", "peer") == "nccl":
        opt.set_exchange(_lib.ZERO1_NCCL)
    state = synth.optimizer_state(P, 0)
    opt.load_state(state["master"], state["moment"], state["variance"], state["bf16"],
                   validate=False)
    opt.validate()
    opt.set_loss_scale(65536.0)
    grads = synth.grads_bf16(P, seed=rank)
    if opt.exchange == _lib.ZERO1_PEER:
        # write this rank's gradient where the other ranks read it
        dev = opt.gradient_buffer("bf16")
        dev.view(torch.int16).copy_(torch.from_numpy(grads.view("int16")))
    else:
        dev = torch.from_numpy(grads).cuda()
    opts = StepOptions(learning_rate=3e-4, one_based_update=10,
                       loss_scale_mode=_lib.SCALE_DYNAMIC)
    stream = torch.cuda.current_stream()
    with _stdout_to_stderr():
        for _ in range(args.warmup):
            opt.step(dev, opts, stream=stream, wait=False)
        first = opt.read_result()
    if first.status != 0 or first.skipped:
        raise RuntimeError(f"warm-up step failed on rank {rank}: {first.as_dict()}")
    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        smi_id = f"GPU-{torch.cuda.get_device_properties(local).uuid}".replace("GPU-GPU-", "GPU-")
    except Exception:
        smi_id = str(local)
    clocks = clock_sampler(smi_id) if rank == 0 else None
    if clocks:
        clocks.start()
    torch.cuda.synchronize()
    dist.barrier()
    start.record(stream)
    for _ in range(K):
        opt.step(dev, opts, stream=stream, wait=False)
    end.record(stream)
    res = opt.read_result()
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop() if clocks else None
    ms_local = start.elapsed_time(end) / K
    t = torch.tensor([ms_local], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if res.status != 0 or res.skipped:
        raise RuntimeError(f"timed step failed on rank {rank}: {res.as_dict()}")

    # Phase split, outside the timed region (with timing on, each step first
    # waits for the previous one); per phase the max over ranks.
    opt.phase_timing(True)
    for _ in range(min(50, max(K, 3))):
        opt.step(dev, opts, stream=stream, wait=False)
    opt.read_result()
    times, _ = opt.phase_times()
    opt.phase_timing(False)
    tp = torch.tensor(list(times.values()), dtype=torch.float64)
    dist.all_reduce(tp, op=dist.ReduceOp.MAX)
    phases_ms = {name: float(v) for name, v in zip(times, tp.tolist())}

    # End to end: the gradient from pinned host memory each step, result read
    # back.  Each update's gradients are uploaded (the handle's copy stream)
    # before stepping on the previous ones, so the PCIe copy overlaps the
    # step; wall clock between device synchronisations, max over ranks.
    host = torch.from_numpy(grads).pin_memory()
    E = max(3, args.e2e_steps)
    opt.step_uploaded(opt.upload(host), opts, stream=stream)  # warm both slots
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    slot = opt.upload(host)
    for i in range(E):
        nxt = opt.upload(host) if i + 1 < E else None
        opt.step_uploaded(slot, opts, stream=stream)
        slot = nxt
    torch.cuda.synchronize()
    mine = (time.perf_counter() - t0) * 1e3 / E
    per_rank = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(per_rank, torch.tensor([mine], dtype=torch.float64))
    per_rank_ms = [float(x.item()) for x in per_rank]
    e2e_ms = max(per_rank_ms)
    parity = _zero1_parity(opt, table, state, grads, dev, opts, rank, world, args) \
        if not getattr(args, "no_parity", False) else {"checked": False, "reason": "--no-parity"}
    opt_exchange = opt.exchange
    opt.close()
    dist.barrier()
    stress_check = _zero1_stress(rank, world) if not getattr(args, "no_parity", False) \
        else {"checked": False, "reason": "--no-parity"}
    dist.barrier()
    if rank == 0:
        peak, peak_kind = hbm_peak()
        part = partition(P, world)
        nvlink_bytes = 2 * 2 * part.stride * (world - 1)  # grads in + weights in, per rank
        line = {
            "metric": metric, "value": P / (ms * 1e-3), "unit": unit, "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy Philox normals; rank r uses seed r)",
            "config": workload_config(args, world, P, len(table)),
            "roofline": {"bound": "nvlink", "achieved": nvlink_bytes / (ms * 1e-3) / 1e9,
                         "peak": NVLINK_PEAK_GBS, "unit": "GB/s",
                         "frac": nvlink_bytes / (ms * 1e-3) / 1e9 / NVLINK_PEAK_GBS,
                         "traffic": None,
                         "peak_source": "measured peer copy per direction "
                                        "(bench.py --nvlink-peak)",
                         "nvlink_bytes_per_rank": nvlink_bytes,
                         "hbm_peak_gbs": peak, "hbm_peak_source": peak_kind},
            "e2e": {"value": P / (e2e_ms * 1e-3), "unit": unit,
                    "h2d_bytes_per_step": int(grads.nbytes), "d2h_bytes_per_step": 80,
                    "ms_per_step": e2e_ms, "per_rank_ms": per_rank_ms,
                    "host_to_device_gbs_all_ranks": world * grads.nbytes / (e2e_ms * 1e-3) / 1e9,
                    "api": "slm_opt_upload_gradients + slm_opt_step_uploaded"},
            "gpu_launches": (2 if opt_exchange == _lib.ZERO1_PEER else 3) * K,
            "exchange": "peer-memory" if opt_exchange == _lib.ZERO1_PEER else "nccl",
            "phases_ms": phases_ms,
            "clocks": clk,
            "result": {"sum_squares": res.sum_squares, "clip_scale": res.clip_scale},
            "parity": parity,
            "stress": stress_check,
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()
    if parity.get("checked") and not parity["bit_exact"]:
        raise SystemExit(f"rank {rank}: ZeRO-1 parity check against the oracle's golden step "
                         "FAILED")
    if stress_check.get("checked") and not stress_check["bit_exact"]:
        raise SystemExit(f"rank {rank}: the 100-step stress trajectory differs from the oracle's")
