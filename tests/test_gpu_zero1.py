"""ZeRO-1 on real GPUs, with both exchanges (peer memory over NVLink, and NCCL):
one child process per GPU, each driving its rank through the C ABI; the
gathered state must equal the oracle's single replica step on the rank-ordered
f32 sum of all ranks' bf16 gradients, bit for bit, and an injected inf on one
rank must make every rank skip.  Needs >= 2 visible GPUs (skipped otherwise)."""
from __future__ import annotations

import hashlib
import multiprocessing as mp
import os
import socket
import time
import traceback

import numpy as np
import pytest

import slm_oracle as oracle
from slmopt import GqaDimensions, TensorTable, synth

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


def _digest(state: dict) -> dict:
    return {k: hashlib.sha256(state[k].tobytes()).hexdigest() for k in state}


def _rank_main(rank, world, port, table_name, exchange, out_q):
    try:
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from slmopt import StepOptions, _lib
        from slmopt.zero1 import Zero1Adamw, unique_id

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120))
        table = _table(table_name)
        P = table.parameter_count
        ids = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        opt = Zero1Adamw(table, rank, world, ids[0], device=rank, timeout_ms=120000)
        if exchange == "nccl":
            opt.set_exchange(_lib.ZERO1_NCCL)
        got_exchange = opt.exchange
        st = synth.optimizer_state(P, 0)
        opt.load_state(st["master"], st["moment"], st["variance"], st["bf16"])
        opt.set_loss_scale(65536.0)
        grads = synth.grads_bf16(P, seed=rank)
        opts = StepOptions(learning_rate=3e-4, one_based_update=10,
                           loss_scale_mode=_lib.SCALE_DYNAMIC)
        opt.phase_timing(True)  # events at the phase boundaries must not change a bit
        r1 = opt.step(torch.from_numpy(grads).cuda(), opts)
        state1 = opt.read_state()  # collective gather
        sha1 = opt.state_sha256()  # collective
        w32 = opt.export_weights_f32().cpu().numpy()  # this rank's full copy
        w32_ok = bool(np.array_equal(w32.view(np.uint32),
                                     synth.bf16_bits_to_f32(state1["bf16"]).view(np.uint32)))
        bad = grads.copy()
        if rank == world - 1:
            synth.inject_nonfinite(bad, 5, table.offsets)
        if got_exchange == _lib.ZERO1_PEER:
            # write straight into the registered buffer the other ranks read
            gbuf = opt.gradient_buffer("bf16")
            gbuf.view(torch.int16).copy_(torch.from_numpy(bad.view(np.int16)))
        else:
            gbuf = torch.from_numpy(bad).cuda()
        r2 = opt.step(gbuf, StepOptions(
            learning_rate=3e-4, one_based_update=11, loss_scale_mode=_lib.SCALE_DYNAMIC))
        state2 = opt.read_state()
        # the same gradients from host memory skip again (scale halves again)
        r3 = opt.step(bad, StepOptions(
            learning_rate=3e-4, one_based_update=12, loss_scale_mode=_lib.SCALE_DYNAMIC))
        state3 = opt.read_state()
        phases = opt.phase_times()
        scale = opt.loss_scale()
        opt.close()
        out_q.put((rank, {"exchange": got_exchange, "r1": r1.as_dict(), "r2": r2.as_dict(),
                          "r3": r3.as_dict(), "d3": _digest(state3), "d1": _digest(state1),
                          "d2": _digest(state2), "sha1": sha1, "scale": scale,
                          "phases": phases, "w32_ok": w32_ok,
                          "bf16": hashlib.sha256(state1["bf16"].tobytes()).hexdigest()}))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, {"error": traceback.format_exc()}))


def _table(name: str) -> TensorTable:
    if name == "smoke":
        return TensorTable.from_dimensions(GqaDimensions.smoke())
    if name == "135m":
        return TensorTable.from_dimensions(GqaDimensions.canonical())
    return TensorTable.from_sizes([65536 * 5 + 17, 768, 4096 + 3], [True, False, True])


def _run(world: int, table_name: str, exchange: str, timeout: float = 600):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, table_name, exchange, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + timeout
    while len(res) < world and time.time() < deadline:
        try:
            r, payload = q.get(timeout=2.0)
            res[r] = payload
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
@pytest.mark.parametrize("table_name", ["ragged", "smoke", "135m"])
def test_zero1_equals_single_replica(table_name, exchange):
    n = _gpus()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(n, 8) if table_name != "ragged" else 2
    res = _run(world, table_name, exchange)
    assert len(res) == world, res
    for r, p in res.items():
        assert "error" not in p, p["error"]
    table = _table(table_name)
    P = table.parameter_count
    grads = [synth.grads_bf16(P, seed=r) for r in range(world)]
    gsum = oracle.rank_sum_bf16(grads, threads=8)
    state = synth.optimizer_state(P, 0)
    scaler = oracle.Scaler(65536.0, 0)
    ref = oracle.step(oracle.make_config(lr=3e-4, t=10, dynamic=True), gsum, table.offsets,
                      table.decay, state, scaler, threads=8)
    want = _digest(state)
    want_sha = oracle.state_sha256(table.names, table.offsets, table.decay, state)[1]
    from slmopt import _lib

    for r, p in res.items():
        assert p["exchange"] == (_lib.ZERO1_PEER if exchange == "peer" else _lib.ZERO1_NCCL)
        assert p["r1"]["status"] == 0 and p["r1"]["skipped"] == 0
        assert p["r1"]["sum_squares"] == ref.sum_squares
        assert np.float32(p["r1"]["clip_scale"]) == np.float32(ref.clip_scale)
        assert p["d1"] == want, f"rank {r} state differs from the single replica"
        assert p["sha1"] == want_sha
        # the injected inf on the last rank makes every rank skip
        assert p["r2"]["skipped"] == 1 and p["r2"]["nonfinite"] == 1
        assert p["r2"]["next_loss_scale"] == 32768.0
        assert p["d2"] == p["d1"]
        assert p["r3"]["skipped"] == 1 and p["r3"]["next_loss_scale"] == 16384.0
        assert p["scale"][0] == 16384.0 and p["d3"] == p["d1"]
        assert p["w32_ok"]
        times, steps = p["phases"]
        assert steps == 3
        assert len(times) == (2 if exchange == "peer" else 6)
        assert all(ms >= 0.0 for ms in times.values()) and sum(times.values()) > 0.0


def _stress_rank(rank, world, port, out_q):
    try:
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from slmopt import StepOptions, _lib, stress
        from slmopt.zero1 import Zero1Adamw, unique_id

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120))
        table = _table("smoke")
        P = table.parameter_count
        runs = []
        for _ in range(2):  # two full runs must be bit-identical
            ids = [unique_id() if rank == 0 else None]
            dist.broadcast_object_list(ids, src=0)
            opt = Zero1Adamw(table, rank, world, ids[0], device=rank, timeout_ms=120000)
            st = synth.optimizer_state(P, 0)
            opt.load_state(st["master"], st["moment"], st["variance"], st["bf16"])
            opt.set_loss_scale(65536.0)
            scale, trace = 65536.0, []
            for t in range(1, stress.STEPS + 1):
                bits = stress.rank_gradient(P, table.offsets, rank, t, scale)
                r = opt.step(torch.from_numpy(bits).cuda(),
                             StepOptions(learning_rate=stress.learning_rate(t),
                                         one_based_update=t,
                                         loss_scale_mode=_lib.SCALE_DYNAMIC))
                trace.append([int(r.skipped), float(r.sum_squares).hex(),
                              int(np.float32(r.clip_scale).view(np.uint32)),
                              float(r.next_loss_scale)])
                scale = r.next_loss_scale
            runs.append((trace, opt.state_sha256()))
            opt.close()
        out_q.put((rank, {"runs": runs}))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, {"error": traceback.format_exc()}))


def _stress_oracle(world: int) -> dict:
    """The oracle's trajectory: the committed golden for 2/4/8 ranks, else
    computed here the way tests/golden/make_stress_golden.py does."""
    import json
    from pathlib import Path

    from slmopt import stress

    golden = Path(__file__).resolve().parent / "golden" / "stress_golden.json"
    worlds = json.loads(golden.read_text())["worlds"]
    if str(world) in worlds:
        return worlds[str(world)]
    table = _table("smoke")
    P = table.parameter_count
    state = synth.optimizer_state(P, 0)
    scaler = oracle.Scaler(65536.0, 0)
    trace = []
    for t in range(1, stress.STEPS + 1):
        lr = oracle.schedule_learning_rate(t, stress.PEAK_LR, stress.MIN_LR, stress.WARMUP,
                                           stress.STEPS)[1]
        g = oracle.rank_sum_bf16([stress.rank_gradient(P, table.offsets, r, t, scaler.scale)
                                  for r in range(world)], threads=8)
        ref = oracle.step(oracle.make_config(lr=lr, t=t, dynamic=True), g, table.offsets,
                          table.decay, state, scaler, threads=8)
        trace.append([int(ref.skipped), float(ref.sum_squares).hex(),
                      int(np.float32(ref.clip_scale).view(np.uint32)),
                      float(ref.next_loss_scale)])
    sha = oracle.state_sha256(table.names, table.offsets, table.decay, state)[1]
    return {"trace": trace, "final_sha256": sha}


def test_zero1_stress_trajectory_matches_oracle():
    # warmup 20 then cosine from 3e-4 over 100 steps, Student-t(3) * 1e-3 bf16
    # gradients per rank, dynamic loss scale, +inf injected at two seeded steps
    from slmopt import stress

    n = _gpus()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(n, 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_stress_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res, deadline = {}, time.time() + 900
    while len(res) < world and time.time() < deadline:
        try:
            r, payload = q.get(timeout=2.0)
            res[r] = payload
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert len(res) == world, res
    want = _stress_oracle(world)
    for r, p in res.items():
        assert "error" not in p, p["error"]
        assert p["runs"][0] == p["runs"][1], f"rank {r}: two runs differ"
        trace, sha = p["runs"][0]
        for t in range(1, stress.STEPS + 1):
            assert trace[t - 1] == want["trace"][t - 1], (r, t)
        assert sum(x[0] for x in trace) == len(stress.INJECT)
        assert sha == want["final_sha256"], f"rank {r} final state differs from the oracle"


def _absent_peer_rank(rank, world, port, out_q):
    # Failure detection on the device, without faulting anything: after one
    # good step rank 1 stops stepping (it stays alive, its memory mapped, none
    # of its kernels in flight).  Rank 0's next step waits at the gradient
    # barrier for a flag nothing sets; the bounded wait gives up after the
    # handle's timeout and the step reports SLM_ERR_TIMEOUT.  Later, rank 1
    # steps alone: it passes the barrier (rank 0 announced itself) and its
    # finalize waits for partials rank 0 never sends, with the same outcome.
    try:
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from slmopt import SlmError, StepOptions, _lib
        from slmopt.zero1 import Zero1Adamw, unique_id

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120))
        table = _table("ragged")
        P = table.parameter_count
        ids = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        opt = Zero1Adamw(table, rank, world, ids[0], device=rank, timeout_ms=2000)
        out = {"exchange": opt.exchange}
        st = synth.optimizer_state(P, 0)
        opt.load_state(st["master"], st["moment"], st["variance"], st["bf16"])
        grads = torch.from_numpy(synth.grads_bf16(P, seed=rank)).cuda()
        opts = StepOptions(learning_rate=3e-4, one_based_update=1, static_loss_scale=65536.0)
        out["r1"] = opt.step(grads, opts).status

        def failing_step(t):
            t0 = time.time()
            try:
                opt.step(grads, StepOptions(learning_rate=3e-4, one_based_update=t,
                                            static_loss_scale=65536.0))
                return ("ok", time.time() - t0)
            except SlmError as e:
                return (e.status, time.time() - t0)

        dist.barrier()
        if rank == 0:
            out["alone"] = failing_step(2)
            out["after"] = failing_step(3)  # the handle is broken: fails at once
            torch.cuda.synchronize()
        dist.barrier()
        if rank == 1:
            out["alone"] = failing_step(2)
            torch.cuda.synchronize()
        dist.barrier()  # nobody's kernels in flight before any memory is released
        opt.close()
        out_q.put((rank, out))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, {"error": traceback.format_exc()}))


def test_absent_peer_times_out_on_device():
    n = _gpus()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    from slmopt import _lib

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_absent_peer_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res, deadline = {}, time.time() + 300
    while len(res) < world and time.time() < deadline:
        try:
            r, payload = q.get(timeout=2.0)
            res[r] = payload
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert len(res) == world, res
    for r, p in res.items():
        assert "error" not in p, p["error"]
        assert p["exchange"] == _lib.ZERO1_PEER
        assert p["r1"] == 0
        status, seconds = p["alone"]
        assert status == _lib.SLM_ERR_TIMEOUT, p
        assert 1.5 < seconds < 10.0, p  # the 2 s device bound, not the host's
    status, seconds = res[0]["after"]
    assert status == _lib.SLM_ERR_TIMEOUT and seconds < 1.0, res[0]
