"""ZeRO-1 host logic on CPU: gloo ranks emulate the device exchange with the
oracle and must reproduce a single replica's step bit for bit.

Each rank takes its chunk-aligned shard from slmopt.zero1.partition, exchanges
gradient slices with all_to_all (the product's grouped ncclSend/ncclRecv),
sums them in rank order, forms its chunk partials, all-gathers partials and
flags, reduces them in global chunk order, updates its shard and all-gathers
the bf16 weights -- the same sequence libslmopt.so runs over NCCL.
A rank that never joins the exchange must surface as a timeout, not a hang.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time
import traceback
from pathlib import Path

import numpy as np
import pytest

import slm_oracle as oracle
from slmopt import TensorTable, synth, zero1

ROOT = Path(__file__).resolve().parents[1]


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))
    return dist


def _rank_step(rank, world, port, sizes, decay, inject, out_q):
    try:
        import torch

        dist = _init(rank, world, port, 60)
        table = TensorTable.from_sizes(sizes, decay)
        P = table.parameter_count
        part = zero1.partition(P, world)
        S, Cr = part.stride, part.chunks_per_rank
        b, L = part.shard(rank)
        scale = 65536.0
        G = synth.grads_bf16(P, seed=rank)
        if inject and rank == world - 1:
            synth.inject_nonfinite(G, 3, table.offsets)
        state = synth.optimizer_state(P, 0)
        shard = {k: v[b:b + L].copy() for k, v in state.items()}
        # 1. all-to-all of gradient slices
        lens = [part.shard(q)[1] for q in range(world)]
        send = np.concatenate([G[q * S:q * S + lens[q]] for q in range(world)])
        # gloo has no 16-bit all-to-all: carry the bf16 bits in int32 lanes
        out = torch.empty(L * world, dtype=torch.int32)
        dist.all_to_all_single(out, torch.from_numpy(send.astype(np.int32)), [L] * world, lens)
        recv = out.numpy().astype(np.uint16).reshape(world, L)
        # 2. rank-ordered f32 sum, unscale, chunk partials of the shard
        gsum = oracle.rank_sum_bf16([recv[q] for q in range(world)]) if L else \
            np.zeros(0, np.float32)
        send_p = np.zeros(Cr + 1, np.float64)
        if L:
            p, flags = oracle.chunk_partials(oracle.unscale(gsum, scale))
            send_p[:p.size] = p
            send_p[Cr] = 1.0 if flags.any() else 0.0
        # 3. all-gather partials + flag, 4. identical finalize on every rank
        gathered = [torch.zeros(Cr + 1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(send_p))
        allp = np.concatenate([x.numpy()[:Cr] for x in gathered])
        nonfinite = any(x.numpy()[Cr] != 0 for x in gathered)
        total = oracle.tree_sum(allp)
        clip, norm_bad = oracle.clip_from_sum(total)
        skipped = nonfinite or norm_bad
        # 5. AdamW on the shard with the group's clip
        cfg = oracle.make_config(lr=3e-4, t=10, static_scale=scale)
        if not skipped and L:
            oracle.adamw_apply_range(cfg, gsum, b, table.offsets, table.decay, scale, clip, shard)
        # 6. all-gather the bf16 weights
        w = np.zeros(S, np.int32)
        w[:L] = shard["bf16"]
        wg = [torch.zeros(S, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(wg, torch.from_numpy(w))
        full_bf16 = np.concatenate([x.numpy().astype(np.uint16) for x in wg])[:P]
        out_q.put((rank, {"total": total, "clip": clip, "skipped": skipped,
                          "master": shard["master"], "moment": shard["moment"],
                          "variance": shard["variance"], "bf16": full_bf16, "range": (b, L)}))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, {"error": traceback.format_exc()}))


def run_ranks(world, target, args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + timeout
    while len(results) < world and time.time() < deadline:
        try:
            r, payload = q.get(timeout=1.0)
            results[r] = payload
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return results


def test_partition_is_chunk_aligned_and_covers_everything():
    for P in (1, 65536, 65537, 4_489_856, 135_285_504):
        for world in (1, 2, 3, 4, 8):
            part = zero1.partition(P, world)
            covered = 0
            for r in range(world):
                b, n = part.shard(r)
                assert b % zero1.CHUNK == 0
                assert n >= 0 and (n == 0 or b == covered)
                covered += n
            assert covered == P
            assert part.padded_chunks() >= part.chunks
            assert part.padded_chunks() % world == 0
    part = zero1.partition(135_285_504, 8)
    assert part.chunks == 2065 and part.chunks_per_rank == 259
    assert part.stride == 259 * 65536


@pytest.mark.parametrize("world,inject", [(2, False), (3, False), (2, True)])
def test_emulated_zero1_equals_single_replica(world, inject):
    sizes = [65536 * 3 + 5, 768, 1000]
    decay = [True, False, True]
    table = TensorTable.from_sizes(sizes, decay)
    P = table.parameter_count
    res = run_ranks(world, _rank_step, (sizes, decay, inject))
    assert len(res) == world, res
    for r, payload in res.items():
        assert "error" not in payload, payload.get("error")
    # single replica: oracle step on the rank-ordered f32 sum of all gradients
    grads = [synth.grads_bf16(P, seed=r) for r in range(world)]
    if inject:
        synth.inject_nonfinite(grads[world - 1], 3, table.offsets)
    gsum = oracle.rank_sum_bf16(grads)
    state = synth.optimizer_state(P, 0)
    ref = oracle.step(oracle.make_config(lr=3e-4, t=10, static_scale=65536.0), gsum,
                      table.offsets, table.decay, state)
    assert bool(ref.skipped) == inject
    for r, payload in res.items():
        assert payload["skipped"] == bool(ref.skipped)
        if not ref.skipped:
            assert payload["total"] == ref.sum_squares
            assert np.float32(payload["clip"]) == np.float32(ref.clip_scale)
        b, L = payload["range"]
        for key in ("master", "moment", "variance"):
            assert np.array_equal(payload[key].view(np.uint32), state[key][b:b + L].view(np.uint32))
        assert np.array_equal(payload["bf16"], state["bf16"])


def _rank_absent(rank, world, port, out_q):
    """Rank 1 joins the group but never the exchange; rank 0 must time out."""
    try:
        import torch

        dist = _init(rank, world, port, 5)
        if rank == 1:
            out_q.put((rank, {"left": True}))
            time.sleep(20)  # alive but silent: the collective never completes
            return
        t0 = time.time()
        try:
            out = torch.empty(4, dtype=torch.int32)
            dist.all_to_all_single(out, torch.zeros(4, dtype=torch.int32), [2, 2], [2, 2])
            out_q.put((rank, {"error": "the collective completed without rank 1"}))
        except Exception as e:  # gloo raises once the group timeout expires
            out_q.put((rank, {"timeout": True, "seconds": time.time() - t0, "what": str(e)[:200]}))
    except Exception:
        out_q.put((rank, {"error": traceback.format_exc()}))


def test_absent_rank_surfaces_as_timeout():
    res = run_ranks(2, _rank_absent, (), timeout=60)
    assert res.get(1, {}).get("left")
    r0 = res.get(0, {})
    assert r0.get("timeout"), r0
    assert r0["seconds"] < 30
