"""Cross-check the C oracle against a second, independent numpy restatement.

The parts of the step the reference has no test for (bf16 gradients, loss
scaling and skip, the fixed f64 norm tree, the rank-ordered ZeRO-1 sum) are
pinned only by restating them twice, in C and here in numpy, and requiring
bit equality.  numpy float32 element-wise operations round once per operation
and never fuse, like the C oracle built with -ffp-contract=off.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest

import slm_oracle as oracle
from slmopt import synth
from slmopt.layout import GqaDimensions, TensorTable

F = np.float32


def np_powi(base: float, exponent: int) -> np.float32:
    """Square-and-multiply in float32 (the compiler-builtins __powisf2 loop)."""
    b = F(base)
    r = F(1.0)
    e = exponent
    with np.errstate(over="ignore"):  # 1.5^t overflows to inf, as in f32
        while True:
            if e & 1:
                r = F(r * b)
            e >>= 1
            if e == 0:
                break
            b = F(b * b)
    return r


def np_tree_fold(lane: np.ndarray) -> np.float64:
    warp = []
    for w in range(8):
        v = lane[32 * w:32 * w + 32].copy()
        off = 16
        while off >= 1:
            v[:off] = v[:off] + v[off:2 * off]
            off //= 2
        warp.append(v[0])
    warp = np.array(warp, np.float64)
    off = 4
    while off >= 1:
        warp[:off] = warp[:off] + warp[off:2 * off]
        off //= 2
    return warp[0]


def np_chunk_partials(g: np.ndarray) -> np.ndarray:
    n = g.size
    c = (n + 65535) // 65536
    padded = np.zeros(c * 65536, np.float32)
    padded[:n] = g
    q = (padded * padded).astype(np.float32)  # f32 squares
    out = np.empty(c, np.float64)
    for ci in range(c):
        blk = q[ci * 65536:(ci + 1) * 65536].reshape(32, 256, 8)  # [k][thread][j]
        # per-vector pairwise f32 sum ((q0+q1)+(q2+q3))+((q4+q5)+(q6+q7))
        p = ((blk[:, :, 0] + blk[:, :, 1]) + (blk[:, :, 2] + blk[:, :, 3])) + \
            ((blk[:, :, 4] + blk[:, :, 5]) + (blk[:, :, 6] + blk[:, :, 7]))
        acc = np.zeros(256, np.float64)
        for k in range(32):
            acc = acc + p[k].astype(np.float64)
        out[ci] = np_tree_fold(acc)
    return out


def np_tree_sum(p: np.ndarray) -> np.float64:
    lane = np.zeros(256, np.float64)
    for start in range(0, p.size, 256):
        seg = p[start:start + 256]
        lane[:seg.size] = lane[:seg.size] + seg
    return np_tree_fold(lane)


def np_step(grads, scale, table, state, lr, t, clip_max=1.0, apply_clip=True,
            b1=0.9, b2=0.95, eps=1e-8, wd=0.1):
    g = (synth.bf16_bits_to_f32(grads) if grads.dtype == np.uint16 else grads).astype(F)
    g = (g / F(scale)).astype(F)
    if not np.all(np.isfinite(g)):
        return {"skipped": True}
    s = np_tree_sum(np_chunk_partials(g))
    sf = F(s)
    clip = F(1.0) if sf == 0 else min(F(F(clip_max) / F(np.sqrt(sf))), F(1.0))
    gc = (g * clip).astype(F) if apply_clip else g
    b1, b2, eps = F(b1), F(b2), F(eps)
    bc1 = F(F(1.0) - np_powi(b1, t))
    bc2 = F(F(1.0) - np_powi(b2, t))
    wdv = np.repeat(np.where(np.asarray(table.decay), F(wd), F(0.0)).astype(F),
                    np.asarray(table.elements))
    th, m, v = state["master"], state["moment"], state["variance"]
    m1 = (b1 * m + F(F(1.0) - b1) * gc).astype(F)
    v1 = (b2 * v + (F(F(1.0) - b2) * gc) * gc).astype(F)
    mh = (m1 / bc1).astype(F)
    vh = (v1 / bc2).astype(F)
    t1 = (th - F(lr) * (mh / (np.sqrt(vh) + eps) + wdv * th)).astype(F)
    return {"skipped": False, "sum": s, "clip": clip, "master": t1, "moment": m1,
            "variance": v1, "bf16": synth.bf16_rne_bits(t1)}


def test_sha256_matches_hashlib():
    rng = np.random.default_rng(1)
    for n in (0, 1, 55, 56, 63, 64, 65, 119, 120, 1000, 65537):
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert oracle.sha256(data) == hashlib.sha256(data).digest(), n


def test_powi_is_square_and_multiply():
    for base in (0.9, 0.95, 0.999, 1.5):
        for t in (1, 2, 3, 7, 10, 20, 100, 1000, 30518, 2**31 - 1):
            assert np.float32(oracle.powi(base, t)) == np_powi(base, t), (base, t)


def test_schedule_matches_python_restatement():
    # config 4 schedule: warmup 20 then cosine 3e-4 -> 3e-5 over 100 updates
    for t in range(1, 101):
        st, lr = oracle.schedule_learning_rate(t, 3e-4, 3e-5, 20, 100)
        assert st == oracle.OK
        if t <= 20:
            expect = F(F(F(3e-4) * F(t)) / F(20))
        else:
            p = (t - 20) / 80
            expect = F(float(F(3e-5)) + 0.5 * float(F(F(3e-4) - F(3e-5))) *
                       (1.0 + math.cos(math.pi * p)))
        assert F(lr) == expect, t


@pytest.mark.parametrize("n", [1, 3, 7, 8, 9, 2047, 2048, 4095, 65536, 65537, 200_003])
def test_chunk_tree_matches_numpy(n):
    g = synth.normal_f32(n, 1e-3, 3, 5)
    p_c, flags = oracle.chunk_partials(g)
    p_np = np_chunk_partials(g)
    assert np.array_equal(p_c.view(np.uint64), p_np.view(np.uint64))
    assert not flags.any()
    assert oracle.tree_sum(p_c) == np_tree_sum(p_np)
    # the fixed tree agrees with the exact sum far inside 1e-6 relative
    exact = math.fsum(float(x) * float(x) for x in g.astype(np.float64))
    assert abs(oracle.tree_sum(p_c) - exact) <= 3e-7 * max(exact, 1e-300)


def test_tree_sum_is_invariant_to_zero_padding():
    # ZeRO-1 pads the chunk count to a multiple of the rank count.
    p = np.abs(synth.normal_f32(2065, 1.0, 1, 1)).astype(np.float64)
    for pad in (1, 3, 7, 100):
        assert oracle.tree_sum(np.concatenate([p, np.zeros(pad)])) == oracle.tree_sum(p)


def test_nonfinite_flags_mark_the_chunk():
    g = np.zeros(3 * 65536 + 5, np.float32)
    g[65536 + 17] = np.inf
    g[3 * 65536 + 2] = np.nan
    _, flags = oracle.chunk_partials(g)
    assert flags.tolist() == [0, 1, 0, 1]


def _table_for(n_sizes, seed=0):
    rng = np.random.default_rng(seed)
    decay = rng.integers(0, 2, len(n_sizes)).astype(bool)
    return TensorTable.from_sizes(n_sizes, decay)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("sizes", [[1], [3, 5], [7, 9, 11, 4095], [65536, 5, 70000],
                                   [768] * 7 + [131072 + 3]])
def test_fused_step_matches_numpy(dtype, sizes):
    table = _table_for(sizes)
    n = table.parameter_count
    state = synth.optimizer_state(n, seed=11)
    scale = 65536.0 if dtype == "bf16" else 1.0
    grads = synth.grads_bf16(n, 11) if dtype == "bf16" else synth.grads_f32(n, 11)
    expect = np_step(grads, scale, table, {k: v.copy() for k, v in state.items()}, 3e-4, 10)
    cfg = oracle.make_config(lr=3e-4, t=10, static_scale=scale)
    res = oracle.step(cfg, grads, table.offsets, table.decay, state)
    assert res.status == oracle.OK and not res.skipped
    assert res.sum_squares == expect["sum"]
    assert np.float32(res.clip_scale) == expect["clip"]
    for key in ("master", "moment", "variance", "bf16"):
        assert np.array_equal(state[key].view(np.uint8), expect[key].view(np.uint8)), key


def test_fused_step_clips_when_norm_exceeds_one():
    table = _table_for([300_000])
    n = table.parameter_count
    state = synth.optimizer_state(n, seed=2)
    grads = (synth.grads_f32(n, 2) * np.float32(10.0)).astype(np.float32)  # norm ~ 5.5
    expect = np_step(grads, 1.0, table, {k: v.copy() for k, v in state.items()}, 3e-4, 10)
    res = oracle.step(oracle.make_config(lr=3e-4, t=10), grads, table.offsets, table.decay, state)
    assert res.clip_scale < 1.0 and np.float32(res.clip_scale) == expect["clip"]
    assert np.array_equal(state["master"].view(np.uint32), expect["master"].view(np.uint32))


def test_skip_and_dynamic_scaler():
    table = _table_for([1000, 24])
    n = table.parameter_count
    state = synth.optimizer_state(n, seed=3)
    before = {k: v.copy() for k, v in state.items()}
    grads = synth.grads_bf16(n, 3)
    synth.inject_nonfinite(grads, 5, table.offsets)
    scaler = oracle.Scaler(65536.0, 7)
    cfg = oracle.make_config(dynamic=True, growth_interval=3)
    res = oracle.step(cfg, grads, table.offsets, table.decay, state, scaler)
    assert res.skipped == 1 and res.nonfinite == 1 and res.status == oracle.OK
    assert res.loss_scale_used == 65536.0 and res.next_loss_scale == 32768.0
    assert scaler.scale == 32768.0 and scaler.good_steps == 0
    for k in state:
        assert np.array_equal(state[k], before[k])
    # three clean steps double the scale
    clean = synth.grads_bf16(n, 4, loss_scale=32768.0)
    for i in range(3):
        res = oracle.step(cfg, clean, table.offsets, table.decay, state, scaler)
        assert not res.skipped
    assert scaler.scale == 65536.0 and scaler.good_steps == 0
    # reference policy: error, state unchanged
    st_before = {k: v.copy() for k, v in state.items()}
    res = oracle.step(oracle.make_config(nonfinite_policy=1, static_scale=65536.0), grads,
                      table.offsets, table.decay, state)
    assert res.status == oracle.MODEL_GRADIENT_NONFINITE and res.skipped
    for k in state:
        assert np.array_equal(state[k], st_before[k])


def test_rank_sum_is_left_to_right():
    n = 10_000
    gs = [synth.grads_bf16(n, r) for r in range(4)]
    out = oracle.rank_sum_bf16(gs)
    s = synth.bf16_bits_to_f32(gs[0]).copy()
    for r in range(1, 4):
        s = (s + synth.bf16_bits_to_f32(gs[r])).astype(np.float32)
    assert np.array_equal(out.view(np.uint32), s.view(np.uint32))


def test_multithreaded_step_equals_single_threaded():
    table = TensorTable.from_dimensions(GqaDimensions.smoke())
    n = table.parameter_count
    s1 = synth.optimizer_state(n, 0)
    s8 = {k: v.copy() for k, v in s1.items()}
    grads = synth.grads_bf16(n, 0)
    cfg = oracle.make_config(t=10, static_scale=65536.0)
    r1 = oracle.step(cfg, grads, table.offsets, table.decay, s1, threads=1)
    r8 = oracle.step(cfg, grads, table.offsets, table.decay, s8, threads=8)
    assert r1.sum_squares == r8.sum_squares
    for k in s1:
        assert np.array_equal(s1[k], s8[k])


@pytest.mark.parametrize("n", [1, 2, 977, 20_000])
def test_reference_sequential_clip_matches_python_restatement(n):
    # src/model/oracle.rs:486-507: `sum += g * g` in f32, one element after
    # another, then min(1 / sqrt(sum), 1) -- restated here element by element
    # with numpy float32 scalars (one rounding per operation).
    g = (((np.arange(n) % 977).astype(np.float32) - F(488.0)) * F(1e-3)).astype(np.float32)
    total = F(0.0)
    for x in g:
        total = F(total + F(x * x))
    expect = F(1.0) if total == 0 else min(F(F(1.0) / F(np.sqrt(total))), F(1.0))
    st, got = oracle.gradient_clip_scale(g)
    assert st == oracle.OK
    assert F(got).view(np.uint32) == expect.view(np.uint32)
