"""The exact parallel method behind the device's sequential clip sum, restated
in numpy and checked against the oracle's one-term-at-a-time f32 loop.

The reference's gradient_clip_scale (src/model/oracle.rs:486-507) adds
fl(g*g) to an f32 sum in order.  The device reproduces that sum with every SM
(seqclip_*_kernel in python-slm_b200/csrc/kernels.cu); this file restates
the same steps on the CPU, term layout and rounding included, so that the
method itself -- not only its CUDA form, which the GPU tests check -- is
pinned without a GPU:

* while the sum s = m * 2^E stays in one binade, fl(s + q) = (m + r) * 2^E
  with r = q / 2^E rounded to the nearest integer, unless q / 2^E is exactly
  halfway (a tie) or m + r reaches 2^24 (the binade changes);
* per 8,192-term window, for the 3 binades around the binade of the exact
  f64 prefix sum, the window's total of r in f32 (per thread of 256, then
  clamped integers) and its tie flags;
* a walk over groups of 32 windows, then windows, accepting totals while
  they fit, and the exact procedure for a window that does not fit.

Which binades are candidates changes only how many windows take the exact
path, never the result: a test moves every base and expects the same bits.
"""
from __future__ import annotations

import numpy as np
import pytest

import slm_oracle as oracle

F = np.float32
W = 8192            # terms per window
THREADS = 256       # threads of the candidate pass
NC = 3              # candidate binades per window
BELOW = 1           # the first candidate's distance below the prefix's binade
BATCH = 1024        # window summaries per chain batch
TWO24 = 1 << 24


def decompose(s: np.float32) -> tuple[int, int]:
    b = int(F(s).view(np.uint32))
    exp, man = (b >> 23) & 0xFF, b & 0x7FFFFF
    return (-149, man) if exp == 0 else (exp - 150, man | 0x800000)


def compose(E: int, m: int) -> np.float32:
    return F(np.ldexp(np.float64(m), E))  # m < 2^24: exact


def increments(q: np.ndarray, E: int) -> tuple[np.ndarray, np.ndarray]:
    """r = round(q / 2^E) with ties flagged (integer form, int64)."""
    b = q.view(np.uint32).astype(np.int64)
    exp, man = (b >> 23) & 0xFF, b & 0x7FFFFF
    Q = np.where(exp == 0, man, man | 0x800000)
    Fx = np.where(exp == 0, -149, exp - 150)
    d = E - Fx
    dc = np.clip(d, 1, 31)
    half = np.left_shift(np.int64(1), dc - 1)
    rem = Q & ((half << 1) - 1)
    r = (Q >> dc) + (rem > half)
    r = np.where(d < 0, np.int64(1) << 25, np.where(d == 0, Q, r))
    tie = (d > 0) & (rem == half)
    return r, tie


def exact_window(state: dict, q: np.ndarray) -> None:
    """Adds the window's squares exactly: the first tie or binade change is
    a real f32 add, the increments before it one integer sum."""
    start = 0
    while not state["bad"] and start < q.size:
        E, m = state["E"], state["m"]
        r, tie = increments(q[start:], E)
        cum = np.cumsum(r)
        stops = np.flatnonzero(tie | (m + cum >= TWO24))
        if stops.size == 0:
            state["m"] = m + int(cum[-1])
            return
        j = int(stops[0])
        before = int(cum[j - 1]) if j else 0
        with np.errstate(over="ignore"):  # an overflow to inf is the reference's too
            s = F(compose(E, m + before) + q[start + j])
        if not np.isfinite(s):
            state["bad"], state["bits"] = True, s
        else:
            state["E"], state["m"] = decompose(s)
        start += j + 1


def seq_binade(s: np.float32) -> int:
    exp = (int(F(s).view(np.uint32)) >> 23) & 0xFF
    return -149 if exp == 0 else exp - 150


def candidate_pass(q: np.ndarray, base: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per window: NC clamped totals and tie bits, the way the candidate
    kernel forms them (thread t holds float4s t + 256k, k = 0..7; its terms
    are added in f32 in that order)."""
    nw = base.size
    x = q.reshape(nw, 8, THREADS, 4).transpose(0, 2, 1, 3).reshape(nw, THREADS, 32)
    k = -base.astype(np.int64)
    split = k > 127
    s0 = np.ldexp(F(1), np.where(split, k - 64, k)).astype(F)
    s1 = np.where(split, F(2.0 ** 64), F(1)).astype(F)
    with np.errstate(over="ignore", invalid="ignore"):
        y = (x * s0[:, None, None]).astype(F) * s1[:, None, None]
        y = y.astype(F)
        totals = np.zeros((nw, NC), np.int64)
        ties = np.zeros((nw, NC), bool)
        for c in range(NC):
            r = np.rint(y).astype(F)  # nearest, ties to even, like rintf
            tot = np.zeros((nw, THREADS), F)
            for j in range(32):
                tot = (tot + r[:, :, j]).astype(F)
            dev = np.abs((y - r).astype(F))
            ties[:, c] = (dev == F(0.5)).any(axis=(1, 2))
            v = np.where(tot < F(TWO24), tot, F(TWO24))
            v = np.where(np.isnan(tot), F(TWO24), v).astype(np.int64)
            warp = np.minimum(v.reshape(nw, 8, 32).sum(axis=2), TWO24)
            totals[:, c] = np.minimum(warp.sum(axis=1), TWO24)
            y = (y * F(0.5)).astype(F)
    return totals, ties


def chain_sum(g: np.ndarray, base_shift: np.ndarray | None = None) -> tuple[bool, np.float32, int]:
    """(non-finite gradient seen, the in-order f32 sum, exact windows)."""
    g = np.ascontiguousarray(g, dtype=F)
    n = g.size
    nw = (n + W - 1) // W
    state = {"E": -149, "m": 0, "bad": False, "bits": F(0)}
    if nw == 0:
        return False, F(0), 0
    x = np.zeros(nw * W, F)
    x[:n] = g
    with np.errstate(over="ignore", invalid="ignore"):
        q = (x * x).astype(F)
    gbad = bool((~np.isfinite(g)).any())
    sums = q.reshape(nw, W).astype(np.float64).sum(axis=1)
    prefix = np.concatenate([[0.0], np.cumsum(sums)[:-1]])
    with np.errstate(over="ignore"):  # an f64 prefix beyond f32 reads as inf
        base = np.array([seq_binade(F(p)) for p in prefix], np.int64) - BELOW
    if base_shift is not None:
        base = base + base_shift
    totals, ties = candidate_pass(q, base)
    exact = 0
    for b0 in range(0, nw, BATCH):
        nb = min(BATCH, nw - b0)
        bb, tt, tie = base[b0:b0 + nb], totals[b0:b0 + nb], ties[b0:b0 + nb]
        ng = (nb + 31) // 32
        g_base, g_tot, g_fit = [], [], []
        for gi in range(ng):
            lo, hi = 32 * gi, min(nb, 32 * gi + 32)
            gb = int(bb[lo])
            tot4, fit = [], []
            for e in range(NC):
                c = gb + e - bb[lo:hi]
                ok = (c >= 0) & (c < NC)
                ok[ok] &= ~tie[lo:hi][ok, c[ok]]
                tot = tt[lo:hi][ok, c[ok]].sum() if ok.all() else 0
                tot4.append(min(int(tot), TWO24))
                fit.append(bool(ok.all()))
            g_base.append(gb)
            g_tot.append(tot4)
            g_fit.append(fit)
        k = 0
        while k < nb:
            if state["bad"]:
                break
            E, m = state["E"], state["m"]
            fine = k % 32 != 0
            miss = False
            while k < nb:
                if fine:
                    end = min((k | 31) + 1, nb)
                    idx = range(k, end)
                    cs = [E - int(bb[i]) for i in idx]
                    oks = [0 <= c < NC and not tie[i, c] for i, c in zip(idx, cs)]
                    tots = [int(tt[i, c]) if ok else 0 for i, c, ok in zip(idx, cs, oks)]
                else:
                    idx = range(k // 32, ng)
                    cs = [E - g_base[gi] for gi in idx]
                    oks = [0 <= c < NC and g_fit[gi][c] for gi, c in zip(idx, cs)]
                    tots = [g_tot[gi][c] if ok else 0 for gi, c, ok in zip(idx, cs, oks)]
                pre = np.cumsum(tots)
                stop = [not ok or m + int(p) >= TWO24 for ok, p in zip(oks, pre)]
                first = stop.index(True) if True in stop else len(stop)
                if first:
                    m += int(pre[first - 1])
                if fine:
                    k += first
                    if first < len(stop):
                        miss = True
                        break
                    fine = False
                else:
                    k = min(nb, k + 32 * first)
                    fine = first < len(stop)
            state["m"] = m
            if not miss:
                break
            w = b0 + k
            exact_window(state, q[w * W:(w + 1) * W])
            exact += 1
            k += 1
    s = state["bits"] if state["bad"] else compose(state["E"], state["m"])
    return gbad, F(s), exact


def _cases() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(7)
    cases = {
        "empty": np.zeros(0, F),
        "kat_3_4": np.array([3.0, 4.0], F),
        "zeros": np.zeros(20_000, F),
        "ragged_8191": rng.standard_normal(8191).astype(F),
        "ragged_8193": rng.standard_normal(8193).astype(F),
        "normal_1M": (rng.standard_normal(1_000_003) * 1e-3).astype(F),
        "powers_of_two": (2.0 ** rng.integers(-70, 8, 300_000)).astype(F),
        "subnormal_squares": (rng.standard_normal(200_000) * 1e-22).astype(F),
        "crossings": np.geomspace(1e-6, 1e3, 400_000).astype(F),
        "overflow": (rng.standard_normal(20_000) * 1e18).astype(F),
    }
    stall = np.full(1_000_000, F(np.sqrt(0.9) * 2.0 ** -12), F)
    stall[:3] = 1.0
    cases["stalled"] = stall
    nan = rng.standard_normal(50_000).astype(F)
    nan[9_000] = np.nan
    cases["nan"] = nan
    return cases


CASES = _cases()


@pytest.mark.parametrize("name", sorted(CASES))
def test_parallel_method_reproduces_the_sequential_f32_sum(name):
    g = CASES[name]
    gbad, got, _ = chain_sum(g)
    st, want = oracle.reference_sum_squares(g)
    assert gbad == (st == oracle.MODEL_GRADIENT_NONFINITE)
    if st == oracle.OK:
        if np.isfinite(want):
            assert F(got).view(np.uint32) == F(want).view(np.uint32), (got, want)
        else:
            assert not np.isfinite(got)


def test_many_batches_and_few_exact_windows():
    # 1,100 windows (two chain batches); a clipped gradient whose in-order sum
    # drifts below the exact one; most windows are added from their summaries
    rng = np.random.default_rng(11)
    g = rng.standard_normal(1_100 * W - 77).astype(F)
    g *= F(0.9 / float(np.sqrt(np.sum(g.astype(np.float64) ** 2))))
    gbad, got, exact = chain_sum(g)
    st, want = oracle.reference_sum_squares(g)
    assert st == oracle.OK and not gbad
    assert F(got).view(np.uint32) == F(want).view(np.uint32)
    assert exact < 60  # binade changes and early ties only


@pytest.mark.parametrize("name", ["normal_1M", "powers_of_two", "crossings"])
def test_candidate_binades_change_only_the_work(name):
    # Moving every window's candidate binades (so that many windows find none
    # that fits) must leave the bits as they are.
    g = CASES[name]
    nw = (g.size + W - 1) // W
    shift = np.random.default_rng(3).integers(-3, 4, nw)
    _, a, exact_a = chain_sum(g)
    _, b, exact_b = chain_sum(g, base_shift=shift)
    assert F(a).view(np.uint32) == F(b).view(np.uint32)
    assert exact_b >= exact_a


def test_f32_candidate_totals_equal_integer_increments():
    # Away from ties, the f32 form of a window's total (exact scaling, rintf,
    # f32 running sums of integers, clamped) equals the
    # integer sum of round-half-down increments, clamped at 2^24.
    rng = np.random.default_rng(5)
    kinds = [
        rng.standard_normal(4 * W).astype(F) * F(1e-3),
        (2.0 ** rng.integers(-80, 60, 4 * W)).astype(F),
        (rng.integers(1, 1 << 12, 4 * W) * 2.0 ** -20).astype(F),
    ]
    for x in kinds:
        q = (x * x).astype(F)
        total = float(q.astype(np.float64).sum())
        E0 = int(np.floor(np.log2(total))) - 23 - 2
        for base in (E0 - 3, E0, E0 + 2, -149, 100):
            bases = np.full(4, base, np.int64)
            totals, ties = candidate_pass(q, bases)
            for c in range(NC):
                if base + c < -149 or base + c > 104:
                    continue
                r, tie = increments(q, base + c)
                per_window_tie = tie.reshape(4, W).any(axis=1)
                assert np.array_equal(ties[:, c], per_window_tie)
                want = np.minimum(r.reshape(4, W).sum(axis=1), TWO24)
                assert np.array_equal(totals[~per_window_tie, c], want[~per_window_tie])


def test_add_based_rounding_is_rint():
    # The candidate kernel rounds some candidates by y + 2^23 - 2^23 below
    # 2^23 (y itself from there on) instead of rintf: the same value for
    # every f32 y >= 0, ties to even included.
    rng = np.random.default_rng(9)
    two23 = F(8388608.0)
    ys = np.concatenate([
        rng.uniform(0, 2**24, 1_000_000).astype(F),
        (rng.integers(0, 2**25, 1_000_000) / 2.0).astype(F),   # every half
        (2.0 ** rng.uniform(-40, 30, 1_000_000)).astype(F),
        np.array([0, 0.5, 1.5, 2.5, 8388607.5, 8388608, 8388609, 16777215, 16777216,
                  3e38, np.inf], F)])
    with np.errstate(over="ignore"):
        r = np.where(ys < two23, ((ys + two23).astype(F) - two23).astype(F), ys)
    assert np.array_equal(r, np.rint(ys))


def _first_stop_two_level(q: np.ndarray, E: int, m: int, start: int) -> int:
    """The device's stop search in one pass of the exact procedure: thread
    totals (8 terms) and warp totals (32 threads) clamped at 2^24, the first
    warp whose running total reaches 2^24 - m, the first tie, and the exact
    term looked up only inside that warp."""
    r, tie = increments(q, E)
    idx = np.arange(q.size)
    r = np.where(idx < start, 0, r)
    tie = tie & (idx >= start)
    per = r.reshape(1024, 8)
    pre = np.cumsum(per, axis=1)                      # inclusive within a thread
    runc = np.minimum(pre[:, -1], TWO24)
    warp_incl = np.cumsum(runc.reshape(32, 32), axis=1)   # within each warp
    warp_tot = np.minimum(warp_incl[:, -1], TWO24)
    scan = np.cumsum(warp_tot)
    first_tie = int(np.flatnonzero(tie)[0]) if tie.any() else None
    leaves = np.flatnonzero(m + scan >= TWO24)
    wstar = int(leaves[0]) if leaves.size else None
    if wstar is None:
        return first_tie if first_tie is not None else -1
    if first_tie is not None and first_tie < 256 * wstar:
        return first_tie
    below = int(scan[wstar - 1]) if wstar else 0
    excl_in_warp = warp_incl[wstar] - runc.reshape(32, 32)[wstar]
    for lane in range(32):
        th = 32 * wstar + lane
        excl = below + int(excl_in_warp[lane])
        for j in range(8):
            k = 8 * th + j
            if k >= start and m + excl + int(pre[th, j]) >= TWO24:
                return k if first_tie is None else min(k, first_tie)
    raise AssertionError("the warp whose total leaves the binade holds the crossing")


@pytest.mark.parametrize("seed", range(6))
def test_clamped_two_level_search_finds_the_first_stop(seed):
    # Huge terms (whose increments would wrap 32-bit sums) mixed with small
    # ones, at several binades and resume points: the clamped search must
    # stop exactly where the plain running sum says.
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(W) * 1e-3).astype(F)
    x[rng.integers(0, W, 40)] = F(1e6)
    x[rng.integers(0, W, 40)] = (2.0 ** rng.integers(-30, 0, 40)).astype(F)
    q = (x * x).astype(F)
    for E in (-149, -60, -40, -30, -20, 10):
        for m in (0, 1 << 23, TWO24 - 5):
            for start in (0, 1, 4097, W - 3):
                r, tie = increments(q, E)
                idx = np.arange(W)
                r = np.where(idx < start, 0, r)
                tie = tie & (idx >= start)
                cum = np.cumsum(r)
                stops = np.flatnonzero(tie | ((m + cum >= TWO24) & (idx >= start)))
                want = int(stops[0]) if stops.size else -1
                assert _first_stop_two_level(q, E, m, start) == want, (E, m, start)
