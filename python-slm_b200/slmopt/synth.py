"""Seeded synthetic optimizer inputs (no dataset or checkpoint is involved).

Every array is drawn from its own numpy ``Philox`` (Philox4x32-10, Salmon et
al. 2011) stream keyed by ``SeedSequence([seed, stream])`` with the float32
ziggurat ``standard_normal``, so a (seed, stream) pair always gives the same
bytes on the same numpy.  Distributions (std, not variance):

* master   ~ N(0, 0.02)            (INIT-001 std, src/model/oracle.rs:21)
* gradient ~ N(0, 1e-3)            fp32, or bf16 RNE of N(0,1e-3) * loss_scale
* moment   ~ N(0, 1e-4)
* variance = N(0, 1e-3)^2
* stress gradient = 1e-3 * Student-t(df=3) = Z / sqrt(chi2_3 / 3)
"""
from __future__ import annotations

import numpy as np

STREAM_MASTER = 1
STREAM_MOMENT = 2
STREAM_VARIANCE = 3
STREAM_GRAD = 4


def generator(seed: int, stream: int) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(np.random.SeedSequence([int(seed), int(stream)])))


def normal_f32(n: int, std: float, seed: int, stream: int) -> np.ndarray:
    z = generator(seed, stream).standard_normal(int(n), dtype=np.float32)
    z *= np.float32(std)
    return z


def bf16_rne_bits(x: np.ndarray) -> np.ndarray:
    """src/model/oracle.rs:300-304 over an f32 array -> uint16 bits."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))
    return ((b + bias) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def _parallel_normals(n: int, specs: list[tuple[float, int]], seed: int) -> list[np.ndarray]:
    """Independent streams drawn on threads (numpy releases the GIL while
    filling); each stream's bytes do not depend on the threading."""
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=len(specs)) as ex:
        futs = [ex.submit(normal_f32, n, std, seed, stream) for std, stream in specs]
        return [f.result() for f in futs]


def optimizer_state(n: int, seed: int = 0) -> dict[str, np.ndarray]:
    """master/m/v with the benchmark distributions and bf16 = RNE(master)."""
    master, moment, v = _parallel_normals(
        n, [(0.02, STREAM_MASTER), (1e-4, STREAM_MOMENT), (1e-3, STREAM_VARIANCE)], seed)
    variance = v * v
    return {"master": master, "moment": moment, "variance": variance,
            "bf16": bf16_rne_bits(master)}


def grads_f32(n: int, seed: int = 0, stream: int = STREAM_GRAD) -> np.ndarray:
    return normal_f32(n, 1e-3, seed, stream)


def grads_bf16(n: int, seed: int = 0, loss_scale: float = 65536.0,
               stream: int = STREAM_GRAD) -> np.ndarray:
    """bf16 bits of N(0, 1e-3) * loss_scale (the multiply is in f32)."""
    g = normal_f32(n, 1e-3, seed, stream)
    g *= np.float32(loss_scale)
    return bf16_rne_bits(g)


def grads_student_t(n: int, seed: int, step: int, scale: float = 1e-3) -> np.ndarray:
    """1e-3 * t(3) draws for one step of the stress run, as float32."""
    t = generator(seed, 1000 + int(step)).standard_t(3, size=int(n))
    return (t * scale).astype(np.float32)


def inject_nonfinite(bits_or_f32: np.ndarray, seed: int, offsets: np.ndarray,
                     value: str = "inf") -> tuple[int, int]:
    """Write one +inf (or nan) at a seeded random index of a seeded random
    tensor, in place; returns (tensor index, flat index)."""
    rng = generator(seed, 9999)
    k = int(rng.integers(0, len(offsets) - 1))
    lo, hi = int(offsets[k]), int(offsets[k + 1])
    i = int(rng.integers(lo, hi))
    if bits_or_f32.dtype == np.uint16:
        bits_or_f32[i] = 0x7F80 if value == "inf" else 0x7FC0
    else:
        bits_or_f32[i] = np.inf if value == "inf" else np.nan
    return k, i
