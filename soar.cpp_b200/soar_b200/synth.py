"""Seeded synthetic inputs for the optimizer-step workloads.

One documented host generator feeds every test, the bench and the oracle, so
device and oracle see identical bits: SplitMix64 over a counter, two 53-bit
uniforms per pair, Box-Muller in float64, then rounded to float32
(csrc/synth.c, OpenMP-parallel, thread-count independent). Seeds are mixed
from (config, tensor, step, rank). The GPU never generates values.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _build

_synth = None


def _lib():
    global _synth
    if _synth is None:
        h = C.CDLL(str(_build.build_synth()))
        h.soar_synth_splitmix64.argtypes = [C.c_uint64, C.c_uint64, C.c_void_p]
        h.soar_synth_normal_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_double, C.c_double,
                                            C.c_void_p]
        _synth = h
    return _synth

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _mix(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def seed_of(config: int, tensor: int = 0, step: int = 0, rank: int = 0) -> int:
    """64-bit seed for one (config, tensor, step, rank) stream."""
    with np.errstate(over="ignore"):
        z = np.array([config * 0x1000193 + 1], dtype=np.uint64)
        for part in (tensor, step, rank):
            z = _mix(z + _GOLDEN + np.uint64(part & 0xFFFFFFFFFFFFFFFF))
    return int(z[0])


def splitmix64(seed: int, n: int) -> np.ndarray:
    """n outputs of SplitMix64 started at `seed` (state advances by the golden gamma)."""
    out = np.empty(n, np.uint64)
    _lib().soar_synth_splitmix64(seed & 0xFFFFFFFFFFFFFFFF, n, out.ctypes.data)
    return out


def splitmix64_np(seed: int, n: int) -> np.ndarray:
    """Pure-numpy restatement of splitmix64 (checks the C generator)."""
    with np.errstate(over="ignore"):
        ctr = np.arange(1, n + 1, dtype=np.uint64)
        state = np.uint64(seed) + ctr * _GOLDEN
        return _mix(state)


def normal(seed: int, n: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    """n float32 samples of N(mean, std^2) by Box-Muller over SplitMix64."""
    out = np.empty(n, np.float32)
    if n:
        _lib().soar_synth_normal_f32(seed & 0xFFFFFFFFFFFFFFFF, n, float(std), float(mean),
                                     out.ctypes.data)
    return out


def uniform_int(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive)."""
    u = splitmix64(seed, n)
    return (lo + (u % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int64)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even; NaN -> 0x7FFF."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    r = ((u + np.uint32(0x7FFF) + lsb) >> np.uint32(16)).astype(np.uint16)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    r[nan] = 0x7FFF
    return r


def from_bf16_bits(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(
        np.float32)


# ---------------------------------------------------------------- configs ---

def config2_shapes() -> list[tuple[str, tuple[int, ...]]]:
    """Segmentation-net tensor list (240 tensors, ~12 M params).

    48 groups of {depthwise [C,1,k,k] (k cycles 3,5,7), 1x1 conv [4C, C],
    GroupNorm gamma [C], GroupNorm beta [C], bias [C]}, C cycling
    32, 64, 128, 256, 512. The depthwise kernel, 1x1 weight, GroupNorm
    gamma/beta and bias are the parameter kinds of the reference's SOAR blocks
    (conv layers [Cout, Cin/groups, k, k], GroupNorm gamma=1 / beta=0)."""
    shapes = []
    cs = (32, 64, 128, 256, 512)
    ks = (3, 5, 7)
    for i in range(48):
        c = cs[i % 5]
        k = ks[i % 3]
        shapes.append(("dw", (c, 1, k, k)))
        shapes.append(("pw", (4 * c, c)))
        shapes.append(("gn_gamma", (c,)))
        shapes.append(("gn_beta", (c,)))
        shapes.append(("bias", (c,)))
    return shapes


def config3_sizes(total: int = 50_000_000, n: int = 400, lo: int = 16384,
                  hi: int = 262144, seed: int | None = None) -> list[int]:
    """n tensor sizes drawn ~U[lo, hi], then rescaled by total/sum so they add
    up to exactly `total` (the last size absorbs the rounding). U[16K, 256K]
    has mean ~139K, so 400 draws sum to ~56M; the rescale maps them onto
    ~U[14.7K, 236K] to keep both the tensor count and the 50M total."""
    s = uniform_int(seed_of(3, 999_999) if seed is None else seed, n, lo, hi).astype(np.float64)
    scaled = np.floor(s * (total / s.sum())).astype(np.int64)
    scaled[-1] += total - int(scaled.sum())
    return [int(x) for x in scaled]
