"""Shared test data and error metrics.

Inputs follow the distributions of the reference benchmark configs: weights
N(0, 0.02) quantized per row by absmax, activations N(0, 1).  Data is made on
the host with numpy's seeded Generator and fed to both the GPU path and the
CPU oracle, so no RNG has to agree across libraries.
"""
from __future__ import annotations

import numpy as np

# Tolerances (normwise: max_j |y - y_ref| / max_j |y_ref|).
TOL_F32 = 1e-5   # fp32-activation path
TOL_F16 = 2e-3   # fp16-activation path (compared after the kernel's fp16 rounding)


def make_weight(N: int, K: int, seed: int, std: float = 0.02) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((N, K), dtype=np.float32) * np.float32(std)).astype(np.float32)


def make_x(M: int, K: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K), dtype=np.float32)


def make_bias(N: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(N, dtype=np.float32) * np.float32(0.1)).astype(np.float32)


def normwise_err(y: np.ndarray, ref: np.ndarray) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    if den == 0:
        return float(np.max(np.abs(y)))
    return float(np.max(np.abs(y - ref)) / den)


def rowwise_normwise_err(y: np.ndarray, ref: np.ndarray) -> float:
    """Worst normwise error over the token rows of [M, N] outputs."""
    y = np.atleast_2d(y)
    ref = np.atleast_2d(ref)
    return max(normwise_err(y[i], ref[i]) for i in range(ref.shape[0]))


def elementwise_rel_err(y: np.ndarray, ref: np.ndarray, floor_frac: float = 1e-3) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    floor = floor_frac * np.max(np.abs(ref))
    return float(np.max(np.abs(y - ref) / np.maximum(np.abs(ref), floor)))


def sample_rows(N: int, n: int, seed: int = 7) -> np.ndarray:
    """First/last rows plus a seeded random sample, sorted, unique."""
    rng = np.random.default_rng(seed)
    pick = set(rng.choice(N, size=min(n, N), replace=False).tolist())
    pick.update([0, N - 1, N // 2])
    return np.array(sorted(pick), dtype=np.int64)
