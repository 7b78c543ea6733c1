"""Row-parallel out_proj with its TP all-reduce (test infrastructure only).

Restates ``RowParallelLinear.forward`` without bias (T/distributed/linear.py:186-191): each TP
rank's local product of its inner-dimension slice, rounded to bf16 (the module's output
dtype), then the all-reduce sum of the partials (T/distributed/collectives.py:18-27), here in
fp32 in rank order and rounded once to bf16 (for two ranks the one correctly rounded sum any
reduction order gives).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np

from .prologue import round_bf16


def local_product(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """bf16 values of x [M, K] @ w [N, K]^T, accumulated in fp64 (the kernel's fp32 tensor-core
    accumulation agrees to rounding)."""

    return round_bf16((np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32))


def tp_reduce(partials: Sequence[np.ndarray]) -> np.ndarray:
    acc = np.zeros_like(np.asarray(partials[0], np.float32))
    for p in partials:
        acc = (acc + np.asarray(p, np.float32)).astype(np.float32)
    return round_bf16(acc)


def row_parallel(xs: Sequence[np.ndarray], ws: Sequence[np.ndarray]) -> np.ndarray:
    return tp_reduce([local_product(x, w) for x, w in zip(xs, ws)])
