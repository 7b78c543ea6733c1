"""W8A8 projection oracle (test infrastructure only).

Restates, in numpy float32 / int64:

* the weight quantiser ``_quantize_weight`` (T/inference/w8a8.py:56-63):
  scale = max(amax_row / 127, 1e-12), q = clamp(round_half_even(w / scale), -127, 127);
* the dynamic per-token activation quantiser the reference calls through vLLM
  (``scaled_int8_quant``, vllm==0.11.1, not vendored): scale = amax_row / 127,
  q = clamp(round_half_even(x * (127 / amax_row)), -128, 127), zero rows -> zeros;
* the scaled int8 GEMM (vLLM ``cutlass_scaled_mm``, same version): exact integer products
  summed exactly, then bf16_rn(a_scale * (b_scale * float32(acc))).

The weight quantiser is pinned to the reference's own code (tests/golden/w8a8.npz); the two
vLLM operations are checked against vLLM itself on the GPU where it loads.
"""

from __future__ import annotations

import numpy as np

from .prologue import round_bf16


def quantize_weight(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    w = np.asarray(w, dtype=np.float32)
    amax = np.abs(w).max(axis=1, keepdims=True)
    scale = np.maximum(amax / np.float32(127.0), np.float32(1.0e-12)).astype(np.float32)
    q = np.clip(np.rint(w / scale), -127, 127).astype(np.int8)
    return q, scale


def quantize_activation(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(axis=1, keepdims=True).astype(np.float32)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        mul = np.where(amax > 0, np.float32(127.0) / amax, np.float32(0.0)).astype(np.float32)
    q = np.clip(np.rint(x * mul), -128, 127).astype(np.int8)
    return q, scale


def scaled_mm(qa: np.ndarray, sa: np.ndarray, qb: np.ndarray, sb: np.ndarray) -> np.ndarray:
    """int8 [M, K], fp32 [M] | [M, 1], int8 [N, K], fp32 [N] | [N, 1] -> bf16 values [M, N]."""

    acc = qa.astype(np.int64) @ qb.astype(np.int64).T
    f = acc.astype(np.float32)
    sa = np.asarray(sa, np.float32).reshape(-1, 1)
    sb = np.asarray(sb, np.float32).reshape(1, -1)
    return round_bf16(sa * (sb * f))
