"""Rectangular SOL-Attn on the B200 kernels (``h3sa_sol_attention``).

Drop-in for ``digitalhuman_h3.inference.sol_attention`` (F/inference/sol_attention.py): the
same ``sol_attn_rectangular`` call, ``SolStaticKVPart`` and ``SolAttentionCallReceipt``. The
caller packs the quality-critical K/V (condition, current media, prefixes, audio history)
first as the exact sink and the routed history after it, as the FL2AV hook does
(F/streaming/attention_hook.py:1379-1470).

The key summaries are rebuilt on the device by every call (one pass over K and V, a few
microseconds), so ``static_parts`` is accepted for interface parity but nothing is cached:
the receipt reports every block as rebuilt, and the threshold always uses the centroids'
mean and population variance (the reference's form without a static cache, :551-554).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, MutableMapping, Sequence

import torch

from ._lib import call, ptr, stream_handle
from .kernels import HEAD_DIM, _require_cuda

BLOCK = 64
GROUP = 32


@dataclass(frozen=True)
class SolStaticKVPart:
    """One immutable K/V part and its summary cache (F/inference/sol_attention.py:24-31)."""

    start_token: int
    key: Any
    value: Any
    summary_cache: MutableMapping[tuple[int, int], Any]


@dataclass(frozen=True)
class SolAttentionCallReceipt:
    static_cache_hits: int = 0
    static_cache_misses: int = 0
    static_summary_reused_blocks: int = 0
    static_summary_built_blocks: int = 0
    dynamic_or_boundary_summary_blocks: int = 0


def _blocks(n: int) -> int:
    return (n + BLOCK - 1) // BLOCK


def sol_attn_rectangular(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *,
                         scale: float, tau: float, sink_tokens: int,
                         static_parts: Sequence[SolStaticKVPart] = (),
                         telemetry_counts: torch.Tensor | None = None,
                         return_receipt: bool = False,
                         exact_blocks: torch.Tensor | None = None,
                         out: torch.Tensor | None = None,
                         device_error: torch.Tensor | None = None,
                         stream: torch.cuda.Stream | None = None):
    """SOL-Attn of ``query`` [Nq, H, 128] over ``key`` / ``value`` [Nk, H, 128] (bf16, CUDA):
    the first ceil(sink_tokens / 64) key blocks exact, the others routed per 64-row query block
    (F/inference/sol_attention.py:366-598). ``telemetry_counts``: int64 CUDA [4] to which the
    routed, exact, routable and candidate block counts are added. ``exact_blocks``: optional
    int32 CUDA [H, ceil(Nq / 64), ceil(ceil(Nk / 64) / 32)] that receives the exact-block
    bitmask. ``out``: optional contiguous bf16 CUDA tensor shaped like ``query`` that receives
    the result. Returns the bf16 output (and the receipt with ``return_receipt``)."""

    _require_cuda(telemetry_counts, exact_blocks, out, device_error)
    for name, t in (("query", query), ("key", key), ("value", value)):
        if not t.is_cuda:
            raise RuntimeError("h3sa kernels require CUDA tensors")
        if t.dtype != torch.bfloat16 or t.ndim != 3 or int(t.shape[-1]) != HEAD_DIM:
            raise RuntimeError(f"sol_attn_rectangular: {name} must be bf16 [tokens, heads, {HEAD_DIM}]")
    if tuple(key.shape) != tuple(value.shape) or key.shape[1] != query.shape[1]:
        raise RuntimeError("sol_attn_rectangular: key and value must match the query's heads")
    nq, heads = int(query.shape[0]), int(query.shape[1])
    nk = int(key.shape[0])
    if nq == 0:
        out = torch.empty_like(query)
        return (out, SolAttentionCallReceipt()) if return_receipt else out
    if nk == 0:
        raise RuntimeError("sol_attn_rectangular: no keys")
    kb, qb = _blocks(nk), _blocks(nq)
    words = (kb + 31) // 32
    if telemetry_counts is not None and (telemetry_counts.dtype != torch.int64
                                         or telemetry_counts.numel() != 4):
        raise RuntimeError("sol_attn_rectangular: telemetry_counts must be int64 [4]")
    if exact_blocks is None:
        exact_blocks = torch.empty(heads, qb, words, dtype=torch.int32, device=query.device)
    elif (exact_blocks.dtype != torch.int32 or tuple(exact_blocks.shape) != (heads, qb, words)
          or not exact_blocks.is_contiguous()):
        raise RuntimeError(f"sol_attn_rectangular: exact_blocks must be int32 [{heads}, {qb}, {words}]")
    q, k, v = query.contiguous(), key.contiguous(), value.contiguous()
    centroids = torch.empty(kb, heads, HEAD_DIM, dtype=torch.bfloat16, device=query.device)
    value_sums = torch.empty_like(centroids)
    stats = torch.empty(heads, 2, HEAD_DIM, dtype=torch.float32, device=query.device)
    if out is None:
        out = torch.empty_like(q)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != tuple(query.shape):
        raise RuntimeError("sol_attn_rectangular: out must be bf16 shaped like the query")
    call("h3sa_sol_attention", ptr(q), nq, ptr(k), ptr(v), nk, heads, HEAD_DIM, float(scale),
         float(tau), int(sink_tokens), ptr(centroids), ptr(value_sums), ptr(stats),
         ptr(exact_blocks), ptr(telemetry_counts), ptr(out), ptr(device_error),
         stream_handle(stream))
    if not return_receipt:
        return out
    return out, SolAttentionCallReceipt(dynamic_or_boundary_summary_blocks=kb)


__all__ = ["BLOCK", "GROUP", "SolAttentionCallReceipt", "SolStaticKVPart", "sol_attn_rectangular"]
