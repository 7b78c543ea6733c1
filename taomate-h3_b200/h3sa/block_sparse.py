"""128-token block-sparse masks on the sm_100a mask kernel.

``history_block_mask`` is the reference rule ``_dynamic_history_mask``
(F/inference/dynamic_block_sparse.py:50-124): per (head, q-block) the top
``max(1, min(full, ceil(full * density)))`` full history blocks by block-mean score, plus the
partial history tail and every current block. ``composite_block_mask`` is the benchmark
policy (audio blocks, sinks, a local band in the KV timeline, top-k fill to a density
budget). Both return the flex ``BlockMask.from_kv_blocks`` inputs consumed by
``attention_fwd``; selections are exact (fixed-order fp64 scores, lower index wins ties).
"""

from __future__ import annotations

import math

import torch

from ._lib import MaskPolicy, call, ptr, stream_handle
from .kernels import PAGE_ROWS


def _run(query: torch.Tensor, paged, *, q_lo: int, q_hi: int, policy: MaskPolicy,
         device_error: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    rows, heads, head_dim = (int(s) for s in query.shape)
    qb = (q_hi - q_lo + PAGE_ROWS - 1) // PAGE_ROWS
    kb = (policy.n_kv + PAGE_ROWS - 1) // PAGE_ROWS
    num = torch.empty(heads, qb, dtype=torch.int32, device=query.device)
    idx = torch.empty(heads, qb, kb, dtype=torch.int32, device=query.device)
    call("h3sa_block_mask", ptr(query), rows, heads, head_dim, int(q_lo), int(q_hi),
         ptr(paged.key), int(paged.key.shape[1]) // PAGE_ROWS, ptr(paged.table),
         int(paged.table.numel()), policy, ptr(num), ptr(idx), kb, ptr(device_error),
         stream_handle(None))
    return num, idx


def history_block_mask(query: torch.Tensor, paged, *, q_lo: int, q_hi: int, n_hist: int,
                       n_kv: int, density: float,
                       device_error: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    if not 0.0 < density <= 1.0:
        raise ValueError("dynamic history density must be in (0, 1]")
    if n_hist // PAGE_ROWS < 1:
        raise ValueError("dynamic sparse history has no complete K/V block")
    pol = MaskPolicy(mode=0, n_hist=int(n_hist), n_kv=int(n_kv), density=float(density))
    return _run(query, paged, q_lo=q_lo, q_hi=q_hi, policy=pol, device_error=device_error)


def composite_block_mask(query: torch.Tensor, paged, *, q_lo: int, q_hi: int, n_hist: int,
                         n_kv: int, q_block_audio: torch.Tensor, kv_block_audio: torch.Tensor,
                         density: float = 0.25, sinks: int = 2, window: int = 4,
                         device_error: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    qa = q_block_audio.to(device=query.device, dtype=torch.uint8).contiguous()
    ka = kv_block_audio.to(device=query.device, dtype=torch.uint8).contiguous()
    # the kernel reads one flag per query block and per KV block through raw pointers
    if qa.numel() < (q_hi - q_lo + PAGE_ROWS - 1) // PAGE_ROWS:
        raise ValueError("q_block_audio needs one flag per 128-row query block")
    if ka.numel() < (n_kv + PAGE_ROWS - 1) // PAGE_ROWS:
        raise ValueError("kv_block_audio needs one flag per 128-row KV block")
    pol = MaskPolicy(mode=1, n_hist=int(n_hist), n_kv=int(n_kv), sinks=int(sinks),
                     window=int(window), density=float(density), q_block_audio=ptr(qa),
                     kv_block_audio=ptr(ka))
    num, idx = _run(query, paged, q_lo=q_lo, q_hi=q_hi, policy=pol, device_error=device_error)
    del qa, ka
    return num, idx


def block_flags(is_audio: torch.Tensor, rows: int) -> torch.Tensor:
    """Per 128-row block: does it hold any audio row (uint8)."""

    blocks = math.ceil(rows / PAGE_ROWS)
    flags = torch.zeros(blocks * PAGE_ROWS, dtype=torch.bool, device=is_audio.device)
    flags[:rows] = is_audio[:rows].to(torch.bool)
    return flags.view(blocks, PAGE_ROWS).any(dim=1).to(torch.uint8)


def history_block_lists(q_src: torch.Tensor, problem, paged, *, n_hist: int, n_kv: int,
                        density: float, scale: float) -> dict:
    """Block lists for the hook's media problem, or {} when the history has no full block
    (the reference then runs dense attention, F/streaming/attention_hook.py:1507)."""

    del scale
    if n_hist < PAGE_ROWS:
        return {}
    num, idx = history_block_mask(q_src, paged, q_lo=problem.q_lo, q_hi=problem.q_hi,
                                  n_hist=n_hist, n_kv=n_kv, density=density)
    return {"kv_num_blocks": num, "kv_indices": idx}


__all__ = ["block_flags", "composite_block_mask", "history_block_lists", "history_block_mask"]
