"""Dense streaming attention oracle (test infrastructure only).

Restates, on CPU:

* ``_sdpa_from_kv_parts`` (F/streaming/attention_hook.py:288-316): concatenate K/V parts
  and run non-causal softmax(Q K^T * scale) V;
* the per-document visibility of ``H3StreamingAttentionHook.__call__``
  (T/streaming/attention_hook.py:118-221): condition rows see condition K/V; media rows see
  [condition, persistent history, current media]; other documents see themselves;
* the FP8 dynamic backend's arithmetic (F/streaming/attention_hook.py:1081-1098 with the
  quantiser of F/inference/fused_kernels.py:826-834): attention on per-head dequantised
  e4m3 Q/K/V.
"""

from __future__ import annotations

from typing import Sequence

import torch


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
              allowed: torch.Tensor | None = None) -> torch.Tensor:
    """q [nq, H, d], k/v [nk, H, d] -> [nq, H, d] float32 (F attention_hook.py:306-315)."""

    s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) * scale
    if allowed is not None:
        s = s.masked_fill(~allowed, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, v.float())


def sdpa_from_kv_parts(query: torch.Tensor, parts: Sequence[tuple[torch.Tensor, torch.Tensor]],
                       scale: float) -> torch.Tensor:
    """Exact SDPA over an ordered K/V plan (F/streaming/attention_hook.py:288-316)."""

    key = parts[0][0] if len(parts) == 1 else torch.cat([p[0] for p in parts], dim=0)
    value = parts[0][1] if len(parts) == 1 else torch.cat([p[1] for p in parts], dim=0)
    out = torch.nn.functional.scaled_dot_product_attention(
        query.float().transpose(0, 1).unsqueeze(0),
        key.float().transpose(0, 1).unsqueeze(0),
        value.float().transpose(0, 1).unsqueeze(0),
        dropout_p=0.0, is_causal=False, scale=scale,
    )
    return out.squeeze(0).transpose(0, 1)


def streaming_hook_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                             commit_mask: torch.Tensor, cu_seqlens: Sequence[int],
                             history: tuple[torch.Tensor, torch.Tensor] | None,
                             scale: float) -> torch.Tensor:
    """Output of the dense streaming hook for one layer call (T attention_hook.py:118-221)."""

    points = [int(p) for p in cu_seqlens]
    boundaries = list(zip(points[:-1], points[1:]))
    live = [i for i, (a, b) in enumerate(boundaries) if bool(commit_mask[a:b].any())]
    if len(live) != 1:
        raise RuntimeError(f"direct streaming expects exactly one live document, got {tuple(live)}")
    outputs = []
    for index, (start, stop) in enumerate(boundaries):
        if start == stop:
            continue
        qd, kd, vd = query[start:stop], key[start:stop], value[start:stop]
        if index != live[0]:
            outputs.append(sdpa_from_kv_parts(qd, [(kd, vd)], scale))
            continue
        media = commit_mask[start:stop].to(torch.bool)
        cond_idx = torch.nonzero(~media).flatten()
        media_idx = torch.nonzero(media).flatten()
        ck, cv = kd.index_select(0, cond_idx), vd.index_select(0, cond_idx)
        cond_out = sdpa_from_kv_parts(qd.index_select(0, cond_idx), [(ck, cv)], scale)
        parts = [(ck, cv)]
        if history is not None:
            parts.append(history)
        parts.append((kd.index_select(0, media_idx), vd.index_select(0, media_idx)))
        media_out = sdpa_from_kv_parts(qd.index_select(0, media_idx), parts, scale)
        doc = torch.zeros(qd.shape, dtype=torch.float32)
        doc.index_copy_(0, cond_idx, cond_out)
        doc.index_copy_(0, media_idx, media_out)
        outputs.append(doc)
    return torch.cat(outputs, dim=0)


def attention_flops(nq: int, nk: int, heads: int, head_dim: int) -> float:
    """Algorithmic FLOPs of non-causal attention: QK^T and PV, 2 FLOPs per MAC."""

    return 4.0 * nq * nk * head_dim * heads


def time_cpu_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                       threads: int) -> float:
    """Seconds for one oracle attention call on ``threads`` host threads."""

    import time

    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        t0 = time.perf_counter()
        sdpa_from_kv_parts(q, [(k, v)], scale)
        return time.perf_counter() - t0
    finally:
        torch.set_num_threads(prev)


__all__ = [
    "attention",
    "attention_flops",
    "sdpa_from_kv_parts",
    "streaming_hook_attention",
    "time_cpu_attention",
]
