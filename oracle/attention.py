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


def segmented_fp8_attention(query: torch.Tensor, parts: Sequence[tuple], scale: float) -> torch.Tensor:
    """The segmented FP8 backend (F/streaming/attention_hook.py:1015-1066): Q quantised per
    head, one FP8 attention per K/V part with that part's own dequantisation scales, the
    partial outputs merged by their log-sum-exp (``_merge_segmented_flash_attention``,
    :319-334). ``parts``: (k_bytes, v_bytes, k_scale [H], v_scale [H]) with e4m3 bytes
    [n, H, d] (numpy uint8). Returns float32 [nq, H, d]."""

    from . import fp8 as ofp8
    import numpy as np

    q8, q_scale = ofp8.quantize_fp8_e4m3_per_head(query.float().numpy()[None])
    q = torch.from_numpy(ofp8.dequantize(q8, q_scale)[0])
    outs, lses = [], []
    for k8, v8, ks, vs in parts:
        k = torch.from_numpy(ofp8.e4m3_decode(k8) * np.asarray(ks, np.float32)[None, :, None])
        v = torch.from_numpy(ofp8.e4m3_decode(v8) * np.asarray(vs, np.float32)[None, :, None])
        s = torch.einsum("qhd,khd->hqk", q.double(), k.double()) * scale
        lse = torch.logsumexp(s, dim=-1)                       # [H, nq]
        p = torch.exp(s - lse[..., None])
        outs.append(torch.einsum("hqk,khd->qhd", p, v.double()))
        lses.append(lse)
    lse = torch.stack(lses, dim=0)                             # [parts, H, nq]
    weights = torch.exp(lse - torch.logsumexp(lse, dim=0, keepdim=True))
    merged = sum(o * w.permute(1, 0)[..., None] for o, w in zip(outs, weights))
    return merged.float()
