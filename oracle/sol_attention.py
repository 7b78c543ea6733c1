"""Rectangular SOL-Attn routing on CPU (test infrastructure only: tests, smoke and the bench's
CPU leg use it as the checker; the product path never calls it).

Restates ``sol_attn_rectangular`` of the FL2AV SOL-Attn adapter
(F/inference/sol_attention.py:366-598) without its static summary cache:

* 64-row key blocks: key centroid = sum of the block's K rows / its length, value sum = sum of
  its V rows, both stored in the summary dtype (bf16 on the GPU; :99-125, reduce_kv);
* 64-row query blocks: query centroid = sum of the rows / length, summary dtype (:157-179);
* per head the centroids' mean and population variance (:551-554), and per (query block,
  head) the route threshold ``mu + tau * sqrt(max(var, 0) + 1e-6)`` of the proxy score
  ``q_bar . k_c * scale * log2(e)`` under a diagonal covariance (:555-566);
* a key block is exact for a query block when it lies in the first ceil(sink / 64) blocks
  (the sink) or when its proxy score averaged over the block's query rows exceeds the
  threshold (:269-283); every other valid block is approximate: it enters the softmax once
  per query row with its proxy score, weight = its row count and value = its value sum
  (:295-322); exact blocks are ordinary attention rows (:324-352).

Softmax statistics run in float64 here; the probabilities that multiply values are rounded to
the value dtype first, as the reference's ``p.to(value.dtype)`` before each ``tl.dot``.
Outputs are returned in float32 before the reference's final bf16 cast, with the exact-block
mask, the route margins (score - threshold) and the four telemetry counts (selected, exact,
routable, candidate; :284-294).
"""

from __future__ import annotations

import math

import torch

BLOCK = 64
LOG2E = 1.4426950408889634


def _blocks(n: int) -> int:
    return (n + BLOCK - 1) // BLOCK


def summaries(x: torch.Tensor, *, mean: bool, dtype: torch.dtype) -> torch.Tensor:
    """Per 64-row block sums (or means) of ``x`` [N, H, D], float32 added in row order, rounded
    to ``dtype``."""

    n = x.shape[0]
    out = []
    for b in range(_blocks(n)):
        rows = x[b * BLOCK:(b + 1) * BLOCK].float()
        s = rows[0].clone()
        for r in range(1, rows.shape[0]):
            s = s + rows[r]
        if mean:
            s = s / float(rows.shape[0])
        out.append(s)
    return torch.stack(out).to(dtype)


def sol_attn_rectangular(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *,
                         scale: float, tau: float, sink_tokens: int,
                         summary_dtype: torch.dtype = torch.bfloat16,
                         exact: torch.Tensor | None = None):
    """query [Nq, H, D], key / value [Nk, H, D] (values exactly representable in
    ``summary_dtype``). ``exact`` (bool [QB, H, KB]) replaces the computed routing when given.

    Returns (out float32 [Nq, H, D], exact bool [QB, H, KB], margin float64 [QB, H, KB],
    telemetry int64 [4])."""

    nq, heads, d = query.shape
    nk = key.shape[0]
    qb_n, kb_n = _blocks(nq), _blocks(nk)
    q32, k32, v32 = query.float(), key.float(), value.float()
    kc = summaries(k32, mean=True, dtype=summary_dtype).float()   # [KB, H, D]
    vs = summaries(v32, mean=False, dtype=summary_dtype).float()
    qbar = summaries(q32, mean=True, dtype=summary_dtype).float()  # [QB, H, D]
    lengths = torch.tensor([min(BLOCK, nk - b * BLOCK) for b in range(kb_n)], dtype=torch.float64)
    log2_scale = float(scale) * LOG2E
    key_mean = kc.mean(dim=0)
    key_var = kc.var(dim=0, unbiased=False)
    proxy_mean = (qbar * key_mean[None]).sum(-1) * log2_scale
    proxy_var = (qbar.square() * key_var[None]).sum(-1) * (log2_scale * log2_scale)
    threshold = proxy_mean + float(tau) * torch.sqrt(proxy_var.clamp_min(0.0) + 1.0e-6)

    sink_blocks = _blocks(int(sink_tokens)) if sink_tokens > 0 else 0
    block_ids = torch.arange(kb_n)
    sink = block_ids < sink_blocks
    margin = torch.zeros(qb_n, heads, kb_n, dtype=torch.float64)
    computed = torch.zeros(qb_n, heads, kb_n, dtype=torch.bool)
    tele = torch.zeros(4, dtype=torch.int64)
    for qb in range(qb_n):
        rows = q32[qb * BLOCK:(qb + 1) * BLOCK]
        for h in range(heads):
            # mean over the block's rows of the fp32 proxy scores (q . k_c per row)
            score = ((rows[:, h] @ kc[:, h].T) * log2_scale).double().sum(0) / rows.shape[0]
            margin[qb, h] = score - float(threshold[qb, h])
            selected = (margin[qb, h] > 0) & ~sink
            computed[qb, h] = selected | sink
            tele += torch.tensor([int(selected.sum()), int(computed[qb, h].sum()),
                                  int((~sink).sum()), kb_n])
    route = computed if exact is None else exact.bool()

    out = torch.zeros(nq, heads, d, dtype=torch.float32)
    vdt = value.dtype if value.dtype != torch.float32 else summary_dtype
    for qb in range(qb_n):
        r0, r1 = qb * BLOCK, min(nq, (qb + 1) * BLOCK)
        for h in range(heads):
            ex = route[qb, h]
            key_rows = torch.cat([torch.arange(b * BLOCK, min(nk, (b + 1) * BLOCK))
                                  for b in range(kb_n) if bool(ex[b])] or [torch.zeros(0, dtype=torch.long)])
            approx = ~ex
            s_exact = (q32[r0:r1, h] @ k32[key_rows, h].T).double() * log2_scale
            s_proxy = (q32[r0:r1, h] @ kc[approx, h].T).double() * log2_scale
            m = torch.full((r1 - r0,), -math.inf, dtype=torch.float64)
            if s_exact.numel():
                m = torch.maximum(m, s_exact.max(1).values)
            if s_proxy.numel():
                m = torch.maximum(m, s_proxy.max(1).values)
            p_exact = torch.exp2(s_exact - m[:, None])
            p_proxy = torch.exp2(s_proxy - m[:, None])
            den = p_exact.sum(1) + (p_proxy * lengths[approx][None]).sum(1)
            # probabilities rounded to the value dtype before they multiply values
            pe = p_exact.float().to(vdt).double()
            pp = p_proxy.float().to(summary_dtype).double()
            num = pe @ v32[key_rows, h].double() + pp @ vs[approx, h].double()
            out[r0:r1, h] = (num / den[:, None]).float()
    return out, route, margin, tele


__all__ = ["BLOCK", "sol_attn_rectangular", "summaries"]
