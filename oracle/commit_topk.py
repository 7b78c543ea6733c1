"""Commit-level top-k of the segmented FP8 backend (test infrastructure only).

Restates, in numpy:

* the key summary of a committed history block: the fp32 mean of its bf16 key rows
  (``key_summary=pair.key.float().mean(dim=0)``, F/streaming/cache.py:854), recomputed over
  the rows a retention keeps (F/streaming/cache.py:1031-1034);
* the selection (F/streaming/attention_hook.py:1256-1302): keep
  ``max(1, min(n, ceil(n * density)))`` blocks; when that is fewer than all of them, score
  block i as the mean over heads of ``sum_d summary[i, h, d] * query_mean[h, d]``, with
  ``query_mean`` the fp32 mean of the media query rows, take the highest scores and attend to
  those blocks in commit order.

Means are taken as the fp64 sum divided in fp64 and rounded to fp32 (the reference's fp32
reduction agrees to an ulp); scores use fp64 products and sums. Equal scores keep the older
block first (torch.topk leaves that order unspecified).
"""

from __future__ import annotations

import math

import numpy as np


def key_summary(rows: np.ndarray) -> np.ndarray:
    """[rows, heads, d] (bf16 values) -> fp32 [heads, d] column means."""

    rows = np.asarray(rows, dtype=np.float64)
    return (rows.sum(axis=0) / rows.shape[0]).astype(np.float32)


def commit_scores(summaries: np.ndarray, query_mean: np.ndarray) -> np.ndarray:
    """[n, heads, d] fp32 and [heads, d] fp32 -> fp64 [n]."""

    s = np.asarray(summaries, dtype=np.float64)
    q = np.asarray(query_mean, dtype=np.float64)
    return (s * q[None]).sum(axis=(1, 2)) / s.shape[1]


def selected_count(n: int, density: float) -> int:
    return max(1, min(n, math.ceil(n * density)))


def select_commits(scores: np.ndarray, density: float) -> list[int]:
    """Indices of the kept commits, ascending."""

    n = int(len(scores))
    if n == 0:
        return []
    count = selected_count(n, density)
    if count >= n:
        return list(range(n))
    order = sorted(range(n), key=lambda i: (-float(scores[i]), i))
    return sorted(order[:count])
