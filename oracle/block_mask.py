"""128-token block-sparse mask oracle (test infrastructure only).

Two selection rules over the logical KV sequence ``[history | current ...]``:

1. ``dynamic_history_mask`` restates ``_dynamic_history_mask``
   (F/inference/dynamic_block_sparse.py:50-124): per (head, q-block), score every *full*
   history block by mean(Q block) . mean(K block) * d^-0.5, keep
   ``max(1, min(full, ceil(full * density)))`` of them, and keep the partial history tail
   and every current block dense. Output: flex ``BlockMask.from_kv_blocks`` inputs
   (``kv_num_blocks [H, QB]``, ``kv_indices [H, QB, KB]`` sorted, zero padded).

2. ``composite_mask`` is the block-sparse policy of the 768p benchmark configuration: every
   block pair touching audio (a q-block holding an audio query row attends to all blocks;
   every q-block attends to blocks holding audio keys), the first ``sinks`` KV blocks, a
   +-``window``-block band around each q-block's position in the KV timeline, and the rest
   of a ``ceil(density * KB)`` budget filled by the highest block-mean scores.

Arithmetic is fixed so that CPU and GPU selections agree bit for bit: block sums of bf16
values in fp64 (exact for these magnitudes, hence order independent), means by one fp64
division, dot products in fp64 with separate multiply and add, as eight partial sums (the
terms d = g, g + 8, g + 16, ... accumulated in order for g = 0..7) combined as
((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)), one fp64 multiply by d^-0.5. Ties rank the lower block index first. The reference
computes the same quantities in fp32 with an unspecified summation order and tie rule; the
two agree wherever the k-th and (k+1)-th scores are further apart than fp32 rounding,
which ``selection_margin`` reports.
"""

from __future__ import annotations

import math

import numpy as np

BLOCK = 128


def block_means(x: np.ndarray, block: int = BLOCK) -> np.ndarray:
    """x [H, N, D] -> [H, ceil(N / block), D] fp64 means (last block over its real rows)."""

    x = np.asarray(x, dtype=np.float64)
    h, n, d = x.shape
    nb = math.ceil(n / block)
    pad = nb * block - n
    xp = np.concatenate([x, np.zeros((h, pad, d))], axis=1) if pad else x
    sums = xp.reshape(h, nb, block, d).sum(axis=2)
    counts = np.full(nb, float(block))
    if pad:
        counts[-1] = n - (nb - 1) * block
    return sums / counts[None, :, None]


PARTIALS = 8


def block_scores(q_mean: np.ndarray, k_mean: np.ndarray, head_dim: int) -> np.ndarray:
    """[H, QB, D] x [H, KB, D] -> [H, QB, KB]: fp64 dot over d in the fixed order above, times
    d^-0.5."""

    shape = (q_mean.shape[0], q_mean.shape[1], k_mean.shape[1])
    part = [np.zeros(shape, dtype=np.float64) for _ in range(PARTIALS)]
    for dd in range(q_mean.shape[2]):
        g = dd % PARTIALS
        part[g] = part[g] + q_mean[:, :, None, dd] * k_mean[:, None, :, dd]
    acc = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]))
    return acc * (float(head_dim) ** -0.5)


def _top(scores: np.ndarray, candidates: np.ndarray, count: int) -> np.ndarray:
    """Indices (into the last axis) of the ``count`` best candidates; ties: lower index."""

    if count <= 0:
        return np.zeros(0, dtype=np.int64)
    idx = np.nonzero(candidates)[0]
    order = np.lexsort((idx, -scores[idx]))
    return np.sort(idx[order[:count]])


def dynamic_history_mask(query: np.ndarray, history_key: np.ndarray, total_key_tokens: int,
                         density: float, block: int = BLOCK) -> dict:
    """query [H, Nq, D], history_key [H, Nh, D] -> mask dict (F dynamic_block_sparse.py:50-124)."""

    h, nq, d = query.shape
    nh = history_key.shape[1]
    full_hist = nh // block
    total_hist = math.ceil(nh / block)
    total_kv = math.ceil(total_key_tokens / block)
    if full_hist < 1:
        raise ValueError("dynamic sparse history has no complete K/V block")
    selected_count = max(1, min(full_hist, math.ceil(full_hist * density)))
    qm = block_means(query, block)
    km = block_means(history_key[:, : full_hist * block], block)
    scores = block_scores(qm, km, d)
    qb = qm.shape[1]
    dense = np.arange(full_hist, total_kv)
    width = selected_count + dense.size
    kv_num = np.full((h, qb), width, dtype=np.int32)
    kv_idx = np.zeros((h, qb, total_kv), dtype=np.int32)
    cand = np.ones(full_hist, dtype=bool)
    for hh in range(h):
        for j in range(qb):
            sel = _top(scores[hh, j], cand, selected_count)
            kv_idx[hh, j, :width] = np.sort(np.concatenate([sel, dense]))
    receipt = {
        "history_tokens": nh,
        "history_blocks": total_hist,
        "selected_history_blocks": selected_count + int(total_hist > full_hist),
        "always_dense_key_blocks": int(dense.size),
    }
    return {"kv_num_blocks": kv_num, "kv_indices": kv_idx, "scores": scores,
            "selected_count": selected_count, "receipt": receipt}


def composite_mask(query: np.ndarray, key: np.ndarray, *, n_hist: int, q_audio: np.ndarray,
                   k_audio: np.ndarray, density: float = 0.25, sinks: int = 2, window: int = 4,
                   block: int = BLOCK) -> dict:
    """query [H, Nq, D] (current chunk), key [H, Nk, D] (the whole logical KV sequence).

    q_audio / k_audio: bool per query row / key row. Query block j sits at KV-timeline block
    floor((n_hist + 128 j) / 128).
    """

    h, nq, d = query.shape
    nk = key.shape[1]
    qb = math.ceil(nq / block)
    kb = math.ceil(nk / block)
    qa = np.zeros(qb * block, dtype=bool)
    qa[:nq] = q_audio
    ka = np.zeros(kb * block, dtype=bool)
    ka[:nk] = k_audio
    q_has_audio = qa.reshape(qb, block).any(axis=1)
    k_has_audio = ka.reshape(kb, block).any(axis=1)
    kpos = np.arange(kb)
    forced = np.zeros((qb, kb), dtype=bool)
    for j in range(qb):
        qpos = (n_hist + block * j) // block
        forced[j] = (q_has_audio[j] | k_has_audio | (kpos < sinks)
                     | (np.abs(kpos - qpos) <= window))
    budget = math.ceil(density * kb)
    qm = block_means(query, block)
    km = block_means(key, block)
    scores = block_scores(qm, km, d)
    kv_num = np.zeros((h, qb), dtype=np.int32)
    kv_idx = np.zeros((h, qb, kb), dtype=np.int32)
    for hh in range(h):
        for j in range(qb):
            f = np.nonzero(forced[j])[0]
            remaining = max(0, budget - f.size)
            sel = _top(scores[hh, j], ~forced[j], remaining)
            keep = np.sort(np.concatenate([f, sel]))
            kv_num[hh, j] = keep.size
            kv_idx[hh, j, : keep.size] = keep
    return {"kv_num_blocks": kv_num, "kv_indices": kv_idx, "scores": scores, "forced": forced,
            "budget": budget}


def selection_margin(scores: np.ndarray, candidates: np.ndarray, count: int) -> float:
    """Gap between the count-th and (count+1)-th best candidate score (inf if no cut)."""

    vals = np.sort(scores[candidates])[::-1]
    if count <= 0 or count >= vals.size:
        return float("inf")
    return float(vals[count - 1] - vals[count])


def kept_fraction(kv_num_blocks: np.ndarray, total_kv_blocks: int) -> float:
    return float(kv_num_blocks.sum()) / (kv_num_blocks.size * total_kv_blocks)


__all__ = [
    "block_means",
    "block_scores",
    "composite_mask",
    "dynamic_history_mask",
    "kept_fraction",
    "selection_margin",
]
