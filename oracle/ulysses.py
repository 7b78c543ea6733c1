"""Ulysses head<->sequence exchange oracle: every rank emulated on one host (test only).

Restates the data movement of ``merged_qkv_sequence_to_heads`` and ``heads_to_sequence``
(T/distributed/ulysses.py:10-55, 103-132; with FL2AV's zero-padded head shards when the heads
do not divide by the world, F/distributed/ulysses.py:107-110, 150-156, 193-251): the send layout each rank builds, the
``all_to_all_single`` exchange (chunk r of rank s's send buffer lands as chunk s of rank
r's receive buffer) and the receive-side reshape. Pure index work, compared bit for bit.
"""

from __future__ import annotations

import numpy as np


def merged_qkv_sequence_to_heads(merged: list[np.ndarray], num_heads: int,
                                 head_dim: int) -> list[tuple[np.ndarray, np.ndarray, np.ndarray]]:
    """Per-rank merged [T, 3*H*d] -> per-rank (q, k, v) [W*T, ceil(H/W), d]."""

    world = len(merged)
    tokens = merged[0].shape[0]
    # heads not divisible by the world: every rank gets ceil(H/W) heads, the missing ones zero
    # (F/distributed/ulysses.py:218-222)
    hl = -(-num_heads // world)
    padded = [np.concatenate([m.reshape(tokens, 3, num_heads, head_dim),
                              np.zeros((tokens, 3, world * hl - num_heads, head_dim), m.dtype)],
                             axis=2) for m in merged]
    send = [m.reshape(tokens, 3, world, hl, head_dim).transpose(2, 1, 0, 3, 4) for m in padded]
    out = []
    for r in range(world):
        recv = np.stack([send[s][r] for s in range(world)])             # [W(src), 3, T, Hl, d]
        x = recv.transpose(1, 0, 2, 3, 4).reshape(3, world * tokens, hl, head_dim)
        out.append((x[0], x[1], x[2]))
    return out


def heads_to_sequence(values: list[np.ndarray], num_heads: int | None = None) -> list[np.ndarray]:
    """Per-rank [W*T, Hl, d] (head shard r) -> per-rank [T, W*Hl, d] (sequence shard r), or
    its first ``num_heads`` heads (dropping the zero padding, F/distributed/ulysses.py:150-156)."""

    world = len(values)
    rows, hl, d = values[0].shape
    tokens = rows // world
    send = [v.reshape(world, tokens, hl, d) for v in values]
    out = []
    for r in range(world):
        recv = np.stack([send[s][r] for s in range(world)])             # [W(head shard), T, Hl, d]
        full = recv.transpose(1, 0, 2, 3).reshape(tokens, world * hl, d)
        out.append(full if num_heads is None else full[:, :num_heads])
    return out


__all__ = ["heads_to_sequence", "merged_qkv_sequence_to_heads"]
