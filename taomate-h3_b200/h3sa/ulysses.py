"""Ulysses sequence<->head exchange on NCCL with h3sa layout kernels.

Mirrors T/distributed/ulysses.py:10-139 (same functions, arguments, errors and result
layouts). The permute+contiguous copies the reference wraps around each
``all_to_all_single`` are done by ``h3sa_permute_rows`` (one 16-byte-vectorised pass each);
the exchange itself is NCCL over NVLink through ``torch.distributed``.

Layouts (W = Ulysses world, T = local rows, Hl = heads per rank, d = head_dim):

* ``merged_qkv_sequence_to_heads``: merged ``[T, 3*H*d]`` -> send ``[W, 3, T, Hl, d]``;
  receive ``[W, 3, T, Hl, d]`` -> q, k, v ``[W*T, Hl, d]`` (source shards in rank order).
* ``heads_to_sequence``: ``[W*T, Hl, d]`` is already the send layout ``[W, T, Hl, d]``;
  receive ``[W, T, Hl, d]`` (head shards) -> ``[T, W*Hl, d]``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from .kernels import permute_rows


@dataclass(frozen=True)
class ParallelContext:
    """Explicit rank topology (T/distributed/parallel.py:9-31)."""

    tp_world_size: int
    tp_rank: int
    ulysses_world_size: int
    ulysses_rank: int
    tp_group: Any
    ulysses_group: Any

    def __post_init__(self) -> None:
        for name in ("tp", "ulysses"):
            size = getattr(self, f"{name}_world_size")
            rank = getattr(self, f"{name}_rank")
            if size <= 0 or not 0 <= rank < size:
                raise ValueError(f"invalid {name} topology: world_size={size}, rank={rank}")
        if self.tp_group is None or self.ulysses_group is None:
            raise ValueError("TP and Ulysses process groups are required")


def _require_dist(context: ParallelContext) -> None:
    if not torch.distributed.is_available() or not torch.distributed.is_initialized():
        raise RuntimeError("Ulysses all-to-all requires initialized torch.distributed")
    if context.ulysses_group is None:
        raise RuntimeError("Ulysses process group is absent")


def pack_qkv_send(merged: torch.Tensor, send: torch.Tensor, *, world: int, num_heads: int,
                  head_dim: int) -> None:
    """merged ``[T, 3, W, Hl, d]`` -> send ``[W, 3, T, Hl, d]``."""

    tokens = int(merged.shape[0])
    hl = num_heads // world
    rb = head_dim * merged.element_size()
    # index space (W, 3, T, Hl); strides in bytes
    src = (hl * rb, num_heads * rb, 3 * num_heads * rb, rb)
    dst = (3 * tokens * hl * rb, tokens * hl * rb, hl * rb, rb)
    permute_rows(merged, send, (world, 3, tokens, hl), src, dst, rb)


def unpack_qkv_recv(recv: torch.Tensor, out: torch.Tensor, *, world: int, tokens: int,
                    local_heads: int, head_dim: int) -> None:
    """recv ``[W, 3, T, Hl, d]`` -> out ``[3, W*T, Hl, d]``."""

    rb = head_dim * recv.element_size()
    hl = local_heads
    src = (3 * tokens * hl * rb, tokens * hl * rb, hl * rb, rb)        # (W, 3, T, Hl)
    dst = (tokens * hl * rb, world * tokens * hl * rb, hl * rb, rb)
    permute_rows(recv, out, (world, 3, tokens, hl), src, dst, rb)


def unpack_o_recv(recv: torch.Tensor, out: torch.Tensor, *, world: int, tokens: int,
                  local_heads: int, head_dim: int) -> None:
    """recv ``[W, T, Hl, d]`` (head shards) -> out ``[T, W*Hl, d]``."""

    rb = head_dim * recv.element_size()
    hl = local_heads
    src = (tokens * hl * rb, hl * rb, rb, 0)                            # (W, T, Hl, 1)
    dst = (hl * rb, world * hl * rb, rb, 0)
    permute_rows(recv, out, (world, tokens, hl, 1), src, dst, rb)


def _all_to_all_swap(value: torch.Tensor, *, world_size: int, group: object,
                     sequence_to_heads: bool) -> torch.Tensor:
    """Swap sequence and head shards with one all-to-all (T/distributed/ulysses.py:10-55)."""

    if sequence_to_heads:
        if value.ndim < 3 or int(value.shape[-2]) % world_size:
            raise ValueError("Ulysses input heads must be divisible by its world size")
        if value.ndim != 3:
            packed = value.contiguous()
            lead = packed.shape[:-3]
            flat = packed.reshape(-1, *packed.shape[-3:])
            outs = [_all_to_all_swap(x, world_size=world_size, group=group,
                                     sequence_to_heads=True) for x in flat]
            return torch.stack(outs).reshape(*lead, *outs[0].shape)
        tokens, heads, d = (int(s) for s in value.shape)
        hl = heads // world_size
        src = value.contiguous()
        send = torch.empty(world_size, tokens, hl, d, dtype=value.dtype, device=value.device)
        rb = d * value.element_size()
        permute_rows(src, send, (world_size, tokens, hl, 1),
                     (hl * rb, heads * rb, rb, 0), (tokens * hl * rb, hl * rb, rb, 0), rb)
        recv = torch.empty_like(send)
        torch.distributed.all_to_all_single(recv, send, group=group)
        return recv.view(world_size * tokens, hl, d)
    if value.ndim < 3 or int(value.shape[-3]) % world_size:
        raise ValueError("Ulysses global rows must be divisible by its world size")
    if value.ndim != 3:
        raise ValueError("heads_to_sequence expects [rows, heads, head_dim]")
    rows, hl, d = (int(s) for s in value.shape)
    tokens = rows // world_size
    send = value.contiguous()
    recv = torch.empty_like(send)
    torch.distributed.all_to_all_single(recv, send, group=group)
    out = torch.empty(tokens, world_size * hl, d, dtype=value.dtype, device=value.device)
    unpack_o_recv(recv, out, world=world_size, tokens=tokens, local_heads=hl, head_dim=d)
    return out


def heads_to_sequence(value: torch.Tensor, *, context: ParallelContext) -> torch.Tensor:
    """Inverse of sequence_to_heads (T/distributed/ulysses.py:77-84)."""

    _require_dist(context)
    return _all_to_all_swap(value, world_size=context.ulysses_world_size,
                            group=context.ulysses_group, sequence_to_heads=False)


def packed_qkv_sequence_to_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                                 context: ParallelContext) -> tuple[torch.Tensor, ...]:
    """Fuse Q/K/V into one collective (T/distributed/ulysses.py:87-100)."""

    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("Ulysses packed Q/K/V shapes differ")
    _require_dist(context)
    world = context.ulysses_world_size
    tokens, heads, d = (int(s) for s in q.shape)
    if heads % world:
        raise ValueError("Ulysses input heads must be divisible by its world size")
    merged = torch.stack((q, k, v), dim=1).reshape(tokens, 3 * heads * d)
    return merged_qkv_sequence_to_heads(merged, num_heads=heads, head_dim=d, context=context)


def merged_qkv_sequence_to_heads(value: torch.Tensor, *, num_heads: int, head_dim: int,
                                 context: ParallelContext) -> tuple[torch.Tensor, ...]:
    """Send an already merged QKV allocation through Ulysses (T/distributed/ulysses.py:103-132)."""

    world_size = context.ulysses_world_size
    tokens = int(value.shape[0])
    if int(value.shape[-1]) != 3 * num_heads * head_dim:
        raise ValueError("merged QKV width differs")
    packed = value.view(tokens, 3, num_heads, head_dim)
    if world_size == 1:
        return tuple(packed.unbind(dim=1))
    if num_heads % world_size:
        raise ValueError("merged QKV heads are not divisible by Ulysses")
    _require_dist(context)
    hl = num_heads // world_size
    send = torch.empty(world_size, 3, tokens, hl, head_dim, dtype=value.dtype, device=value.device)
    pack_qkv_send(value.contiguous(), send, world=world_size, num_heads=num_heads, head_dim=head_dim)
    recv = torch.empty_like(send)
    torch.distributed.all_to_all_single(recv, send, group=context.ulysses_group)
    out = torch.empty(3, world_size * tokens, hl, head_dim, dtype=value.dtype, device=value.device)
    unpack_qkv_recv(recv, out, world=world_size, tokens=tokens, local_heads=hl, head_dim=head_dim)
    return tuple(out.unbind(dim=0))


__all__ = [
    "ParallelContext",
    "heads_to_sequence",
    "merged_qkv_sequence_to_heads",
    "packed_qkv_sequence_to_heads",
    "pack_qkv_send",
    "unpack_o_recv",
    "unpack_qkv_recv",
]
