"""Ulysses sequence<->head exchange on NCCL with h3sa layout kernels.

Mirrors T/distributed/ulysses.py:10-139 (same functions, arguments, errors and result
layouts) with FL2AV's head padding (F/distributed/ulysses.py:94-251): when the heads do not
divide by the Ulysses world, every rank receives ceil(H/W) heads and the missing ones are
zero; ``heads_to_sequence(..., num_heads=H)`` drops them again. The permute+contiguous copies the reference wraps around each
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


def build_parallel_context(tp_size: int, ulysses_degree: int, *,
                           backend: str | None = None) -> ParallelContext:
    """This rank's view of a TP x Ulysses layout over the whole world, built as the reference
    runtime builds it (T/runtime/direct.py:169-190): global rank = ulysses_rank * tp_size +
    tp_rank; TP groups are runs of ``tp_size`` consecutive ranks, Ulysses group t holds the
    ranks t, t + tp_size, t + 2 * tp_size, ... (e.g. {t, t+2, t+4, t+6} for TP2 x SP4).
    Collective: every rank creates every group, in the same order."""

    dist = torch.distributed
    world = dist.get_world_size()
    if tp_size <= 0 or ulysses_degree <= 0 or tp_size * ulysses_degree != world:
        raise ValueError(f"TP {tp_size} x Ulysses {ulysses_degree} does not cover world {world}")
    rank = dist.get_rank()
    tp_groups = [dist.new_group(ranks=[u * tp_size + t for t in range(tp_size)], backend=backend)
                 for u in range(ulysses_degree)]
    ulysses_groups = [dist.new_group(ranks=[u * tp_size + t for u in range(ulysses_degree)],
                                     backend=backend)
                      for t in range(tp_size)]
    return ParallelContext(tp_world_size=tp_size, tp_rank=rank % tp_size,
                           ulysses_world_size=ulysses_degree, ulysses_rank=rank // tp_size,
                           tp_group=tp_groups[rank // tp_size],
                           ulysses_group=ulysses_groups[rank % tp_size])

def _require_dist(context: ParallelContext) -> None:
    if not torch.distributed.is_available() or not torch.distributed.is_initialized():
        raise RuntimeError("Ulysses all-to-all requires initialized torch.distributed")
    if context.ulysses_group is None:
        raise RuntimeError("Ulysses process group is absent")


def _tail(t: torch.Tensor, byte_offset: int) -> torch.Tensor:
    """Flat view of a contiguous tensor from ``byte_offset`` on (the permute kernel addresses
    records by byte strides from the view's start)."""

    return t.reshape(-1)[byte_offset // t.element_size():]


def _shards(num_heads: int, world: int) -> tuple[int, int, int]:
    """(heads per rank, ranks whose shard holds only real heads, real heads of the next rank):
    with H % W != 0 every rank gets ceil(H/W) heads and the missing ones are zero padding
    (F/distributed/ulysses.py:218-222)."""

    hl = -(-num_heads // world)
    full = num_heads // hl
    return hl, full, num_heads - full * hl


def pack_qkv_send(merged: torch.Tensor, send: torch.Tensor, *, world: int, num_heads: int,
                  head_dim: int) -> None:
    """merged ``[T, 3, H, d]`` -> send ``[W, 3, T, Hl, d]`` (Hl = ceil(H/W); padded heads
    zero)."""

    tokens = int(merged.shape[0])
    hl, full, rest = _shards(num_heads, world)
    rb = head_dim * merged.element_size()
    if full < world:
        send.zero_()
    # index space (W, 3, T, heads of the shard); strides in bytes
    src = (hl * rb, num_heads * rb, 3 * num_heads * rb, rb)
    dst = (3 * tokens * hl * rb, tokens * hl * rb, hl * rb, rb)
    if full:
        permute_rows(merged, send, (full, 3, tokens, hl), src, dst, rb)
    if rest:
        permute_rows(_tail(merged, full * hl * rb), _tail(send, full * dst[0]),
                     (1, 3, tokens, rest), src, dst, rb)


def unpack_qkv_recv(recv: torch.Tensor, out: torch.Tensor, *, world: int, tokens: int,
                    local_heads: int, head_dim: int) -> None:
    """recv ``[W, 3, T, Hl, d]`` -> out ``[3, W*T, Hl, d]``."""

    rb = head_dim * recv.element_size()
    hl = local_heads
    src = (3 * tokens * hl * rb, tokens * hl * rb, hl * rb, rb)        # (W, 3, T, Hl)
    dst = (tokens * hl * rb, world * tokens * hl * rb, hl * rb, rb)
    permute_rows(recv, out, (world, 3, tokens, hl), src, dst, rb)


def unpack_o_recv(recv: torch.Tensor, out: torch.Tensor, *, world: int, tokens: int,
                  local_heads: int, head_dim: int, num_heads: int | None = None) -> None:
    """recv ``[W, T, Hl, d]`` (head shards) -> out ``[T, H, d]``, H = ``num_heads`` (default
    W*Hl): the zero padding of the last shards is dropped."""

    rb = head_dim * recv.element_size()
    hl = local_heads
    heads = world * hl if num_heads is None else int(num_heads)
    full, rest = heads // hl, heads % hl
    src = (tokens * hl * rb, hl * rb, rb, 0)                            # (W, T, Hl, 1)
    dst = (hl * rb, heads * rb, rb, 0)
    if full:
        permute_rows(recv, out, (full, tokens, hl, 1), src, dst, rb)
    if rest:
        permute_rows(_tail(recv, full * src[0]), _tail(out, full * dst[0]), (1, tokens, rest, 1),
                     src, dst, rb)


def qkv_send_layout(value: torch.Tensor, *, num_heads: int, head_dim: int,
                    world_size: int) -> torch.Tensor:
    """The FL2AV send layout (F/distributed/ulysses_layout.py:26-37): merged QKV
    ``[T, 3 * H * d]`` -> ``[W, 3, T, ceil(H / W), d]`` with the missing heads of the last
    shards zero."""

    tokens = int(value.shape[0])
    hl = -(-num_heads // world_size)
    out = torch.empty(world_size, 3, tokens, hl, head_dim, dtype=value.dtype, device=value.device)
    pack_qkv_send(value.contiguous(), out, world=world_size, num_heads=num_heads,
                  head_dim=head_dim)
    return out


def attention_receive_layout(value: torch.Tensor, *, num_heads: int) -> torch.Tensor:
    """The FL2AV receive layout (F/distributed/ulysses_layout.py:54-60): head shards
    ``[W, T, Hl, d]`` -> ``[T, H, d]``, the zero padding dropped."""

    world, tokens, local, dim = (int(x) for x in value.shape)
    out = torch.empty(tokens, num_heads, dim, dtype=value.dtype, device=value.device)
    unpack_o_recv(value.contiguous(), out, world=world, tokens=tokens, local_heads=local,
                  head_dim=dim, num_heads=num_heads)
    return out


def _all_to_all_swap(value: torch.Tensor, *, world_size: int, group: object,
                     sequence_to_heads: bool, num_heads: int | None = None) -> torch.Tensor:
    """Swap sequence and head shards with one all-to-all (T/distributed/ulysses.py:10-55)."""

    if sequence_to_heads:
        if value.ndim < 3:
            raise ValueError("Ulysses input heads must be divisible by its world size")
        padding = (-int(value.shape[-2])) % world_size
        if padding:  # zero heads up to a multiple of the world (F/distributed/ulysses.py:107-110)
            value = torch.nn.functional.pad(value, (0, 0, 0, padding))
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
    heads = world_size * hl if num_heads is None else int(num_heads)
    out = torch.empty(tokens, heads, d, dtype=value.dtype, device=value.device)
    unpack_o_recv(recv, out, world=world_size, tokens=tokens, local_heads=hl, head_dim=d,
                  num_heads=heads)
    return out


def sequence_to_heads(value: torch.Tensor, *, context: ParallelContext) -> torch.Tensor:
    """Trade Ulysses-local sequence rows for attention heads (F/distributed/ulysses.py:119-127);
    heads are zero-padded to a multiple of the world first."""

    if context.ulysses_world_size == 1:
        return value
    _require_dist(context)
    return _all_to_all_swap(value, world_size=context.ulysses_world_size,
                            group=context.ulysses_group, sequence_to_heads=True)


def heads_to_sequence(value: torch.Tensor, *, context: ParallelContext,
                      num_heads: int | None = None) -> torch.Tensor:
    """Inverse of sequence_to_heads (T/distributed/ulysses.py:77-84); ``num_heads`` drops the
    zero-padded heads of the last shards (F/distributed/ulysses.py:130-156)."""

    _require_dist(context)
    return _all_to_all_swap(value, world_size=context.ulysses_world_size,
                            group=context.ulysses_group, sequence_to_heads=False,
                            num_heads=num_heads)


def packed_qkv_sequence_to_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                                 context: ParallelContext) -> tuple[torch.Tensor, ...]:
    """Fuse Q/K/V into one collective (T/distributed/ulysses.py:87-100)."""

    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("Ulysses packed Q/K/V shapes differ")
    _require_dist(context)
    world = context.ulysses_world_size
    tokens, heads, d = (int(s) for s in q.shape)
    merged = torch.stack((q, k, v), dim=1).reshape(tokens, 3 * heads * d)
    return merged_qkv_sequence_to_heads(merged, num_heads=heads, head_dim=d, context=context)


def merged_qkv_sequence_to_heads(value: torch.Tensor, *, num_heads: int, head_dim: int,
                                 context: ParallelContext) -> tuple[torch.Tensor, ...]:
    """Send an already merged QKV allocation through Ulysses (T/distributed/ulysses.py:103-132);
    with H % W != 0 every rank receives ceil(H/W) heads, the missing ones zero
    (F/distributed/ulysses.py:193-251)."""

    world_size = context.ulysses_world_size
    tokens = int(value.shape[0])
    if int(value.shape[-1]) != 3 * num_heads * head_dim:
        raise ValueError("merged QKV width differs")
    packed = value.view(tokens, 3, num_heads, head_dim)
    if world_size == 1:
        return tuple(packed.unbind(dim=1))
    _require_dist(context)
    hl = -(-num_heads // world_size)  # zero-padded shards when H % W != 0
    send = torch.empty(world_size, 3, tokens, hl, head_dim, dtype=value.dtype, device=value.device)
    pack_qkv_send(value.contiguous(), send, world=world_size, num_heads=num_heads, head_dim=head_dim)
    recv = torch.empty_like(send)
    torch.distributed.all_to_all_single(recv, send, group=context.ulysses_group)
    out = torch.empty(3, world_size * tokens, hl, head_dim, dtype=value.dtype, device=value.device)
    unpack_qkv_recv(recv, out, world=world_size, tokens=tokens, local_heads=hl, head_dim=head_dim)
    return tuple(out.unbind(dim=0))


__all__ = [
    "ParallelContext",
    "attention_receive_layout",
    "qkv_send_layout",
    "build_parallel_context",
    "heads_to_sequence",
    "merged_qkv_sequence_to_heads",
    "packed_qkv_sequence_to_heads",
    "sequence_to_heads",
    "pack_qkv_send",
    "unpack_o_recv",
    "unpack_qkv_recv",
]
