"""QK-RMSNorm + RoPE prologue on merged QKV (drop-in for the reference's fused prologue).

``fused_qkv_qk_norm_rope_`` mirrors T/inference/fused_kernels.py:805-855 (same arguments,
in-place result and ValueError messages) on the sm_100a kernel; ``qkv_norm_rope_pack`` fuses
the same prologue with the Ulysses send-side permute so the merged projection is read once
and written once.
"""

from __future__ import annotations

import torch

from ._lib import call, ptr, stream_handle


def _check(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
           cos_sin_cache: torch.Tensor, positions: torch.Tensor) -> tuple[int, int, int, torch.Tensor, torch.Tensor]:
    if qkv.ndim != 2 or not qkv.is_contiguous():
        raise ValueError("fused QKV preprocessing requires contiguous [tokens, width]")
    if q_weight.shape != k_weight.shape or q_weight.ndim != 1:
        raise ValueError("fused QKV Q/K norm weights differ")
    if any(t.dtype != torch.bfloat16 for t in (qkv, q_weight, k_weight, cos_sin_cache)):
        raise ValueError("fused QKV preprocessing requires BF16 tensors")
    tokens = int(qkv.shape[0])
    head_dim = int(q_weight.numel())
    projection_width, remainder = divmod(int(qkv.shape[-1]), 3)
    heads, head_remainder = divmod(projection_width, head_dim)
    if remainder or head_remainder:
        raise ValueError("fused QKV width does not contain three complete projections")
    positions = positions.reshape(-1).to(torch.int64).contiguous()
    if int(positions.numel()) != tokens:
        raise ValueError("fused QKV RoPE positions do not cover every token")
    cache = cos_sin_cache.contiguous()
    rotary = int(cache.shape[-1])
    if cache.ndim != 2 or rotary > head_dim or rotary % 2:
        raise ValueError("fused QKV RoPE cache span is invalid")
    for t in (qkv, q_weight, k_weight, cache, positions):
        if not t.is_cuda:
            raise RuntimeError("h3sa kernels require CUDA tensors")
    return tokens, heads, head_dim, cache, positions


def fused_qkv_qk_norm_rope_(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                            cos_sin_cache: torch.Tensor, positions: torch.Tensor,
                            eps: float) -> torch.Tensor:
    """Normalise and rotate Q/K in place in a merged bf16 QKV projection; V untouched."""

    tokens, heads, head_dim, cache, positions = _check(qkv, q_weight, k_weight, cos_sin_cache, positions)
    call("h3sa_qkv_norm_rope", ptr(qkv), ptr(q_weight.contiguous()), ptr(k_weight.contiguous()),
         ptr(cache), int(cache.shape[0]), int(cache.shape[1]), ptr(positions), tokens, heads,
         head_dim, float(eps), None, stream_handle(None))
    return qkv


def fused_qk_norm_rope(value: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor,
                       sin: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm + rotate-half RoPE of one of Q or K, out of place (T/inference/fused_kernels.py:
    775-802, used by the processor when the merged prologue is off, T/model/layers.py:390-398).

    ``value`` ``[T, H, d]`` bf16 (any strides), ``cos`` / ``sin`` ``[T, rotary]`` per token
    with duplicated halves, as the processor builds them from the cos/sin cache. Runs the
    merged prologue kernel (same arithmetic and bf16 rounding points) on a ``[T, 3, H, d]``
    staging copy whose Q plane is ``value``; returns a contiguous ``[T, H, d]`` bf16 tensor."""

    if value.ndim != 3:
        raise ValueError("SOL QKNorm/RoPE takes [tokens, heads, head_dim]")
    tokens, heads, head_dim = (int(x) for x in value.shape)
    rotary = int(cos.shape[-1])
    if rotary > head_dim or rotary % 2:
        raise ValueError("SOL QKNorm/RoPE requires an even rotary span within a head")
    if tuple(cos.shape) != (tokens, rotary) or tuple(sin.shape) != (tokens, rotary):
        raise ValueError("SOL QKNorm/RoPE needs one cos/sin row per token")
    half = rotary // 2
    merged = torch.zeros(tokens, 3, heads, head_dim, dtype=torch.bfloat16, device=value.device)
    merged[:, 0].copy_(value)
    cache = torch.cat((cos[:, :half], sin[:, :half]), dim=-1).to(torch.bfloat16).contiguous()
    positions = torch.arange(tokens, device=value.device)
    w = weight.to(torch.bfloat16).contiguous()
    fused_qkv_qk_norm_rope_(merged.view(tokens, 3 * heads * head_dim), w, w, cache, positions, eps)
    return merged[:, 0].contiguous()


def qkv_norm_rope_pack(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                       cos_sin_cache: torch.Tensor, positions: torch.Tensor, eps: float, *,
                       world: int, send: torch.Tensor | None = None) -> torch.Tensor:
    """Prologue written into the Ulysses send buffer ``[world, 3, tokens, heads/world, d]``."""

    tokens, heads, head_dim, cache, positions = _check(qkv, q_weight, k_weight, cos_sin_cache, positions)
    if heads % world:
        raise ValueError("merged QKV heads are not divisible by Ulysses")
    if send is None:
        send = torch.empty(world, 3, tokens, heads // world, head_dim, dtype=qkv.dtype,
                           device=qkv.device)
    call("h3sa_qkv_norm_rope_pack", ptr(qkv), ptr(send), ptr(q_weight.contiguous()),
         ptr(k_weight.contiguous()), ptr(cache), int(cache.shape[0]), int(cache.shape[1]),
         ptr(positions), tokens, heads, head_dim, int(world), float(eps), None,
         stream_handle(None))
    return send




def qkv_norm_rope_scatter_paged(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                                cos_sin_cache: torch.Tensor, positions: torch.Tensor, eps: float,
                                *, q, key_pool, value_pool, page_table: torch.Tensor,
                                dst_start: int, device_error: torch.Tensor | None = None,
                                stream: torch.cuda.Stream | None = None) -> None:
    """The layer prologue fused with the sequence -> heads exchange and the cache append.

    ``qkv`` is this rank's raw merged projection ``[T, 3*H*d]`` (read only). ``q``,
    ``key_pool`` and ``value_pool`` are ``h3sa.peer.PeerBuffer`` objects (or
    ``h3sa.peer.LocalBuffer`` for one GPU): the all-rank Q plane ``[W*T, H/W, d]`` and the
    paged pools ``[H/W, pages*128, d]`` of every rank. Q rows land in their owners' planes and
    K/V rows in their owners' caches at logical rows ``dst_start + rank*T + t``.
    """

    from .kernels import PAGE_ROWS

    tokens, heads, head_dim, cache, positions = _check(qkv, q_weight, k_weight, cos_sin_cache,
                                                       positions)
    world, rank = q.world, q.rank
    if heads % world:
        raise ValueError("merged QKV heads are not divisible by Ulysses")
    hl = heads // world
    if tuple(q.shape) != (world * tokens, hl, head_dim):
        raise ValueError(f"Q plane must be [{world * tokens}, {hl}, {head_dim}], got {list(q.shape)}")
    if (tuple(key_pool.shape) != tuple(value_pool.shape) or len(key_pool.shape) != 3
            or key_pool.shape[0] != hl or key_pool.shape[2] != head_dim
            or key_pool.shape[1] % PAGE_ROWS):
        raise ValueError(f"KV pools must both be [{hl}, pages * {PAGE_ROWS}, {head_dim}]")
    if key_pool.world != world or value_pool.world != world:
        raise ValueError("Q plane and KV pools must span the same ranks")
    if page_table.dtype != torch.int32 or not page_table.is_cuda:
        raise ValueError("page_table must be an int32 CUDA tensor")
    call("h3sa_qkv_norm_rope_scatter_paged", ptr(qkv), ptr(q_weight.contiguous()),
         ptr(k_weight.contiguous()), ptr(cache), int(cache.shape[0]), int(cache.shape[1]),
         ptr(positions), tokens, heads, head_dim, world, rank, ptr(q.peer_table),
         ptr(key_pool.peer_table), ptr(value_pool.peer_table), int(key_pool.shape[1]) // PAGE_ROWS,
         ptr(page_table), int(page_table.numel()), int(dst_start), float(eps), ptr(device_error),
         stream_handle(stream))


def _e4m3_shape(buf) -> tuple[int, ...]:
    """Shape of a peer / local buffer seen as e4m3 (bf16 buffers hold two e4m3 bytes each)."""

    t = buf.tensor
    if t.dtype == torch.float8_e4m3fn:
        return tuple(int(x) for x in t.shape)
    if t.dtype == torch.bfloat16:
        return tuple(int(x) for x in t.shape[:-1]) + (2 * int(t.shape[-1]),)
    raise ValueError("e4m3 destinations must be e4m3 (or bf16-typed byte) buffers")


def qkv_norm_rope_scatter_fp8(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                              cos_sin_cache: torch.Tensor, positions: torch.Tensor, eps: float,
                              *, q8, key_pool8, value_pool8, page_table8: torch.Tensor,
                              dst8_start: int, amax_rows: torch.Tensor | None = None,
                              group=None, peer_max=None, q=None, key_pool=None,
                              value_pool=None, page_table: torch.Tensor | None = None,
                              dst_start: int = 0, bf16_unflagged_only: bool = False,
                              device_error: torch.Tensor | None = None,
                              stream: torch.cuda.Stream | None = None
                              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The fused RMSNorm + RoPE + per-head e4m3 prologue writing Q and the chunk's K/V part
    straight into the owners' e4m3 plane and paged caches (two passes: amax, then quantise and
    store; with more than one rank the maxima are reduced over ``group`` in between).

    ``q8`` / ``key_pool8`` / ``value_pool8``: ``h3sa.peer.PeerBuffer`` / ``LocalBuffer`` of the
    e4m3 Q plane ``[W*T, H/W, 128]`` and pools ``[H/W, pages * 128, 128]``. ``amax_rows``:
    uint8 ``[T]`` flags of the rows the scales cover (None: all). With ``q`` (the bf16 plane)
    and ``key_pool`` / ``value_pool`` (+ ``page_table``, ``dst_start``) the bf16 rows are stored
    too (only the unflagged ones with ``bf16_unflagged_only``). With more than one rank the
    maxima are reduced over ``group`` by NCCL, or over peer memory with ``peer_max`` (an
    ``h3sa.peer.PeerGroupMax`` of 3 * heads words). Returns this rank's fp32 ``[H/W]`` Q, K
    and V scales."""

    from .kernels import PAGE_ROWS

    tokens, heads, head_dim, cache, positions = _check(qkv, q_weight, k_weight, cos_sin_cache,
                                                       positions)
    world, rank = q8.world, q8.rank
    if heads % world:
        raise ValueError("merged QKV heads are not divisible by Ulysses")
    hl = heads // world
    if _e4m3_shape(q8) != (world * tokens, hl, head_dim):
        raise ValueError(f"e4m3 Q plane must be [{world * tokens}, {hl}, {head_dim}]")
    ks, vs = _e4m3_shape(key_pool8), _e4m3_shape(value_pool8)
    if ks != vs or len(ks) != 3 or ks[0] != hl or ks[2] != head_dim or ks[1] % PAGE_ROWS:
        raise ValueError(f"e4m3 KV pools must both be [{hl}, pages * {PAGE_ROWS}, {head_dim}]")
    if key_pool8.world != world or value_pool8.world != world:
        raise ValueError("Q plane and KV pools must span the same ranks")
    if page_table8.dtype != torch.int32 or not page_table8.is_cuda:
        raise ValueError("page_table8 must be an int32 CUDA tensor")
    if amax_rows is not None and (amax_rows.dtype != torch.uint8 or amax_rows.numel() != tokens
                                  or not amax_rows.is_cuda):
        raise ValueError("amax_rows must be a uint8 CUDA tensor with one flag per token")
    keep = key_pool is not None
    if keep:
        if value_pool is None or page_table is None:
            raise ValueError("bf16 K/V destinations need both pools and their page table")
        if (tuple(key_pool.shape) != tuple(value_pool.shape) or key_pool.shape[0] != hl
                or key_pool.shape[1] % PAGE_ROWS or key_pool.world != world):
            raise ValueError(f"bf16 KV pools must both be [{hl}, pages * {PAGE_ROWS}, {head_dim}]")
    if q is not None and (tuple(q.shape) != (world * tokens, hl, head_dim) or q.world != world):
        raise ValueError(f"bf16 Q plane must be [{world * tokens}, {hl}, {head_dim}]")
    if bf16_unflagged_only and amax_rows is None:
        raise ValueError("bf16_unflagged_only needs amax_rows")
    if peer_max is not None and (peer_max.count != 3 * heads or peer_max.world != world):
        raise ValueError(f"peer_max must carry {3 * heads} words over {world} ranks")
    dev = qkv.device
    amax = torch.empty(3 * heads, dtype=torch.int32, device=dev)
    call("h3sa_qkv_norm_rope_amax", ptr(qkv), ptr(q_weight.contiguous()),
         ptr(k_weight.contiguous()), ptr(cache), int(cache.shape[0]), int(cache.shape[1]),
         ptr(positions), tokens, heads, head_dim, ptr(amax_rows), ptr(amax), float(eps),
         ptr(device_error), stream_handle(stream))
    sets, words = 1, amax
    if world > 1 and peer_max is not None:
        words, sets = peer_max(amax), world
    elif world > 1:  # non-negative floats order like their bits
        torch.distributed.all_reduce(amax, op=torch.distributed.ReduceOp.MAX, group=group)
    scales = torch.empty(3, hl, dtype=torch.float32, device=dev)
    call("h3sa_qkv_norm_rope_scatter_fp8", ptr(qkv), ptr(q_weight.contiguous()),
         ptr(k_weight.contiguous()), ptr(cache), int(cache.shape[0]), int(cache.shape[1]),
         ptr(positions), tokens, heads, head_dim, world, rank, ptr(words), sets, ptr(amax_rows),
         1 if bf16_unflagged_only else 0, ptr(q8.peer_table),
         ptr(key_pool8.peer_table), ptr(value_pool8.peer_table), ks[1] // PAGE_ROWS,
         ptr(page_table8), int(page_table8.numel()), int(dst8_start), ptr(scales[0]),
         ptr(scales[1]), ptr(scales[2]), ptr(q.peer_table) if q is not None else None,
         ptr(key_pool.peer_table) if keep else None, ptr(value_pool.peer_table) if keep else None,
         int(key_pool.shape[1]) // PAGE_ROWS if keep else 0, ptr(page_table),
         int(page_table.numel()) if keep else 0, int(dst_start), float(eps), ptr(device_error),
         stream_handle(stream))
    return scales[0], scales[1], scales[2]


__all__ = ["fused_qk_norm_rope", "fused_qkv_qk_norm_rope_", "qkv_norm_rope_pack", "qkv_norm_rope_scatter_fp8",
           "qkv_norm_rope_scatter_paged"]
