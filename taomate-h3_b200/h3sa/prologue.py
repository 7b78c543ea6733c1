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


__all__ = ["fused_qkv_qk_norm_rope_", "qkv_norm_rope_pack"]
