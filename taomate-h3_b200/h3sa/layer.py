"""The attention part of one DiT layer call, composed from the h3sa drop-ins.

``attention_from_projection`` is the stretch of ``MiniMaxH3Attention.forward``
(T/model/layers.py:351-443) between the QKV projection and the output projection, with the
reference's own order of operations:

    merged QKV [T, 3*H*d]  --fused_qkv_qk_norm_rope_ (in place)-->
    --merged_qkv_sequence_to_heads--> q, k, v [W*T, H/W, d]
    --streaming hook (cache append + attention)--> O [W*T, H/W, d]
    --heads_to_sequence--> [T, H, d] -> [T, H*d] (the out_proj input)

With ``exchange=None`` the two Ulysses steps are the NCCL drop-ins of ``h3sa.ulysses`` (the
reference's structure). With a ``PeerUlysses`` they are stores over NVLink: the QKV shard is
scattered into every owner's q/k/v planes by one kernel, and the attention epilogue stores
each output row into the sequence shard of the rank that owns it.
"""

from __future__ import annotations

from typing import Sequence

import torch

from . import _lib
from .kernels import HEAD_DIM
from .peer import PeerBarrier, PeerBuffer, scatter_qkv
from .prologue import fused_qkv_qk_norm_rope_
from .ulysses import ParallelContext, heads_to_sequence, merged_qkv_sequence_to_heads


class PeerUlysses:
    """Both Ulysses exchanges of a layer call as peer stores over NVLink, for one node.

    Collective to construct (every rank of ``group`` with the same sizes). Holds this rank's
    q/k/v planes ``[3, W*T, H/W, d]`` and output shard ``[T, H, d]``, mapped by every rank,
    and a peer barrier whose waits give up after ``timeout_s`` (reported in
    ``device_error``). ``T`` is the per-rank sequence shard, as in the reference.
    """

    def __init__(self, tokens: int, num_heads: int, head_dim: int = HEAD_DIM, group=None, *,
                 device_error: torch.Tensor | None = None, timeout_s: float = 2.0) -> None:
        import torch.distributed as dist

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_heads % self.world:
            raise ValueError("merged QKV heads are not divisible by Ulysses")
        self.tokens, self.num_heads, self.head_dim = int(tokens), int(num_heads), int(head_dim)
        self.local_heads = num_heads // self.world
        self.qkv = PeerBuffer((3, self.world * tokens, self.local_heads, head_dim), group)
        self.out = PeerBuffer((tokens, num_heads, head_dim), group)
        self.barrier = PeerBarrier(group, device_error=device_error, timeout_s=timeout_s)

    def sequence_to_heads(self, merged: torch.Tensor) -> tuple[torch.Tensor, ...]:
        """This rank's post-prologue merged shard -> the attention-ready q, k, v of its heads
        (views of its planes, valid once every rank has scattered: the barrier)."""

        if tuple(merged.shape) != (self.tokens, 3 * self.num_heads * self.head_dim):
            raise ValueError("merged QKV shard does not match the exchange's sizes")
        scatter_qkv(merged, self.qkv, num_heads=self.num_heads, head_dim=self.head_dim)
        self.barrier()
        return tuple(self.qkv.tensor.unbind(0))

    def store_output_rows(self, out: torch.Tensor) -> None:
        """Attention output ``[W*T, H/W, d]`` of this rank's heads -> every owner's sequence
        shard, one strided row copy per owner (used when the attention epilogue could not
        store the rows itself). The caller then runs ``finish``."""

        rows, hl, d = (int(s) for s in out.shape)
        if rows != self.world * self.tokens or hl != self.local_heads or d != self.head_dim:
            raise ValueError("attention output does not match the exchange's sizes")
        if not out.is_contiguous() or out.dtype != torch.bfloat16:
            raise ValueError("attention output must be contiguous bf16")
        import ctypes

        rb = d * 2
        dims = (ctypes.c_int64 * 4)(self.tokens, hl, 1, 1)
        src_strides = (ctypes.c_int64 * 4)(hl * rb, rb, 0, 0)
        dst_strides = (ctypes.c_int64 * 4)(self.num_heads * rb, rb, 0, 0)
        for owner in range(self.world):
            src = out.data_ptr() + owner * self.tokens * hl * rb
            dst = self.out.addresses[owner] + self.rank * hl * rb
            _lib.call("h3sa_permute_rows", src, dst, dims, src_strides, dst_strides, rb,
                      _lib.stream_handle(None))

    def finish(self) -> torch.Tensor:
        """Wait for every rank's output stores; returns this rank's ``[T, H, d]`` shard."""

        self.barrier()
        return self.out.tensor

    def close(self) -> None:
        self.barrier.close()
        self.out.close()
        self.qkv.close()


def attention_from_projection(
    qkv: torch.Tensor,
    *,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    rope_cache: tuple[torch.Tensor, torch.Tensor] | None,
    eps: float,
    num_heads: int,
    head_dim: int,
    hook,
    attention: object,
    layer_name: str,
    token_tags: torch.Tensor,
    commit_mask: torch.Tensor,
    cu_seqlens_host: Sequence[int],
    context: ParallelContext | None = None,
    exchange: PeerUlysses | None = None,
) -> torch.Tensor:
    """QKV projection output ``[T, 3*H*d]`` (this rank's sequence shard, bf16, modified in
    place by the prologue) -> the out_proj input ``[T, H*d]``.

    ``H`` is the heads of this TP rank; Ulysses runs when ``context`` has a world above one
    (NCCL drop-ins) or when ``exchange`` is given (peer stores). ``token_tags``,
    ``commit_mask`` and ``cu_seqlens_host`` describe the full post-Ulysses sequence, as the
    reference hook receives them (T/model/layers.py:414-431).
    """

    tokens = int(qkv.shape[0])
    if rope_cache is not None:
        cos_sin_cache, positions = rope_cache
        fused_qkv_qk_norm_rope_(qkv, q_weight, k_weight, cos_sin_cache, positions, eps)
    ulysses = exchange is not None or (context is not None and context.ulysses_world_size > 1)
    if exchange is not None:
        q, k, v = exchange.sequence_to_heads(qkv)
    elif ulysses:
        q, k, v = merged_qkv_sequence_to_heads(qkv, num_heads=num_heads, head_dim=head_dim,
                                               context=context)
    else:
        q, k, v = qkv.view(tokens, 3, num_heads, head_dim).unbind(1)
    if exchange is not None:
        hook.output_exchange = exchange
        try:
            output = hook(attention=attention, layer_name=layer_name, query=q, key=k, value=v,
                          token_tags=token_tags, commit_mask=commit_mask,
                          cu_seqlens_host=cu_seqlens_host)
        finally:
            hook.output_exchange = None
        if not hook.last_output_exchanged:
            exchange.store_output_rows(output)
        output = exchange.finish()
    else:
        output = hook(attention=attention, layer_name=layer_name, query=q, key=k, value=v,
                      token_tags=token_tags, commit_mask=commit_mask,
                      cu_seqlens_host=cu_seqlens_host)
        if ulysses:
            output = heads_to_sequence(output, context=context, num_heads=num_heads)
    return output.reshape(tokens, num_heads * head_dim)


__all__ = ["PeerUlysses", "attention_from_projection"]
