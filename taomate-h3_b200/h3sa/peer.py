"""Peer buffers and the fused Ulysses exchanges over NVLink (one process per GPU, one node).

The reference exchanges Ulysses shards with ``torch.distributed.all_to_all_single`` plus a
layout copy on each side (``T/distributed/ulysses.py:10-132``). Here every rank maps every
other rank's exchange buffers through CUDA IPC once, and the kernels store across NVLink
directly: ``scatter_qkv`` writes this rank's rows of every head into the attention-ready q/k/v
planes of the rank owning the head; ``attention_fwd_scatter`` writes each output row into the
sequence shard of the rank owning the row. A ``barrier`` (a one-element all-reduce, ordered on
the stream) separates the writers from the readers.
"""

from __future__ import annotations

import ctypes
import math
from typing import Sequence

import torch

from . import _lib
from ._lib import call, ptr, stream_handle
from .kernels import PAGE_ROWS, AttentionProblem, _problems, _require_cuda

_IPC_HANDLE_BYTES = 64


class _CudaArray:
    """Minimal ``__cuda_array_interface__`` owner so torch can wrap a raw allocation."""

    def __init__(self, address: int, shape: tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (address, False), "version": 3,
                                         "strides": None}


class PeerBuffer:
    """A bf16 device buffer of the same shape on every rank of ``group``, mapped by all.

    ``tensor`` is this rank's buffer; ``peer_table`` is an int64 device tensor holding the
    address of every rank's buffer as mapped in this process (its own at index ``rank``).
    Collective: every rank of the group constructs it with the same shape.
    """

    def __init__(self, shape: Sequence[int], group=None) -> None:
        import torch.distributed as dist

        self.shape = tuple(int(s) for s in shape)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        nbytes = math.prod(self.shape) * 2
        addr = ctypes.c_void_p()
        call("h3sa_peer_alloc", ctypes.c_size_t(nbytes), ctypes.byref(addr))
        self._local = int(addr.value)
        self._opened: list[int] = []
        self._owner = _CudaArray(self._local, self.shape, "<i2")
        self.tensor = torch.as_tensor(self._owner, device="cuda").view(torch.bfloat16)
        handle = (ctypes.c_char * _IPC_HANDLE_BYTES)()
        call("h3sa_ipc_handle", self._local, handle)
        handles: list[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        addresses = []
        for r, h in enumerate(handles):
            if r == self.rank:
                addresses.append(self._local)
                continue
            opened = ctypes.c_void_p()
            buf = (ctypes.c_char * _IPC_HANDLE_BYTES).from_buffer_copy(h)
            call("h3sa_ipc_open", buf, ctypes.byref(opened))
            self._opened.append(int(opened.value))
            addresses.append(int(opened.value))
        self.addresses = addresses  # host copy of peer_table
        self.peer_table = torch.tensor(addresses, dtype=torch.int64, device="cuda")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective in practice: peers
        must be done with this rank's buffer)."""

        for a in self._opened:
            _lib.LIB.h3sa_ipc_close(a)
        self._opened = []
        if self._local:
            del self.tensor
            _lib.LIB.h3sa_peer_free(self._local)
            self._local = 0


class LocalBuffer:
    """One rank's tensor in the form the peer kernels take (``peer_table`` of one address,
    world 1): runs the fused exchange kernels on a single GPU, where every row is local."""

    def __init__(self, tensor: torch.Tensor) -> None:
        if not tensor.is_cuda or not tensor.is_contiguous():
            raise ValueError("LocalBuffer needs a contiguous CUDA tensor")
        self.tensor = tensor
        self.shape = tuple(int(s) for s in tensor.shape)
        self.world, self.rank = 1, 0
        self.addresses = [tensor.data_ptr()]
        self.peer_table = torch.tensor(self.addresses, dtype=torch.int64, device=tensor.device)

    def close(self) -> None:
        self.peer_table = None


class PeerBarrier:
    """Barrier of the group's ranks over peer memory (``h3sa_peer_barrier``), ordered on the
    stream like a kernel: a few microseconds over NVLink instead of a NCCL all-reduce.
    Collective to construct; every rank then calls it the same number of times."""

    def __init__(self, group=None, device_error: torch.Tensor | None = None,
                 timeout_s: float = 2.0) -> None:
        import torch.distributed as dist

        if not 0.0 < timeout_s <= 60.0:
            raise ValueError("peer barrier wait limit must be in (0, 60] seconds")
        self.flags = PeerBuffer((2 * dist.get_world_size(group),), group)  # uint32 per rank
        self.flags.tensor.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=group)
        self.epoch = 0
        self.err = device_error
        self.limit_ns = int(timeout_s * 1e9)

    def __call__(self, stream: torch.cuda.Stream | None = None) -> None:
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        call("h3sa_peer_barrier_limit", ptr(self.flags.peer_table), self.flags.world,
             self.flags.rank, ctypes.c_uint32(self.epoch), ctypes.c_int64(self.limit_ns),
             ptr(self.err), stream_handle(stream))

    def close(self) -> None:
        self.flags.close()


class PeerGroupMax:
    """Maximum over the group's ranks of a small vector of non-negative int32 words, over peer
    memory: each rank stores its words into its slot of every rank's slot array
    (``h3sa_publish_words``), one peer barrier, and every rank then holds all ranks' words
    (the consumer takes the maximum). Two slot sets alternate, so a set is rewritten only
    after every rank has passed the barrier of the call in between. Collective to construct."""

    def __init__(self, count: int, group=None, device_error: torch.Tensor | None = None) -> None:
        import torch.distributed as dist

        self.count = int(count)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.slots = PeerBuffer((2, self.world, 2 * self.count), group)  # int32 words
        self.slots.tensor.zero_()
        self.barrier = PeerBarrier(group, device_error=device_error)
        set_bytes = self.world * self.count * 4
        self._tables = [torch.tensor([a + s * set_bytes for a in self.slots.addresses],
                                     dtype=torch.int64, device="cuda") for s in range(2)]
        self._calls = 0

    def __call__(self, words: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """int32 ``[world * count]``: every rank's words (rank-major), once all have arrived."""

        if words.dtype != torch.int32 or words.numel() != self.count or not words.is_cuda:
            raise ValueError(f"PeerGroupMax takes {self.count} int32 CUDA words")
        s = self._calls & 1
        self._calls += 1
        call("h3sa_publish_words", ptr(words), ptr(self._tables[s]), self.world, self.rank,
             self.count, stream_handle(stream))
        self.barrier(stream)
        return self.slots.tensor[s].view(torch.int32).reshape(-1)

    def close(self) -> None:
        self.barrier.close()
        self.slots.close()


def barrier(group=None, flag: torch.Tensor | None = None) -> None:
    """Stream-ordered barrier: a one-element all-reduce. Kernels enqueued after it on any rank
    start after every rank's kernels enqueued before it have finished."""

    import torch.distributed as dist

    t = flag if flag is not None else torch.zeros(1, dtype=torch.float32, device="cuda")
    dist.all_reduce(t, group=group)


def scatter_qkv(merged: torch.Tensor, qkv: PeerBuffer, *, num_heads: int, head_dim: int = 128,
                stream: torch.cuda.Stream | None = None) -> None:
    """Sequence -> heads: this rank's post-prologue shard ``[T, 3 * H * d]`` (or
    ``[T, 3, H, d]``) stored into every owner rank's ``[3, W * T, H / W, d]`` planes."""

    _require_cuda(merged)
    if merged.dtype != torch.bfloat16 or not merged.is_contiguous():
        raise ValueError("scatter_qkv expects a contiguous bf16 merged QKV shard")
    tokens = int(merged.shape[0])
    world = qkv.world
    if num_heads % world:
        raise ValueError(f"num_heads={num_heads} must be divisible by Ulysses world size {world}")
    if merged.numel() != tokens * 3 * num_heads * head_dim:
        raise ValueError("merged QKV shard must hold 3 * num_heads * head_dim values per token")
    if qkv.shape != (3, world * tokens, num_heads // world, head_dim):
        raise ValueError(f"peer q/k/v planes must be [3, {world * tokens}, "
                         f"{num_heads // world}, {head_dim}], got {list(qkv.shape)}")
    call("h3sa_scatter_qkv", ptr(merged), tokens, num_heads, head_dim, world, qkv.rank,
         ptr(qkv.peer_table), stream_handle(stream))


def scatter_qkv_paged(merged: torch.Tensor, q: PeerBuffer, key_pool: PeerBuffer,
                      value_pool: PeerBuffer, page_table: torch.Tensor, *, dst_start: int,
                      num_heads: int, head_dim: int = 128,
                      device_error: torch.Tensor | None = None,
                      stream: torch.cuda.Stream | None = None) -> None:
    """Sequence -> heads with the cache append folded in: this rank's post-prologue shard
    ``[T, 3 * H * d]`` goes to every owner rank's ``[W * T, H / W, d]`` Q plane and, for K and
    V, straight into the owner's paged pools ``[H / W, pages * 128, d]`` at logical rows
    ``dst_start + rank * T + t`` through ``page_table``, which must be the same on every rank
    (the ranks of a Ulysses group commit the same rows)."""

    _require_cuda(merged, page_table, device_error)
    if merged.dtype != torch.bfloat16 or not merged.is_contiguous():
        raise ValueError("scatter_qkv_paged expects a contiguous bf16 merged QKV shard")
    tokens = int(merged.shape[0])
    world = q.world
    if num_heads % world:
        raise ValueError(f"num_heads={num_heads} must be divisible by Ulysses world size {world}")
    if merged.numel() != tokens * 3 * num_heads * head_dim:
        raise ValueError("merged QKV shard must hold 3 * num_heads * head_dim values per token")
    hl = num_heads // world
    if q.shape != (world * tokens, hl, head_dim):
        raise ValueError(f"peer Q plane must be [{world * tokens}, {hl}, {head_dim}], "
                         f"got {list(q.shape)}")
    if key_pool.shape != value_pool.shape or key_pool.shape[0] != hl or key_pool.shape[2] != head_dim \
            or key_pool.shape[1] % PAGE_ROWS:
        raise ValueError(f"peer KV pools must both be [{hl}, pages * {PAGE_ROWS}, {head_dim}]")
    if page_table.dtype != torch.int32:
        raise ValueError("page_table must be int32")
    call("h3sa_scatter_qkv_paged", ptr(merged), tokens, num_heads, head_dim, world, q.rank,
         ptr(q.peer_table), ptr(key_pool.peer_table), ptr(value_pool.peer_table),
         key_pool.shape[1] // PAGE_ROWS, ptr(page_table), int(page_table.numel()), int(dst_start),
         ptr(device_error), stream_handle(stream))


def attention_fwd_scatter(
    query: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    page_table: torch.Tensor,
    problems: Sequence[AttentionProblem],
    softmax_scale: float,
    out: PeerBuffer,
    *,
    kv_num_blocks: torch.Tensor | None = None,
    kv_indices: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Attention whose output rows go straight to the owning rank's sequence shard
    ``out`` (``[T, H, d]`` on every rank): heads -> sequence fused into the store."""

    _require_cuda(query, key_pool, value_pool, page_table, kv_num_blocks, kv_indices)
    rows, heads, head_dim = (int(s) for s in query.shape)
    if query.dtype != torch.bfloat16 or key_pool.dtype != torch.bfloat16:
        raise RuntimeError("attention takes bf16 query and KV pools")
    if key_pool.shape != value_pool.shape or key_pool.ndim != 3 or key_pool.shape[0] != heads \
            or value_pool.dtype != key_pool.dtype:
        raise RuntimeError("KV pools must be [heads, pages*128, head_dim] with matching shapes")
    tokens, heads_total = out.shape[0], out.shape[1]
    if out.shape[2] != head_dim or tokens * out.world < rows:
        raise ValueError("output shard must be [T, H, d] with W * T covering the query rows")
    pool_pages = int(key_pool.shape[1]) // PAGE_ROWS
    q_blocks = stride = 0
    if kv_num_blocks is not None:
        q_blocks = int(kv_num_blocks.shape[-1])
        stride = int(kv_indices.shape[-1])
    call("h3sa_attention_fwd_scatter", ptr(query), rows, heads, head_dim, ptr(key_pool),
         ptr(value_pool), pool_pages, ptr(page_table), int(page_table.numel()),
         _problems(problems), len(problems), float(softmax_scale), ptr(kv_num_blocks),
         ptr(kv_indices), q_blocks, stride, ptr(out.peer_table), out.world, tokens, heads_total,
         out.rank * heads, ptr(device_error), stream_handle(stream))


__all__ = ["LocalBuffer", "PeerBarrier", "PeerBuffer", "PeerGroupMax", "attention_fwd_scatter", "barrier", "scatter_qkv",
           "scatter_qkv_paged"]
