"""The attention's row-parallel out_proj with its TP all-reduce, on the sm_100a kernels.

The reference ends the attention with ``heads_to_sequence`` and ``out_proj``, a
``RowParallelLinear`` (T/model/layers.py:441-443): each TP rank multiplies its slice of the
inner dimension, ``[T, inner / TP] @ W_local^T``, and the partial outputs are summed with a NCCL
all-reduce over the TP group (T/distributed/linear.py:142-198, collectives.py:51-55). Here the
heads -> sequence exchange already happens in the attention epilogue (peer stores), and
``PeerRowParallelLinear`` fuses the rest: the tcgen05 bf16 GEMM's epilogue stores each tile of
this rank's partial into its slot of every TP rank's partial buffer over NVLink while the next
tiles are multiplied, one peer barrier, then each rank sums the slots in rank order
(``h3sa_tp_reduce``). ``row_parallel_linear`` is the same product with the reference's NCCL
all-reduce, for comparison.
"""

from __future__ import annotations

import torch

from ._lib import call, ptr, stream_handle


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, *,
              partial_peers: torch.Tensor | None = None, ranks: int = 0, slot: int = 0,
              device_error: torch.Tensor | None = None,
              stream: torch.cuda.Stream | None = None) -> torch.Tensor | None:
    """bf16 ``[M, N]`` = a ``[M, K]`` @ b ``[N, K]``^T (fp32 accumulation); with
    ``partial_peers`` also into slot ``slot`` of every rank's ``[ranks, M, N]`` buffer."""

    for t in (a, b, out, partial_peers, device_error):
        if t is not None and not t.is_cuda:
            raise RuntimeError("gemm_bf16 tensors must be CUDA tensors")
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or a.ndim != 2 or b.ndim != 2:
        raise RuntimeError("gemm_bf16 takes bf16 [M, K] and [N, K] operands")
    m, k = (int(s) for s in a.shape)
    n = int(b.shape[0])
    if int(b.shape[1]) != k:
        raise RuntimeError(f"gemm_bf16: K differs ({k} vs {int(b.shape[1])})")
    a, b = a.contiguous(), b.contiguous()
    if out is None and partial_peers is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    ldo = n
    if out is not None:
        if out.dtype != torch.bfloat16 or tuple(out.shape) != (m, n) or not out.is_contiguous():
            raise RuntimeError("gemm_bf16 output must be a contiguous bf16 [M, N] tensor")
    if partial_peers is not None and (partial_peers.dtype != torch.int64
                                      or partial_peers.numel() < ranks):
        raise RuntimeError("partial_peers must be int64 with one address per rank")
    call("h3sa_gemm_bf16", ptr(a), ptr(b), ptr(out), m, n, k, ldo, ptr(partial_peers), int(ranks),
         int(slot), ptr(device_error), stream_handle(stream))
    return out


def tp_reduce(slots: torch.Tensor, out: torch.Tensor | None = None, *,
              stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """bf16 ``[M, N]`` = sum over the leading axis of ``slots`` ``[ranks, M, N]`` (fp32, in
    rank order, rounded once)."""

    if not slots.is_cuda or slots.dtype != torch.bfloat16 or slots.ndim != 3:
        raise RuntimeError("tp_reduce takes bf16 [ranks, M, N] CUDA slots")
    ranks, m, n = (int(s) for s in slots.shape)
    slots = slots.contiguous()
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=slots.device)
    call("h3sa_tp_reduce", ptr(slots), ptr(out), m, n, n, ranks, stream_handle(stream))
    return out


def row_parallel_linear(inputs: torch.Tensor, weight: torch.Tensor, *, group=None) -> torch.Tensor:
    """The reference's RowParallelLinear.forward without bias: the local product (tcgen05
    bf16 GEMM) then a NCCL all-reduce over ``group`` (skipped when it has one rank)."""

    out = gemm_bf16(inputs.reshape(-1, int(inputs.shape[-1])), weight)
    if group is not None and torch.distributed.get_world_size(group) > 1:
        torch.distributed.all_reduce(out, group=group)
    return out.reshape(*inputs.shape[:-1], int(weight.shape[0]))


class PeerRowParallelLinear:
    """out_proj with the TP all-reduce fused into the GEMM over peer memory.

    ``weight``: this TP rank's ``[N, inner / TP]`` slice (bf16). ``max_rows``: the most rows a
    call may carry. Collective to construct (maps every TP rank's partial buffers); every rank
    then calls it with the same row count. Partial buffers alternate between two sets, so one
    peer barrier per call orders both the exchange and the reuse."""

    def __init__(self, weight: torch.Tensor, max_rows: int, group=None,
                 device_error: torch.Tensor | None = None) -> None:
        import torch.distributed as dist

        from .peer import PeerBarrier, PeerBuffer

        self.weight = weight.contiguous()
        self.n = int(weight.shape[0])
        self.group = group
        self.ranks = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_rows = int(max_rows)
        self.err = device_error
        self.partials = PeerBuffer((2, self.ranks, self.max_rows, self.n), group)
        self.barrier = PeerBarrier(group, device_error=device_error)
        base = self.partials.addresses
        half = self.ranks * self.max_rows * self.n * 2  # bytes of one set
        self._tables = [torch.tensor([a + s * half for a in base], dtype=torch.int64,
                                     device=weight.device) for s in range(2)]
        self._calls = 0

    def __call__(self, inputs: torch.Tensor) -> torch.Tensor:
        rows = int(inputs.reshape(-1, int(inputs.shape[-1])).shape[0])
        if rows > self.max_rows:
            raise ValueError(f"{rows} rows exceed the {self.max_rows} the buffers hold")
        s = self._calls & 1
        self._calls += 1
        flat = inputs.reshape(rows, -1)
        # slots of this set viewed with this call's row count: [ranks, rows, N] at the head of
        # each rank's [ranks, max_rows, N] set, laid out with the rows stride of `rows`
        gemm_bf16(flat, self.weight, None, partial_peers=self._tables[s], ranks=self.ranks,
                  slot=self.rank, device_error=self.err)
        self.barrier()
        slots = self.partials.tensor[s].reshape(-1)[: self.ranks * rows * self.n]
        out = tp_reduce(slots.view(self.ranks, rows, self.n))
        return out.reshape(*inputs.shape[:-1], self.n)

    def close(self) -> None:
        self.barrier.close()
        self.partials.close()


__all__ = ["PeerRowParallelLinear", "gemm_bf16", "row_parallel_linear", "tp_reduce"]
