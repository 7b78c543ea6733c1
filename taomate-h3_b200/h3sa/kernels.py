"""Tensor-level wrappers over the C ABI: attention, KV row copies, e4m3 quantisation.

Shapes follow the reference's post-Ulysses layout: packed rows ``[rows, heads, 128]``.
KV pools are head-major and paged: ``[heads, pages * 128, 128]``; a page table (int32,
device) maps logical 128-row blocks to pages.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _lib
from ._lib import Problem, Rows, call, ptr, stream_handle

PAGE_ROWS = 128
HEAD_DIM = 128


@dataclass(frozen=True)
class AttentionProblem:
    """Queries ``[q_lo, q_hi)`` attend to logical KV rows ``[kv_lo, kv_hi)``."""

    q_lo: int
    q_hi: int
    kv_lo: int
    kv_hi: int
    sparse: bool = False


def _problems(problems: Sequence[AttentionProblem]) -> ctypes.Array:
    if not 1 <= len(problems) <= _lib.MAX_PROBLEMS:
        raise ValueError(f"1..{_lib.MAX_PROBLEMS} attention problems per launch")
    arr = (Problem * len(problems))()
    for dst, src in zip(arr, problems):
        dst.q_lo, dst.q_hi = int(src.q_lo), int(src.q_hi)
        dst.kv_lo, dst.kv_hi = int(src.kv_lo), int(src.kv_hi)
        dst.sparse = 1 if src.sparse else 0
    return arr


def _require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("h3sa kernels require CUDA tensors")
        if t is not None and not t.is_contiguous():
            raise RuntimeError("h3sa kernels require contiguous tensors")


def _check_attention_args(
    query: torch.Tensor,
    out: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    page_table: torch.Tensor,
    kv_num_blocks: torch.Tensor | None,
    kv_indices: torch.Tensor | None,
    q_scale: torch.Tensor | None,
    k_scale: torch.Tensor | None,
    v_scale: torch.Tensor | None,
) -> None:
    """Shape, dtype and device checks of ``attention_fwd`` that the C ABI cannot make: it
    sees raw pointers, so a short scale or block-list tensor would be read past its end."""

    if query.ndim != 3:
        raise RuntimeError("attention query must be [rows, heads, head_dim]")
    heads = int(query.shape[1])
    others = [out, key_pool, value_pool, page_table, kv_num_blocks, kv_indices, q_scale, k_scale,
              v_scale]
    if any(t is not None and t.device != query.device for t in others):
        raise RuntimeError("attention tensors must all be on the query's device")
    if out.shape != query.shape or out.dtype != torch.bfloat16:
        raise RuntimeError("attention output must be bf16 with the query's shape")
    if key_pool.shape != value_pool.shape or key_pool.ndim != 3 or key_pool.shape[0] != heads:
        raise RuntimeError("KV pools must be [heads, pages*128, head_dim] with matching shapes")
    if value_pool.dtype != key_pool.dtype:
        raise RuntimeError("key and value pools must have the same dtype")
    if page_table.dtype != torch.int32:
        raise RuntimeError("page table must be int32")
    if (kv_num_blocks is None) != (kv_indices is None):
        raise RuntimeError("block lists need both kv_num_blocks and kv_indices")
    if kv_num_blocks is not None and kv_indices is not None:
        if kv_num_blocks.dtype != torch.int32 or kv_indices.dtype != torch.int32:
            raise RuntimeError("block lists must be int32 kv_num_blocks and kv_indices")
        q_blocks = int(kv_num_blocks.shape[-1])
        stride = int(kv_indices.shape[-1])
        if (kv_indices.ndim < 2 or int(kv_indices.shape[-2]) != q_blocks
                or kv_num_blocks.numel() < heads * q_blocks
                or kv_indices.numel() < heads * q_blocks * stride):
            raise RuntimeError("block lists must be kv_num_blocks [heads, q_blocks] and "
                               "kv_indices [heads, q_blocks, stride] for every query head")
    scales = (q_scale, k_scale, v_scale)
    if any(t is not None for t in scales):
        if any(t is None for t in scales):
            raise RuntimeError("fp8 attention needs q_scale, k_scale and v_scale")
        if any(t.dtype != torch.float32 or t.numel() < heads for t in scales):  # type: ignore[union-attr]
            raise RuntimeError("fp8 attention scales must be float32 with one value per head")


def attention_fwd(
    query: torch.Tensor,
    out: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    page_table: torch.Tensor,
    problems: Sequence[AttentionProblem],
    softmax_scale: float,
    *,
    kv_num_blocks: torch.Tensor | None = None,
    kv_indices: torch.Tensor | None = None,
    q_scale: torch.Tensor | None = None,
    k_scale: torch.Tensor | None = None,
    v_scale: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> torch.Tensor:
    """Launch the sm_100a attention kernel (bf16, or e4m3 when scales are given)."""

    _require_cuda(query, out, key_pool, value_pool, page_table, kv_num_blocks, kv_indices,
                  q_scale, k_scale, v_scale)
    _check_attention_args(query, out, key_pool, value_pool, page_table, kv_num_blocks, kv_indices,
                          q_scale, k_scale, v_scale)
    rows, heads, head_dim = (int(s) for s in query.shape)
    pool_pages = int(key_pool.shape[1]) // PAGE_ROWS
    q_blocks = stride = 0
    if kv_num_blocks is not None and kv_indices is not None:
        q_blocks = int(kv_num_blocks.shape[-1])
        stride = int(kv_indices.shape[-1])
    probs = _problems(problems)
    fp8 = q_scale is not None
    common = (
        ptr(query), ptr(out), rows, heads, head_dim, ptr(key_pool), ptr(value_pool), pool_pages,
        ptr(page_table), int(page_table.numel()), probs, len(problems), float(softmax_scale),
    )
    tail = (ptr(kv_num_blocks), ptr(kv_indices), q_blocks, stride, ptr(device_error),
            stream_handle(stream))
    if fp8:
        if query.dtype != torch.float8_e4m3fn or key_pool.dtype != torch.float8_e4m3fn:
            raise RuntimeError("fp8 attention takes e4m3 query and KV pools")
        call("h3sa_attention_fwd_fp8", *common, ptr(q_scale), ptr(k_scale), ptr(v_scale), *tail)
    else:
        if query.dtype != torch.bfloat16 or key_pool.dtype != torch.bfloat16:
            raise RuntimeError("attention takes bf16 query and KV pools")
        call("h3sa_attention_fwd", *common, *tail)
    return out


def _rows(t: torch.Tensor, page_table: torch.Tensor | None) -> Rows:
    r = Rows()
    r.base = ptr(t)
    if page_table is None:
        r.paged = 0
        r.extent = int(t.shape[0])
        r.page_table = None
        r.table_blocks = 0
    else:
        r.paged = 1
        r.extent = int(t.shape[1]) // PAGE_ROWS
        r.page_table = ptr(page_table)
        r.table_blocks = int(page_table.numel())
    return r


def _check_copy_args(src: Sequence[torch.Tensor], dst: Sequence[torch.Tensor],
                     src_table: torch.Tensor | None, dst_table: torch.Tensor | None) -> tuple[int, int]:
    """Every src/dst tensor of one ``kv_copy_rows`` call must have the same heads and row size:
    the kernel addresses all of them with the first source's (its row bounds are checked on
    the device, its head and row extents are not). Returns (heads, row_bytes)."""

    if len(src) != len(dst) or not 1 <= len(src) <= 2:
        raise ValueError("one or two src/dst tensor pairs")
    shapes = []
    for tensors, table in ((src, src_table), (dst, dst_table)):
        for t in tensors:
            if t.ndim != 3:
                raise RuntimeError("kv_copy_rows takes [heads, pages*128, d] pages or [rows, heads, d] rows")
            heads = int(t.shape[0] if table is not None else t.shape[1])
            shapes.append((heads, int(t.shape[-1]) * t.element_size()))
    if any(sh != shapes[0] for sh in shapes):
        raise RuntimeError("kv_copy_rows tensors must all have the same heads and row size")
    return shapes[0]


def kv_copy_rows(
    src: Sequence[torch.Tensor],
    dst: Sequence[torch.Tensor],
    *,
    count: int,
    src_table: torch.Tensor | None = None,
    dst_table: torch.Tensor | None = None,
    src_index: torch.Tensor | None = None,
    src_start: int = 0,
    dst_index: torch.Tensor | None = None,
    dst_start: int = 0,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Copy ``count`` rows (all heads) from each src tensor to the matching dst tensor.

    A tensor is paged (``[heads, pages*128, d]``) when its side has a page table, else
    packed (``[rows, heads, d]``). Row i goes from ``src_index[i]`` (or ``src_start + i``)
    to ``dst_index[i]`` (or ``dst_start + i``).
    """

    if len(src) != len(dst) or not 1 <= len(src) <= 2:
        raise ValueError("one or two src/dst tensor pairs")
    _require_cuda(*src, *dst, src_table, dst_table, src_index, dst_index)
    heads, row_bytes = _check_copy_args(src, dst, src_table, dst_table)
    if count == 0:
        return
    s_arr = (Rows * len(src))(*[_rows(t, src_table) for t in src])
    d_arr = (Rows * len(dst))(*[_rows(t, dst_table) for t in dst])
    for idx in (src_index, dst_index):
        if idx is not None and idx.dtype != torch.int32:
            raise RuntimeError("row indices must be int32")
    call(
        "h3sa_kv_copy_rows", s_arr, d_arr, len(src), ptr(src_index), int(src_start),
        ptr(dst_index), int(dst_start), int(count), heads, row_bytes, ptr(device_error),
        stream_handle(stream),
    )


def quantize_fp8_e4m3_per_head(value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``[B, S, H, D]`` bf16 -> (e4m3 of the same shape, fp32 scales ``[B, H]``).

    Drop-in for ``quantize_fp8_e4m3_per_head`` (F/inference/fused_kernels.py:823-877):
    scale = max(amax over (S, D) / 448, 1e-12); q = RTNE(clamp(x / scale, +-448)).
    """

    if value.ndim != 4 or value.dtype != torch.bfloat16:
        raise ValueError("quantize_fp8_e4m3_per_head expects [B, S, H, D] bf16")
    _require_cuda(value)
    x = value.contiguous()
    b, s, h, d = (int(v) for v in x.shape)
    out = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    scale = torch.empty((b, h), dtype=torch.float32, device=x.device)
    call("h3sa_quantize_fp8_per_head", ptr(x), ptr(out), ptr(scale), b, s, h, d,
         stream_handle(None))
    return out, scale


def _check_quant_pool_args(pool: torch.Tensor, pool_fp8: torch.Tensor, scale: torch.Tensor,
                           page_table: torch.Tensor) -> None:
    """The e4m3 pool and the scales are written through raw pointers sized from ``pool``."""

    if pool.ndim != 3 or pool.dtype != torch.bfloat16:
        raise RuntimeError("quantize_fp8_pool takes a bf16 pool [heads, pages*128, head_dim]")
    if pool_fp8.shape != pool.shape or pool_fp8.dtype != torch.float8_e4m3fn:
        raise RuntimeError("the e4m3 pool must be float8_e4m3fn with the bf16 pool's shape")
    if scale.dtype != torch.float32 or scale.numel() < int(pool.shape[0]):
        raise RuntimeError("quantize_fp8_pool scales must be float32 with one value per head")
    if page_table.dtype != torch.int32:
        raise RuntimeError("page table must be int32")
    if any(t.device != pool.device for t in (pool_fp8, scale, page_table)):
        raise RuntimeError("quantize_fp8_pool tensors must all be on the pool's device")


def quantize_fp8_pool(
    pool: torch.Tensor,
    pool_fp8: torch.Tensor,
    scale: torch.Tensor,
    page_table: torch.Tensor,
    rows: int,
    *,
    device_error: torch.Tensor | None = None,
) -> None:
    """Per-head e4m3 quantisation of logical rows ``[0, rows)`` of a paged bf16 pool."""

    _require_cuda(pool, pool_fp8, scale, page_table)
    _check_quant_pool_args(pool, pool_fp8, scale, page_table)
    heads = int(pool.shape[0])
    pages = int(pool.shape[1]) // PAGE_ROWS
    call("h3sa_quantize_fp8_pool", ptr(pool), ptr(pool_fp8), ptr(scale), heads, pages,
         ptr(page_table), int(page_table.numel()), int(rows), ptr(device_error),
         stream_handle(None))


def _check_permute_extent(src: torch.Tensor, dst: torch.Tensor, dims: Sequence[int],
                          src_strides: Sequence[int], dst_strides: Sequence[int],
                          row_bytes: int) -> None:
    """Every record the index space addresses must lie inside its tensor: the kernel gets
    only base pointers and byte strides."""

    if len(dims) != 4 or len(src_strides) != 4 or len(dst_strides) != 4:
        raise ValueError("permute_rows takes a 4-D index space")
    if any(int(x) < 0 for x in (*dims, *src_strides, *dst_strides)) or int(row_bytes) <= 0:
        raise ValueError("permute_rows takes non-negative extents and strides")
    # the kernel moves 16-byte vectors: every record must start on a 16-byte boundary
    if int(row_bytes) % 16 or any(int(x) % 16 for x in (*src_strides, *dst_strides)):
        raise ValueError("permute_rows row_bytes and strides must be multiples of 16 bytes")
    if src.data_ptr() % 16 or dst.data_ptr() % 16:
        raise ValueError("permute_rows tensors must start on a 16-byte boundary")
    if any(int(x) == 0 for x in dims):
        return
    for t, strides, side in ((src, src_strides, "source"), (dst, dst_strides, "destination")):
        last = sum((int(n) - 1) * int(st) for n, st in zip(dims, strides)) + int(row_bytes)
        if last > t.numel() * t.element_size():
            raise ValueError(f"permute_rows {side} holds {t.numel() * t.element_size()} bytes, "
                             f"the index space reaches byte {last}")


def permute_rows(src: torch.Tensor, dst: torch.Tensor, dims: Sequence[int],
                 src_strides: Sequence[int], dst_strides: Sequence[int], row_bytes: int,
                 *, stream: torch.cuda.Stream | None = None) -> None:
    """Copy ``row_bytes`` records over a 4-D index space with byte strides on both sides."""

    _require_cuda(src, dst)
    _check_permute_extent(src, dst, dims, src_strides, dst_strides, row_bytes)
    d = (ctypes.c_int64 * 4)(*[int(x) for x in dims])
    ss = (ctypes.c_int64 * 4)(*[int(x) for x in src_strides])
    ds = (ctypes.c_int64 * 4)(*[int(x) for x in dst_strides])
    call("h3sa_permute_rows", ptr(src), ptr(dst), d, ss, ds, int(row_bytes), stream_handle(stream))


def quantize_fp8_rows(
    src: Sequence[torch.Tensor],
    dst: Sequence[torch.Tensor],
    scales: Sequence[torch.Tensor],
    workspace: torch.Tensor,
    *,
    count: int,
    src_start: int = 0,
    dst_start: int = 0,
    src_table: torch.Tensor | None = None,
    dst_table: torch.Tensor | None = None,
    zero_tail: bool = False,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Per-head e4m3 quantisation of rows ``[src_start, src_start + count)`` of each bf16
    ``src`` (packed ``[rows, heads, 128]`` or paged when ``src_table`` is given) into the
    matching e4m3 ``dst`` at ``dst_start``; tensor t's scales go to ``scales[t]`` (fp32
    ``[heads]``). ``workspace``: int32 ``[len(src) * heads]`` scratch owned by the caller.
    ``zero_tail`` zeroes the paged destination rows after the part up to its block's end."""

    if len(src) != len(dst) or len(src) != len(scales) or not 1 <= len(src) <= 2:
        raise ValueError("one or two src/dst/scale triples")
    _require_cuda(*src, *dst, *scales, workspace, src_table, dst_table, device_error)
    heads = int(src[0].shape[0] if src_table is not None else src[0].shape[1])
    for t, table, dtype in ((src, src_table, torch.bfloat16), (dst, dst_table, torch.float8_e4m3fn)):
        for x in t:
            h = int(x.shape[0] if table is not None else x.shape[1])
            if x.ndim != 3 or h != heads or int(x.shape[-1]) != HEAD_DIM or x.dtype != dtype:
                raise RuntimeError("quantize_fp8_rows takes bf16 sources and e4m3 destinations "
                                   f"with {heads} heads of {HEAD_DIM}")
    if any(s.dtype != torch.float32 or s.numel() < heads for s in scales):
        raise RuntimeError("quantize_fp8_rows scales must be float32 with one value per head")
    if workspace.dtype != torch.int32 or workspace.numel() < len(src) * heads:
        raise RuntimeError("quantize_fp8_rows workspace must be int32 with len(src) * heads entries")
    if count == 0:
        return
    s_arr = (Rows * len(src))(*[_rows(t, src_table) for t in src])
    d_arr = (Rows * len(dst))(*[_rows(t, dst_table) for t in dst])
    call("h3sa_quantize_fp8_rows", s_arr, d_arr, len(src), int(src_start), int(dst_start),
         int(count), heads, ptr(scales[0]), ptr(scales[1]) if len(scales) > 1 else None,
         ptr(workspace), 1 if zero_tail else 0, ptr(device_error), stream_handle(stream))


def segment_row_means(
    src: torch.Tensor,
    segments: Sequence[tuple[int, int]],
    *,
    src_table: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> torch.Tensor:
    """fp32 ``[len(segments), heads, 128]`` column means of bf16 rows: entry i is the mean over
    rows ``[start, start + rows)`` of segment i of ``src`` (packed ``[rows, heads, 128]``, or
    paged ``[heads, pages * 128, 128]`` with ``src_table``), from exact fp64 sums. The key
    summary of a committed block and the media query summary of commit-level top-k
    (F/streaming/cache.py:854; F/streaming/attention_hook.py:1279)."""

    _require_cuda(src, src_table, device_error)
    heads = int(src.shape[0] if src_table is not None else src.shape[1])
    if src.ndim != 3 or src.dtype != torch.bfloat16 or int(src.shape[-1]) != HEAD_DIM:
        raise RuntimeError(f"segment_row_means takes bf16 rows of {HEAD_DIM}")
    # paged rows beyond the table are refused on the device (bad-index flag)
    limit = int(src.shape[0]) if src_table is None else int(src_table.numel()) * PAGE_ROWS
    seg = [(int(a), int(n)) for a, n in segments]
    if any(a < 0 or n < 0 or a + n > limit for a, n in seg):
        raise RuntimeError("segment_row_means: a segment reaches outside the rows")
    means = torch.empty(len(seg), heads, HEAD_DIM, dtype=torch.float32, device=src.device)
    if not seg:
        return means
    table = torch.tensor([v for pair in seg for v in pair], dtype=torch.int32)
    table = table.pin_memory().to(src.device, non_blocking=True)
    work = torch.empty(len(seg) * heads * HEAD_DIM, dtype=torch.float64, device=src.device)
    rows = _rows(src, src_table)
    call("h3sa_segment_row_means", ctypes.byref(rows), ptr(table), len(seg),
         max(n for _, n in seg), heads, ptr(work), ptr(means), ptr(device_error),
         stream_handle(stream))
    return means


def commit_scores(summaries: torch.Tensor, query_mean: torch.Tensor, *,
                  stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """fp64 ``[parts]`` scores of commit-level top-k: the mean over heads of each summary's
    dot product with the query mean (F/streaming/attention_hook.py:1281-1286)."""

    _require_cuda(summaries, query_mean)
    if (summaries.dtype != torch.float32 or query_mean.dtype != torch.float32
            or summaries.ndim != 3 or tuple(summaries.shape[1:]) != tuple(query_mean.shape)
            or int(query_mean.shape[-1]) != HEAD_DIM):
        raise RuntimeError("commit_scores takes fp32 summaries [parts, heads, 128] and a "
                           "query mean [heads, 128]")
    summaries = summaries.contiguous()
    query_mean = query_mean.contiguous()
    scores = torch.empty(int(summaries.shape[0]), dtype=torch.float64, device=summaries.device)
    call("h3sa_commit_scores", ptr(summaries), ptr(query_mean), int(summaries.shape[0]),
         int(query_mean.shape[0]), ptr(scores), stream_handle(stream))
    return scores


def attention_fwd_fp8_parts(
    query: torch.Tensor,
    out: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    page_table: torch.Tensor,
    problems: Sequence[AttentionProblem],
    softmax_scale: float,
    *,
    q_scale: torch.Tensor,
    block_part: torch.Tensor,
    part_k_scale: torch.Tensor,
    part_v_scale: torch.Tensor,
    kv_num_blocks: torch.Tensor | None = None,
    kv_indices: torch.Tensor | None = None,
    device_error: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> torch.Tensor:
    """e4m3 attention over a segmented KV sequence: ``block_part[b]`` = part of logical block
    b | valid rows << 16, ``part_k_scale`` / ``part_v_scale`` fp32 ``[parts, heads]``."""

    _require_cuda(query, out, key_pool, value_pool, page_table, kv_num_blocks, kv_indices,
                  q_scale, block_part, part_k_scale, part_v_scale)
    _check_attention_args(query, out, key_pool, value_pool, page_table, kv_num_blocks, kv_indices,
                          q_scale, q_scale, q_scale)
    rows, heads, head_dim = (int(s) for s in query.shape)
    if query.dtype != torch.float8_e4m3fn or key_pool.dtype != torch.float8_e4m3fn:
        raise RuntimeError("fp8 attention takes e4m3 query and KV pools")
    if block_part.dtype != torch.int32 or block_part.numel() < page_table.numel():
        raise RuntimeError("block_part must be int32 with one entry per page-table block")
    if (part_k_scale.shape != part_v_scale.shape or part_k_scale.ndim != 2
            or int(part_k_scale.shape[1]) != heads or part_k_scale.dtype != torch.float32
            or part_v_scale.dtype != torch.float32):
        raise RuntimeError("part scales must be float32 [parts, heads] with matching shapes")
    if any(t.device != query.device for t in (block_part, part_k_scale, part_v_scale)):
        raise RuntimeError("attention tensors must all be on the query's device")
    q_blocks = stride = 0
    if kv_num_blocks is not None and kv_indices is not None:
        q_blocks = int(kv_num_blocks.shape[-1])
        stride = int(kv_indices.shape[-1])
    call("h3sa_attention_fwd_fp8_parts", ptr(query), ptr(out), rows, heads, head_dim,
         ptr(key_pool), ptr(value_pool), int(key_pool.shape[1]) // PAGE_ROWS, ptr(page_table),
         int(page_table.numel()), _problems(problems), len(problems), float(softmax_scale),
         ptr(q_scale), ptr(block_part), int(part_k_scale.shape[0]), ptr(part_k_scale),
         ptr(part_v_scale), ptr(kv_num_blocks), ptr(kv_indices), q_blocks, stride,
         ptr(device_error), stream_handle(stream))
    return out
