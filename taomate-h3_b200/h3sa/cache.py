"""Paged, head-major clean audio/video KV cache with the CleanAVKVCache interface.

Mirrors ``CleanAVKVCache`` (T/streaming/cache.py:77-294): the same transactional
stage -> commit protocol, the same retention and audio-drop row selection and the same
error messages, but the storage is a per-layer pool of 128-row pages laid out
``[heads, pages * 128, head_dim]`` plus a page table, instead of one dense tensor that
``torch.cat`` re-allocates on every commit.

Logical layout of one layer's page sequence::

    [ history (committed clean rows, logical commit order) | tail ]

The streaming hook writes the current chunk's media rows straight after the history
(the tail), so a clean commit only advances the history length: staged rows are already
in place. Retention and audio drop gather the selected rows into fresh pages in one
kernel launch per layer (T/streaming/cache.py:246-284 selects the same rows).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from .kernels import PAGE_ROWS, kv_copy_rows

MAIN_LAYER_NAMES = tuple(f"blocks.{index}.attn" for index in range(50))
VIDEO_TOKEN_TAG = 0
AUDIO_TOKEN_TAG = 2


@dataclass(frozen=True)
class KVContract:
    """Shape contract for the local attention shard (T/streaming/cache.py:16-23)."""

    local_heads: int = 14
    head_dim: int = 128
    dtype: torch.dtype = torch.bfloat16
    device_type: str = "cuda"


def kv_contract_from_model(model: object) -> KVContract:
    """Build the KV shape contract from an installed model (T/streaming/cache.py:26-48)."""

    blocks = getattr(model, "blocks", None)
    if blocks is None:
        raise RuntimeError("model does not expose transformer blocks")
    layers = len(blocks)
    if layers != len(MAIN_LAYER_NAMES):
        raise RuntimeError(f"expected {len(MAIN_LAYER_NAMES)} transformer layers, got {layers}")
    architecture = getattr(model, "arch", None)
    context = getattr(model, "parallel_context", None)
    total_heads = int(getattr(architecture, "num_attention_heads", 0))
    head_dim = int(getattr(architecture, "attention_head_dim", 0))
    tp_size = int(getattr(context, "tp_world_size", 0))
    ulysses_size = int(getattr(context, "ulysses_world_size", 0))
    parallel_size = tp_size * ulysses_size
    if total_heads <= 0 or head_dim <= 0 or parallel_size <= 0 or total_heads % parallel_size:
        raise RuntimeError("model topology cannot resolve post-Ulysses local KV heads")
    return KVContract(local_heads=total_heads // parallel_size, head_dim=head_dim)


@dataclass(frozen=True)
class AVKV:
    """Dense clean audio/video keys and values for one attention layer."""

    key: torch.Tensor
    value: torch.Tensor


@dataclass(frozen=True)
class VideoKV:
    """Dense video-only keys and values for one attention layer (F/streaming/cache.py:44-54)."""

    key: torch.Tensor
    value: torch.Tensor


def _check_prefix_pair(pair, contract: KVContract, layer: str) -> None:
    tail = (contract.local_heads, contract.head_dim)
    if (pair.key.ndim != 3 or pair.key.shape != pair.value.shape
            or tuple(pair.key.shape[1:]) != tail or pair.key.dtype != contract.dtype
            or pair.value.dtype != contract.dtype):
        raise ValueError(f"{layer} temporary full-prefix K/V must be [tokens, {tail[0]}, "
                         f"{tail[1]}] {contract.dtype}")


class TemporaryVideoPrefix:
    """Per-layer video K/V a full-prefix capture recorded, seen by later calls as an extra
    part and never committed (F/streaming/cache.py:118-147)."""

    def __init__(self, layers, *, contract: KVContract,
                 layer_names: tuple[str, ...] | None = None) -> None:
        names = tuple(layer_names or MAIN_LAYER_NAMES)
        self.contract = contract
        if set(layers) != set(names):
            raise ValueError("temporary full-prefix must cover every main attention layer")
        self._layers = {name: layers[name] for name in names}
        for name, pair in self._layers.items():
            _check_prefix_pair(pair, contract, name)
        self.token_count = int(self._layers[names[0]].key.shape[0])
        if any(int(p.key.shape[0]) != self.token_count for p in self._layers.values()):
            raise ValueError("temporary full-prefix token counts differ by layer")

    def get(self, layer: str):
        return self._layers[layer]

    def release(self) -> None:
        self._layers.clear()


class TemporaryAVPrefix(TemporaryVideoPrefix):
    """Per-layer captured audio (two channels) and video K/V (F/streaming/cache.py:150-196)."""

    def __init__(self, layers, *, video_token_count: int, audio_token_count_per_channel: int,
                 contract: KVContract, layer_names: tuple[str, ...] | None = None) -> None:
        for name, count in (("video count", video_token_count),
                            ("per-channel audio count", audio_token_count_per_channel)):
            if isinstance(count, bool) or not isinstance(count, int) or count <= 0:
                raise ValueError(f"temporary AV full-prefix {name} must be positive")
        super().__init__(layers, contract=contract, layer_names=layer_names)
        self.video_token_count = video_token_count
        self.audio_token_count_per_channel = audio_token_count_per_channel
        self.audio_token_count = 2 * audio_token_count_per_channel
        if self.token_count != video_token_count + self.audio_token_count:
            raise ValueError("temporary AV full-prefix token count differs")


def _upload_pages(table: torch.Tensor, pages: list[int]) -> None:
    """Copy a page list into the head of a device page table, ordered on the current stream
    without blocking the host: the list goes through a pinned staging tensor, which the
    host allocator keeps alive until the copy has run."""

    if not pages:
        return
    host = torch.tensor(pages, dtype=torch.int32)
    if table.is_cuda:
        host = host.pin_memory()
    table[: len(pages)].copy_(host, non_blocking=table.is_cuda)


class PagedLayerKV:
    """Page pool and page sequence of one layer.

    ``key``/``value`` are ``[heads, capacity_pages * 128, head_dim]``; ``pages`` lists the
    physical page of each logical 128-row block; ``table`` is its int32 device copy
    (length = capacity, unused entries 0). Pages are recycled through a free list; a
    fresh or grown pool is zero-filled, so rows beyond a sequence's end are always finite.
    """

    def __init__(self, heads: int, head_dim: int, dtype: torch.dtype, device: torch.device,
                 initial_pages: int = 8) -> None:
        self.heads = heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device
        self.capacity = 0
        self.key = torch.empty(0, device=device, dtype=dtype)
        self.value = torch.empty(0, device=device, dtype=dtype)
        self.free: list[int] = []
        self.pages: list[int] = []
        self.table = torch.zeros(0, dtype=torch.int32, device=device)
        self.history_rows = 0
        self.fp8: SegmentedFp8History | None = None  # e4m3 history (segmented FP8 caches)
        self._grow(max(1, initial_pages))

    def _grow(self, capacity: int) -> None:
        key = torch.zeros(self.heads, capacity * PAGE_ROWS, self.head_dim, dtype=self.dtype,
                          device=self.device)
        value = torch.zeros_like(key)
        if self.capacity:
            rows = self.capacity * PAGE_ROWS
            key[:, :rows].copy_(self.key)
            value[:, :rows].copy_(self.value)
        self.free.extend(range(capacity - 1, self.capacity - 1, -1))
        self.key, self.value = key, value
        self.capacity = capacity
        table = torch.zeros(capacity, dtype=torch.int32, device=self.device)
        _upload_pages(table, self.pages)
        self.table = table

    def _take(self, count: int) -> list[int]:
        if count > len(self.free):
            self._grow(max(2 * self.capacity, self.capacity + count - len(self.free)))
        taken = [self.free.pop() for _ in range(count)]
        return taken

    def _sync_table(self) -> None:
        _upload_pages(self.table, self.pages)

    def reserve(self, rows: int) -> None:
        """Make the page sequence cover logical rows [0, rows)."""

        need = (rows + PAGE_ROWS - 1) // PAGE_ROWS
        if need > len(self.pages):
            self.pages.extend(self._take(need - len(self.pages)))
            self._sync_table()

    def write(self, key: torch.Tensor, value: torch.Tensor, *, start: int, count: int,
              src_start: int = 0, src_index: torch.Tensor | None = None) -> None:
        """Copy ``count`` packed rows of key/value into logical rows [start, start+count)."""

        self.reserve(start + count)
        kv_copy_rows([key, value], [self.key, self.value], count=count, dst_table=self.table,
                     src_start=src_start, src_index=src_index, dst_start=start)

    def gather(self, rows: torch.Tensor) -> "PagedLayerKV":
        """Build the sequence made of the given logical rows, in order, in fresh pages."""

        count = int(rows.numel())
        new_pages = self._take((count + PAGE_ROWS - 1) // PAGE_ROWS)
        table = torch.zeros(self.capacity, dtype=torch.int32, device=self.device)
        _upload_pages(table, new_pages)
        if count:
            kv_copy_rows([self.key, self.value], [self.key, self.value], count=count,
                         src_table=self.table, dst_table=table,
                         src_index=rows.to(device=self.device, dtype=torch.int32))
        self.free.extend(reversed(self.pages))
        self.pages = new_pages
        self.table = table
        self.history_rows = count
        return self

    def materialize(self, rows: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense ``[rows, heads, head_dim]`` copies of logical rows [0, rows)."""

        key = torch.empty(rows, self.heads, self.head_dim, dtype=self.dtype, device=self.device)
        value = torch.empty_like(key)
        if rows:
            kv_copy_rows([self.key, self.value], [key, value], count=rows, src_table=self.table)
        return key, value

    def release(self) -> None:
        self.free.extend(reversed(self.pages))
        self.pages = []
        self.history_rows = 0


class SegmentedFp8History:
    """The e4m3 copy of one layer's committed history, one part per commit.

    Each committed block is quantised once, at commit, with its own per-head K and V scales
    (F/streaming/cache.py:835-855), and keeps them when retention later drops rows from it.
    Parts are stored in an e4m3 page sequence of their own, each starting on a 128-row block
    boundary, so every KV block belongs to one part: ``block_part`` holds, per logical block,
    the part index and the block's valid rows (``part | rows << 16``), the layout
    ``h3sa_attention_fwd_fp8_parts`` reads. The rows after a part in its last block hold
    zeros or earlier quantiser outputs, always finite, and are masked by the kernel.
    """

    def __init__(self, heads: int, head_dim: int, device: torch.device) -> None:
        self.heads = heads
        self.store = PagedLayerKV(heads, head_dim, torch.float8_e4m3fn, device)
        self.starts: list[int] = []   # first logical e4m3 row of each part (block aligned)
        self.rows: list[int] = []     # rows of each part
        self.k_scale = torch.zeros(0, heads, dtype=torch.float32, device=device)
        self.v_scale = torch.zeros(0, heads, dtype=torch.float32, device=device)
        # fp32 [parts, heads, head_dim]: each part's mean bf16 key row, the summary that
        # commit-level top-k scores against the media queries (F/streaming/cache.py:854)
        self.key_summary = torch.zeros(0, heads, head_dim, dtype=torch.float32, device=device)
        self.workspace = torch.zeros(2 * heads, dtype=torch.int32, device=device)

    @property
    def end(self) -> int:
        """First block-aligned logical row after the last part."""

        if not self.starts:
            return 0
        last = self.starts[-1] + self.rows[-1]
        return (last + PAGE_ROWS - 1) // PAGE_ROWS * PAGE_ROWS

    def block_part(self, extra: list[tuple[int, int]] = ()) -> torch.Tensor:
        """int32 device table over the store's capacity: the parts plus ``extra`` (start,
        rows) parts that follow them (their indices continue the numbering)."""

        entries = [0] * self.store.capacity
        for i, (s0, n) in enumerate(list(zip(self.starts, self.rows)) + list(extra)):
            for b in range(s0 // PAGE_ROWS, (s0 + n + PAGE_ROWS - 1) // PAGE_ROWS):
                entries[b] = i | (min(PAGE_ROWS, s0 + n - b * PAGE_ROWS) << 16)
        table = torch.zeros(self.store.capacity, dtype=torch.int32, device=self.store.device)
        _upload_pages(table, entries)
        return table

    def subset_tables(self, selected: list[int], current: list[tuple[int, int, int]]
                      ) -> tuple[torch.Tensor, torch.Tensor, int]:
        """Page table and block_part of a sequence made of the selected history parts (in the
        given order) followed by ``current`` (part index, start, rows) parts of the store, all
        keeping their part indices; returns them with the sequence's row count."""

        pages, entries = [], []
        parts = [(i, self.starts[i], self.rows[i]) for i in selected] + list(current)
        for index, s0, n in parts:
            for b in range(s0 // PAGE_ROWS, (s0 + n + PAGE_ROWS - 1) // PAGE_ROWS):
                pages.append(self.store.pages[b])
                entries.append(index | (min(PAGE_ROWS, s0 + n - b * PAGE_ROWS) << 16))
        dev = self.store.device
        table = torch.zeros(max(1, len(pages)), dtype=torch.int32, device=dev)
        block_part = torch.zeros_like(table)
        _upload_pages(table, pages)
        _upload_pages(block_part, entries)
        kv_end = (len(pages) - 1) * PAGE_ROWS + (entries[-1] >> 16) if pages else 0
        return table, block_part, kv_end

    def append_part(self, key: torch.Tensor, value: torch.Tensor, *, src_start: int, count: int,
                    src_table: torch.Tensor | None, k_scale: torch.Tensor,
                    v_scale: torch.Tensor, start: int | None = None) -> int:
        """Quantise ``count`` bf16 rows of key/value (paged when ``src_table`` is given) into
        a part at ``start`` (default: after the last part); scales into ``k_scale`` /
        ``v_scale`` (fp32 [heads]). Returns the part's start. Does not record the part."""

        from .kernels import quantize_fp8_rows

        s0 = self.end if start is None else start
        self.store.reserve(s0 + count)
        quantize_fp8_rows([key, value], [self.store.key, self.store.value], [k_scale, v_scale],
                          self.workspace, count=count, src_start=src_start, dst_start=s0,
                          src_table=src_table, dst_table=self.store.table, zero_tail=True)
        return s0

    def commit_part(self, key: torch.Tensor, value: torch.Tensor, *, src_start: int, count: int,
                    src_table: torch.Tensor | None) -> None:
        """Quantise a committed block into a new part with its own scales, and record its
        key summary (the mean of its bf16 key rows)."""

        from .kernels import segment_row_means

        ks = torch.empty(1, self.heads, dtype=torch.float32, device=self.store.device)
        vs = torch.empty_like(ks)
        s0 = self.append_part(key, value, src_start=src_start, count=count, src_table=src_table,
                              k_scale=ks[0], v_scale=vs[0])
        summary = segment_row_means(key, [(src_start, count)], src_table=src_table)
        self.starts.append(s0)
        self.rows.append(count)
        self.k_scale = torch.cat((self.k_scale, ks))
        self.v_scale = torch.cat((self.v_scale, vs))
        self.key_summary = torch.cat((self.key_summary, summary))

    def refresh_summaries(self, key: torch.Tensor, table: torch.Tensor) -> None:
        """Recompute every part's key summary from the bf16 history rows, where the parts'
        rows follow one another in order (after retention, which keeps a part's scales but
        recomputes its summary over the rows it kept: F/streaming/cache.py:1031-1034)."""

        from .kernels import segment_row_means

        segments, cursor = [], 0
        for n in self.rows:
            segments.append((cursor, n))
            cursor += n
        self.key_summary = segment_row_means(key, segments, src_table=table)

    def retain(self, selection: list[tuple[int, list[int]]]) -> None:
        """Keep, in order, the given (part, local rows) selections: each becomes a part of its
        own in fresh block-aligned pages, with its original scales."""

        old_table = self.store.table
        old_pages = self.store.pages
        starts, rows, src_rows, dst_rows = [], [], [], []
        cursor = 0
        for part, local in selection:
            if not local:
                continue
            starts.append(cursor)
            rows.append(len(local))
            src_rows.extend(self.starts[part] + r for r in local)
            dst_rows.extend(cursor + i for i in range(len(local)))
            cursor = (cursor + len(local) + PAGE_ROWS - 1) // PAGE_ROWS * PAGE_ROWS
        keep = [part for part, local in selection if local]
        new_pages = self.store._take(cursor // PAGE_ROWS)
        table = torch.zeros(self.store.capacity, dtype=torch.int32, device=self.store.device)
        _upload_pages(table, new_pages)
        if src_rows:
            dev = self.store.device
            kv_copy_rows([self.store.key, self.store.value], [self.store.key, self.store.value],
                         count=len(src_rows), src_table=old_table, dst_table=table,
                         src_index=torch.tensor(src_rows, dtype=torch.int32).pin_memory().to(dev, non_blocking=True),
                         dst_index=torch.tensor(dst_rows, dtype=torch.int32).pin_memory().to(dev, non_blocking=True))
        self.store.free.extend(reversed(old_pages))
        self.store.pages = new_pages
        self.store.table = table
        idx = torch.tensor(keep, dtype=torch.long, device=self.store.device)
        self.k_scale = self.k_scale.index_select(0, idx)
        self.v_scale = self.v_scale.index_select(0, idx)
        self.key_summary = self.key_summary.index_select(0, idx)  # refreshed by the cache
        self.starts, self.rows = starts, rows

    def release(self) -> None:
        self.store.release()
        self.starts, self.rows = [], []
        self.k_scale = self.k_scale[:0]
        self.v_scale = self.v_scale[:0]
        self.key_summary = self.key_summary[:0]


def _validate_layer_name(layer_name: str, names: tuple[str, ...]) -> None:
    if layer_name not in names:
        raise KeyError(f"unexpected transformer layer: {layer_name}")


class CleanAVKVCache:
    """Transactional persistent cache containing clean media KV only.

    Clean commits append one streaming chunk. Retention preserves the first video's rows
    as a long-term sink and the two most recent clean chunks.
    """

    def __init__(self, contract: KVContract, *, layer_names: tuple[str, ...] = MAIN_LAYER_NAMES,
                 device: torch.device | str | None = None, initial_pages: int = 8,
                 segmented_fp8_history: bool = False) -> None:
        self.contract = contract
        # also keep every committed block as an e4m3 part quantised once, at commit
        # (F/streaming/cache.py:205-211, 835-855)
        self.segmented_fp8_history = bool(segmented_fp8_history)
        self.layer_names = tuple(layer_names)
        self._device = torch.device(device) if device is not None else None
        self._initial_pages = initial_pages
        self._layers: dict[str, PagedLayerKV] = {}
        self._staged: dict[str, int] = {}
        self._staged_block: int | None = None
        self._staged_tags: tuple[int, ...] | None = None
        self._staged_indices: torch.Tensor | None = None
        self._block_index = 0
        self._commit_token_counts: list[int] = []
        self._commit_token_tags: list[tuple[int, ...]] = []
        self._invalid_after_failed_commit = False
        # set by the FL2AV sink + recent retention; read by history_for_fused_current
        self._sink_video_only = False

    # ------------------------------------------------------------------ properties
    @property
    def committed_blocks(self) -> int:
        """Logical number of clean chunks committed since the last clear."""

        self._require_valid()
        return self._block_index

    @property
    def history_tokens(self) -> int:
        self._require_valid()
        return sum(self._commit_token_counts)

    @property
    def history_audio_tokens(self) -> int:
        return sum(tag == AUDIO_TOKEN_TAG for tags in self._commit_token_tags for tag in tags)

    @property
    def history_video_tokens(self) -> int:
        return sum(tag == VIDEO_TOKEN_TAG for tags in self._commit_token_tags for tag in tags)

    @property
    def clean_commit_active(self) -> bool:
        return self._staged_block is not None

    def commit_token_tags(self) -> list[tuple[int, ...]]:
        return list(self._commit_token_tags)

    @property
    def commit_token_counts(self) -> tuple[int, ...]:
        """Rows of each retained clean block, oldest first (F/streaming/cache.py:259-262)."""

        self._require_valid()
        return tuple(self._commit_token_counts)

    @property
    def retained_blocks(self) -> int:
        return len(self._commit_token_counts)

    def _require_valid(self) -> None:
        if self._invalid_after_failed_commit:
            raise RuntimeError("H3 cache is invalid after a failed clean commit")

    def _invalidate_failed_commit(self) -> None:
        for paged in self._layers.values():
            paged.release()
            if paged.fp8 is not None:
                paged.fp8.release()
        self._clear_staging()
        self._block_index = 0
        self._commit_token_counts.clear()
        self._commit_token_tags.clear()
        self._invalid_after_failed_commit = True

    # ------------------------------------------------------------------ snapshots
    def save_snapshot(self, path) -> None:
        """Write the committed history and its bookkeeping to ``path`` (h3sa.snapshot)."""

        from .snapshot import save_cache

        save_cache(self, path)

    @classmethod
    def load_snapshot(cls, path, *, device=None, contract: KVContract | None = None
                      ) -> "CleanAVKVCache":
        """A cache restored from a snapshot, ready to attend and commit where it stopped."""

        from .snapshot import load_cache

        return load_cache(path, device=device, contract=contract)

    # ------------------------------------------------------------------ paged access
    def layer(self, layer_name: str, device: torch.device | None = None) -> PagedLayerKV:
        """The layer's page sequence, created on first use."""

        _validate_layer_name(layer_name, self.layer_names)
        paged = self._layers.get(layer_name)
        if paged is None:
            dev = device or self._device or torch.device("cuda", torch.cuda.current_device())
            paged = PagedLayerKV(self.contract.local_heads, self.contract.head_dim,
                                 self.contract.dtype, dev, self._initial_pages)
            if self.segmented_fp8_history:
                paged.fp8 = SegmentedFp8History(self.contract.local_heads, self.contract.head_dim,
                                                dev)
            self._layers[layer_name] = paged
        return paged

    def history_rows(self, layer_name: str) -> int:
        _validate_layer_name(layer_name, self.layer_names)
        paged = self._layers.get(layer_name)
        return 0 if paged is None else paged.history_rows

    def history(self, layer_name: str) -> AVKV | None:
        """Dense copies of the layer's committed rows (None when empty)."""

        self._require_valid()
        _validate_layer_name(layer_name, self.layer_names)
        paged = self._layers.get(layer_name)
        if paged is None or paged.history_rows == 0:
            return None
        key, value = paged.materialize(paged.history_rows)
        return AVKV(key=key, value=value)

    # ------------------------------------------------------------------ transactions
    def begin_clean_commit(self, block_index: int) -> None:
        if self.clean_commit_active:
            raise RuntimeError("a clean KV commit is already active")
        if block_index != self._block_index:
            raise RuntimeError(f"expected clean chunk {self._block_index}, got {block_index}")
        self._staged_block = block_index
        self._staged.clear()
        self._staged_tags = None
        self._staged_indices = None

    def _resolve_stage(self, token_tags: torch.Tensor, commit_mask: torch.Tensor,
                       commit_indices: torch.Tensor | None = None) -> torch.Tensor:
        if self._staged_indices is None:
            if commit_indices is None:
                indices = torch.nonzero(commit_mask.to(torch.bool), as_tuple=False).flatten()
            else:
                # FL2AV: the caller names the committed rows (a fused forward commits the
                # previous document's media only, F/streaming/cache.py:589-640)
                if (commit_indices.ndim != 1 or commit_indices.dtype != torch.long
                        or commit_indices.device != token_tags.device):
                    raise ValueError("clean H3 block contains no valid audio/video rows")
                indices = commit_indices
            if indices.numel() == 0:
                raise RuntimeError("clean commit did not contain audio/video rows")
            selected_tags = token_tags.index_select(0, indices)
            tags = tuple(int(tag) for tag in selected_tags.detach().cpu().tolist())
            if frozenset(tags) != frozenset((VIDEO_TOKEN_TAG, AUDIO_TOKEN_TAG)):
                raise RuntimeError("each clean chunk must contain both video and audio KV")
            self._staged_indices = indices
            self._staged_tags = tags
        return self._staged_indices

    def _check_stage_args(self, layer_name: str, key: torch.Tensor, value: torch.Tensor,
                          token_tags: torch.Tensor, commit_mask: torch.Tensor) -> None:
        if not self.clean_commit_active:
            raise RuntimeError("begin_clean_commit() must be called before stage()")
        _validate_layer_name(layer_name, self.layer_names)
        if layer_name in self._staged:
            raise RuntimeError(f"{layer_name}: KV was staged more than once")
        if key.shape != value.shape or key.ndim != 3:
            raise RuntimeError(f"{layer_name}: key/value must have matching rank-3 shapes")
        if token_tags.ndim != 1 or commit_mask.ndim != 1:
            raise RuntimeError("token_tags and commit_mask must be rank-1")
        if token_tags.shape[0] != key.shape[0] or commit_mask.shape[0] != key.shape[0]:
            raise RuntimeError(f"{layer_name}: packed metadata length does not match KV rows")
        expected_tail = (self.contract.local_heads, self.contract.head_dim)
        if tuple(key.shape[1:]) != expected_tail:
            raise RuntimeError(
                f"{layer_name}: expected key shape [tokens, {expected_tail[0]}, {expected_tail[1]}], "
                f"got {tuple(key.shape)}"
            )
        if key.dtype != self.contract.dtype or value.dtype != self.contract.dtype:
            raise RuntimeError(f"{layer_name}: persistent KV must be {self.contract.dtype}")
        if key.device.type != self.contract.device_type or value.device.type != self.contract.device_type:
            raise RuntimeError(f"{layer_name}: persistent KV must reside on {self.contract.device_type}")

    def stage(self, layer_name: str, key: torch.Tensor, value: torch.Tensor,
              token_tags: torch.Tensor, commit_mask: torch.Tensor, *,
              commit_indices: torch.Tensor | None = None) -> None:
        """Stage clean audio/video rows produced by one transformer layer.

        The committed rows (``nonzero(commit_mask)`` in packed order, or ``commit_indices``)
        are written into the layer's tail, directly after its history.
        """

        self._check_stage_args(layer_name, key, value, token_tags, commit_mask)
        indices = self._resolve_stage(token_tags, commit_mask, commit_indices)
        paged = self.layer(layer_name, key.device)
        paged.write(key.contiguous(), value.contiguous(), start=paged.history_rows,
                    count=int(indices.numel()), src_index=indices.to(torch.int32))
        self._staged[layer_name] = int(indices.numel())

    def stage_in_place(self, layer_name: str, key: torch.Tensor, value: torch.Tensor,
                       token_tags: torch.Tensor, commit_mask: torch.Tensor, *,
                       commit_indices: torch.Tensor | None = None) -> None:
        """Stage rows the streaming hook already wrote to the tail, in commit order."""

        self._check_stage_args(layer_name, key, value, token_tags, commit_mask)
        indices = self._resolve_stage(token_tags, commit_mask, commit_indices)
        self._staged[layer_name] = int(indices.numel())

    def commit(self, *, retain_recent_commit_count: int | None = None) -> None:
        """Atomically append all staged layers to persistent history; with
        ``retain_recent_commit_count`` keep only that many newest blocks (FL2AV,
        F/streaming/cache.py:780-821)."""

        if retain_recent_commit_count is not None:
            self.commit_bounded(retain_recent_commit_count)
            return
        self._require_valid()
        if not self.clean_commit_active:
            raise RuntimeError("no clean KV commit is active")
        missing = [name for name in self.layer_names if name not in self._staged]
        if missing:
            raise RuntimeError(f"clean KV commit is missing {len(missing)} transformer layers")
        assert self._staged_tags is not None
        token_count = len(self._staged_tags)
        for layer_name in self.layer_names:
            staged = self._staged[layer_name]
            if staged != token_count:
                raise RuntimeError(f"{layer_name}: staged {staged} rows, expected {token_count}")
        try:
            for layer_name in self.layer_names:
                paged = self._layers[layer_name]
                if paged.fp8 is not None:
                    # the staged rows sit right after the history: quantise them as one part
                    paged.fp8.commit_part(paged.key, paged.value, src_start=paged.history_rows,
                                          count=token_count, src_table=paged.table)
                paged.history_rows += token_count
        except BaseException:
            # a commit that stops half way leaves layers out of step: the cache refuses further
            # use until clear() (F/streaming/cache.py:766-778)
            self._invalidate_failed_commit()
            raise
        self._commit_token_counts.append(token_count)
        self._commit_token_tags.append(self._staged_tags)
        self._block_index += 1
        self._clear_staging()

    def commit_bounded(self, count: int, *, advance_serial: bool = True) -> None:
        """Commit the staged block keeping only the newest ``count`` blocks, the staged one
        included (F/streaming/cache.py:857-927); without ``advance_serial`` the logical
        chunk count stays."""

        self._require_valid()
        if isinstance(count, bool) or not isinstance(count, int) or count < 1:
            raise ValueError("bounded clean commit count must be positive")
        serial = self._block_index
        self.commit()
        if not advance_serial:
            self._block_index = serial
        blocks = len(self._commit_token_counts)
        if blocks > count:
            self._retain_commit_rows([(index, False) for index in range(blocks - count, blocks)])

    def retain_recent_commits(self, count: int) -> None:
        """Keep the newest ``count`` clean blocks (F/streaming/cache.py:929-962)."""

        self._require_valid()
        if isinstance(count, bool) or not isinstance(count, int) or count < 1:
            raise ValueError("retained clean commit count must be a positive integer")
        if self.clean_commit_active:
            raise RuntimeError("cannot evict H3 history during a clean commit")
        blocks = len(self._commit_token_counts)
        if blocks <= count:
            return
        self._retain_commit_rows([(index, False) for index in range(blocks - count, blocks)])

    def retain_sink_and_recent_commits(self, recent_count: int | None = None, *,
                                       sink_video_only: bool = True) -> None:
        """Keep the first chunk's video sink and the most recent clean chunks.

        Without arguments, the T recipe: block 0's video rows and the two newest blocks
        (T/streaming/cache.py:206-218). With ``recent_count`` (FL2AV,
        F/streaming/cache.py:964-995): block 0, whole while it is still among the newest
        ``recent_count`` blocks and otherwise its video rows only (all of it without
        ``sink_video_only``), plus the newest ``recent_count`` blocks.
        """

        self._require_valid()
        if self.clean_commit_active:
            raise RuntimeError("cannot trim persistent KV during an active clean commit")
        block_count = len(self._commit_token_counts)
        if recent_count is None:
            if block_count <= 2:
                return
            recent_start = max(1, block_count - 2)
            selection = [(0, True)] + [(index, False) for index in range(recent_start, block_count)]
            self._retain_commit_rows(selection)
            return
        if isinstance(recent_count, bool) or not isinstance(recent_count, int) or recent_count < 0:
            raise ValueError("recent clean commit count must be non-negative")
        self._sink_video_only = bool(sink_video_only)
        if block_count == 0:
            return
        recent_start = max(0, block_count - recent_count)
        selection = [(0, bool(sink_video_only and recent_start > 0))]
        selection += [(index, False) for index in range(max(1, recent_start), block_count)]
        if selection == [(index, False) for index in range(block_count)]:
            return
        self._retain_commit_rows(selection)

    def drop_audio_history(self) -> int:
        """Remove audio rows while preserving every retained video row."""

        if self.clean_commit_active:
            raise RuntimeError("cannot drop audio history during an active clean commit")
        removed_tokens = self.history_audio_tokens
        if not self._commit_token_counts:
            return 0
        self._retain_commit_rows([(index, True) for index in range(len(self._commit_token_counts))])
        return removed_tokens

    def rollback(self) -> None:
        """Discard the currently staged clean chunk (its tail rows are simply not adopted)."""

        self._clear_staging()

    # ------------------------------------------------------------------ FL2AV history views
    def _block_offsets(self) -> list[int]:
        offsets = [0]
        for count in self._commit_token_counts:
            offsets.append(offsets[-1] + count)
        return offsets

    def _rows_view(self, layer_name: str, rows: list[int]) -> AVKV | None:
        """Dense copies of the given logical history rows, in order (one gather launch)."""

        paged = self._layers.get(layer_name)
        if paged is None or not rows:
            return None
        key = torch.empty(len(rows), paged.heads, paged.head_dim, dtype=paged.dtype,
                          device=paged.device)
        value = torch.empty_like(key)
        index = torch.tensor(rows, dtype=torch.int32).pin_memory().to(paged.device, non_blocking=True)
        kv_copy_rows([paged.key, paged.value], [key, value], count=len(rows), src_table=paged.table,
                     src_index=index)
        return AVKV(key=key, value=value)

    def history_blocks(self, layer_name: str) -> tuple[AVKV, ...]:
        """One dense copy per retained clean block (F/streaming/cache.py:344-366)."""

        self._require_valid()
        _validate_layer_name(layer_name, self.layer_names)
        offsets = self._block_offsets()
        views = (self._rows_view(layer_name, list(range(offsets[i], offsets[i + 1])))
                 for i in range(len(self._commit_token_counts)))
        return tuple(v for v in views if v is not None)

    def sink_and_recent_history_blocks(self, layer_name: str,
                                       recent_count: int) -> tuple[AVKV, ...]:
        """Block 0 plus the newest ``recent_count`` other blocks, one copy per block
        (F/streaming/cache.py:325-342)."""

        if isinstance(recent_count, bool) or not isinstance(recent_count, int) or recent_count < 0:
            raise ValueError("recent H3 history count must be non-negative")
        blocks = self.history_blocks(layer_name)
        if not blocks:
            return ()
        return (blocks[0], *blocks[max(1, len(blocks) - recent_count):])

    def history_modality_parts_rows(self, block_indices: Sequence[int]
                                    ) -> tuple[list[list[int]], list[list[int]]]:
        """Logical rows of ``history_modality_parts``: per selected block its audio rows and
        its video rows (blocks without rows of a kind contribute no part)."""

        self._require_valid()
        offsets = self._block_offsets()
        audio: list[list[int]] = []
        video: list[list[int]] = []
        for b in block_indices:
            start, tags = offsets[b], self._commit_token_tags[b]
            for tag, parts in ((AUDIO_TOKEN_TAG, audio), (VIDEO_TOKEN_TAG, video)):
                rows = [start + i for i, t in enumerate(tags) if t == tag]
                if rows:
                    parts.append(rows)
        return audio, video

    def history_modality_parts(self, layer_name: str, block_indices: Sequence[int]
                               ) -> tuple[tuple[tuple[torch.Tensor, torch.Tensor], ...],
                                          tuple[tuple[torch.Tensor, torch.Tensor], ...]]:
        """The selected blocks' history as exact audio and routable video (key, value) parts
        for SOL-Attn (F/streaming/cache.py:439-475)."""

        _validate_layer_name(layer_name, self.layer_names)
        audio, video = self.history_modality_parts_rows(block_indices)
        views = lambda parts: tuple((v.key, v.value) for v in  # noqa: E731
                                    (self._rows_view(layer_name, rows) for rows in parts))
        return views(audio), views(video)

    def sol_history_modality_parts(self, layer_name: str, *, fused_current: bool,
                                   use_sink: bool = False, recent_blocks: int | None = None):
        """``history_modality_parts`` over every retained block, or in a fused forward's
        current document the sink and recent window (F/streaming/cache.py:477-499)."""

        retained = self.retained_blocks
        if retained == 0:
            return (), ()
        if fused_current and recent_blocks is not None:
            recent = max(0, recent_blocks - 1)
            if use_sink:
                blocks = (0, *range(max(1, retained - recent), retained))
            else:
                blocks = tuple(range(max(0, retained - recent), retained))
        else:
            blocks = tuple(range(retained))
        return self.history_modality_parts(layer_name, blocks)

    def recent_history(self, layer_name: str, count: int) -> AVKV | None:
        """The newest ``count`` blocks (F/streaming/cache.py:287-300)."""

        if isinstance(count, bool) or not isinstance(count, int) or count < 0:
            raise ValueError("recent H3 history count must be non-negative")
        self._require_valid()
        _validate_layer_name(layer_name, self.layer_names)
        if count == 0 or not self._commit_token_counts:
            return None
        offsets = self._block_offsets()
        first = max(0, len(self._commit_token_counts) - count)
        return self._rows_view(layer_name, list(range(offsets[first], offsets[-1])))

    def sink_and_recent_history(self, layer_name: str, recent_count: int) -> AVKV | None:
        """Block 0 plus the newest ``recent_count`` other blocks (F/streaming/cache.py:302-342)."""

        if isinstance(recent_count, bool) or not isinstance(recent_count, int) or recent_count < 0:
            raise ValueError("recent H3 history count must be non-negative")
        self._require_valid()
        _validate_layer_name(layer_name, self.layer_names)
        blocks = len(self._commit_token_counts)
        if blocks == 0:
            return None
        offsets = self._block_offsets()
        start = max(1, blocks - recent_count)
        rows = list(range(offsets[0], offsets[1])) + list(range(offsets[start], offsets[-1]))
        return self._rows_view(layer_name, rows)

    def history_for_fused_current_rows(self, *, use_sink: bool = False,
                                       recent_blocks: int | None = None) -> list[int] | None:
        """Logical history rows of ``history_for_fused_current`` (None: no history)."""

        self._require_valid()
        offsets = self._block_offsets()
        blocks = len(self._commit_token_counts)
        if blocks == 0:
            return None
        if recent_blocks is None:
            return list(range(offsets[-1]))
        persistent_recent = max(0, recent_blocks - 1)
        if not use_sink:
            if persistent_recent == 0:
                return None
            first = max(0, blocks - persistent_recent)
            return list(range(offsets[first], offsets[-1]))
        start = max(1, blocks - persistent_recent)
        sink_tags = self._commit_token_tags[0]
        if (self._sink_video_only and self.retained_blocks + 1 > recent_blocks
                and AUDIO_TOKEN_TAG in sink_tags):
            # the pending document ages the sink out of the recent window: its audio rows go
            sink = [row for row, tag in enumerate(sink_tags) if tag == VIDEO_TOKEN_TAG]
        else:
            sink = list(range(offsets[1]))
        return sink + list(range(offsets[start], offsets[-1]))

    def history_for_fused_current(self, layer_name: str, *, use_sink: bool = False,
                                  recent_blocks: int | None = None) -> AVKV | None:
        """The persistent part a fused forward's current document sees: all history, or
        with ``recent_blocks`` one recent slot fewer (the packed previous document supplies
        the newest block), optionally with the sink (F/streaming/cache.py:368-407)."""

        _validate_layer_name(layer_name, self.layer_names)
        rows = self.history_for_fused_current_rows(use_sink=use_sink, recent_blocks=recent_blocks)
        return None if not rows else self._rows_view(layer_name, rows)

    def attention_history_rows(self, *, count: int, recent_full_blocks: int,
                               older_video_stride: int, preserve_sink: bool = False) -> list[int] | None:
        """Logical history rows of ``attention_history``, in order (None: no history)."""

        if recent_full_blocks < 0 or older_video_stride < 1:
            raise ValueError("invalid H3 attention-history policy")
        self._require_valid()
        n = len(self._commit_token_counts)
        if n == 0 or count <= 0:
            return None
        if preserve_sink:
            blocks = [0, *range(max(1, n - max(0, count - 1)), n)]
        else:
            blocks = list(range(max(0, n - count), n))
        offsets = self._block_offsets()
        dense = older_video_stride == 1 or recent_full_blocks >= len(blocks)
        dense_start = max(0, len(blocks) - recent_full_blocks)
        rows: list[int] = []
        for position, block in enumerate(blocks):
            start, tags = offsets[block], self._commit_token_tags[block]
            if dense or position >= dense_start:
                rows.extend(range(start, start + len(tags)))
                continue
            ordinal = 0
            for i, tag in enumerate(tags):
                if tag == AUDIO_TOKEN_TAG:
                    rows.append(start + i)
                elif tag == VIDEO_TOKEN_TAG:
                    if ordinal % older_video_stride == 0:
                        rows.append(start + i)
                    ordinal += 1
        return rows

    def history_for_attention_rows(self, *, fused_current: bool, recent_full_blocks: int,
                                   older_video_stride: int, use_sink: bool = False,
                                   recent_blocks: int | None = None) -> list[int] | None:
        """Logical rows of ``history_for_attention`` (None: no history)."""

        retained = self.retained_blocks
        if fused_current and recent_blocks is not None:
            retained_recent = max(0, recent_blocks - 1)
            count = min(retained, (1 if use_sink and retained else 0) + retained_recent)
            recent_full_blocks = max(0, recent_full_blocks - 1)
        else:
            count = retained
        return self.attention_history_rows(count=count, recent_full_blocks=recent_full_blocks,
                                           older_video_stride=older_video_stride,
                                           preserve_sink=use_sink)

    def history_for_attention(self, layer_name: str, *, fused_current: bool,
                              recent_full_blocks: int, older_video_stride: int,
                              use_sink: bool = False,
                              recent_blocks: int | None = None) -> AVKV | None:
        """History for dense-recent / sparse-older attention: every block, or in a fused
        forward's current document the sink and recent window, with the older blocks' video
        rows strided (F/streaming/cache.py:409-437)."""

        _validate_layer_name(layer_name, self.layer_names)
        rows = self.history_for_attention_rows(
            fused_current=fused_current, recent_full_blocks=recent_full_blocks,
            older_video_stride=older_video_stride, use_sink=use_sink, recent_blocks=recent_blocks)
        return None if not rows else self._rows_view(layer_name, rows)

    def attention_history(self, layer_name: str, *, count: int, recent_full_blocks: int,
                          older_video_stride: int, preserve_sink: bool = False) -> AVKV | None:
        """Dense recent blocks and structured-sparse older video rows (every audio row and
        every ``older_video_stride``-th video row of the older blocks) of the newest ``count``
        blocks, or of block 0 plus the newest ``count - 1`` (F/streaming/cache.py:501-575)."""

        _validate_layer_name(layer_name, self.layer_names)
        rows = self.attention_history_rows(count=count, recent_full_blocks=recent_full_blocks,
                                           older_video_stride=older_video_stride,
                                           preserve_sink=preserve_sink)
        return None if rows is None else self._rows_view(layer_name, rows)

    def advance_serial_without_history_commit(self, block_index: int) -> None:
        """Close one generated block without committing it (F/streaming/cache.py:1111-1122)."""

        if self.clean_commit_active:
            raise RuntimeError("cannot advance H3 serial during a clean commit")
        if block_index != self._block_index:
            raise ValueError(f"clean block order mismatch: expected {self._block_index}, "
                             f"got {block_index}")
        self._block_index += 1

    def discard_retained_history_preserve_serial(self) -> int:
        """Drop the retained history, keep the logical chunk count (F/streaming/cache.py:1123-1138)."""

        if self.clean_commit_active:
            raise RuntimeError("cannot discard H3 history during a clean commit")
        removed = self.history_tokens
        for paged in self._layers.values():
            paged.release()
            if paged.fp8 is not None:
                paged.fp8.release()
        self._commit_token_counts.clear()
        self._commit_token_tags.clear()
        return removed

    def clear(self) -> None:
        """Clear persistent and staged KV and reset the logical chunk count."""

        for paged in self._layers.values():
            paged.release()
            if paged.fp8 is not None:
                paged.fp8.release()
        self._commit_token_counts.clear()
        self._commit_token_tags.clear()
        self._block_index = 0
        self._clear_staging()
        self._invalid_after_failed_commit = False
        self._sink_video_only = False

    def retained_rows(self, selection: list[tuple[int, bool]]) -> tuple[list[int], list[int], list[tuple[int, ...]]]:
        """Logical rows kept by a ``(commit, video_only)`` selection, with counts and tags."""

        offsets = [0]
        for count in self._commit_token_counts:
            offsets.append(offsets[-1] + count)
        selected_rows: list[int] = []
        selected_counts: list[int] = []
        selected_tags: list[tuple[int, ...]] = []
        for block_index, video_only in selection:
            tags = self._commit_token_tags[block_index]
            start = offsets[block_index]
            local_rows = [i for i, tag in enumerate(tags) if not video_only or tag == VIDEO_TOKEN_TAG]
            if not local_rows:
                continue
            selected_rows.extend(start + row for row in local_rows)
            kept_tags = tuple(tags[row] for row in local_rows)
            selected_counts.append(len(kept_tags))
            selected_tags.append(kept_tags)
        return selected_rows, selected_counts, selected_tags

    def _retain_commit_rows(self, selection: list[tuple[int, bool]]) -> None:
        selected_rows, selected_counts, selected_tags = self.retained_rows(selection)
        if not selected_rows:
            for paged in self._layers.values():
                paged.release()
                if paged.fp8 is not None:
                    paged.fp8.release()
            self._commit_token_counts.clear()
            self._commit_token_tags.clear()
            return
        rows = torch.tensor(selected_rows, dtype=torch.int32)
        parts = [(block, [i for i, tag in enumerate(self._commit_token_tags[block])
                          if not video_only or tag == VIDEO_TOKEN_TAG])
                 for block, video_only in selection]
        for paged in self._layers.values():
            if paged.history_rows:
                paged.gather(rows)
            if paged.fp8 is not None and paged.fp8.starts:
                paged.fp8.retain(parts)
                paged.fp8.refresh_summaries(paged.key, paged.table)
        self._commit_token_counts = selected_counts
        self._commit_token_tags = selected_tags

    def _clear_staging(self) -> None:
        self._staged.clear()
        self._staged_block = None
        self._staged_tags = None
        self._staged_indices = None


__all__ = [
    "AUDIO_TOKEN_TAG",
    "AVKV",
    "TemporaryAVPrefix",
    "TemporaryVideoPrefix",
    "VideoKV",
    "CleanAVKVCache",
    "KVContract",
    "MAIN_LAYER_NAMES",
    "PagedLayerKV",
    "VIDEO_TOKEN_TAG",
    "kv_contract_from_model",
]
