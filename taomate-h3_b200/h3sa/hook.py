"""Streaming attention hook with the reference's call protocol, on the sm_100a kernels.

Mirrors ``H3StreamingAttentionHook`` (T/streaming/attention_hook.py:39-252): the same
keyword call, validation order and messages, live-document rule, modes and receipt
counters. Per packed document the visibility is unchanged:

* the live document's condition (text) rows attend to condition K/V only;
* its media rows attend to [condition, persistent clean AV history, current media];
* every other (pad) document attends to itself.

What changes is the data path. Instead of ``index_select`` + ``torch.cat`` of the whole
history and one FlashAttention-3 launch per part, the hook writes the current media,
condition and other-document K/V rows into the layer's page sequence right after the
persistent history::

    logical KV rows: [history | media | condition | other documents]

and runs every document's attention in one kernel launch over that sequence. In
CLEAN_COMMIT mode the media rows written there are exactly the rows the cache stages, so
the commit needs no further copy.

Backends (``attention_backend``): ``"flash_attn_3"``/``"flash_attn3"``/``"sdpa"`` (dense
bf16), ``"flash_attn3_fp8_dynamic"`` (per-call per-head e4m3 Q/K/V,
F/streaming/attention_hook.py:1081-1098), ``"flash_attn3_fp8_segmented"`` (e4m3 history
parts quantised once at commit, :1015-1066), ``"flash_attn3_fp8_segmented_topk"`` (the same
over the committed blocks whose key summaries score highest against the media queries,
:1256-1302) and ``"flex_dynamic_blocksparse"`` (history block top-k,
F/inference/dynamic_block_sparse.py:50-172).
"""

from __future__ import annotations

from enum import Enum
from typing import Sequence

import torch

from . import _lib
from .cache import CleanAVKVCache
from .kernels import PAGE_ROWS
from .kernels import (AttentionProblem, attention_fwd, attention_fwd_fp8_parts, kv_copy_rows,
                      quantize_fp8_e4m3_per_head, quantize_fp8_pool)
from .peer import attention_fwd_scatter

DENSE_BACKENDS = ("flash_attn_3", "flash_attn3", "sdpa", "h3sa_dense")
FP8_BACKENDS = ("flash_attn3_fp8_dynamic", "flash_attn3_fp8_segmented",
                "flash_attn3_fp8_segmented_topk")
SEGMENTED_BACKENDS = ("flash_attn3_fp8_segmented", "flash_attn3_fp8_segmented_topk")
SPARSE_BACKENDS = ("flex_dynamic_blocksparse",)


class HookMode(str, Enum):
    IDLE = "idle"
    NOISY = "noisy"
    CLEAN_COMMIT = "clean_commit"


def _live_documents_from_mask(commit_mask: torch.Tensor,
                              boundaries: Sequence[tuple[int, int]]) -> tuple[int, ...]:
    """Documents holding any committed row (T/streaming/attention_hook.py:28-36)."""

    live: list[int] = []
    for document_index, (start, stop) in enumerate(boundaries):
        if bool(commit_mask[start:stop].any().item()):
            live.append(document_index)
    return tuple(live)


def _live_documents_from_mask_or_hint(commit_mask: torch.Tensor,
                                      boundaries: Sequence[tuple[int, int]],
                                      live_documents_hint: tuple[int, ...] | None) -> tuple[int, ...]:
    """The FL2AV form: a caller that knows the live documents passes them and the commit mask
    is not read for it (F/streaming/attention_hook.py:337-371, same checks and messages)."""

    if live_documents_hint is None:
        return _live_documents_from_mask(commit_mask, boundaries)
    if not isinstance(live_documents_hint, tuple):
        raise TypeError("live document hint must be a tuple")
    count = len(boundaries)
    if any(isinstance(i, bool) or not isinstance(i, int) or i < 0 or i >= count
           for i in live_documents_hint):
        raise ValueError("live document hint contains an invalid document index")
    if tuple(sorted(set(live_documents_hint))) != live_documents_hint:
        raise ValueError("live document hint must be sorted and unique")
    if any(boundaries[i][0] == boundaries[i][1] for i in live_documents_hint):
        raise ValueError("live document hint references an empty document")
    return live_documents_hint


def _as_range(indices: torch.Tensor) -> tuple[int, int] | None:
    """(first, stop) when the sorted host index list is one contiguous run."""

    n = int(indices.numel())
    if n == 0:
        return None
    first = int(indices[0])
    last = int(indices[-1])
    return (first, last + 1) if last - first + 1 == n else None


class _DocumentPlan:
    """Row bookkeeping of one activation, resolved on the first layer call."""

    def __init__(self, boundaries: tuple[tuple[int, int], ...], live: int,
                 commit_mask_host: torch.Tensor, device: torch.device) -> None:
        start, stop = boundaries[live]
        media_mask = commit_mask_host[start:stop]
        cond = torch.nonzero(~media_mask, as_tuple=False).flatten() + start
        media = torch.nonzero(media_mask, as_tuple=False).flatten() + start
        if cond.numel() == 0 or media.numel() == 0:
            raise RuntimeError("live streaming document must contain condition and media rows")
        self.boundaries = boundaries
        self.live = live
        self.n_cond = int(cond.numel())
        self.n_media = int(media.numel())
        self.cond_range = _as_range(cond)
        self.media_range = _as_range(media)
        self.cond_index = cond.to(device=device, dtype=torch.int32)
        self.media_index = media.to(device=device, dtype=torch.int32)
        self.others = [(a, b) for i, (a, b) in enumerate(boundaries) if i != live and b > a]


class H3StreamingAttentionHook:
    """Condition current media on text, persistent clean AV KV, and current KV."""

    def __init__(self, cache: CleanAVKVCache, *, backend: str = "flash_attn_3",
                 history_density: float = 0.5, attention_backend: str | None = None,
                 history_kv_dynamic_density: float | None = None) -> None:
        # the FL2AV constructor's names for the same two knobs (F/streaming/attention_hook.py:377-394)
        if attention_backend is not None:
            backend = attention_backend
        if history_kv_dynamic_density is not None:
            history_density = history_kv_dynamic_density
        if backend not in DENSE_BACKENDS + FP8_BACKENDS + SPARSE_BACKENDS:
            raise ValueError(f"unsupported H3 streaming attention backend: {backend}")
        if not 0.0 < history_density <= 1.0:
            raise ValueError("dynamic history KV density must be in (0, 1]")
        self.cache = cache
        self.backend = backend
        self.history_density = float(history_density)
        self.kernel_calls = 0
        self.query_tokens = 0
        self.key_tokens = 0
        self.launches = 0
        # commit-level top-k counters (F/streaming/attention_hook.py:1292-1298)
        self.dynamic_block_sparse_call_count = 0
        self.dynamic_block_sparse_selected_blocks = 0
        self.dynamic_block_sparse_history_blocks = 0
        self.mode = HookMode.IDLE
        self._plan: _DocumentPlan | None = None
        self._plan_key: tuple[int, ...] | None = None
        self._device_error: torch.Tensor | None = None
        self._fp8_pools: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
        # Set by h3sa.layer for a call whose heads -> sequence exchange is peer stores: the
        # attention epilogue then writes every output row into its owner's sequence shard
        # (last_output_exchanged tells the caller whether that happened).
        self.output_exchange = None
        self.last_output_exchanged = False

    def receipt(self) -> dict[str, object]:
        return {
            "backend": f"h3sa_sm100a_{self.backend}",
            "tensor_layout": "NHD",
            "is_causal": False,
            "kernel_calls": self.kernel_calls,
            "query_tokens": self.query_tokens,
            "key_tokens": self.key_tokens,
            "launches": self.launches,
        }

    @property
    def active(self) -> bool:
        return self.mode is not HookMode.IDLE

    def activate(self, mode: HookMode) -> None:
        if self.active:
            raise RuntimeError("streaming attention hook is already active")
        if mode not in (HookMode.NOISY, HookMode.CLEAN_COMMIT):
            raise ValueError(f"unsupported streaming hook mode: {mode}")
        self.mode = mode
        self._plan = None
        self._plan_key = None

    def deactivate(self) -> None:
        self.mode = HookMode.IDLE
        self._plan = None
        self._plan_key = None

    def device_error(self, device: torch.device) -> torch.Tensor:
        if self._device_error is None or self._device_error.device != device:
            self._device_error = torch.zeros(1, dtype=torch.int32, device=device)
        return self._device_error

    def check_device_error(self) -> None:
        """Raise if any kernel of this hook reported a device-side failure (synchronises)."""

        if self._device_error is not None:
            code = int(self._device_error.item())
            if code:
                raise RuntimeError(f"h3sa device error flags {code:#x}")

    def _validate_qkv(self, layer_name: str, query: torch.Tensor, key: torch.Tensor,
                      value: torch.Tensor) -> None:
        contract = self.cache.contract
        expected_tail = (contract.local_heads, contract.head_dim)
        if query.shape != key.shape or value.shape != key.shape or key.ndim != 3:
            raise RuntimeError(f"{layer_name}: query/key/value must have matching rank-3 shapes")
        if tuple(key.shape[1:]) != expected_tail:
            raise RuntimeError(
                f"{layer_name}: expected local attention tail {expected_tail}, "
                f"got {tuple(key.shape[1:])}"
            )
        if query.dtype != contract.dtype or key.dtype != contract.dtype or value.dtype != contract.dtype:
            raise RuntimeError(f"{layer_name}: streaming attention requires {contract.dtype} QKV")
        if (query.device.type != contract.device_type or key.device.type != contract.device_type
                or value.device.type != contract.device_type):
            raise RuntimeError(f"{layer_name}: streaming attention requires {contract.device_type} QKV")

    def _resolve_plan(self, boundaries: tuple[tuple[int, int], ...],
                      commit_mask: torch.Tensor, device: torch.device,
                      live_documents_hint: tuple[int, ...] | None = None) -> _DocumentPlan:
        points = tuple(b for _, b in boundaries)
        if self._plan is not None and self._plan_key == points:
            return self._plan
        live = _live_documents_from_mask_or_hint(commit_mask, boundaries, live_documents_hint)
        if len(live) != 1:
            raise RuntimeError(f"direct streaming expects exactly one live document, got {live}")
        plan = _DocumentPlan(boundaries, live[0], commit_mask.detach().to("cpu", torch.bool), device)
        self._plan, self._plan_key = plan, points
        return plan

    def __call__(self, *, attention: object, layer_name: str, query: torch.Tensor,
                 key: torch.Tensor, value: torch.Tensor, token_tags: torch.Tensor,
                 commit_mask: torch.Tensor, cu_seqlens_host: Sequence[int] | None = None,
                 cu_seqlens: torch.Tensor | None = None, max_seqlen: int | None = None,
                 live_documents_hint: tuple[int, ...] | None = None) -> torch.Tensor:
        """The T call (T/streaming/attention_hook.py:118-129) or the FL2AV one
        (F/streaming/attention_hook.py:739-753): ``cu_seqlens`` (device) stands in for
        ``cu_seqlens_host`` when that is None, ``max_seqlen`` is not needed, and
        ``live_documents_hint`` names the live document without reading the commit mask."""

        del max_seqlen
        if not self.active:
            raise RuntimeError("streaming attention hook was called while inactive")
        self._validate_qkv(layer_name, query, key, value)
        if commit_mask.ndim != 1 or commit_mask.shape[0] != query.shape[0]:
            raise RuntimeError(f"{layer_name}: commit_mask does not match packed QKV rows")
        if token_tags.ndim != 1 or token_tags.shape[0] != query.shape[0]:
            raise RuntimeError(f"{layer_name}: token_tags does not match packed QKV rows")
        if cu_seqlens_host is None:
            if cu_seqlens is None:
                raise RuntimeError(f"{layer_name}: packed sequence boundaries are missing")
            cu_seqlens_host = cu_seqlens.tolist()
        points = tuple(int(point) for point in cu_seqlens_host)
        if (len(points) < 2 or points[0] != 0 or points[-1] != query.shape[0]
                or any(left > right for left, right in zip(points, points[1:]))):
            raise RuntimeError(f"{layer_name}: invalid packed sequence boundaries")
        boundaries = tuple(zip(points[:-1], points[1:]))
        plan = self._resolve_plan(boundaries, commit_mask, query.device, live_documents_hint)
        scale = float(getattr(attention, "softmax_scale"))

        query = query.contiguous()
        key = key.contiguous()
        value = value.contiguous()
        paged = self.cache.layer(layer_name, query.device)
        err = self.device_error(query.device)
        n_hist = paged.history_rows
        m0 = n_hist
        c0 = m0 + plan.n_media
        o0 = c0 + plan.n_cond

        # 1. current K/V rows into the tail of the layer's page sequence
        if plan.media_range is not None:
            paged.write(key, value, start=m0, count=plan.n_media, src_start=plan.media_range[0])
        else:
            paged.write(key, value, start=m0, count=plan.n_media, src_index=plan.media_index)
        if plan.cond_range is not None:
            paged.write(key, value, start=c0, count=plan.n_cond, src_start=plan.cond_range[0])
        else:
            paged.write(key, value, start=c0, count=plan.n_cond, src_index=plan.cond_index)
        other_kv: list[tuple[int, int, int]] = []
        cursor = o0
        for a, b in plan.others:
            paged.write(key, value, start=cursor, count=b - a, src_start=a)
            other_kv.append((a, b, cursor))
            cursor += b - a

        # 2. attention problems over packed query rows (gathered when not contiguous)
        out = torch.empty_like(query)
        q_src = query
        media_q = plan.media_range
        cond_q = plan.cond_range
        gathered = None
        if media_q is None or cond_q is None:
            gathered = torch.empty(plan.n_media + plan.n_cond, *query.shape[1:], dtype=query.dtype,
                                   device=query.device)
            kv_copy_rows([query], [gathered], count=plan.n_media, src_index=plan.media_index)
            kv_copy_rows([query], [gathered], count=plan.n_cond, src_index=plan.cond_index,
                         dst_start=plan.n_media)
            q_src = gathered
            media_q = (0, plan.n_media)
            cond_q = (plan.n_media, plan.n_media + plan.n_cond)
        n_kv_media = o0  # history + media + condition
        media_problem = AttentionProblem(media_q[0], media_q[1], 0, n_kv_media,
                                         sparse=self.backend in SPARSE_BACKENDS)
        cond_problem = AttentionProblem(cond_q[0], cond_q[1], c0, o0)
        out_main = out if gathered is None else torch.empty_like(gathered)
        # rows stored straight into the owners' sequence shards when the output rows are the
        # query rows (no gather) and the launch is bf16
        exchange = self.output_exchange
        if exchange is not None and (gathered is not None or self.backend in FP8_BACKENDS):
            exchange = None
        self.last_output_exchanged = exchange is not None
        self._launch(layer_name, paged, q_src, out_main, [media_problem, cond_problem], scale,
                     n_kv_media, n_hist, plan, err, exchange)
        if other_kv:
            probs = [AttentionProblem(a, b, c, c + (b - a)) for a, b, c in other_kv]
            for i in range(0, len(probs), _lib.MAX_PROBLEMS):
                chunk = probs[i:i + _lib.MAX_PROBLEMS]
                if exchange is not None:
                    attention_fwd_scatter(query, paged.key, paged.value, paged.table, chunk, scale,
                                          exchange.out, device_error=err)
                else:
                    attention_fwd(query, out, paged.key, paged.value, paged.table, chunk, scale,
                                  device_error=err)
                self.launches += 1
        if gathered is not None:
            kv_copy_rows([out_main], [out], count=plan.n_media, src_start=0,
                         dst_index=plan.media_index)
            kv_copy_rows([out_main], [out], count=plan.n_cond, src_start=plan.n_media,
                         dst_index=plan.cond_index)

        self.kernel_calls += 2 + len(other_kv)
        self.query_tokens += int(query.shape[0])
        self.key_tokens += n_kv_media + plan.n_cond + sum(b - a for a, b, _ in other_kv)

        if self.mode is HookMode.CLEAN_COMMIT:
            self.cache.stage_in_place(layer_name, key, value, token_tags, commit_mask)
        return out

    # ------------------------------------------------------------------ launches
    def _launch(self, layer_name: str, paged, q_src: torch.Tensor, out: torch.Tensor,
                problems: list[AttentionProblem], scale: float, n_kv: int, n_hist: int,
                plan: _DocumentPlan, err: torch.Tensor, exchange=None) -> None:
        if self.backend in SEGMENTED_BACKENDS:
            self._launch_fp8_segmented(paged, q_src, out, problems, scale, n_hist, err)
            return
        if self.backend in FP8_BACKENDS:
            self._launch_fp8(layer_name, paged, q_src, out, problems, scale, n_kv, err)
            return
        lists = {}
        if self.backend in SPARSE_BACKENDS:
            from .block_sparse import history_block_lists

            lists = history_block_lists(q_src, problems[0], paged, n_hist=n_hist, n_kv=n_kv,
                                        density=self.history_density, scale=scale)
            if not lists:
                problems = [AttentionProblem(p.q_lo, p.q_hi, p.kv_lo, p.kv_hi) for p in problems]
        if exchange is not None:
            attention_fwd_scatter(q_src, paged.key, paged.value, paged.table, problems, scale,
                                  exchange.out, device_error=err, **lists)
        else:
            attention_fwd(q_src, out, paged.key, paged.value, paged.table, problems, scale,
                          device_error=err, **lists)
        self.launches += 1

    def _launch_fp8(self, layer_name: str, paged, q_src: torch.Tensor, out: torch.Tensor,
                    problems: list[AttentionProblem], scale: float, n_kv: int,
                    err: torch.Tensor) -> None:
        media, cond = problems
        pools = self._fp8_pools.get(layer_name)
        if pools is None or pools[0].shape != paged.key.shape:
            pools = (torch.zeros_like(paged.key, dtype=torch.float8_e4m3fn),
                     torch.zeros_like(paged.value, dtype=torch.float8_e4m3fn))
            self._fp8_pools[layer_name] = pools
        k8, v8 = pools
        heads = paged.heads
        k_scale = torch.empty(heads, dtype=torch.float32, device=q_src.device)
        v_scale = torch.empty_like(k_scale)
        quantize_fp8_pool(paged.key, k8, k_scale, paged.table, n_kv, device_error=err)
        quantize_fp8_pool(paged.value, v8, v_scale, paged.table, n_kv, device_error=err)
        q_media = q_src[media.q_lo:media.q_hi].unsqueeze(0)
        q8, q_scale = quantize_fp8_e4m3_per_head(q_media)
        out_media = torch.empty(media.q_hi - media.q_lo, *q_src.shape[1:], dtype=torch.bfloat16,
                                device=q_src.device)
        attention_fwd(q8.squeeze(0), out_media, k8, v8, paged.table,
                      [AttentionProblem(0, media.q_hi - media.q_lo, media.kv_lo, media.kv_hi)],
                      scale, q_scale=q_scale.reshape(-1).contiguous(), k_scale=k_scale,
                      v_scale=v_scale, device_error=err)
        out[media.q_lo:media.q_hi].copy_(out_media)
        # condition rows attend to condition K/V only; that tiny call stays in bf16
        attention_fwd(q_src, out, paged.key, paged.value, paged.table, [cond], scale,
                      device_error=err)
        self.launches += 2


    def _launch_fp8_segmented(self, paged, q_src: torch.Tensor, out: torch.Tensor,
                              problems: list[AttentionProblem], scale: float, n_hist: int,
                              err: torch.Tensor) -> None:
        """The segmented FP8 backend (F/streaming/attention_hook.py:1015-1066): every committed
        history block is a part with the scales it was given at commit; the current media rows
        and the condition rows are quantised now, each as a part of its own; one launch
        attends over all parts with their own dequantisation (no LSE merge needed)."""

        seg = paged.fp8
        if seg is None:
            raise RuntimeError("segmented FP8 attention needs a cache built with "
                               "segmented_fp8_history=True")
        media, cond = problems
        heads = paged.heads
        n_media = media.q_hi - media.q_lo
        n_cond = cond.kv_hi - cond.kv_lo
        n_parts = len(seg.starts)
        ks = torch.empty(n_parts + 2, heads, dtype=torch.float32, device=q_src.device)
        vs = torch.empty_like(ks)
        if n_parts:
            ks[:n_parts].copy_(seg.k_scale)
            vs[:n_parts].copy_(seg.v_scale)
        # current media rows [n_hist, n_hist + n_media) and condition rows [cond.kv_lo, ...) of
        # the bf16 page sequence -> e4m3 parts after the history parts
        m0 = seg.append_part(paged.key, paged.value, src_start=n_hist, count=n_media,
                             src_table=paged.table, k_scale=ks[n_parts], v_scale=vs[n_parts])
        c0 = (m0 + n_media + PAGE_ROWS - 1) // PAGE_ROWS * PAGE_ROWS
        seg.append_part(paged.key, paged.value, src_start=cond.kv_lo, count=n_cond,
                        src_table=paged.table, k_scale=ks[n_parts + 1],
                        v_scale=vs[n_parts + 1], start=c0)
        selected = self._select_commits(seg, q_src, media, err)
        if selected is None:
            table = seg.store.table
            block_part = seg.block_part([(m0, n_media), (c0, n_cond)])
            kv_end = c0 + n_cond
        else:
            table, block_part, kv_end = seg.subset_tables(
                selected, [(n_parts, m0, n_media), (n_parts + 1, c0, n_cond)])
        q8, q_scale = quantize_fp8_e4m3_per_head(q_src[media.q_lo:media.q_hi].unsqueeze(0))
        out_media = torch.empty(n_media, *q_src.shape[1:], dtype=torch.bfloat16,
                                device=q_src.device)
        attention_fwd_fp8_parts(q8.squeeze(0), out_media, seg.store.key, seg.store.value,
                                table, [AttentionProblem(0, n_media, 0, kv_end)],
                                scale, q_scale=q_scale.reshape(-1).contiguous(),
                                block_part=block_part, part_k_scale=ks, part_v_scale=vs,
                                device_error=err)
        out[media.q_lo:media.q_hi].copy_(out_media)
        # condition rows attend to condition K/V only; that small call stays in bf16
        attention_fwd(q_src, out, paged.key, paged.value, paged.table, [cond], scale,
                      device_error=err)
        self.launches += 2

    def _select_commits(self, seg, q_src: torch.Tensor, media: AttentionProblem,
                        err: torch.Tensor) -> list[int] | None:
        """Commit-level top-k of the segmented backend (F/streaming/attention_hook.py:1256-1302):
        keep max(1, min(n, ceil(n * density))) committed blocks, those whose key summaries
        have the highest mean-over-heads dot product with the media queries' mean row, in
        commit order. None: attend to every committed block."""

        import math

        from .kernels import commit_scores, segment_row_means

        n = len(seg.starts)
        if self.backend != "flash_attn3_fp8_segmented_topk" or n == 0:
            return None
        count = max(1, min(n, math.ceil(n * self.history_density)))
        self.dynamic_block_sparse_call_count += 1
        self.dynamic_block_sparse_history_blocks += n
        self.dynamic_block_sparse_selected_blocks += count
        if count >= n:
            return None
        q_mean = segment_row_means(q_src, [(media.q_lo, media.q_hi - media.q_lo)],
                                   device_error=err)
        # the reference reads its selection back to the host (.tolist()); so does this
        scores = commit_scores(seg.key_summary, q_mean[0]).cpu().tolist()
        order = sorted(range(n), key=lambda i: (-scores[i], i))  # equal scores: older first
        return sorted(order[:count])


__all__ = ["H3StreamingAttentionHook", "HookMode"]
