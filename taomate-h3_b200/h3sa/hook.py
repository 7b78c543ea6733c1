"""Streaming attention hook with the reference's call protocol, on the sm_100a kernels.

Mirrors ``H3StreamingAttentionHook`` in both of its forms: the T hook
(T/streaming/attention_hook.py:39-252: ``activate(mode)``, NOISY / CLEAN_COMMIT) and the
FL2AV one (F/streaming/attention_hook.py:373-1593: ``activate(*, mode, block_index,
full_prefix, ...)``, the PROGRESS_COMMIT, FUSED_PROGRESS_DENOISE and FULL_PREFIX_CAPTURE
modes, temporary full prefixes), with the same keyword call, validation order and messages,
live-document rule and receipt counters. Per packed document the visibility is unchanged:

* a live document's condition (text) rows attend to its condition K/V only;
* its media rows attend to [condition, temporary prefix, persistent clean AV history,
  current media] (F/streaming/attention_hook.py:193-216); in a fused progress-denoise
  forward the current document sees the fused-current history view plus the previous
  document's media rows instead of the full history, and the previous document is the block
  being committed;
* every other (pad) document attends to itself.

What changes is the data path. Instead of ``index_select`` + ``torch.cat`` of the whole
history and one FlashAttention-3 launch per part, the hook writes each live document's
media, condition and extra K/V rows into the layer's page sequence after the persistent
history::

    logical KV rows: [history | doc A: media, condition, prefix | doc B: ... | others]

so that every query set attends to one contiguous range, and runs the live documents'
attention in one kernel launch. The first live document's media rows sit right after the
history: they are exactly the rows a clean commit stages, so the commit needs no copy.

Backends (``attention_backend``): ``"flash_attn_3"``/``"flash_attn3"``/``"sdpa"`` (dense
bf16), ``"flash_attn3_fp8_dynamic"`` (per-call per-head e4m3 Q/K/V,
F/streaming/attention_hook.py:1081-1098), ``"flash_attn3_fp8_segmented"`` (e4m3 history
parts quantised once at commit, :1015-1066), ``"flash_attn3_fp8_segmented_topk"`` (the same
over the committed blocks whose key summaries score highest against the media queries,
:1256-1302), ``"flex_dynamic_blocksparse"`` (history block top-k,
F/inference/dynamic_block_sparse.py:50-172) and ``"sol_attn"`` (rectangular SOL-Attn routing
of the history video, F/streaming/attention_hook.py:909-991, 1361-1492: dense in the commit
and capture modes, the first ``sol_attn_dense_layers`` layers and the first
``sol_attn_dense_denoise_steps`` denoise steps). The e4m3 and block-sparse backends run the
NOISY / CLEAN_COMMIT / PROGRESS_COMMIT modes without a temporary prefix; fused forwards,
prefix captures and temporary prefixes run on the dense and SOL backends.
"""

from __future__ import annotations

from enum import Enum
from typing import Sequence

import torch

from . import _lib
from .cache import (AUDIO_TOKEN_TAG, VIDEO_TOKEN_TAG, AVKV, CleanAVKVCache, TemporaryAVPrefix,
                    TemporaryVideoPrefix, VideoKV)
from .kernels import PAGE_ROWS
from .kernels import (AttentionProblem, attention_fwd, attention_fwd_fp8_parts, kv_copy_rows,
                      quantize_fp8_e4m3_per_head, quantize_fp8_pool)
from .peer import attention_fwd_scatter

DENSE_BACKENDS = ("flash_attn_3", "flash_attn3", "sdpa", "h3sa_dense")
FP8_BACKENDS = ("flash_attn3_fp8_dynamic", "flash_attn3_fp8_segmented",
                "flash_attn3_fp8_segmented_topk")
SEGMENTED_BACKENDS = ("flash_attn3_fp8_segmented", "flash_attn3_fp8_segmented_topk")
SPARSE_BACKENDS = ("flex_dynamic_blocksparse",)
SOL_BACKENDS = ("sol_attn",)


class HookMode(str, Enum):
    IDLE = "idle"
    NOISY = "noisy"
    CLEAN_COMMIT = "clean_commit"
    PROGRESS_COMMIT = "progress_commit"
    FUSED_PROGRESS_DENOISE = "fused_progress_denoise"
    FULL_PREFIX_CAPTURE = "full_prefix_capture"


_COMMIT_MODES = (HookMode.CLEAN_COMMIT, HookMode.PROGRESS_COMMIT)


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


def _full_prefix_capture_rows(tags: torch.Tensor, commit: torch.Tensor, video_rows: int,
                              audio_rows_per_channel: int | None) -> torch.Tensor:
    """Rows a full-prefix capture keeps: the newest ``video_rows`` committed video rows,
    preceded by the newest ``audio_rows_per_channel`` audio rows of each of the two channels
    (channel-major), F/streaming/attention_hook.py:254-285. Host tensors in and out."""

    video = torch.nonzero(commit & (tags == VIDEO_TOKEN_TAG), as_tuple=False).view(-1)
    if int(video.numel()) < video_rows:
        raise RuntimeError("full-prefix capture contains too few video rows")
    video = video[-video_rows:]
    if audio_rows_per_channel is None:
        return video
    audio = torch.nonzero(commit & (tags == AUDIO_TOKEN_TAG), as_tuple=False).view(-1)
    if int(audio.numel()) % 2:
        raise RuntimeError("full-prefix capture contains incomplete audio channels")
    available = int(audio.numel()) // 2
    if available < audio_rows_per_channel:
        raise RuntimeError("full-prefix capture contains too few audio rows")
    audio = audio.reshape(2, available)[:, -audio_rows_per_channel:].reshape(-1)
    return torch.cat((audio, video))


class _Rows:
    """One set of packed rows: host indices, their device copy, and the run they form."""

    def __init__(self, host: torch.Tensor, device: torch.device) -> None:
        self.host = host
        self.n = int(host.numel())
        self.range = _as_range(host)
        self.index = host.to(device=device, dtype=torch.int32)


class _LiveDoc:
    def __init__(self, index: int, start: int, stop: int, commit_host: torch.Tensor,
                 device: torch.device) -> None:
        media_mask = commit_host[start:stop]
        cond = torch.nonzero(~media_mask, as_tuple=False).flatten() + start
        media = torch.nonzero(media_mask, as_tuple=False).flatten() + start
        if cond.numel() == 0 or media.numel() == 0:
            raise RuntimeError("live streaming document must contain condition and media rows")
        self.index = index
        self.cond = _Rows(cond, device)
        self.media = _Rows(media, device)


class _DocumentPlan:
    """Row bookkeeping of one activation, resolved on the first layer call.

    ``docs``: the live documents in the order their rows follow the history (one; or, in a
    fused forward, the previous document, whose media rows the commit stages, then the
    current one). ``previous_media``: the previous document's media rows the current one
    attends to (video only with ``fused_previous_video_only``)."""

    def __init__(self, boundaries: tuple[tuple[int, int], ...], live: tuple[int, ...],
                 commit_mask_host: torch.Tensor, tags_host: torch.Tensor | None,
                 device: torch.device, previous_video_only: bool = False) -> None:
        self.boundaries = boundaries
        self.live = live
        self.docs = [_LiveDoc(i, *boundaries[i], commit_mask_host, device) for i in live]
        self.others = [(a, b) for i, (a, b) in enumerate(boundaries) if i not in live and b > a]
        self.previous_media: _Rows | None = None
        if len(self.docs) == 2:
            prev = self.docs[0].media.host
            if previous_video_only:
                assert tags_host is not None
                prev = prev[tags_host[prev] == VIDEO_TOKEN_TAG]
            self.previous_media = _Rows(prev, device)


class H3StreamingAttentionHook:
    """Condition current media on text, persistent clean AV KV, and current KV."""

    def __init__(self, cache: CleanAVKVCache, *, backend: str = "flash_attn_3",
                 history_density: float = 0.5, attention_backend: str | None = None,
                 history_kv_dynamic_density: float | None = None, sol_attn_tau: float = 1.0,
                 sol_attn_thresh_type: str = "diag", sol_attn_dense_layers: int = 2,
                 sol_attn_dense_denoise_steps: int = 1,
                 sol_attn_route_current_video: bool = False,
                 sol_attn_static_summary_cache: bool = False,
                 history_kv_recent_full_blocks: int = 5, history_kv_older_video_stride: int = 1,
                 current_video_kv_stride: int = 1,
                 dense_current_document_when_empty: bool = False,
                 direct_sage_kv_workspace: bool = False) -> None:
        # the FL2AV constructor's names for the same two knobs (F/streaming/attention_hook.py:377-394)
        if attention_backend is not None:
            backend = attention_backend
        if history_kv_dynamic_density is not None:
            history_density = history_kv_dynamic_density
        if backend not in DENSE_BACKENDS + FP8_BACKENDS + SPARSE_BACKENDS + SOL_BACKENDS:
            raise ValueError(f"unsupported H3 streaming attention backend: {backend}")
        # SOL-Attn knobs (F/streaming/attention_hook.py:387-434)
        self.sol_attn_tau = float(sol_attn_tau)
        if sol_attn_thresh_type != "diag":
            raise ValueError("SOL-Attn rectangular adapter supports only diag thresholding")
        self.sol_attn_thresh_type = sol_attn_thresh_type
        self.sol_attn_dense_layers = int(sol_attn_dense_layers)
        self.sol_attn_dense_denoise_steps = int(sol_attn_dense_denoise_steps)
        self.sol_attn_route_current_video = bool(sol_attn_route_current_video)
        self.sol_attn_static_summary_cache = bool(sol_attn_static_summary_cache)
        self.sol_attn_kernel_calls = 0
        self.sol_attn_dense_calls = 0
        self.sol_attn_query_tokens = 0
        self.sol_attn_key_tokens = 0
        self._sol_attn_density_counts: torch.Tensor | None = None
        if not 0.0 < history_density <= 1.0:
            raise ValueError("dynamic history KV density must be in (0, 1]")
        # the FL2AV history / current-video policies (F/streaming/attention_hook.py:382-441)
        if current_video_kv_stride < 1:
            raise ValueError("current video KV stride must be positive")
        if history_kv_recent_full_blocks < 0 or history_kv_older_video_stride < 1:
            raise ValueError("invalid H3 attention-history policy")
        if direct_sage_kv_workspace:
            raise ValueError("Direct dense K/V workspace requires SageAttention")
        if dense_current_document_when_empty and current_video_kv_stride != 1:
            raise ValueError(
                "dense current-document compatibility requires current video KV stride 1")
        if ((history_kv_older_video_stride > 1 or current_video_kv_stride > 1)
                and backend not in DENSE_BACKENDS + SOL_BACKENDS):
            raise ValueError(f"the {backend} backend reads the whole history and every current "
                             "row; strided history or current video needs a dense or SOL backend")
        self.history_kv_recent_full_blocks = int(history_kv_recent_full_blocks)
        self.history_kv_older_video_stride = int(history_kv_older_video_stride)
        self.current_video_kv_stride = int(current_video_kv_stride)
        self.dense_current_document_when_empty = bool(dense_current_document_when_empty)
        self.direct_sage_kv_workspace = False
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
        self._fl2av = False  # activated through the FL2AV form
        self.block_index: int | None = None
        self.full_prefix: TemporaryAVPrefix | TemporaryVideoPrefix | None = None
        self.fused_previous_full_prefix: TemporaryAVPrefix | TemporaryVideoPrefix | None = None
        self.fused_previous_video_only = False
        self.fused_current_use_sink: bool | None = None
        self.fused_current_recent_blocks: int | None = None
        self._denoise_step_index: int | None = None
        self._phase_index: int | None = None
        self._capture_video_rows = 0
        self._capture_audio_rows_per_channel: int | None = None
        self._captured_full_prefix_layers: dict[str, AVKV | VideoKV] = {}
        self._capture_index: torch.Tensor | None = None
        self._plan: _DocumentPlan | None = None
        self._plan_key: tuple[int, ...] | None = None
        self._plan_hint: tuple[int, ...] | None = None
        self._device_error: torch.Tensor | None = None
        self._fp8_pools: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
        # Set by h3sa.layer for a call whose heads -> sequence exchange is peer stores: the
        # attention epilogue then writes every output row into its owner's sequence shard
        # (last_output_exchanged tells the caller whether that happened).
        self.output_exchange = None
        self.last_output_exchanged = False

    def sol_attn_receipt(self) -> dict[str, object] | None:
        """Counters of the SOL-Attn backend, with the reference's keys
        (F/streaming/attention_hook.py:496-552). The routing counts come from the device
        telemetry of every SOL call (always collected here); the summaries are rebuilt on
        every call, so the static summary cache counters stay zero."""

        if self.backend not in SOL_BACKENDS:
            return None
        counts = ([0, 0, 0, 0] if self._sol_attn_density_counts is None
                  else [int(x) for x in self._sol_attn_density_counts.detach().cpu().tolist()])
        selected, exact, routable, candidate = counts
        return {
            "backend": "h3sa_sm100a_sol_attn_rectangular",
            "tau": self.sol_attn_tau,
            "thresh_type": self.sol_attn_thresh_type,
            "dense_layers": self.sol_attn_dense_layers,
            "dense_denoise_steps": self.sol_attn_dense_denoise_steps,
            "route_current_video": self.sol_attn_route_current_video,
            "static_summary_cache": self.sol_attn_static_summary_cache,
            "density_telemetry_enabled": True,
            "kernel_calls": self.sol_attn_kernel_calls,
            "dense_calls": self.sol_attn_dense_calls,
            "query_tokens": self.sol_attn_query_tokens,
            "key_tokens": self.sol_attn_key_tokens,
            "static_cache_hits": 0,
            "static_cache_misses": 0,
            "static_summary_reused_blocks": 0,
            "static_summary_built_blocks": 0,
            "dynamic_or_boundary_summary_blocks": 0,
            "route_selected_blocks": selected,
            "exact_blocks": exact,
            "routable_blocks": routable,
            "candidate_blocks": candidate,
            "selected_density": None if routable == 0 else selected / routable,
            "exact_density": None if candidate == 0 else exact / candidate,
            "history_policy": (
                "rectangular_exact_condition_prefix_audio_sparse_current_and_history_video"
                if self.sol_attn_route_current_video
                else "rectangular_exact_condition_current_prefix_audio_sparse_history_video"),
        }

    def sage_attn_receipt(self) -> dict[str, object] | None:
        """The SageAttention backend is not built here (an sm90 library): always None."""

        return None

    def attention_backend_receipt(self) -> dict[str, object] | None:
        """The alternative backend's receipt (F/streaming/attention_hook.py:574-575)."""

        return self.sol_attn_receipt() or self.sage_attn_receipt()

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

    # ------------------------------------------------------------------ modes
    def activate(self, mode: HookMode | None = None, *, block_index: int | None = None,
                 full_prefix: TemporaryAVPrefix | TemporaryVideoPrefix | None = None,
                 fused_previous_full_prefix: TemporaryAVPrefix | TemporaryVideoPrefix | None = None,
                 fused_previous_video_only: bool = False,
                 fused_current_use_sink: bool | None = None,
                 fused_current_recent_blocks: int | None = None,
                 denoise_step_index: int | None = None,
                 phase_index: int | None = None) -> None:
        """``activate(mode)``: the T form (NOISY or CLEAN_COMMIT,
        T/streaming/attention_hook.py:104-116). With ``block_index``: the FL2AV form and its
        checks (F/streaming/attention_hook.py:577-643)."""

        if block_index is None:
            if self.active:
                raise RuntimeError("streaming attention hook is already active")
            if mode not in (HookMode.NOISY, HookMode.CLEAN_COMMIT):
                raise ValueError(f"unsupported streaming hook mode: {mode}")
            self._reset(mode)
            return
        mode = HookMode(mode)
        if self.active:
            raise RuntimeError("H3 streaming attention hook is already active")
        if block_index != self.cache.committed_blocks:
            raise ValueError("streaming attention block differs from clean history")
        if full_prefix is not None and full_prefix.contract != self.cache.contract:
            raise ValueError("temporary prefix and persistent cache contracts differ")
        if (fused_previous_full_prefix is not None
                and fused_previous_full_prefix.contract != self.cache.contract):
            raise ValueError("fused previous prefix and persistent cache contracts differ")
        if fused_previous_full_prefix is not None and mode is not HookMode.FUSED_PROGRESS_DENOISE:
            raise ValueError("fused previous prefix requires fused progress-denoise mode")
        if fused_previous_video_only and mode is not HookMode.FUSED_PROGRESS_DENOISE:
            raise ValueError(
                "fused previous video-only visibility requires fused progress-denoise mode")
        if ((fused_current_use_sink is not None or fused_current_recent_blocks is not None)
                and mode is not HookMode.FUSED_PROGRESS_DENOISE):
            raise ValueError("fused current history policy requires fused progress-denoise mode")
        if denoise_step_index is not None and mode not in (HookMode.NOISY,
                                                            HookMode.FUSED_PROGRESS_DENOISE):
            raise ValueError("denoise step index requires noisy or fused progress-denoise mode")
        if mode in (HookMode.IDLE, HookMode.FULL_PREFIX_CAPTURE):
            raise ValueError(f"{mode.value} is not an activation mode")
        self._require_dense_for(mode is HookMode.FUSED_PROGRESS_DENOISE
                                or full_prefix is not None)
        self._reset(mode)
        self._fl2av = True
        self.block_index = block_index
        self.full_prefix = full_prefix
        self.fused_previous_full_prefix = fused_previous_full_prefix
        self.fused_previous_video_only = bool(fused_previous_video_only)
        self.fused_current_use_sink = fused_current_use_sink
        self.fused_current_recent_blocks = fused_current_recent_blocks
        self._denoise_step_index = denoise_step_index
        self._phase_index = phase_index

    def _require_dense_for(self, extras: bool) -> None:
        if extras and self.backend not in DENSE_BACKENDS + SOL_BACKENDS:
            raise ValueError(f"the {self.backend} backend runs NOISY, CLEAN_COMMIT and "
                             "PROGRESS_COMMIT without a temporary prefix; fused forwards, "
                             "prefix captures and temporary prefixes need a dense backend")

    def _reset(self, mode: HookMode) -> None:
        self.mode = mode
        self._fl2av = False
        self.block_index = None
        self.full_prefix = None
        self.fused_previous_full_prefix = None
        self.fused_previous_video_only = False
        self.fused_current_use_sink = None
        self.fused_current_recent_blocks = None
        self._denoise_step_index = None
        self._phase_index = None
        self._capture_video_rows = 0
        self._capture_audio_rows_per_channel = None
        self._captured_full_prefix_layers = {}
        self._capture_index = None
        self._plan = None
        self._plan_key = None
        self._plan_hint = None

    def deactivate(self) -> None:
        self._reset(HookMode.IDLE)

    def begin_full_prefix_capture(self, *, video_rows: int,
                                  audio_rows_per_channel: int | None = None) -> None:
        """Start a forward whose committed media rows become a temporary full prefix
        (F/streaming/attention_hook.py:658-684): its media attend to the current document
        only, and every layer's selected K/V rows are kept."""

        if self.active:
            raise RuntimeError("H3 streaming attention hook is already active")
        if isinstance(video_rows, bool) or not isinstance(video_rows, int) or video_rows <= 0:
            raise ValueError("full-prefix capture video_rows must be positive")
        if audio_rows_per_channel is not None and (
                isinstance(audio_rows_per_channel, bool)
                or not isinstance(audio_rows_per_channel, int) or audio_rows_per_channel <= 0):
            raise ValueError("full-prefix capture audio_rows_per_channel must be positive")
        self._require_dense_for(True)
        self._reset(HookMode.FULL_PREFIX_CAPTURE)
        self._fl2av = True
        self.block_index = self.cache.committed_blocks
        self._capture_video_rows = video_rows
        self._capture_audio_rows_per_channel = audio_rows_per_channel

    def finish_full_prefix_capture(self) -> TemporaryAVPrefix | TemporaryVideoPrefix:
        """The captured prefix, once every layer has run (F/streaming/attention_hook.py:709-735)."""

        if self.mode is not HookMode.FULL_PREFIX_CAPTURE:
            raise RuntimeError("no H3 full-prefix capture is active")
        layers = self._captured_full_prefix_layers
        names = self.cache.layer_names
        if tuple(layers) != names:
            missing = [name for name in names if name not in layers]
            self.deactivate()
            raise RuntimeError(f"full-prefix capture did not traverse all H3 layers: {missing}")
        audio = self._capture_audio_rows_per_channel
        if audio is None:
            prefix = TemporaryVideoPrefix(layers, contract=self.cache.contract, layer_names=names)
        else:
            prefix = TemporaryAVPrefix(layers, video_token_count=self._capture_video_rows,
                                       audio_token_count_per_channel=audio,
                                       contract=self.cache.contract, layer_names=names)
        self.deactivate()
        return prefix

    def _transient(self, layer_name: str, doc_position: int, fused: bool):
        """The temporary prefix a live document sees: in a fused forward the previous
        document keeps the prefix of its own time (F/streaming/attention_hook.py:686-707)."""

        if self.mode is HookMode.FULL_PREFIX_CAPTURE:
            return None
        prefix = (self.fused_previous_full_prefix if fused and doc_position == 0
                  else self.full_prefix)
        return None if prefix is None else prefix.get(layer_name)

    # ------------------------------------------------------------------ helpers
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
                      commit_mask: torch.Tensor, token_tags: torch.Tensor, device: torch.device,
                      live_documents_hint: tuple[int, ...] | None = None) -> _DocumentPlan:
        points = tuple(b for _, b in boundaries)
        if self._plan is not None:
            if self._plan_key == points:
                if (self._fl2av and live_documents_hint is not None
                        and live_documents_hint != self._plan.live):
                    raise ValueError("live document hint changed within one streaming step")
                return self._plan
            if self._fl2av:
                raise ValueError("packed H3 boundaries changed within one streaming step")
        live = _live_documents_from_mask_or_hint(commit_mask, boundaries, live_documents_hint)
        fused = self.mode is HookMode.FUSED_PROGRESS_DENOISE
        if self._fl2av:
            expected = 2 if fused else 1
            if len(live) != expected:
                raise ValueError("streaming session target-document count differs from hook "
                                 f"mode: expected={expected}, actual={len(live)}")
        elif len(live) != 1:
            raise RuntimeError(f"direct streaming expects exactly one live document, got {live}")
        tags_host = token_tags.detach().to("cpu") if fused else None
        plan = _DocumentPlan(boundaries, live, commit_mask.detach().to("cpu", torch.bool),
                             tags_host, device, self.fused_previous_video_only)
        self._plan, self._plan_key = plan, points
        return plan

    # ------------------------------------------------------------------ the call
    def __call__(self, *, attention: object, layer_name: str, query: torch.Tensor,
                 key: torch.Tensor, value: torch.Tensor, token_tags: torch.Tensor,
                 commit_mask: torch.Tensor, cu_seqlens_host: Sequence[int] | None = None,
                 cu_seqlens: torch.Tensor | None = None, max_seqlen: int | None = None,
                 live_documents_hint: tuple[int, ...] | None = None) -> torch.Tensor:
        """The T call (T/streaming/attention_hook.py:118-129) or the FL2AV one
        (F/streaming/attention_hook.py:739-753): ``cu_seqlens`` (device) stands in for
        ``cu_seqlens_host`` when that is None, ``max_seqlen`` is not needed, and
        ``live_documents_hint`` names the live documents without reading the commit mask."""

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
        plan = self._resolve_plan(boundaries, commit_mask, token_tags, query.device,
                                  live_documents_hint)
        scale = float(getattr(attention, "softmax_scale"))
        fused = self.mode is HookMode.FUSED_PROGRESS_DENOISE
        capture = self.mode is HookMode.FULL_PREFIX_CAPTURE

        query = query.contiguous()
        key = key.contiguous()
        value = value.contiguous()
        paged = self.cache.layer(layer_name, query.device)
        err = self.device_error(query.device)
        n_hist = paged.history_rows

        # 1. K/V rows of every live document into the page sequence after the history
        cursor = n_hist
        regions = []  # per live document: (media kv start, condition start, region end)

        def put_rows(rows: _Rows) -> None:
            nonlocal cursor
            if rows.range is not None:
                paged.write(key, value, start=cursor, count=rows.n, src_start=rows.range[0])
            else:
                paged.write(key, value, start=cursor, count=rows.n, src_index=rows.index)
            cursor += rows.n

        def put_dense(pair) -> None:
            nonlocal cursor
            n = int(pair.key.shape[0])
            paged.write(pair.key.contiguous(), pair.value.contiguous(), start=cursor, count=n)
            cursor += n

        sparse_history = self.history_kv_older_video_stride > 1
        video_stride = self.current_video_kv_stride
        # doc -> (first row, rows, media positions) of its strided current media keys
        selected_media: dict[int, tuple[int, int, torch.Tensor]] = {}

        def copy_rows(rows: list[int]) -> None:
            nonlocal cursor
            if not rows:
                return
            index = torch.tensor(rows, dtype=torch.int32).pin_memory().to(
                query.device, non_blocking=True)
            paged.reserve(cursor + len(rows))
            kv_copy_rows([paged.key, paged.value], [paged.key, paged.value], count=len(rows),
                         src_table=paged.table, dst_table=paged.table, src_index=index,
                         dst_start=cursor)
            cursor += len(rows)

        for position, doc in enumerate(plan.docs):
            first = cursor
            put_rows(doc.media)
            c_start = cursor
            put_rows(doc.cond)
            transient = self._transient(layer_name, position, fused)
            if transient is not None:
                put_dense(transient)
            # the persistent history this document's media see, appended as a row view when
            # it is not the whole history in place: the fused current document's view, a
            # strided older history, or any history once the current video is strided
            view: list[int] | None = None
            own_view = False
            if fused and position == 1:
                assert plan.previous_media is not None
                if plan.previous_media.n:
                    put_rows(plan.previous_media)
                policy = ({} if self.fused_current_recent_blocks is None else
                          {"use_sink": bool(self.fused_current_use_sink),
                           "recent_blocks": self.fused_current_recent_blocks})
                if sparse_history:
                    view = self.cache.history_for_attention_rows(
                        fused_current=True, recent_full_blocks=self.history_kv_recent_full_blocks,
                        older_video_stride=self.history_kv_older_video_stride, **policy)
                else:
                    view = self.cache.history_for_fused_current_rows(
                        use_sink=bool(self.fused_current_use_sink),
                        recent_blocks=self.fused_current_recent_blocks)
                own_view = True
            elif not capture and (sparse_history or video_stride > 1):
                if sparse_history:
                    view = self.cache.history_for_attention_rows(
                        fused_current=False, recent_full_blocks=self.history_kv_recent_full_blocks,
                        older_video_stride=self.history_kv_older_video_stride)
                else:
                    view = list(range(n_hist))
                own_view = True
            if view:
                copy_rows(view)
            if video_stride > 1:
                # every committed audio row and every video_stride-th committed video row of
                # the document (F/streaming/attention_hook.py:219-236)
                tags_media = token_tags.detach().to("cpu")[doc.media.host]
                video_pos = torch.nonzero(tags_media == VIDEO_TOKEN_TAG).flatten()
                keep = torch.ones(doc.media.n, dtype=torch.bool)
                keep[video_pos] = False
                keep[video_pos[::video_stride]] = True
                sel_first = cursor
                kept = torch.nonzero(keep).flatten()
                copy_rows((kept + first).tolist())
                selected_media[position] = (sel_first, cursor - sel_first, kept)
                kv_start = c_start  # skips the unstrided media rows
            elif own_view:
                kv_start = first
            else:
                # the first document's media see the persistent history (none while capturing)
                kv_start = n_hist if capture else 0
            regions.append((kv_start, first, c_start, cursor))
        other_kv: list[tuple[int, int, int]] = []
        for a, b in plan.others:
            paged.write(key, value, start=cursor, count=b - a, src_start=a)
            other_kv.append((a, b, cursor))
            cursor += b - a

        # 2. one problem per query set (gathered into a compact buffer unless every set is a
        # contiguous run of the packed rows)
        sets = [rows for doc in plan.docs for rows in (doc.media, doc.cond)]
        out = torch.empty_like(query)
        gathered = None
        if all(r.range is not None for r in sets):
            q_src = query
            q_ranges = [r.range for r in sets]
        else:
            total = sum(r.n for r in sets)
            gathered = torch.empty(total, *query.shape[1:], dtype=query.dtype, device=query.device)
            q_ranges, at = [], 0
            for r in sets:
                kv_copy_rows([query], [gathered], count=r.n, src_index=r.index, dst_start=at)
                q_ranges.append((at, at + r.n))
                at += r.n
            q_src = gathered
        # the first packed document with nothing before it: its condition rows see the whole
        # document too (F/streaming/attention_hook.py:1308-1316)
        whole_document = (self.dense_current_document_when_empty
                          and self.mode is HookMode.NOISY and self.block_index == 0
                          and n_hist == 0 and self._transient(layer_name, 0, fused) is None
                          and not fused)
        problems = []
        for d, (kv_start, m_start, c_start, end) in enumerate(regions):
            mq, cq = q_ranges[2 * d], q_ranges[2 * d + 1]
            problems.append(AttentionProblem(mq[0], mq[1], kv_start, end,
                                             sparse=self.backend in SPARSE_BACKENDS))
            if whole_document:
                problems.append(AttentionProblem(cq[0], cq[1], kv_start, end))
            else:
                problems.append(AttentionProblem(cq[0], cq[1], c_start,
                                                 c_start + (cq[1] - cq[0])))
        out_main = out if gathered is None else torch.empty_like(gathered)
        # SOL-Attn backend: the media rows of the document(s) it routes go through
        # h3sa_sol_attention instead of the dense launch
        sol_docs = self._sol_documents(layer_name, fused)
        # rows stored straight into the owners' sequence shards when the output rows are the
        # query rows (no gather) and the launch is bf16
        exchange = self.output_exchange
        if exchange is not None and (gathered is not None or self.backend in FP8_BACKENDS
                                     or sol_docs):
            exchange = None
        self.last_output_exchanged = exchange is not None
        n_kv_media = regions[0][3]
        dense_problems = [pr for i, pr in enumerate(problems)
                          if not (i % 2 == 0 and i // 2 in sol_docs)]
        self._launch(layer_name, paged, q_src, out_main, dense_problems, scale, n_kv_media,
                     n_hist, plan, err, exchange)
        if self.backend in SOL_BACKENDS:
            self.sol_attn_dense_calls += len(dense_problems)
        for d in sol_docs:
            self._sol_media(paged, plan, d, regions[d], q_src, q_ranges[2 * d], out_main, scale,
                            fused, token_tags, layer_name, err, selected_media.get(d))
        if other_kv and self.backend in FP8_BACKENDS:
            # every other document is its own one-part e4m3 call in the reference's FP8 backends
            for a, b, c in other_kv:
                self._fp8_condition(paged, query, out, AttentionProblem(a, b, c, c + (b - a)),
                                    scale, err)
                self.launches += 1
        elif other_kv:
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
            for r, (lo, hi) in zip(sets, q_ranges):
                kv_copy_rows([out_main], [out], count=r.n, src_start=lo, dst_index=r.index)

        self.kernel_calls += len(problems) + len(other_kv)
        self.query_tokens += int(query.shape[0])
        self.key_tokens += sum(p.kv_hi - p.kv_lo for p in problems) + sum(
            b - a for a, b, _ in other_kv)

        # 3. what the mode keeps
        if capture:
            self._capture(layer_name, key, value, token_tags, commit_mask)
        elif self.mode in _COMMIT_MODES:
            # the live document's media rows were written right after the history
            self.cache.stage_in_place(layer_name, key, value, token_tags, commit_mask)
        elif fused:
            # the previous document is the committed block (F/streaming/attention_hook.py:1580-1590)
            self.cache.stage_in_place(layer_name, key, value, token_tags, commit_mask,
                                      commit_indices=plan.docs[0].media.host.to(
                                          token_tags.device, torch.long))
        return out

    # ------------------------------------------------------------------ SOL-Attn
    def _sol_documents(self, layer_name: str, fused: bool) -> list[int]:
        """Live documents (positions in the plan) whose media rows are routed this call: none
        in the commit and capture modes, in the first ``sol_attn_dense_denoise_steps`` denoise
        steps or the first ``sol_attn_dense_layers`` layers; in a fused forward only the
        current document (F/streaming/attention_hook.py:909-929, 1487)."""

        if self.backend not in SOL_BACKENDS:
            return []
        if self.mode in (HookMode.CLEAN_COMMIT, HookMode.PROGRESS_COMMIT,
                         HookMode.FULL_PREFIX_CAPTURE):
            return []
        if (self._denoise_step_index is not None
                and self._denoise_step_index < self.sol_attn_dense_denoise_steps):
            return []
        if int(layer_name.split(".")[1]) < self.sol_attn_dense_layers:
            return []
        return [1] if fused else [0]

    def _sol_history_rows(self, fused_current: bool,
                          device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        """Logical history rows (int32 device tensors) split into audio and video, block by
        block, over the blocks the SOL call sees (F/streaming/cache.py:439-499). Built once
        per history state and policy, then shared by every layer's call."""

        cache = self.cache
        retained = cache.retained_blocks
        recent_blocks = self.fused_current_recent_blocks
        counts = tuple(cache.commit_token_counts)
        if fused_current and recent_blocks is not None:
            recent = max(0, recent_blocks - 1)
            if self.fused_current_use_sink:
                blocks = (0, *range(max(1, retained - recent), retained)) if retained else ()
            else:
                blocks = tuple(range(max(0, retained - recent), retained))
        else:
            blocks = tuple(range(retained))
        tags = cache.commit_token_tags()
        # a block's tag tuple is replaced whenever its rows change (retention, audio drop)
        key = (cache.committed_blocks, counts, blocks, tuple(id(tags[b]) for b in blocks),
               str(device))
        hit = getattr(self, "_sol_history_cache", None)
        if hit is not None and hit[0] == key:
            return hit[2]
        offsets = cache._block_offsets()
        audio, video = [], []
        for b in blocks:
            t = torch.tensor(tags[b], dtype=torch.int64)
            audio.append(torch.nonzero(t == AUDIO_TOKEN_TAG).flatten() + offsets[b])
            video.append(torch.nonzero(t == VIDEO_TOKEN_TAG).flatten() + offsets[b])
        empty = torch.zeros(0, dtype=torch.int64)
        split = tuple((torch.cat(x) if x else empty).to(torch.int32).pin_memory().to(
            device, non_blocking=True) for x in (audio, video))
        self._sol_history_cache = (key, [tags[b] for b in blocks], split)  # keeps the ids alive
        return split

    def _sol_media(self, paged, plan: _DocumentPlan, d: int, region: tuple[int, int, int, int],
                   q_src: torch.Tensor, q_range: tuple[int, int], out: torch.Tensor,
                   scale: float, fused: bool, token_tags: torch.Tensor, layer_name: str,
                   err: torch.Tensor,
                   selected: tuple[int, int, torch.Tensor] | None = None) -> None:
        """One live document's media rows through SOL-Attn. The K/V sequence is gathered from
        the page sequence in the reference's part order: exact parts [condition, current
        media, temporary prefix, previous document's media, audio history] as the sink, then
        the video history routed; with ``sol_attn_route_current_video`` the current video
        moves from the sink to the routed part and the audio queries attend densely
        (F/streaming/attention_hook.py:1379-1492)."""

        from .sol_attention import sol_attn_rectangular

        kv_start, first, c_start, end = region
        doc = plan.docs[d]
        n_media, n_cond = doc.media.n, doc.cond.n
        transient = self._transient(layer_name, d, fused)
        n_prefix = 0 if transient is None else int(transient.key.shape[0])
        n_prev = plan.previous_media.n if (fused and d == 1 and plan.previous_media is not None) else 0
        device = q_src.device

        def span(a: int, n: int) -> torch.Tensor:
            return torch.arange(a, a + n, dtype=torch.int32, device=device)

        # the current media keys: every media row, or the strided copy with
        # current_video_kv_stride > 1 (the reference's current_media_key)
        media_rows = span(first, n_media) if selected is None else span(selected[0], selected[1])
        cond_rows = span(c_start, n_cond)
        prefix_rows = span(c_start + n_cond, n_prefix)
        prev_rows = span(c_start + n_cond + n_prefix, n_prev)
        audio_hist, video_hist = self._sol_history_rows(fused and d == 1, device)
        lo, hi = q_range
        route_video = self.sol_attn_route_current_video and not fused
        if route_video:
            tags = token_tags.detach().to("cpu")[doc.media.host]
            q_audio = torch.nonzero(tags == AUDIO_TOKEN_TAG).flatten().tolist()
            q_video = torch.nonzero(tags == VIDEO_TOKEN_TAG).flatten().tolist()
            key_tags = tags if selected is None else tags[selected[2]]
            k_audio = torch.nonzero(key_tags == AUDIO_TOKEN_TAG).flatten().to(device)
            k_video = torch.nonzero(key_tags == VIDEO_TOKEN_TAG).flatten().to(device)
            cur_audio, cur_video = media_rows[k_audio], media_rows[k_video]
            exact = (cond_rows, cur_audio, prefix_rows, audio_hist)
            routed = (cur_video, video_hist)
        else:
            exact = (cond_rows, media_rows, prefix_rows, prev_rows, audio_hist)
            routed = (video_hist,)
            q_audio, q_video = [], None
        n_exact = sum(int(t.numel()) for t in exact)
        index = torch.cat(exact + routed)
        n_rows = int(index.numel())
        heads = q_src.shape[1]
        k = torch.empty(n_rows, heads, q_src.shape[2], dtype=q_src.dtype, device=device)
        v = torch.empty_like(k)
        kv_copy_rows([paged.key, paged.value], [k, v], count=n_rows, src_table=paged.table,
                     src_index=index, device_error=err)
        if self._sol_attn_density_counts is None or self._sol_attn_density_counts.device != device:
            self._sol_attn_density_counts = torch.zeros(4, dtype=torch.int64, device=device)

        def subset(positions: list[int]):
            idx = torch.tensor([lo + i for i in positions], dtype=torch.int32).pin_memory().to(
                device, non_blocking=True)
            qs = torch.empty(len(positions), *q_src.shape[1:], dtype=q_src.dtype, device=device)
            kv_copy_rows([q_src], [qs], count=len(positions), src_index=idx)
            return qs, idx

        if q_video is None:
            sol_attn_rectangular(q_src[lo:hi], k, v, scale=scale, tau=self.sol_attn_tau,
                                 sink_tokens=n_exact,
                                 telemetry_counts=self._sol_attn_density_counts,
                                 out=out[lo:hi], device_error=err)
            n_sol = hi - lo
        else:
            if q_audio:
                qa, ia = subset(q_audio)
                oa = torch.empty_like(qa)
                attention_fwd(qa, oa, paged.key, paged.value, paged.table,
                              [AttentionProblem(0, len(q_audio), kv_start, end)], scale,
                              device_error=err)
                kv_copy_rows([oa], [out], count=len(q_audio), dst_index=ia)
                self.sol_attn_dense_calls += 1
                self.launches += 1
            n_sol = len(q_video)
            if q_video:
                qv, iv = subset(q_video)
                ov = sol_attn_rectangular(qv, k, v, scale=scale, tau=self.sol_attn_tau,
                                          sink_tokens=n_exact,
                                          telemetry_counts=self._sol_attn_density_counts,
                                          device_error=err)
                kv_copy_rows([ov], [out], count=n_sol, dst_index=iv)
        if n_sol:
            self.sol_attn_kernel_calls += 1
            self.sol_attn_query_tokens += n_sol
            self.sol_attn_key_tokens += n_rows
            self.launches += 1

    def _capture(self, layer_name: str, key: torch.Tensor, value: torch.Tensor,
                 token_tags: torch.Tensor, commit_mask: torch.Tensor) -> None:
        if layer_name in self._captured_full_prefix_layers:
            raise ValueError(f"duplicate full-prefix K/V layer: {layer_name}")
        if self._capture_index is None:
            rows = _full_prefix_capture_rows(token_tags.detach().cpu(),
                                             commit_mask.detach().cpu().to(torch.bool),
                                             self._capture_video_rows,
                                             self._capture_audio_rows_per_channel)
            self._capture_index = rows.to(device=key.device, dtype=torch.int32)
        n = int(self._capture_index.numel())
        k = torch.empty(n, *key.shape[1:], dtype=key.dtype, device=key.device)
        v = torch.empty_like(k)
        kv_copy_rows([key, value], [k, v], count=n, src_index=self._capture_index)
        pair = (VideoKV if self._capture_audio_rows_per_channel is None else AVKV)(key=k, value=v)
        self._captured_full_prefix_layers[layer_name] = pair

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
        self._fp8_condition(paged, q_src, out, cond, scale, err)
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
        self._fp8_condition(paged, q_src, out, cond, scale, err)
        self.launches += 2

    def _fp8_condition(self, paged, q_src: torch.Tensor, out: torch.Tensor,
                       cond: AttentionProblem, scale: float, err: torch.Tensor) -> None:
        """A one-part call (the condition rows, or another document) in e4m3, as the
        reference's FP8 backends run it (F/streaming/attention_hook.py:1081-1107): the rows'
        Q, K and V quantised per head over those rows alone, one attention launch."""

        from .kernels import quantize_fp8_rows

        n_kv, n_q = cond.kv_hi - cond.kv_lo, cond.q_hi - cond.q_lo
        heads, dim, dev = paged.heads, paged.head_dim, q_src.device
        pad = (n_kv + PAGE_ROWS - 1) // PAGE_ROWS * PAGE_ROWS
        k8 = torch.empty(heads, pad, dim, dtype=torch.float8_e4m3fn, device=dev)
        v8 = torch.empty_like(k8)
        table = torch.arange(pad // PAGE_ROWS, dtype=torch.int32, device=dev)
        kv_scale = torch.empty(2, heads, dtype=torch.float32, device=dev)
        work = torch.empty(2 * heads, dtype=torch.int32, device=dev)
        quantize_fp8_rows([paged.key, paged.value], [k8, v8], [kv_scale[0], kv_scale[1]], work,
                          count=n_kv, src_start=cond.kv_lo, src_table=paged.table,
                          dst_table=table, zero_tail=True, device_error=err)
        q8, q_scale = quantize_fp8_e4m3_per_head(q_src[cond.q_lo:cond.q_hi].unsqueeze(0))
        o = torch.empty(n_q, heads, dim, dtype=torch.bfloat16, device=dev)
        attention_fwd(q8.squeeze(0), o, k8, v8, table, [AttentionProblem(0, n_q, 0, n_kv)], scale,
                      q_scale=q_scale.reshape(-1).contiguous(), k_scale=kv_scale[0],
                      v_scale=kv_scale[1], device_error=err)
        out[cond.q_lo:cond.q_hi].copy_(o)

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
