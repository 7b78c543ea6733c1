"""FL2AV streaming hook modes on CPU (test infrastructure only).

Restates the dense path of the FL2AV ``H3StreamingAttentionHook`` (F/streaming/
attention_hook.py) with its cache (F/streaming/cache.py), one layer, fp32 SDPA:

* NOISY / CLEAN_COMMIT / PROGRESS_COMMIT: one live document; media rows see
  [condition, temporary prefix, persistent history, current media], condition rows their own
  condition rows, other documents themselves (:1112-1236, plan :193-216); the two commit
  modes stage the live document's media rows (:1577-1578);
* FULL_PREFIX_CAPTURE: no history and no prefix; the kept rows are the newest committed video
  rows preceded by the newest audio rows of each channel (:254-285, :1560-1576);
* FUSED_PROGRESS_DENOISE: two live documents; the previous one sees its own prefix and the
  whole history, the current one its prefix, the fused-current history view
  (F/streaming/cache.py:368-407) and the previous document's media rows (video only on
  request, :239-251); the previous document's media rows are the commit (:1579-1590).

The history / current-video policies of the FL2AV hook constructor are restated too:
strided older history (``history_for_attention``, F/streaming/cache.py:409-437, 501-575),
strided current video keys (F/streaming/attention_hook.py:219-236) and the whole first
document (:1308-1336).

The history is kept as dense per-block K/V with their token tags, the way the reference's
cache ledger does (F/streaming/cache.py:199-262, 964-995).
"""

from __future__ import annotations

from typing import Sequence

import torch

from .attention import sdpa_from_kv_parts

VIDEO, AUDIO = 0, 2


class FL2AVHookOracle:
    def __init__(self, scale: float) -> None:
        self.scale = scale
        self.blocks: list[tuple[torch.Tensor, torch.Tensor, list[int]]] = []  # (k, v, tags)
        self.sink_video_only = False

    # ---------------------------------------------------------------- cache views
    def _cat(self, blocks) -> tuple[torch.Tensor, torch.Tensor] | None:
        if not blocks:
            return None
        return (torch.cat([b[0] for b in blocks]), torch.cat([b[1] for b in blocks]))

    def history(self):
        return self._cat(self.blocks)  # (key, value) of every block, oldest first

    def fused_current_history(self, use_sink: bool, recent_blocks: int | None):
        if recent_blocks is None:
            return self.history()
        recent = max(0, recent_blocks - 1)
        if not use_sink:
            if recent == 0 or not self.blocks:
                return None
            return self._cat(self.blocks[max(0, len(self.blocks) - recent):])
        if not self.blocks:
            return None
        start = max(1, len(self.blocks) - recent)
        sink_k, sink_v, sink_tags = self.blocks[0]
        if self.sink_video_only and len(self.blocks) + 1 > recent_blocks and AUDIO in sink_tags:
            keep = torch.tensor([t == VIDEO for t in sink_tags])
            sink = (sink_k[keep], sink_v[keep], [t for t in sink_tags if t == VIDEO])
        else:
            sink = self.blocks[0]
        return self._cat([sink] + self.blocks[start:])

    def attention_history(self, count: int, recent_full_blocks: int, older_video_stride: int,
                          preserve_sink: bool = False):
        """Dense newest ``recent_full_blocks`` blocks and the older blocks' audio rows plus
        every ``older_video_stride``-th video row, over the newest ``count`` blocks or block
        0 plus the newest ``count - 1`` (F/streaming/cache.py:501-575)."""

        n = len(self.blocks)
        if n == 0 or count <= 0:
            return None
        if preserve_sink:
            chosen = [0, *range(max(1, n - max(0, count - 1)), n)]
        else:
            chosen = list(range(max(0, n - count), n))
        dense = older_video_stride == 1 or recent_full_blocks >= len(chosen)
        dense_start = max(0, len(chosen) - recent_full_blocks)
        parts = []
        for position, b in enumerate(chosen):
            k, v, tags = self.blocks[b]
            if dense or position >= dense_start:
                parts.append((k, v, tags))
                continue
            keep, ordinal = [], 0
            for i, tag in enumerate(tags):
                if tag == AUDIO:
                    keep.append(i)
                elif tag == VIDEO:
                    if ordinal % older_video_stride == 0:
                        keep.append(i)
                    ordinal += 1
            parts.append((k[keep], v[keep], [tags[i] for i in keep]))
        return self._cat(parts)

    def history_for_attention(self, fused_current: bool, recent_full_blocks: int,
                              older_video_stride: int, use_sink: bool = False,
                              recent_blocks: int | None = None):
        """F/streaming/cache.py:409-437."""

        retained = len(self.blocks)
        if fused_current and recent_blocks is not None:
            count = min(retained, (1 if use_sink and retained else 0) + max(0, recent_blocks - 1))
            recent_full_blocks = max(0, recent_full_blocks - 1)
        else:
            count = retained
        return self.attention_history(count, recent_full_blocks, older_video_stride,
                                      preserve_sink=use_sink)

    def retain_sink_and_recent(self, recent_count: int, sink_video_only: bool = True) -> None:
        self.sink_video_only = bool(sink_video_only)
        n = len(self.blocks)
        if n == 0:
            return
        recent_start = max(0, n - recent_count)
        kept = []
        k, v, tags = self.blocks[0]
        if sink_video_only and recent_start > 0:
            keep = torch.tensor([t == VIDEO for t in tags])
            kept.append((k[keep], v[keep], [t for t in tags if t == VIDEO]))
        else:
            kept.append(self.blocks[0])
        kept += self.blocks[max(1, recent_start):]
        self.blocks = kept

    # ---------------------------------------------------------------- one call
    def call(self, mode: str, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
             tags: Sequence[int], cu: Sequence[int], *, prefix=None, previous_prefix=None,
             previous_video_only: bool = False, use_sink: bool | None = None,
             recent_blocks: int | None = None, capture: tuple[int, int | None] | None = None,
             older_video_stride: int = 1, recent_full_blocks: int = 5, video_stride: int = 1,
             whole_first_document: bool = False):
        """Output rows of one layer call; commits (or returns the captured rows) as the mode
        says. ``prefix`` / ``previous_prefix``: (key, value) pairs. ``older_video_stride`` /
        ``recent_full_blocks``: the strided-history policy; ``video_stride``: the current
        media keys keep every audio row and every ``video_stride``-th video row
        (F/streaming/attention_hook.py:219-236, 831-850, 1147-1200);
        ``whole_first_document``: a noisy call with nothing before the document lets its
        condition rows see the whole document (:1308-1336)."""

        tags_t = torch.as_tensor(list(tags))
        commit = (tags_t == VIDEO) | (tags_t == AUDIO)
        bounds = list(zip(cu[:-1], cu[1:]))
        live = [i for i, (a, b) in enumerate(bounds) if bool(commit[a:b].any())]
        fused = mode == "fused"
        out = torch.zeros(q.shape, dtype=torch.float32)
        for index, (a, b) in enumerate(bounds):
            if a == b:
                continue
            if index not in live:
                out[a:b] = sdpa_from_kv_parts(q[a:b], [(k[a:b], v[a:b])], self.scale)
                continue
            rows = torch.arange(a, b)
            cond = rows[~commit[a:b]]
            media = rows[commit[a:b]]
            if mode == "capture":
                transient = None
            elif fused and index == live[0]:
                transient = previous_prefix
            else:
                transient = prefix
            extra = []
            sparse = older_video_stride > 1
            if fused and index == live[-1]:
                pa, pb = bounds[live[0]]
                prev = torch.arange(pa, pb)[commit[pa:pb]]
                if previous_video_only:
                    prev = prev[tags_t[prev] == VIDEO]
                if sparse:
                    policy = ({} if recent_blocks is None else
                              {"use_sink": bool(use_sink), "recent_blocks": recent_blocks})
                    persistent = self.history_for_attention(True, recent_full_blocks,
                                                            older_video_stride, **policy)
                else:
                    persistent = self.fused_current_history(bool(use_sink), recent_blocks)
                extra = [p for p in (transient, persistent) if p is not None]
                extra.append((k[prev], v[prev]))
            else:
                if mode == "capture":
                    persistent = None
                elif sparse:
                    persistent = self.history_for_attention(False, recent_full_blocks,
                                                            older_video_stride)
                else:
                    persistent = self.history()
                extra = [p for p in (transient, persistent) if p is not None]
            current = media
            if video_stride > 1:
                video_rows = media[tags_t[media] == VIDEO]
                keep = set(media[tags_t[media] != VIDEO].tolist()) | set(video_rows[::video_stride].tolist())
                current = torch.tensor(sorted(keep), dtype=torch.long)
            whole = (whole_first_document and mode == "noisy" and not self.blocks
                     and transient is None and not fused)
            cond_parts = [(k[cond], v[cond])] + ([(k[media], v[media])] if whole else [])
            out[cond] = sdpa_from_kv_parts(q[cond], cond_parts, self.scale)
            parts = [(k[cond], v[cond]), *extra, (k[current], v[current])]
            out[media] = sdpa_from_kv_parts(q[media], parts, self.scale)
        captured = None
        if mode == "capture":
            video_rows, audio_per_channel = capture
            vid = torch.nonzero(commit & (tags_t == VIDEO)).view(-1)[-video_rows:]
            keep = vid
            if audio_per_channel is not None:
                aud = torch.nonzero(commit & (tags_t == AUDIO)).view(-1)
                aud = aud.reshape(2, -1)[:, -audio_per_channel:].reshape(-1)
                keep = torch.cat((aud, vid))
            captured = (k[keep], v[keep])
        elif mode in ("clean_commit", "progress_commit"):
            a, b = bounds[live[0]]
            media = torch.arange(a, b)[commit[a:b]]
            self.blocks.append((k[media], v[media], [int(t) for t in tags_t[media]]))
        elif fused:
            a, b = bounds[live[0]]
            media = torch.arange(a, b)[commit[a:b]]
            self.blocks.append((k[media], v[media], [int(t) for t in tags_t[media]]))
        return out, captured
