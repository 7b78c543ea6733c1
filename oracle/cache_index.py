"""Clean AV KV cache row-index oracle (test infrastructure only).

Restates the row bookkeeping of ``CleanAVKVCache`` (T/streaming/cache.py:77-294, and the
FL2AV additions of F/streaming/cache.py:199-1151: bounded commits, count-based and sink +
recent retention, the strided attention history) on plain
Python lists: which packed rows a clean commit stages (``nonzero(commit_mask)`` in packed
order, :155-165), how commits append (:175-204), and which logical rows retention and audio
drop keep (:206-230, :246-284). History rows are identified by (commit serial, row within
that commit's staged rows), so tables from different implementations compare exactly.
"""

from __future__ import annotations

VIDEO_TOKEN_TAG = 0
AUDIO_TOKEN_TAG = 2


class CacheIndexOracle:
    def __init__(self) -> None:
        self.rows: list[tuple[int, int]] = []     # logical history row -> (commit serial, local row)
        self.counts: list[int] = []
        self.tags: list[tuple[int, ...]] = []
        self.serial = 0
        self.committed_blocks = 0

    @staticmethod
    def staged_rows(token_tags: list[int], commit_mask: list[bool]) -> tuple[list[int], tuple[int, ...]]:
        """Packed rows and tags a clean commit stages (T/streaming/cache.py:155-165)."""

        indices = [i for i, m in enumerate(commit_mask) if m]
        if not indices:
            raise RuntimeError("clean commit did not contain audio/video rows")
        tags = tuple(int(token_tags[i]) for i in indices)
        if frozenset(tags) != frozenset((VIDEO_TOKEN_TAG, AUDIO_TOKEN_TAG)):
            raise RuntimeError("each clean chunk must contain both video and audio KV")
        return indices, tags

    def commit(self, token_tags: list[int], commit_mask: list[bool]) -> None:
        _, tags = self.staged_rows(token_tags, commit_mask)
        self.rows.extend((self.serial, r) for r in range(len(tags)))
        self.counts.append(len(tags))
        self.tags.append(tags)
        self.serial += 1
        self.committed_blocks += 1

    def _retain(self, selection: list[tuple[int, bool]]) -> None:
        offsets = [0]
        for c in self.counts:
            offsets.append(offsets[-1] + c)
        rows: list[tuple[int, int]] = []
        counts: list[int] = []
        tags: list[tuple[int, ...]] = []
        for block, video_only in selection:
            t = self.tags[block]
            local = [i for i, tag in enumerate(t) if not video_only or tag == VIDEO_TOKEN_TAG]
            if not local:
                continue
            rows.extend(self.rows[offsets[block] + i] for i in local)
            counts.append(len(local))
            tags.append(tuple(t[i] for i in local))
        self.rows, self.counts, self.tags = rows, counts, tags

    def retain_sink_and_recent_commits(self) -> None:
        n = len(self.counts)
        if n <= 2:
            return
        recent_start = max(1, n - 2)
        self._retain([(0, True)] + [(i, False) for i in range(recent_start, n)])

    def drop_audio_history(self) -> int:
        removed = sum(t == AUDIO_TOKEN_TAG for tags in self.tags for t in tags)
        if not self.counts:
            return 0
        self._retain([(i, True) for i in range(len(self.counts))])
        return removed

    # ------------------------------------------------------------------ FL2AV (F/streaming/cache.py)
    def commit_bounded(self, token_tags: list[int], commit_mask: list[bool], count: int,
                       advance_serial: bool = True) -> None:
        """Commit keeping only the newest ``count`` blocks (:857-927)."""

        if count < 1:
            raise ValueError("bounded clean commit count must be positive")
        _, tags = self.staged_rows(token_tags, commit_mask)
        keep = count - 1
        if keep:
            kept = sum(self.counts[-keep:])
            self.rows = self.rows[len(self.rows) - kept:]
            self.counts, self.tags = self.counts[-keep:], self.tags[-keep:]
        else:
            self.rows, self.counts, self.tags = [], [], []
        self.rows.extend((self.serial, r) for r in range(len(tags)))
        self.counts.append(len(tags))
        self.tags.append(tags)
        self.serial += 1
        if advance_serial:
            self.committed_blocks += 1

    def retain_recent_commits(self, count: int) -> None:
        """Keep the newest ``count`` blocks (:929-962)."""

        if count < 1:
            raise ValueError("retained clean commit count must be a positive integer")
        if len(self.counts) <= count:
            return
        self._retain([(i, False) for i in range(len(self.counts) - count, len(self.counts))])

    def retain_sink_and_recent(self, recent_count: int, sink_video_only: bool = True) -> None:
        """Block 0 (video rows only once it has aged out of the recent window) plus the newest
        ``recent_count`` blocks (:964-995)."""

        n = len(self.counts)
        if n == 0:
            return
        recent_start = max(0, n - recent_count)
        selection = [(0, bool(sink_video_only and recent_start > 0))]
        selection += [(i, False) for i in range(max(1, recent_start), n)]
        if selection == [(i, False) for i in range(n)]:
            return
        self._retain(selection)

    def attention_history_rows(self, count: int, recent_full_blocks: int, older_video_stride: int,
                               preserve_sink: bool = False) -> list[tuple[int, int]] | None:
        """Rows ``attention_history`` selects (:501-575): the newest ``count`` blocks (or block
        0 plus the newest ``count - 1``), dense for the newest ``recent_full_blocks`` of them,
        and for older ones every audio row and every ``older_video_stride``-th video row."""

        if recent_full_blocks < 0 or older_video_stride < 1:
            raise ValueError("invalid H3 attention-history policy")
        n = len(self.counts)
        if n == 0 or count == 0:
            return None
        if preserve_sink:
            recent_start = max(1, n - max(0, count - 1))
            blocks = [0, *range(recent_start, n)]
        else:
            blocks = list(range(max(0, n - count), n)) if count < n else list(range(n))
        offsets = [0]
        for c in self.counts:
            offsets.append(offsets[-1] + c)
        dense_start = max(0, len(blocks) - recent_full_blocks)
        dense = older_video_stride == 1 or recent_full_blocks >= len(blocks)
        out: list[tuple[int, int]] = []
        for position, block in enumerate(blocks):
            tags = self.tags[block]
            if dense or position >= dense_start:
                local = list(range(len(tags)))
            else:
                local, ordinal = [], 0
                for i, tag in enumerate(tags):
                    if tag == AUDIO_TOKEN_TAG:
                        local.append(i)
                    elif tag == VIDEO_TOKEN_TAG:
                        if ordinal % older_video_stride == 0:
                            local.append(i)
                        ordinal += 1
            out.extend(self.rows[offsets[block] + i] for i in local)
        return out

    @property
    def history_tokens(self) -> int:
        return len(self.rows)


__all__ = ["AUDIO_TOKEN_TAG", "CacheIndexOracle", "VIDEO_TOKEN_TAG"]
