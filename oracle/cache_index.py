"""Clean AV KV cache row-index oracle (test infrastructure only).

Restates the row bookkeeping of ``CleanAVKVCache`` (T/streaming/cache.py:77-294) on plain
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

    @property
    def history_tokens(self) -> int:
        return len(self.rows)


__all__ = ["AUDIO_TOKEN_TAG", "CacheIndexOracle", "VIDEO_TOKEN_TAG"]
