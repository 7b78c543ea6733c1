"""Seeded inputs shared by the golden generator and the tests (numpy PCG64 + bf16 RNE)."""

from __future__ import annotations

import numpy as np


def bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16 values, returned as float32."""

    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def rms(x: np.ndarray) -> np.ndarray:
    return (x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True) + 1e-5)).astype(np.float32)


def hook_cpu_inputs(seed: int = 0, heads: int = 8, head_dim: int = 64, seq: int = 320,
                    hist: int = 1024) -> dict:
    """CPU benchmark configuration: q/k RMS-normalised N(0,1), v N(0,1), bf16 values.

    Packed rows [16 text | 16 + 16 audio | 256 video | 16 pad] (seq 320), 1024 cached rows.
    """

    rng = np.random.default_rng(seed)
    q = bf16(rms(rng.standard_normal((seq, heads, head_dim)).astype(np.float32)))
    k = bf16(rms(rng.standard_normal((seq, heads, head_dim)).astype(np.float32)))
    v = bf16(rng.standard_normal((seq, heads, head_dim)).astype(np.float32))
    hist_k = bf16(rms(rng.standard_normal((hist, heads, head_dim)).astype(np.float32)))
    hist_v = bf16(rng.standard_normal((hist, heads, head_dim)).astype(np.float32))
    tags = np.full(seq, -1, dtype=np.int64)
    tags[:16] = 1
    tags[16:48] = 2
    tags[48:304] = 0
    return {"q": q, "k": k, "v": v, "hist_k": hist_k, "hist_v": hist_v, "token_tags": tags,
            "commit_mask": (tags == 0) | (tags == 2), "cu_seqlens": [0, 304, 320],
            "scale": head_dim ** -0.5}


def fp8_input(seed: int = 5) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, 300, 3, 128)).astype(np.float32)
    x = np.where(rng.random(x.shape) < 0.01, x * 8.0, x)
    return bf16(x)


def mask_inputs(seed: int = 3, heads: int = 2, nq: int = 384, nh: int = 1000) -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(seed)
    q = bf16(rng.standard_normal((1, heads, nq, 128)).astype(np.float32))
    hk = bf16(rng.standard_normal((1, heads, nh, 128)).astype(np.float32))
    return q, hk


def prologue_inputs(seed: int = 11, seq: int = 128, heads: int = 4, head_dim: int = 128) -> dict:
    rng = np.random.default_rng(seed)
    qkv = bf16(rng.standard_normal((seq, 3 * heads * head_dim)).astype(np.float32) * 1.7)
    q_w = bf16(1.0 + 0.1 * rng.standard_normal(head_dim).astype(np.float32))
    k_w = bf16(1.0 + 0.1 * rng.standard_normal(head_dim).astype(np.float32))
    return {"qkv": qkv, "q_weight": q_w, "k_weight": k_w}


def ulysses_merged(rank: int, tokens: int = 6, heads: int = 4, d: int = 16) -> np.ndarray:
    return np.random.default_rng(100 + rank).standard_normal((tokens, 3 * heads * d)).astype(np.float32)


# FL2AV hook schedule: (mode, live documents in the packed sequence, extra activate arguments)
HOOK_F_SCHEDULE = (
    ("clean_commit", 1, {}),
    ("progress_commit", 1, {}),
    ("capture", 1, {"video_rows": 24, "audio_rows_per_channel": 3}),
    ("noisy_prefix", 1, {"denoise_step_index": 0}),
    ("fused_recent", 2, {"fused_previous_video_only": True, "fused_current_use_sink": True,
                         "fused_current_recent_blocks": 2}),
    ("fused", 2, {}),
    ("noisy", 1, {}),
)


# FL2AV hook history / current-video policies and their schedule
HOOK_F_POLICY = {"history_kv_older_video_stride": 3, "history_kv_recent_full_blocks": 1,
                 "current_video_kv_stride": 2}
HOOK_F_POLICY_SCHEDULE = (
    ("clean_commit", 1, {}),
    ("clean_commit", 1, {}),
    ("clean_commit", 1, {}),
    ("noisy", 1, {"denoise_step_index": 1}),
    ("fused", 2, {"fused_current_use_sink": True, "fused_current_recent_blocks": 2}),
    ("noisy", 1, {}),
)


def hook_f_inputs(step: int, live: int, heads: int = 2, head_dim: int = 128) -> dict:
    """One packed call of the FL2AV hook schedule: ``live`` documents of [8 text | 4 + 4
    audio | 48 video] rows each, then an 8-row pad document; q/k RMS-normalised, bf16."""

    rng = np.random.default_rng(1000 + step)
    doc = [1] * 8 + [2] * 8 + [0] * 48
    tags = np.array(doc * live + [-1] * 8, dtype=np.int64)
    n = len(tags)
    q = bf16(rms(rng.standard_normal((n, heads, head_dim)).astype(np.float32)))
    k = bf16(rms(rng.standard_normal((n, heads, head_dim)).astype(np.float32)))
    v = bf16(rng.standard_normal((n, heads, head_dim)).astype(np.float32))
    cu = [0] + [64 * (i + 1) for i in range(live)] + [n]
    return {"q": q, "k": k, "v": v, "token_tags": tags, "commit_mask": (tags == 0) | (tags == 2),
            "cu_seqlens": cu, "scale": head_dim ** -0.5}


def hook_topk_inputs(step: int, heads: int = 2, head_dim: int = 128) -> dict:
    """One call of the commit-level top-k schedule: hook_f_inputs' single-document layout
    with K (commit steps) or Q (the final call) shifted by a per-step offset row, so the
    blocks' key summaries score clearly apart against the media queries."""

    x = hook_f_inputs(100 + step, 1, heads, head_dim)
    rng = np.random.default_rng(2000 + step)
    offset = 0.5 * rng.standard_normal((1, heads, head_dim)).astype(np.float32)
    x["k"] = bf16(x["k"] + offset)
    x["q"] = bf16(x["q"] + offset)
    return x


# SOL-Attn cases: (query rows, key rows, heads, tau, sink tokens)
SOL_CASES = ((150, 700, 2, 0.5, 200), (64, 1283, 1, 1.0, 0), (200, 640, 3, -0.5, 130))


def sol_inputs(case: int, head_dim: int = 128) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """bf16-exact float32 query / key / value [N, H, D] with block-clustered keys (each 64-row
    key block drawn around its own centre), so that the routing keeps some blocks and not
    others."""

    nq, nk, heads, _, _ = SOL_CASES[case]
    rng = np.random.default_rng(700 + case)
    kb = (nk + 63) // 64
    centre = rng.standard_normal((kb, heads, head_dim)).astype(np.float32)
    k = 0.6 * rng.standard_normal((nk, heads, head_dim)).astype(np.float32)
    k += np.repeat(centre, 64, axis=0)[:nk]
    q = rng.standard_normal((nq, heads, head_dim)).astype(np.float32)
    v = rng.standard_normal((nk, heads, head_dim)).astype(np.float32)
    return bf16(q), bf16(k), bf16(v)


def sol_hook_document(rng: np.random.Generator, heads: int = 2, head_dim: int = 128) -> dict:
    """One packed call for the hook's SOL backend: 16 text, 32 audio, 256 video rows and a
    16-row pad document, keys clustered around a centre per 64 rows (bf16-exact float32)."""

    centre = rng.standard_normal((5, heads, head_dim))
    tags = np.full(320, -1, np.int64)
    tags[:16] = 1
    tags[16:48] = 2
    tags[48:304] = 0
    k = 0.7 * rng.standard_normal((320, heads, head_dim)) + np.repeat(centre, 64, axis=0)[:320]
    return {"q": bf16(rng.standard_normal((320, heads, head_dim)).astype(np.float32)),
            "k": bf16(k.astype(np.float32)),
            "v": bf16(rng.standard_normal((320, heads, head_dim)).astype(np.float32)),
            "token_tags": tags, "commit_mask": (tags == 0) | (tags == 2), "cu_seqlens": [0, 304, 320]}


def sol_hook_inputs(seed: int = 5) -> tuple[list[dict], dict]:
    """Three committed documents and the noisy call of the SOL hook fixture."""

    rng = np.random.default_rng(seed)
    docs = [sol_hook_document(rng) for _ in range(4)]
    return docs[:3], docs[3]
