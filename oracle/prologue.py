"""QKV prologue oracle: packed layout, 3-axis RoPE cache, QK-RMSNorm + RoPE (test only).

Restates, in numpy:

* the packed text/audio/video/pad layout and its fp64 position grid
  (``minimax_h3_packed_sequence``, T/model/packed_sequence.py:42-104);
* the RoPE frequency table and bf16 cos/sin cache (``MiniMaxH3Rope.forward`` and
  ``rope_cos_sin_cache``, T/model/layers.py:138-165);
* the in-place merged-QKV QK-RMSNorm + rotate-half RoPE with its explicit bf16 rounding
  points (``_merged_qkv_preprocess_kernel``, T/inference/fused_kernels.py:413-485):
  normalized = bf16(v * rsqrt(mean(v^2) + eps) * w); rope = bf16(bf16(normalized * cos) +
  bf16(rotated * sin)) on dims [0, rotary), normalized elsewhere; V untouched.

The sum of squares is exact (fp64), the mean is rounded to fp32, eps is added in fp32 as
the reference adds it, and the reciprocal square root is evaluated in fp64 and rounded
once, so a GPU kernel following the same steps reproduces these values bit for bit.
"""

from __future__ import annotations

import numpy as np

INTERP = 32
T_GROUP = 5
FRAME_PER_TOKEN = (1, 4, 4, 4, 4)
FRAME_RESCALE = 5.0 / 3.0
ALIGN = 64


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 value (returned as float32)."""

    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def _axis(dim: int, patch: int, sqrt_area: float) -> np.ndarray:
    ratio = dim / sqrt_area
    left = (1.0 - ratio) / 2.0
    return np.linspace(left, left + ratio, dim // patch, endpoint=False) * INTERP


def packed_layout(*, text_len: int, latent_t: int, latent_h: int, latent_w: int,
                  audio_t: int, audio_channel: int = 2, align: int = ALIGN) -> dict:
    """Rows [text | audio ch0 | audio ch1 | video | pad] with positions and token tags."""

    ph, pw = latent_h // 2, latent_w // 2
    frame_rows = ph * pw
    video_rows = latent_t * frame_rows
    audio_rows = audio_t * audio_channel
    used = text_len + audio_rows + video_rows
    seq_len = (used + align - 1) // align * align
    grid = np.zeros((seq_len, 3), dtype=np.float64)
    grid[:text_len, 0] = np.arange(text_len, dtype=np.float64)
    spans = np.array([FRAME_RESCALE * FRAME_PER_TOKEN[k % T_GROUP] for k in range(latent_t)])
    t_grid = float(text_len) + np.concatenate([[0.0], np.cumsum(spans[:-1])])
    sqrt_area = np.sqrt(latent_h * latent_w)
    h_grid = _axis(latent_h, 2, sqrt_area)
    w_grid = _axis(latent_w, 2, sqrt_area)
    hh, ww = np.meshgrid(h_grid, w_grid, indexing="ij")
    a0 = text_len
    v0 = a0 + audio_rows
    video = grid[v0:v0 + video_rows].reshape(latent_t, frame_rows, 3)
    video[:, :, 0] = t_grid[:, None]
    video[:, :, 1] = hh.reshape(-1)[None]
    video[:, :, 2] = ww.reshape(-1)[None]
    grid[a0:v0, 0] = np.tile(float(text_len) + np.arange(audio_t, dtype=np.float64), audio_channel)
    grid[a0:a0 + audio_t, 2] = float(w_grid[0])
    grid[a0 + audio_t:v0, 2] = float(w_grid[-1])
    tags = np.full(seq_len, -1, dtype=np.int64)
    tags[:text_len] = 1
    tags[a0:v0] = 2
    tags[v0:v0 + video_rows] = 0
    commit = (tags == 0) | (tags == 2)
    return {"seq_len": seq_len, "used": used, "grid": grid, "token_tags": tags,
            "commit_mask": commit, "cu_seqlens": [0, used, seq_len],
            "text": (0, text_len), "audio": (a0, v0), "video": (v0, v0 + video_rows)}


def default_inv_freq(per_axis: int, base: float = 10000.0) -> np.ndarray:
    """Synthetic RoPE frequencies (the model loads its own): base^(-2i / (2 * per_axis))."""

    i = np.arange(per_axis, dtype=np.float64)
    return (base ** (-2.0 * i / (2.0 * per_axis))).astype(np.float32)


def rope_cos_sin(grid: np.ndarray, inv_freq: np.ndarray) -> np.ndarray:
    """[S, 3] fp64 positions -> [S, 6F] bf16 cos|sin cache (T/model/layers.py:149-165)."""

    pos = grid.astype(np.float32)
    per_axis = pos[:, :, None] * inv_freq[None, None, :].astype(np.float32)   # fp32 product
    half = np.concatenate([per_axis[:, 0], per_axis[:, 1], per_axis[:, 2]], axis=-1)
    freqs = np.concatenate([half, half], axis=-1)
    h = freqs.shape[-1] // 2
    cs = np.concatenate([np.cos(freqs[:, :h].astype(np.float64)),
                         np.sin(freqs[:, :h].astype(np.float64))], axis=-1).astype(np.float32)
    return round_bf16(cs)


def qkv_norm_rope(qkv: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray,
                  cos_sin: np.ndarray, positions: np.ndarray, heads: int, head_dim: int,
                  eps: float) -> np.ndarray:
    """Merged [T, 3*H*d] (bf16 values) -> same with Q and K normalised and rotated."""

    out = np.array(qkv, dtype=np.float32, copy=True)
    t = out.shape[0]
    rot = cos_sin.shape[-1]
    half = rot // 2
    view = out.reshape(t, 3, heads, head_dim)
    cs = cos_sin[np.asarray(positions, dtype=np.int64)]
    idx = np.arange(head_dim)
    partner = np.where(idx < half, idx + half, idx - half)
    rotating = idx < rot
    phase = idx % half
    cos = np.where(rotating[None], cs[:, np.minimum(phase, half - 1)], 1.0).astype(np.float32)
    sin = np.where(rotating[None], cs[:, half + np.minimum(phase, half - 1)], 0.0).astype(np.float32)
    for qk, w in ((0, q_weight), (1, k_weight)):
        v = view[:, qk].astype(np.float32)                                  # [T, H, d]
        var = (v.astype(np.float64) ** 2).sum(axis=-1) / head_dim
        ve = (var.astype(np.float32) + np.float32(eps)).astype(np.float32)
        inv = (1.0 / np.sqrt(ve.astype(np.float64))).astype(np.float32)
        w = np.asarray(w, dtype=np.float32)
        normalized = round_bf16((v * inv[..., None]).astype(np.float32) * w)
        vp = v[..., np.where(rotating, partner, idx)]
        paired = round_bf16((vp * inv[..., None]).astype(np.float32) * w[np.where(rotating, partner, idx)])
        rotated = np.where(idx < half, -paired, paired).astype(np.float32)
        a = round_bf16(normalized * cos[:, None, :])
        b = round_bf16(rotated * sin[:, None, :])
        rope = round_bf16(a + b)
        view[:, qk] = np.where(rotating, rope, normalized)
    return out


__all__ = [
    "default_inv_freq",
    "packed_layout",
    "qkv_norm_rope",
    "rope_cos_sin",
    "round_bf16",
]
