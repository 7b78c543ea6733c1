"""The hook's ``sol_attn`` backend against the SOL oracle composed the reference's way.

Four clean commits (dense in the commit modes) build a history of 4 x (32 audio + 256 video)
rows with block-clustered keys; then NOISY calls:

* at a routed layer (index >= ``sol_attn_dense_layers``) the media rows equal the oracle's
  SOL-Attn over [condition, current media, audio history] as the exact sink and the video
  history routed (F/streaming/attention_hook.py:1452-1492), rel-L2 <= 1e-2, and the receipt
  counts one SOL call with the oracle's routing counts;
* with ``sol_attn_route_current_video`` the current video moves into the routed part and the
  audio queries attend densely (:1379-1451);
* in a dense layer the media rows equal dense attention over the same keys;
* a fused progress-denoise forward with the sink + recent policy routes the current
  document over [condition, media, previous document's media, audio history] exact and the
  policy's video history (F/streaming/cache.py:477-499), the previous document dense.

The inputs are seeded so that no routing decision lies within 5e-5 (log2 units) of its
threshold, far above the fp32 noise of the scores (~1e-6).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sol_attention as osol

pytestmark = pytest.mark.gpu
HEADS = 2
SCALE = 128 ** -0.5
TAU = 0.5


class Attn:
    softmax_scale = SCALE


def _document(rng: np.random.Generator, centre: np.ndarray) -> dict:
    """16 text, 32 audio, 256 video rows and a 16-row pad document; keys clustered around
    a centre per 64 rows."""

    seq = 320
    tags = np.full(seq, -1, np.int64)
    tags[:16] = 1
    tags[16:48] = 2
    tags[48:304] = 0
    k = 0.7 * rng.standard_normal((seq, HEADS, 128)) + np.repeat(centre, 64, axis=0)[:seq]
    to = lambda x: torch.from_numpy(x.astype(np.float32)).bfloat16()  # noqa: E731
    return {"q": to(rng.standard_normal((seq, HEADS, 128))), "k": to(k),
            "v": to(rng.standard_normal((seq, HEADS, 128))), "tags": torch.from_numpy(tags),
            "commit": torch.from_numpy((tags == 0) | (tags == 2)), "cu": (0, 304, 320)}


def _inputs(seed: int = 11):
    rng = np.random.default_rng(seed)
    docs = [_document(rng, rng.standard_normal((5, HEADS, 128))) for _ in range(5)]
    return docs[:4], docs[4]


def _oracle_parts(history: list[dict], y: dict, route_video: bool):
    cond, media = slice(0, 16), slice(16, 304)
    audio_hist = [(d["k"][16:48], d["v"][16:48]) for d in history]
    video_hist = [(d["k"][48:304], d["v"][48:304]) for d in history]
    if route_video:
        exact = [(y["k"][cond], y["v"][cond]), (y["k"][16:48], y["v"][16:48]), *audio_hist]
        routed = [(y["k"][48:304], y["v"][48:304]), *video_hist]
    else:
        exact = [(y["k"][cond], y["v"][cond]), (y["k"][media], y["v"][media]), *audio_hist]
        routed = video_hist
    k = torch.cat([p[0] for p in exact + routed]).float()
    v = torch.cat([p[1] for p in exact + routed]).float()
    return k, v, sum(int(p[0].shape[0]) for p in exact)


def _dense(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    p = torch.softmax(torch.einsum("qhd,khd->hqk", q.float(), k.float()) * SCALE, -1)
    return torch.einsum("hqk,khd->qhd", p, v.float())


def _hook_with_history(layers, **kw):
    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    history, y = _inputs()
    cache = CleanAVKVCache(KVContract(local_heads=HEADS, head_dim=128), layer_names=layers)
    hook = H3StreamingAttentionHook(cache, attention_backend="sol_attn", sol_attn_tau=TAU, **kw)
    for x in history:
        cache.begin_clean_commit(cache.committed_blocks)
        hook.activate(HookMode.CLEAN_COMMIT)
        for layer in layers:
            hook(attention=Attn(), layer_name=layer, query=x["q"].cuda(), key=x["k"].cuda(),
                 value=x["v"].cuda(), token_tags=x["tags"].cuda(),
                 commit_mask=x["commit"].cuda(), cu_seqlens_host=x["cu"])
        hook.deactivate()
        cache.commit()
    hook.check_device_error()
    assert hook.sol_attn_kernel_calls == 0  # commits stay dense
    return hook, history, y


def _noisy(hook, layer: str, y: dict) -> torch.Tensor:
    from h3sa.hook import HookMode

    hook.activate(HookMode.NOISY)
    out = hook(attention=Attn(), layer_name=layer, query=y["q"].cuda(), key=y["k"].cuda(),
               value=y["v"].cuda(), token_tags=y["tags"].cuda(), commit_mask=y["commit"].cuda(),
               cu_seqlens_host=y["cu"])
    hook.deactivate()
    hook.check_device_error()
    return out.float().cpu()


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a - b).norm() / b.norm())


def test_hook_sol_routes_history_video() -> None:
    hook, history, y = _hook_with_history(("blocks.0.attn", "blocks.2.attn"))
    k, v, sink = _oracle_parts(history, y, route_video=False)
    q = y["q"][16:304].float()
    want, _, margin, tele = osol.sol_attn_rectangular(q, k, v, scale=SCALE, tau=TAU,
                                                      sink_tokens=sink)
    assert float(margin.abs().min()) > 5e-5
    assert 0 < tele[0] < tele[2]  # some history video blocks routed, not all
    out = _noisy(hook, "blocks.2.attn", y)
    assert _rel(out[16:304], want) <= 1e-2
    assert _rel(out[:16], _dense(y["q"][:16], y["k"][:16], y["v"][:16])) <= 1e-2
    receipt = hook.sol_attn_receipt()
    assert receipt["kernel_calls"] == 1 and receipt["query_tokens"] == 288
    assert receipt["key_tokens"] == k.shape[0]
    assert [receipt[n] for n in ("route_selected_blocks", "exact_blocks", "routable_blocks",
                                 "candidate_blocks")] == tele.tolist()
    assert hook.attention_backend_receipt() == receipt and hook.sage_attn_receipt() is None
    # the cache's SOL history split: per block its audio rows and its video rows
    audio_parts, video_parts = hook.cache.sol_history_modality_parts("blocks.2.attn",
                                                                     fused_current=False)
    assert len(audio_parts) == 4 and len(video_parts) == 4
    for (ak, av), (vk, vv), d in zip(audio_parts, video_parts, history):
        assert torch.equal(ak.cpu(), d["k"][16:48]) and torch.equal(av.cpu(), d["v"][16:48])
        assert torch.equal(vk.cpu(), d["k"][48:304]) and torch.equal(vv.cpu(), d["v"][48:304])
    # a dense layer: the media rows see the same keys densely
    out0 = _noisy(hook, "blocks.0.attn", y)
    assert hook.sol_attn_kernel_calls == 1
    assert _rel(out0[16:304], _dense(q, k, v)) <= 1e-2
    assert _rel(out[16:304], out0[16:304]) > 2e-2  # the routing changed something


def test_hook_sol_routes_current_video() -> None:
    hook, history, y = _hook_with_history(("blocks.3.attn",), sol_attn_route_current_video=True)
    k, v, sink = _oracle_parts(history, y, route_video=True)
    qa, qv = y["q"][16:48].float(), y["q"][48:304].float()
    want, _, margin, _ = osol.sol_attn_rectangular(qv, k, v, scale=SCALE, tau=TAU,
                                                   sink_tokens=sink)
    assert float(margin.abs().min()) > 5e-5
    out = _noisy(hook, "blocks.3.attn", y)
    assert _rel(out[48:304], want) <= 1e-2
    assert _rel(out[16:48], _dense(qa, k, v)) <= 1e-2
    assert hook.sol_attn_receipt()["history_policy"].endswith("current_and_history_video")


def test_hook_sol_rejects_other_thresholds() -> None:
    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook

    cache = CleanAVKVCache(KVContract(local_heads=HEADS, head_dim=128), layer_names=("blocks.0.attn",))
    with pytest.raises(ValueError, match="diag"):
        H3StreamingAttentionHook(cache, attention_backend="sol_attn", sol_attn_thresh_type="full")


def _fused_inputs(seed: int):
    rng = np.random.default_rng(seed)
    history = [_document(rng, rng.standard_normal((5, HEADS, 128))) for _ in range(3)]
    a = _document(rng, rng.standard_normal((5, HEADS, 128)))
    b = _document(rng, rng.standard_normal((5, HEADS, 128)))
    # the packed call: document A (previous, committed by this forward), document B, a pad
    cat = lambda key: torch.cat((a[key][:304], b[key][:304], b[key][304:]))  # noqa: E731
    y = {key: cat(key) for key in ("q", "k", "v", "tags", "commit")}
    y["cu"] = (0, 304, 608, 624)
    return history, a, b, y


def _fused_oracle_parts(history: list[dict], a: dict, b: dict):
    """Document B's SOL parts in a fused forward with the sink + one recent block policy:
    [condition, current media, previous document's media, audio history of blocks 0 and 2]
    exact, the video history of blocks 0 and 2 routed (F/streaming/cache.py:477-499)."""

    seen = [history[0], history[2]]
    exact = [(b["k"][:16], b["v"][:16]), (b["k"][16:304], b["v"][16:304]),
             (a["k"][16:304], a["v"][16:304]), *[(d["k"][16:48], d["v"][16:48]) for d in seen]]
    routed = [(d["k"][48:304], d["v"][48:304]) for d in seen]
    k = torch.cat([p[0] for p in exact + routed]).float()
    v = torch.cat([p[1] for p in exact + routed]).float()
    return k, v, sum(int(p[0].shape[0]) for p in exact)


FUSED_SEED = 31


def test_hook_sol_fused_progress_denoise() -> None:
    """FUSED_PROGRESS_DENOISE with fused_current_use_sink / fused_current_recent_blocks: the
    previous document attends densely to its condition, the whole history and its media; the
    current one through SOL over the parts above; the previous document is committed."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    layer = "blocks.2.attn"
    history, a, b, y = _fused_inputs(FUSED_SEED)
    k, v, sink = _fused_oracle_parts(history, a, b)
    qb = b["q"][16:304].float()
    want, _, margin, _ = osol.sol_attn_rectangular(qb, k, v, scale=SCALE, tau=TAU,
                                                   sink_tokens=sink)
    assert float(margin.abs().min()) > 5e-5

    cache = CleanAVKVCache(KVContract(local_heads=HEADS, head_dim=128), layer_names=(layer,))
    hook = H3StreamingAttentionHook(cache, attention_backend="sol_attn", sol_attn_tau=TAU)
    for i, x in enumerate(history):
        cache.begin_clean_commit(cache.committed_blocks)
        hook.activate(mode=HookMode.CLEAN_COMMIT, block_index=i)
        hook(attention=Attn(), layer_name=layer, query=x["q"].cuda(), key=x["k"].cuda(),
             value=x["v"].cuda(), token_tags=x["tags"].cuda(), commit_mask=x["commit"].cuda(),
             cu_seqlens_host=x["cu"])
        hook.deactivate()
        cache.commit()
    cache.begin_clean_commit(cache.committed_blocks)
    hook.activate(mode=HookMode.FUSED_PROGRESS_DENOISE, block_index=3, denoise_step_index=1,
                  fused_current_use_sink=True, fused_current_recent_blocks=2)
    out = hook(attention=Attn(), layer_name=layer, query=y["q"].cuda(), key=y["k"].cuda(),
               value=y["v"].cuda(), token_tags=y["tags"].cuda(), commit_mask=y["commit"].cuda(),
               cu_seqlens_host=y["cu"]).float().cpu()
    hook.deactivate()
    cache.commit()
    hook.check_device_error()
    assert hook.sol_attn_kernel_calls == 1
    assert _rel(out[320:608], want) <= 1e-2
    hk = torch.cat([d["k"][16:304] for d in history])
    hv = torch.cat([d["v"][16:304] for d in history])
    ka = torch.cat((a["k"][:16], hk, a["k"][16:304]))
    va = torch.cat((a["v"][:16], hv, a["v"][16:304]))
    assert _rel(out[16:304], _dense(a["q"][16:304], ka, va)) <= 1e-2
    assert cache.committed_blocks == 4 and cache.commit_token_counts[-1] == 288
