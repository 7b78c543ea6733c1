"""The drop-in hook and paged cache on the GPU, against the oracle and reference goldens.

* Cache: the reference's own commit / retain / audio-drop schedule (tests/golden/cache.npz)
  replayed through the paged cache; history row tables must match exactly.
* Hook: the CPU benchmark configuration's structure (16 text, 32 audio, 256 video, 16 pad
  rows, 1024 cached rows) at head_dim 128, dense / FP8 / block-sparse backends, contiguous
  and scattered condition rows, NOISY and CLEAN_COMMIT modes.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from oracle import attention as oatt  # noqa: E402
from oracle import block_mask as omask  # noqa: E402

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
FP8_TOL = 3e-2


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm())


class Attn:
    softmax_scale = 128 ** -0.5


def test_cache_schedule_matches_reference_golden() -> None:
    from h3sa.cache import MAIN_LAYER_NAMES, CleanAVKVCache, KVContract

    with np.load(GOLDEN / "cache.npz") as f:
        g = {k: f[k] for k in f.files}
    cache = CleanAVKVCache(KVContract(local_heads=1, head_dim=8), initial_pages=1)
    serial = 0
    for i, op in enumerate(g["ops"]):
        if op == "commit":
            tags = torch.from_numpy(g[f"tags_{i}"])
            commit = (tags == 0) | (tags == 2)
            ids = torch.zeros(len(tags), 1, 8)
            staged = torch.nonzero(commit).flatten()
            ids[staged, 0, 0] = serial
            ids[staged, 0, 1] = torch.arange(staged.numel(), dtype=torch.float32)
            kv = ids.to(torch.bfloat16).cuda()
            cache.begin_clean_commit(cache.committed_blocks)
            for name in MAIN_LAYER_NAMES:
                cache.stage(name, kv, kv.clone(), tags.cuda(), commit.cuda())
            cache.commit()
            serial += 1
        elif op == "retain":
            cache.retain_sink_and_recent_commits()
        else:
            assert cache.drop_audio_history() == int(g[f"removed_{i}"])
        for name in ("blocks.0.attn", "blocks.49.attn"):
            hist = cache.history(name)
            rows = np.zeros((0, 2), np.int64) if hist is None else \
                hist.key[:, 0, :2].float().cpu().numpy().astype(np.int64)
            assert np.array_equal(rows, g[f"rows_{i}"]), (i, op, name)
        assert cache.history_tokens == g[f"rows_{i}"].shape[0]


def _layout(heads: int, hist: int, scattered: bool, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    seq = 320
    tags = np.full(seq, -1, np.int64)
    tags[:16] = 1
    tags[16:48] = 2
    tags[48:304] = 0
    if scattered:  # condition rows interleaved with media inside the live document
        tags[:304] = np.concatenate([tags[16:48], tags[:8], tags[48:304], tags[8:16]])
    def rms(x):
        return x / np.sqrt((x ** 2).mean(-1, keepdims=True) + 1e-5)
    t = lambda x: torch.from_numpy(x.astype(np.float32)).bfloat16().cuda()  # noqa: E731
    return {
        "q": t(rms(rng.standard_normal((seq, heads, 128)))),
        "k": t(rms(rng.standard_normal((seq, heads, 128)))),
        "v": t(rng.standard_normal((seq, heads, 128))),
        "hist_k": t(rms(rng.standard_normal((hist, heads, 128)))),
        "hist_v": t(rng.standard_normal((hist, heads, 128))),
        "tags": torch.from_numpy(tags).cuda(),
        "commit": torch.from_numpy((tags == 0) | (tags == 2)).cuda(),
        "cu": (0, 304, 320),
    }


def _cache_with_history(heads: int, x: dict, layer: str = "blocks.0.attn"):
    from h3sa.cache import CleanAVKVCache, KVContract

    cache = CleanAVKVCache(KVContract(local_heads=heads, head_dim=128),
                           layer_names=(layer,))
    n = x["hist_k"].shape[0]
    if n:
        paged = cache.layer(layer)
        paged.write(x["hist_k"], x["hist_v"], start=0, count=n)
        paged.history_rows = n
        cache._commit_token_counts.append(n)
        cache._commit_token_tags.append(tuple([0] * n))
    return cache


def _oracle(x: dict, hist: bool = True) -> torch.Tensor:
    return oatt.streaming_hook_attention(
        x["q"].float().cpu(), x["k"].float().cpu(), x["v"].float().cpu(), x["commit"].cpu(),
        x["cu"], (x["hist_k"].float().cpu(), x["hist_v"].float().cpu()) if hist else None,
        Attn.softmax_scale)


@pytest.mark.parametrize("scattered", [False, True])
def test_hook_dense_matches_oracle(scattered: bool) -> None:
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads = 4
    x = _layout(heads, 1024, scattered)
    cache = _cache_with_history(heads, x)
    hook = H3StreamingAttentionHook(cache)
    hook.activate(HookMode.NOISY)
    out = hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
               value=x["v"], token_tags=x["tags"], commit_mask=x["commit"],
               cu_seqlens_host=x["cu"])
    hook.check_device_error()
    assert rel_l2(out, _oracle(x)) <= BF16_TOL
    assert cache.history_rows("blocks.0.attn") == 1024  # NOISY never mutates history


def test_hook_clean_commit_then_reads_new_history() -> None:
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads = 4
    x = _layout(heads, 0, False, seed=5)
    cache = _cache_with_history(heads, x)
    hook = H3StreamingAttentionHook(cache)
    cache.begin_clean_commit(cache.committed_blocks)
    hook.activate(HookMode.CLEAN_COMMIT)
    out = hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
               value=x["v"], token_tags=x["tags"], commit_mask=x["commit"],
               cu_seqlens_host=x["cu"])
    hook.deactivate()
    cache.commit()
    assert rel_l2(out, _oracle(x, hist=False)) <= BF16_TOL
    hist = cache.history("blocks.0.attn")
    media = torch.nonzero(x["commit"]).flatten()
    assert torch.equal(hist.key, x["k"][media]) and torch.equal(hist.value, x["v"][media])
    # next chunk attends to the committed media rows as history
    y = _layout(heads, 0, False, seed=6)
    hook.activate(HookMode.NOISY)
    out2 = hook(attention=Attn(), layer_name="blocks.0.attn", query=y["q"], key=y["k"],
                value=y["v"], token_tags=y["tags"], commit_mask=y["commit"],
                cu_seqlens_host=y["cu"])
    y["hist_k"], y["hist_v"] = hist.key, hist.value
    assert rel_l2(out2, _oracle(y)) <= BF16_TOL


def test_hook_fp8_dynamic_matches_dequantised_oracle() -> None:
    import h3sa
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads = 4
    x = _layout(heads, 1024, False, seed=2)
    cache = _cache_with_history(heads, x)
    hook = H3StreamingAttentionHook(cache, backend="flash_attn3_fp8_dynamic")
    hook.activate(HookMode.NOISY)
    out = hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
               value=x["v"], token_tags=x["tags"], commit_mask=x["commit"],
               cu_seqlens_host=x["cu"])
    hook.check_device_error()
    # media rows: per-head e4m3 over [cond | history | media] K and V and over media Q
    media = torch.arange(16, 304, device="cuda")  # audio + video rows of the live document
    cond = torch.arange(0, 16, device="cuda")
    k_all = torch.cat([x["k"][cond], x["hist_k"], x["k"][media]])
    v_all = torch.cat([x["v"][cond], x["hist_v"], x["v"][media]])
    deq = lambda t: (lambda q, s: q.float() * s.reshape(1, 1, -1, 1))(*h3sa.quantize_fp8_e4m3_per_head(t.unsqueeze(0)))  # noqa: E731
    ref_media = oatt.attention(deq(x["q"][media])[0].cpu(), deq(k_all)[0].cpu(), deq(v_all)[0].cpu(),
                               Attn.softmax_scale)
    assert rel_l2(out[16:304], ref_media) <= FP8_TOL
    # condition rows: their own e4m3 call over the condition rows' Q/K/V
    ref_cond = oatt.attention(deq(x["q"][cond])[0].cpu(), deq(x["k"][cond])[0].cpu(),
                              deq(x["v"][cond])[0].cpu(), Attn.softmax_scale)
    assert rel_l2(out[:16], ref_cond) <= FP8_TOL


def test_hook_block_sparse_matches_masked_oracle() -> None:
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads, hist = 2, 2048
    x = _layout(heads, hist, False, seed=3)
    cache = _cache_with_history(heads, x)
    density = 0.3
    hook = H3StreamingAttentionHook(cache, backend="flex_dynamic_blocksparse",
                                    history_density=density)
    hook.activate(HookMode.NOISY)
    out = hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
               value=x["v"], token_tags=x["tags"], commit_mask=x["commit"],
               cu_seqlens_host=x["cu"])
    hook.check_device_error()
    media = slice(16, 304)  # audio + video rows of the live document
    q = x["q"][media].float().cpu()
    # logical KV [history | media | cond], mask per the reference rule on that sequence
    k_all = torch.cat([x["hist_k"], x["k"][media], x["k"][:16]]).float().cpu()
    v_all = torch.cat([x["hist_v"], x["v"][media], x["v"][:16]]).float().cpu()
    m = omask.dynamic_history_mask(q.numpy().transpose(1, 0, 2),
                                   k_all[:hist].numpy().transpose(1, 0, 2), k_all.shape[0], density)
    nq, nk = q.shape[0], k_all.shape[0]
    allowed = torch.zeros(heads, nq, nk, dtype=torch.bool)
    for h in range(heads):
        for j in range(m["kv_num_blocks"].shape[1]):
            for b in m["kv_indices"][h, j, : m["kv_num_blocks"][h, j]]:
                allowed[h, j * 128:(j + 1) * 128, b * 128:(b + 1) * 128] = True
    ref = oatt.attention(q, k_all, v_all, Attn.softmax_scale, allowed)
    assert rel_l2(out[media], ref) <= BF16_TOL
    assert math.isclose(float(m["selected_count"]), math.ceil(hist // 128 * density))


def test_hook_rejects_like_reference() -> None:
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads = 4
    x = _layout(heads, 0, False)
    cache = _cache_with_history(heads, x)
    hook = H3StreamingAttentionHook(cache)
    with pytest.raises(RuntimeError, match="called while inactive"):
        hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
             value=x["v"], token_tags=x["tags"], commit_mask=x["commit"], cu_seqlens_host=x["cu"])
    hook.activate(HookMode.NOISY)
    with pytest.raises(RuntimeError, match="invalid packed sequence boundaries"):
        hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
             value=x["v"], token_tags=x["tags"], commit_mask=x["commit"], cu_seqlens_host=(0, 5))
    two_live = x["commit"].clone()
    two_live[310] = True
    with pytest.raises(RuntimeError, match="exactly one live document"):
        hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
             value=x["v"], token_tags=x["tags"], commit_mask=two_live, cu_seqlens_host=x["cu"])


def test_hook_fp8_segmented_history_matches_merged_oracle() -> None:
    """Three clean commits with different value ranges build a segmented e4m3 history (each
    block quantised once at commit with its own scales); retention then keeps block 0's video
    rows (with block 0's scales) and the recent blocks. A NOISY call attends over the parts plus
    the current media and condition parts; the media rows must match the reference's
    segmented backend (one FP8 attention per part, LSE merge) on the same quantised bytes."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode
    from oracle import fp8 as ofp8

    heads = 2
    cache = CleanAVKVCache(KVContract(local_heads=heads, head_dim=128),
                           layer_names=("blocks.0.attn",), segmented_fp8_history=True)
    hook = H3StreamingAttentionHook(cache, backend="flash_attn3_fp8_segmented")
    committed = []
    for i in range(3):
        x = _layout(heads, 0, False, seed=20 + i)
        x["k"] = (x["k"].float() * (1 + i)).bfloat16()
        x["v"] = (x["v"].float() / (1 + 2 * i)).bfloat16()
        cache.begin_clean_commit(cache.committed_blocks)
        hook.activate(HookMode.CLEAN_COMMIT)
        hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
             value=x["v"], token_tags=x["tags"], commit_mask=x["commit"], cu_seqlens_host=x["cu"])
        hook.deactivate()
        cache.commit()
        media = torch.nonzero(x["commit"]).flatten()
        committed.append((x["k"][media], x["v"][media], x["tags"][media]))
    hook.check_device_error()
    cache.retain_sink_and_recent_commits()  # block 0 keeps its video rows only

    def q8(t: torch.Tensor):
        q, s = ofp8.quantize_fp8_e4m3_per_head(t.float().cpu().numpy()[None])
        return q[0], s[0]

    parts = []
    for i, (k, v, tags) in enumerate(committed):
        (k8, ks), (v8, vs) = q8(k), q8(v)
        if i == 0:
            video = (tags == 0).cpu().numpy()
            k8, v8 = k8[video], v8[video]
        parts.append((k8, v8, ks, vs))
    y = _layout(heads, 0, False, seed=30)
    hook.activate(HookMode.NOISY)
    out = hook(attention=Attn(), layer_name="blocks.0.attn", query=y["q"], key=y["k"],
               value=y["v"], token_tags=y["tags"], commit_mask=y["commit"], cu_seqlens_host=y["cu"])
    hook.check_device_error()
    media = torch.arange(16, 304, device="cuda")
    cond = torch.arange(0, 16, device="cuda")
    (ck8, cks), (cv8, cvs) = q8(y["k"][cond]), q8(y["v"][cond])
    (mk8, mks), (mv8, mvs) = q8(y["k"][media]), q8(y["v"][media])
    ref = oatt.segmented_fp8_attention(y["q"][media].float().cpu(),
                                       [(ck8, cv8, cks, cvs), *parts, (mk8, mv8, mks, mvs)],
                                       Attn.softmax_scale)
    assert rel_l2(out[16:304], ref) <= FP8_TOL
    # condition rows see condition K/V only, in their own e4m3 call
    ref_cond = oatt.segmented_fp8_attention(y["q"][cond].float().cpu(), [(ck8, cv8, cks, cvs)],
                                            Attn.softmax_scale)
    assert rel_l2(out[:16], ref_cond) <= FP8_TOL


def test_fl2av_cache_schedule_matches_reference_golden() -> None:
    """The FL2AV cache operations on the paged cache (bounded commits, count-based and sink +
    recent retention, audio drop, strided attention history) against the row tables of the
    reference's own F CleanAVKVCache (tests/golden/cache_f.npz), with a segmented e4m3
    history kept alongside."""

    from h3sa.cache import CleanAVKVCache, KVContract

    with np.load(GOLDEN / "cache_f.npz") as f:
        g = {k: f[k] for k in f.files}
    layer = "blocks.0.attn"
    cache = CleanAVKVCache(KVContract(local_heads=1, head_dim=128), layer_names=(layer,),
                           segmented_fp8_history=True)
    serial = 0

    def table(view) -> np.ndarray:
        if view is None:
            return np.zeros((0, 2), np.int64)
        return view.key[:, 0, :2].float().cpu().numpy().astype(np.int64)

    for i, step in enumerate(g["schedule"]):
        op, *args = str(step).split("|")
        if op in ("commit", "bounded"):
            tags = g[f"tags_{i}"]
            commit = (tags == 0) | (tags == 2)
            ids = torch.zeros(len(tags), 1, 128)
            staged = torch.from_numpy(np.nonzero(commit)[0])
            ids[staged, 0, 0] = serial
            ids[staged, 0, 1] = torch.arange(staged.numel()).float()
            kv = ids.bfloat16().cuda()
            cache.begin_clean_commit(cache.committed_blocks)
            cache.stage(layer, kv, kv.clone(), torch.from_numpy(tags).cuda(),
                        torch.from_numpy(commit).cuda())
            if op == "commit":
                cache.commit()
            else:
                cache.commit(retain_recent_commit_count=int(args[0]))
            serial += 1
        elif op == "sink_recent":
            cache.retain_sink_and_recent_commits(int(args[0]), sink_video_only=args[1] == "True")
        elif op == "retain_recent":
            cache.retain_recent_commits(int(args[0]))
        elif op == "drop":
            assert cache.drop_audio_history() == int(g[f"removed_{i}"])
        elif op == "attn":
            got = cache.attention_history(layer, count=int(args[0]), recent_full_blocks=int(args[1]),
                                          older_video_stride=int(args[2]),
                                          preserve_sink=args[3] == "True")
            assert np.array_equal(table(got), g[f"attn_{i}"]), i
        assert np.array_equal(table(cache.history(layer)), g[f"rows_{i}"]), i
        assert list(cache.commit_token_counts) == g[f"counts_{i}"].tolist(), i
        assert cache.committed_blocks == int(g[f"blocks_{i}"]), i
        # the e4m3 history holds one part per retained block, with the same row counts
        seg = cache.layer(layer).fp8
        assert seg.rows == list(cache.commit_token_counts), i
        blocks = cache.history_blocks(layer)
        assert [int(b.key.shape[0]) for b in blocks] == list(cache.commit_token_counts), i


def test_hook_fl2av_call_form_matches_t_form() -> None:
    """The FL2AV call (device cu_seqlens, max_seqlen, live_documents_hint) gives the same
    bits as the T call with host boundaries."""

    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads = 2
    x = _layout(heads, 512, False, seed=8)
    outs = []
    for form in ("t", "f"):
        cache = _cache_with_history(heads, x)
        hook = H3StreamingAttentionHook(cache)
        hook.activate(HookMode.NOISY)
        kw = dict(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
                  value=x["v"], token_tags=x["tags"], commit_mask=x["commit"])
        if form == "t":
            out = hook(**kw, cu_seqlens_host=x["cu"])
        else:
            out = hook(**kw, cu_seqlens_host=None,
                       cu_seqlens=torch.tensor(x["cu"], dtype=torch.int32, device="cuda"),
                       max_seqlen=304, live_documents_hint=(0,))
        hook.check_device_error()
        outs.append(out)
    assert torch.equal(outs[0], outs[1])


def test_hook_fp8_segmented_topk_attends_selected_commits() -> None:
    """flash_attn3_fp8_segmented_topk: four commits whose keys carry different offsets, then a
    NOISY call at density 0.5. The hook must keep the two commits the oracle's summaries and
    scores select (F/streaming/attention_hook.py:1256-1302) and its media rows must match the
    segmented oracle over [condition, selected commits, current media]; the counters follow
    the reference's."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode
    from oracle import commit_topk as otopk
    from oracle import fp8 as ofp8

    heads = 2
    cache = CleanAVKVCache(KVContract(local_heads=heads, head_dim=128),
                           layer_names=("blocks.0.attn",), segmented_fp8_history=True)
    hook = H3StreamingAttentionHook(cache, attention_backend="flash_attn3_fp8_segmented_topk",
                                    history_kv_dynamic_density=0.5)
    gen = torch.Generator(device="cuda").manual_seed(3)
    committed = []
    for i in range(4):
        x = _layout(heads, 0, False, seed=40 + i)
        offset = torch.randn(1, heads, 128, device="cuda", generator=gen)
        x["k"] = (x["k"].float() + 0.5 * offset).bfloat16()
        cache.begin_clean_commit(cache.committed_blocks)
        hook.activate(HookMode.CLEAN_COMMIT)
        hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"],
             value=x["v"], token_tags=x["tags"], commit_mask=x["commit"], cu_seqlens_host=x["cu"])
        hook.deactivate()
        cache.commit()
        media = torch.nonzero(x["commit"]).flatten()
        committed.append((x["k"][media], x["v"][media]))
    hook.check_device_error()
    calls_before = hook.dynamic_block_sparse_call_count

    y = _layout(heads, 0, False, seed=50)
    y["q"] = (y["q"].float() + 0.5 * torch.randn(1, heads, 128, device="cuda",
                                                 generator=gen)).bfloat16()
    media = torch.arange(16, 304, device="cuda")
    cond = torch.arange(0, 16, device="cuda")
    summaries = np.stack([otopk.key_summary(k.float().cpu().numpy()) for k, _ in committed])
    scores = otopk.commit_scores(summaries, otopk.key_summary(y["q"][media].float().cpu().numpy()))
    selected = otopk.select_commits(scores, 0.5)
    assert len(selected) == 2
    hook.activate(HookMode.NOISY)
    out = hook(attention=Attn(), layer_name="blocks.0.attn", query=y["q"], key=y["k"],
               value=y["v"], token_tags=y["tags"], commit_mask=y["commit"], cu_seqlens_host=y["cu"])
    hook.deactivate()
    hook.check_device_error()
    assert hook.dynamic_block_sparse_call_count == calls_before + 1
    assert hook.dynamic_block_sparse_selected_blocks >= 2

    def q8(t: torch.Tensor):
        q, s = ofp8.quantize_fp8_e4m3_per_head(t.float().cpu().numpy()[None])
        return q[0], s[0]

    def part(k: torch.Tensor, v: torch.Tensor):
        (k8, ks), (v8, vs) = q8(k), q8(v)
        return k8, v8, ks, vs

    parts = [part(*committed[i]) for i in selected]
    (ck8, cks), (cv8, cvs) = q8(y["k"][cond]), q8(y["v"][cond])
    (mk8, mks), (mv8, mvs) = q8(y["k"][media]), q8(y["v"][media])
    ref = oatt.segmented_fp8_attention(y["q"][media].float().cpu(),
                                       [(ck8, cv8, cks, cvs), *parts, (mk8, mv8, mks, mvs)],
                                       Attn.softmax_scale)
    assert rel_l2(out[16:304], ref) <= FP8_TOL
    # attending to every commit instead gives a measurably different result
    every = oatt.segmented_fp8_attention(
        y["q"][media].float().cpu(),
        [(ck8, cv8, cks, cvs), *[part(k, v) for k, v in committed], (mk8, mv8, mks, mvs)],
        Attn.softmax_scale)
    assert rel_l2(every, ref) > 2 * FP8_TOL


@pytest.mark.parametrize("segmented", [False, True])
def test_cache_snapshot_round_trip_resumes_bit_exact(tmp_path, segmented: bool) -> None:
    """A cache written to disk and loaded into a fresh process-side object (h3sa.snapshot)
    holds the same history bytes, e4m3 parts, scales, summaries and bookkeeping; a NOISY call
    and a further clean commit on the restored cache give bit-identical results to the
    original's."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads = 2
    layers = ("blocks.0.attn", "blocks.1.attn")
    backend = "flash_attn3_fp8_segmented" if segmented else "flash_attn_3"
    cache = CleanAVKVCache(KVContract(local_heads=heads, head_dim=128), layer_names=layers,
                           segmented_fp8_history=segmented)

    def step(c: CleanAVKVCache, x: dict, mode: HookMode) -> list[torch.Tensor]:
        hook = H3StreamingAttentionHook(c, backend=backend)
        if mode is HookMode.CLEAN_COMMIT:
            c.begin_clean_commit(c.committed_blocks)
        hook.activate(mode)
        outs = [hook(attention=Attn(), layer_name=name, query=x["q"], key=x["k"], value=x["v"],
                     token_tags=x["tags"], commit_mask=x["commit"], cu_seqlens_host=x["cu"])
                for name in layers]
        hook.deactivate()
        if mode is HookMode.CLEAN_COMMIT:
            c.commit()
        hook.check_device_error()
        return outs

    for i in range(3):
        step(cache, _layout(heads, 0, False, seed=60 + i), HookMode.CLEAN_COMMIT)
    cache.retain_sink_and_recent_commits()  # block 0 keeps its video rows only
    path = tmp_path / "cache.h3kv"
    cache.save_snapshot(path)
    restored = CleanAVKVCache.load_snapshot(path, contract=KVContract(local_heads=heads,
                                                                     head_dim=128))
    assert restored.committed_blocks == cache.committed_blocks
    assert restored.commit_token_counts == cache.commit_token_counts
    assert restored.commit_token_tags() == cache.commit_token_tags()
    for name in layers:
        a, b = cache.history(name), restored.history(name)
        assert torch.equal(a.key, b.key) and torch.equal(a.value, b.value), name
        if segmented:
            sa, sb = cache.layer(name).fp8, restored.layer(name).fp8
            assert sa.rows == sb.rows
            assert torch.equal(sa.k_scale, sb.k_scale) and torch.equal(sa.v_scale, sb.v_scale)
            assert torch.equal(sa.key_summary, sb.key_summary)
            for (s0, n), (t0, m) in zip(zip(sa.starts, sa.rows), zip(sb.starts, sb.rows)):
                ka, kb = sa.store.materialize(s0 + n), sb.store.materialize(t0 + m)
                assert torch.equal(ka[0][s0:].view(torch.uint8), kb[0][t0:].view(torch.uint8))
                assert torch.equal(ka[1][s0:].view(torch.uint8), kb[1][t0:].view(torch.uint8))
    y = _layout(heads, 0, False, seed=70)
    for got, want in zip(step(restored, y, HookMode.NOISY), step(cache, y, HookMode.NOISY)):
        assert torch.equal(got, want)
    z = _layout(heads, 0, False, seed=71)
    step(cache, z, HookMode.CLEAN_COMMIT)
    step(restored, z, HookMode.CLEAN_COMMIT)
    for got, want in zip(step(restored, y, HookMode.NOISY), step(cache, y, HookMode.NOISY)):
        assert torch.equal(got, want)
    # a flipped byte is refused before anything reaches the device
    from h3sa.snapshot import read_header

    header, base = read_header(path)
    last = header["sections"][-1]
    raw = bytearray(path.read_bytes())
    raw[base + last["offset"] + last["nbytes"] - 5] ^= 0x40
    bad = tmp_path / "bad.h3kv"
    bad.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="CRC-32"):
        CleanAVKVCache.load_snapshot(bad)


def test_fl2av_hook_modes_match_reference_golden() -> None:
    """The FL2AV activation form through every mode, replaying tests/golden/hook_f.npz (the
    reference hook's own outputs): clean and progress commits, a full-prefix capture (its
    rows bit-exact), a noisy call over the captured prefix, fused progress-denoise forwards
    with and without the recent / sink / previous-video-only policy (each committing the
    previous document) and a final noisy call. Layer 0's outputs within 1e-2 relative L2 of
    the reference's bf16 SDPA, commit ledgers identical."""

    sys.path.insert(0, str(GOLDEN))
    from inputs import HOOK_F_SCHEDULE, hook_f_inputs

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    g = np.load(GOLDEN / "hook_f.npz")
    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128))
    hook = H3StreamingAttentionHook(cache, attention_backend="sdpa")
    modes = {"clean_commit": HookMode.CLEAN_COMMIT, "progress_commit": HookMode.PROGRESS_COMMIT,
             "noisy_prefix": HookMode.NOISY, "noisy": HookMode.NOISY,
             "fused_recent": HookMode.FUSED_PROGRESS_DENOISE,
             "fused": HookMode.FUSED_PROGRESS_DENOISE}
    t = lambda a, dt=torch.bfloat16: torch.from_numpy(a).to(dt).cuda()  # noqa: E731
    prefix = None
    for step, (name, live, extra) in enumerate(HOOK_F_SCHEDULE):
        x = hook_f_inputs(step, live)
        commit = False
        if name == "capture":
            hook.begin_full_prefix_capture(**extra)
        else:
            kw = dict(extra)
            kw["full_prefix"] = prefix if name in ("noisy_prefix", "fused_recent") else None
            if name == "fused_recent":
                kw["fused_previous_full_prefix"] = prefix
                cache.retain_sink_and_recent_commits(cache.retained_blocks, sink_video_only=True)
            mode = modes[name]
            commit = mode in (HookMode.CLEAN_COMMIT, HookMode.PROGRESS_COMMIT,
                              HookMode.FUSED_PROGRESS_DENOISE)
            if commit:
                cache.begin_clean_commit(cache.committed_blocks)
            hook.activate(mode=mode, block_index=cache.committed_blocks, **kw)
        q, k, v = t(x["q"]), t(x["k"]), t(x["v"])
        tags, mask = t(x["token_tags"], torch.int64), t(x["commit_mask"], torch.bool)
        for layer in cache.layer_names:
            out = hook(attention=Attn(), layer_name=layer, query=q, key=k, value=v,
                       token_tags=tags, commit_mask=mask, cu_seqlens=None,
                       cu_seqlens_host=tuple(x["cu_seqlens"]), max_seqlen=64)
            if layer == cache.layer_names[0]:
                first = out
        hook.check_device_error()
        assert rel_l2(first, torch.from_numpy(g[f"out_{step}"])) <= BF16_TOL, (step, name)
        if name == "capture":
            prefix = hook.finish_full_prefix_capture()
            pair = prefix.get(cache.layer_names[0])
            assert torch.equal(pair.key.float().cpu(), torch.from_numpy(g["prefix_key"]))
            assert torch.equal(pair.value.float().cpu(), torch.from_numpy(g["prefix_value"]))
        else:
            hook.deactivate()
            if commit:
                cache.commit()
        assert list(cache.commit_token_counts) == list(g[f"counts_{step}"]), step
        assert cache.committed_blocks == int(g[f"blocks_{step}"]), step


def test_fl2av_activation_checks_match_reference() -> None:
    """The FL2AV activate() checks and messages (F/streaming/attention_hook.py:577-620)."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128), layer_names=("blocks.0.attn",))
    hook = H3StreamingAttentionHook(cache, attention_backend="sdpa")
    with pytest.raises(ValueError, match="block differs from clean history"):
        hook.activate(mode=HookMode.NOISY, block_index=1, full_prefix=None)
    with pytest.raises(ValueError, match="requires fused progress-denoise mode"):
        hook.activate(mode=HookMode.NOISY, block_index=0, full_prefix=None,
                      fused_previous_video_only=True)
    with pytest.raises(ValueError, match="fused current history policy"):
        hook.activate(mode=HookMode.CLEAN_COMMIT, block_index=0, full_prefix=None,
                      fused_current_recent_blocks=2)
    with pytest.raises(ValueError, match="denoise step index requires"):
        hook.activate(mode=HookMode.CLEAN_COMMIT, block_index=0, full_prefix=None,
                      denoise_step_index=1)
    hook.activate(mode=HookMode.NOISY, block_index=0, full_prefix=None)
    with pytest.raises(RuntimeError, match="already active"):
        hook.activate(mode=HookMode.NOISY, block_index=0, full_prefix=None)
    hook.deactivate()
    with pytest.raises(RuntimeError, match="no H3 full-prefix capture is active"):
        hook.finish_full_prefix_capture()
    with pytest.raises(ValueError, match="video_rows must be positive"):
        hook.begin_full_prefix_capture(video_rows=0)
    fp8 = H3StreamingAttentionHook(cache, attention_backend="flash_attn3_fp8_dynamic")
    with pytest.raises(ValueError, match="need a dense backend"):
        fp8.activate(mode=HookMode.FUSED_PROGRESS_DENOISE, block_index=0, full_prefix=None)
    # a fused forward needs two live documents
    x = _layout(2, 0, False, seed=80)
    hook.activate(mode=HookMode.FUSED_PROGRESS_DENOISE, block_index=0, full_prefix=None)
    with pytest.raises(ValueError, match="target-document count differs"):
        hook(attention=Attn(), layer_name="blocks.0.attn", query=x["q"], key=x["k"], value=x["v"],
             token_tags=x["tags"], commit_mask=x["commit"], cu_seqlens_host=x["cu"])
    hook.deactivate()


def test_hook_fp8_segmented_topk_matches_reference_hook_golden() -> None:
    """The top-k segmented backend against the reference FL2AV hook itself
    (tests/golden/hook_topk.npz: its own e4m3 quantisation, commit-level selection at density
    0.5 and LSE merge, FlashAttention-3's FP8 call replaced by exact attention on the
    dequantised inputs) over four clean commits and a noisy call: every step's layer-0 output
    within the FP8 tolerance, selection counters equal."""

    sys.path.insert(0, str(GOLDEN))
    from inputs import hook_topk_inputs

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    g = np.load(GOLDEN / "hook_topk.npz")
    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128), segmented_fp8_history=True)
    hook = H3StreamingAttentionHook(cache, attention_backend="flash_attn3_fp8_segmented_topk",
                                    history_kv_dynamic_density=0.5)
    t = lambda a, dt=torch.bfloat16: torch.from_numpy(a).to(dt).cuda()  # noqa: E731
    for step in range(5):
        x = hook_topk_inputs(step)
        commit = step < 4
        if commit:
            cache.begin_clean_commit(cache.committed_blocks)
        hook.activate(mode=HookMode.CLEAN_COMMIT if commit else HookMode.NOISY,
                      block_index=cache.committed_blocks, full_prefix=None)
        q, k, v = t(x["q"]), t(x["k"]), t(x["v"])
        tags, mask = t(x["token_tags"], torch.int64), t(x["commit_mask"], torch.bool)
        for layer in cache.layer_names:
            out = hook(attention=Attn(), layer_name=layer, query=q, key=k, value=v,
                       token_tags=tags, commit_mask=mask, cu_seqlens=None,
                       cu_seqlens_host=tuple(x["cu_seqlens"]), max_seqlen=64)
            if layer == cache.layer_names[0]:
                first = out
        hook.deactivate()
        hook.check_device_error()
        if commit:
            cache.commit()
        ref = torch.from_numpy(g[f"out_{step}"])
        assert rel_l2(first[:64], ref[:64]) <= FP8_TOL, step          # the live document
        assert rel_l2(first[64:], ref[64:]) <= FP8_TOL, step          # the pad document
        assert hook.dynamic_block_sparse_selected_blocks == int(g[f"selected_blocks_{step}"])


def test_fl2av_hook_policies_match_reference_golden() -> None:
    """The FL2AV hook's strided older history (history_kv_older_video_stride,
    history_kv_recent_full_blocks) and strided current video keys (current_video_kv_stride)
    through commits, noisy and fused calls, and dense_current_document_when_empty on a first
    call with no history, replaying tests/golden/hook_f_policy.npz (the reference hook's own
    outputs). A hook without the policies gives measurably different outputs."""

    sys.path.insert(0, str(GOLDEN))
    from inputs import HOOK_F_POLICY, HOOK_F_POLICY_SCHEDULE, hook_f_inputs

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    g = np.load(GOLDEN / "hook_f_policy.npz")
    modes = {"clean_commit": HookMode.CLEAN_COMMIT, "noisy": HookMode.NOISY,
             "fused": HookMode.FUSED_PROGRESS_DENOISE}
    t = lambda a, dt=torch.bfloat16: torch.from_numpy(a).to(dt).cuda()  # noqa: E731

    def run(hook, cache, step, name, live, extra):
        x = hook_f_inputs(100 + step, live)
        mode = modes[name]
        commit = mode is not HookMode.NOISY
        if commit:
            cache.begin_clean_commit(cache.committed_blocks)
        hook.activate(mode=mode, block_index=cache.committed_blocks, full_prefix=None, **extra)
        q, k, v = t(x["q"]), t(x["k"]), t(x["v"])
        tags, mask = t(x["token_tags"], torch.int64), t(x["commit_mask"], torch.bool)
        first = None
        for layer in cache.layer_names:
            out = hook(attention=Attn(), layer_name=layer, query=q, key=k, value=v,
                       token_tags=tags, commit_mask=mask, cu_seqlens=None,
                       cu_seqlens_host=tuple(x["cu_seqlens"]), max_seqlen=64)
            if first is None:
                first = out
        hook.check_device_error()
        hook.deactivate()
        if commit:
            cache.commit()
        return first

    caches = [CleanAVKVCache(KVContract(local_heads=2, head_dim=128)) for _ in range(2)]
    hooks = [H3StreamingAttentionHook(caches[0], attention_backend="sdpa", **HOOK_F_POLICY),
             H3StreamingAttentionHook(caches[1], attention_backend="sdpa")]
    for step, (name, live, extra) in enumerate(HOOK_F_POLICY_SCHEDULE):
        out = run(hooks[0], caches[0], step, name, live, extra)
        plain = run(hooks[1], caches[1], step, name, live, extra)
        want = torch.from_numpy(g[f"out_{step}"])
        assert rel_l2(out, want) <= BF16_TOL, (step, name)
        assert list(caches[0].commit_token_counts) == list(g[f"counts_{step}"]), step
        if step > 0:  # with history or strided current keys the policies change the result
            assert rel_l2(plain, want) > 2 * BF16_TOL, (step, name)
    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128))
    hook = H3StreamingAttentionHook(cache, attention_backend="sdpa",
                                    dense_current_document_when_empty=True)
    whole = run(hook, cache, 50, "noisy", 1, {})
    assert rel_l2(whole, torch.from_numpy(g["whole_out"])) <= BF16_TOL
    plain_hook = H3StreamingAttentionHook(CleanAVKVCache(KVContract(local_heads=2, head_dim=128)),
                                          attention_backend="sdpa")
    plain = run(plain_hook, plain_hook.cache, 50, "noisy", 1, {})
    assert rel_l2(plain, torch.from_numpy(g["whole_out"])) > 2 * BF16_TOL
