"""Generate the golden fixtures by running the REFERENCE's own Python code on CPU.

Run where the reference sources are checked out: by default a ``reference`` checkout beside
this repository's directory, or the path in H3SA_REFERENCE. The GPU box and the test suite
only read the committed .npz outputs.

    python tests/golden/make_golden.py [fixture.npz ...]

Inputs come from numpy's PCG64 generator (platform independent) so the tests can rebuild
them from the seeds recorded in each fixture. Fixtures:

* prologue.npz   QK-RMSNorm + RoPE of a merged QKV shard through the reference's unfused
                 CPU path (nn.RMSNorm, rope_cos_sin_cache, apply_rope_qk;
                 T/model/layers.py:138-196) with positions from minimax_h3_packed_sequence.
* hook_cpu.npz   the CPU benchmark configuration (H=8, d=64, 256 video + 32 audio queries,
                 1024 cached + 288 current keys, 16 text rows) through the reference
                 H3StreamingAttentionHook (T/streaming/attention_hook.py) with
                 FlashAttention-3 replaced by torch SDPA (the math FA3 implements).
* fp8.npz        quantize_fp8_e4m3_per_head (F/inference/fused_kernels.py:823-834).
* mask.npz       _dynamic_history_mask (F/inference/dynamic_block_sparse.py:50-124).
* cache.npz      CleanAVKVCache row tables through a commit / retain / audio-drop schedule
                 (T/streaming/cache.py), rows tagged by (commit, local row) in the K values.
* ulysses.npz    merged_qkv_sequence_to_heads / heads_to_sequence on two gloo ranks
                 (T/distributed/ulysses.py).
* cache_f.npz    the FL2AV CleanAVKVCache (F/streaming/cache.py) row tables through bounded
                 commits, count-based and sink + recent retention, audio drop and strided
                 attention-history queries.
* ulysses_pad.npz the FL2AV versions with 3 heads over 2 ranks (zero-padded head shards,
                 F/distributed/ulysses.py).
* hook_f.npz     the FL2AV H3StreamingAttentionHook (F/streaming/attention_hook.py) with its
                 sdpa backend through every mode: clean and progress commits, a full-prefix
                 capture, a noisy call over a temporary prefix, fused progress-denoise forwards
                 (with the recent / sink / previous-video-only policy and without) and a final
                 noisy call; layer 0's outputs, the captured prefix and the commit ledger. The
                 hook insists on CUDA tensors: CPU tensors of a subclass that reports is_cuda
                 stand in, and the K/V pair validators are stubbed.
* hook_f_policy.npz the FL2AV hook (sdpa backend) with strided older history, strided
                 current video keys and, separately, dense_current_document_when_empty:
                 layer 0's outputs and the commit counts of every step.
* hook_sol.npz   the FL2AV hook with its sol_attn backend (tests/golden/make_hook_sol.py):
                 layer 0 and layer 2 outputs of a noisy call over three commits, default and
                 route-current-video policies, the adapter in Triton's CPU interpreter.
* hook_topk.npz  the FL2AV hook with its flash_attn3_fp8_segmented_topk backend at density
                 0.5 over four clean commits, then a noisy call (layer 0 outputs of every
                 step): FlashAttention-3's FP8 call is replaced by exact attention on the
                 dequantised e4m3 inputs plus its log-sum-exp, so the reference's own
                 quantisation, commit-level selection and LSE merge run as written.
* w8a8.npz       the reference's int8 weight quantiser _quantize_weight
                 (T/inference/w8a8.py:56-63) on a bf16 weight with outliers and an all-zero
                 row (the 1e-12 scale floor).
* sol.npz        the SOL-Attn rectangular adapter (F/inference/sol_attention.py:366-598),
                 its Triton kernels run by Triton's CPU interpreter with float32 buffers, on
                 three block-clustered cases: outputs and the four telemetry counts.
* topk.npz       key summaries of the FL2AV segmented-FP8 CleanAVKVCache
                 (F/streaming/cache.py:836-855) over six commits and after a sink + recent
                 retention, with the commit-level top-k selection of the segmented top-k
                 backend (F/streaming/attention_hook.py:1256-1302) evaluated on them.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
# the reference checkout: a sibling of this repository unless H3SA_REFERENCE names it
REF = Path(os.environ.get("H3SA_REFERENCE", HERE.parents[2] / "reference"))
sys.path.insert(0, str(HERE))

from inputs import bf16, fp8_input, hook_cpu_inputs, mask_inputs, prologue_inputs, ulysses_merged  # noqa: E402


def _import_reference():
    sys.path.insert(0, str(REF / "src"))
    sys.path.insert(0, str(REF / "src" / "taomate-fl2av" / "src"))
    import torch

    stub = types.ModuleType("flash_attn_interface")

    def flash_attn_func(q, k, v, softmax_scale=None, causal=False, num_splits=1,
                        q_descale=None, k_descale=None, v_descale=None):
        if q_descale is None:
            o = torch.nn.functional.scaled_dot_product_attention(
                q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=softmax_scale,
                is_causal=causal)
            return o.transpose(1, 2)
        # FP8 form: e4m3 [B, S, H, D] inputs with fp32 [B, H] descales; exact attention on the
        # dequantised values, returned with its log-sum-exp [B, H, S] as FA3 does
        deq = lambda x, s: torch.Tensor(x).float() * torch.Tensor(s).float()[:, None, :, None]  # noqa: E731
        qf, kf, vf = deq(q, q_descale), deq(k, k_descale), deq(v, v_descale)
        scores = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * softmax_scale
        lse = torch.logsumexp(scores, dim=-1)
        o = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(scores, dim=-1), vf)
        return o.to(torch.bfloat16), lse

    stub.flash_attn_func = flash_attn_func
    sys.modules["flash_attn_interface"] = stub


# ----------------------------------------------------------------------------- prologue
def make_prologue(path: Path) -> None:
    import torch
    from taomate_h3.model.layers import MiniMaxH3Rope, apply_rope_qk, rope_cos_sin_cache
    from taomate_h3.model.packed_sequence import minimax_h3_packed_sequence

    seed, heads, head_dim, per_axis = 11, 4, 128, 16
    layout = minimax_h3_packed_sequence(text_len=16, latent_t=2, latent_h=8, latent_w=12,
                                        audio_t=8)
    seq = int(layout["seq_len"])
    inp = prologue_inputs(seed, seq, heads, head_dim)
    qkv, q_w, k_w = inp["qkv"], inp["q_weight"], inp["k_weight"]
    inv_freq = (10000.0 ** (-2.0 * np.arange(per_axis) / (2.0 * per_axis))).astype(np.float32)
    rope = MiniMaxH3Rope(per_axis)
    rope.inv_freq.copy_(torch.from_numpy(inv_freq))
    freqs = rope(layout["img_position_ids"].unsqueeze(0))
    cache = rope_cos_sin_cache(freqs, dtype=torch.bfloat16)
    positions = torch.arange(seq)
    t = torch.from_numpy(qkv).bfloat16().view(seq, 3, heads, head_dim)
    q_norm = torch.nn.RMSNorm(head_dim, eps=1e-5, dtype=torch.bfloat16)
    k_norm = torch.nn.RMSNorm(head_dim, eps=1e-5, dtype=torch.bfloat16)
    with torch.no_grad():
        q_norm.weight.copy_(torch.from_numpy(q_w))
        k_norm.weight.copy_(torch.from_numpy(k_w))
        q, k = apply_rope_qk(q_norm(t[:, 0]), k_norm(t[:, 1]), cache, positions)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    np.savez(path, seed=seed, heads=heads, head_dim=head_dim, per_axis=per_axis, seq=seq,
             inv_freq=inv_freq, grid=layout["img_position_ids"].numpy(),
             cos_sin_bf16=bits(cache), q_bf16=bits(q), k_bf16=bits(k))


# ----------------------------------------------------------------------------- hook
def make_hook(path: Path) -> None:
    import torch
    from taomate_h3.streaming.attention_hook import H3StreamingAttentionHook, HookMode
    from taomate_h3.streaming.cache import AVKV, CleanAVKVCache, KVContract

    seed = 0
    inp = hook_cpu_inputs(seed)
    heads, head_dim = inp["q"].shape[1:]
    contract = KVContract(local_heads=heads, head_dim=head_dim, dtype=torch.float32,
                          device_type="cpu")
    cache = CleanAVKVCache(contract)
    cache._history["blocks.0.attn"] = AVKV(torch.from_numpy(inp["hist_k"]),
                                           torch.from_numpy(inp["hist_v"]))
    hook = H3StreamingAttentionHook(cache)
    hook.activate(HookMode.NOISY)

    class Attn:
        softmax_scale = inp["scale"]

    out = hook(attention=Attn(), layer_name="blocks.0.attn", query=torch.from_numpy(inp["q"]),
               key=torch.from_numpy(inp["k"]), value=torch.from_numpy(inp["v"]),
               token_tags=torch.from_numpy(inp["token_tags"]),
               commit_mask=torch.from_numpy(inp["commit_mask"]),
               cu_seqlens_host=tuple(inp["cu_seqlens"])).numpy()
    np.savez(path, seed=seed, rows=np.arange(0, out.shape[0], 4), out=out[::4],
             out_sum=np.float64(out.astype(np.float64).sum()),
             out_l2=np.float64(np.sqrt((out.astype(np.float64) ** 2).sum())),
             receipt=np.array([hook.kernel_calls, hook.query_tokens, hook.key_tokens]))


# ----------------------------------------------------------------------------- fp8
def make_fp8(path: Path) -> None:
    import torch
    from digitalhuman_h3.inference.fused_kernels import quantize_fp8_e4m3_per_head

    seed = 5
    x = fp8_input(seed)
    q, s = quantize_fp8_e4m3_per_head(torch.from_numpy(x).bfloat16())
    np.savez(path, seed=seed, q=q.view(torch.uint8).numpy(), scale=s.numpy())


# ----------------------------------------------------------------------------- mask
def make_mask(path: Path) -> None:
    import torch
    from digitalhuman_h3.inference.dynamic_block_sparse import _dynamic_history_mask

    seed, heads, nq, nh, extra, density = 3, 2, 384, 1000, 400, 0.3
    q, hk = mask_inputs(seed, heads, nq, nh)
    mask, receipt = _dynamic_history_mask(torch, query=torch.from_numpy(q),
                                          history_key=torch.from_numpy(hk),
                                          total_key_tokens=nh + extra, density=density,
                                          block_size=128)
    np.savez(path, seed=seed, heads=heads, nq=nq, nh=nh, total=nh + extra, density=density,
             kv_num_blocks=mask.kv_num_blocks.numpy(), kv_indices=mask.kv_indices.numpy(),
             selected=receipt["selected_history_blocks"])


# ----------------------------------------------------------------------------- cache
def make_cache(path: Path) -> None:
    import torch
    from taomate_h3.streaming.cache import MAIN_LAYER_NAMES, CleanAVKVCache, KVContract

    rng = np.random.default_rng(9)
    contract = KVContract(local_heads=1, head_dim=2, dtype=torch.float32, device_type="cpu")
    cache = CleanAVKVCache(contract)
    steps = []
    schedule = ["commit", "retain", "commit", "retain", "commit", "retain", "commit", "retain",
                "drop", "commit", "retain", "commit", "retain"]
    serial = 0
    for op in schedule:
        if op == "commit":
            text = 3 + int(rng.integers(0, 3))
            audio = 2 * int(rng.integers(2, 5))
            video = int(rng.integers(5, 12))
            pad = int(rng.integers(0, 3))
            tags = np.array([1] * text + [2] * audio + [0] * video + [-1] * pad)
            commit = (tags == 0) | (tags == 2)
            n = len(tags)
            ids = np.zeros((n, 1, 2), dtype=np.float32)
            staged = np.nonzero(commit)[0]
            ids[staged, 0, 0] = serial
            ids[staged, 0, 1] = np.arange(staged.size)
            cache.begin_clean_commit(cache.committed_blocks)
            for name in MAIN_LAYER_NAMES:
                t = torch.from_numpy(ids)
                cache.stage(name, t, t.clone(), torch.from_numpy(tags), torch.from_numpy(commit))
            cache.commit()
            steps.append(("commit", tags, serial))
            serial += 1
        elif op == "retain":
            cache.retain_sink_and_recent_commits()
            steps.append(("retain", None, None))
        else:
            removed = cache.drop_audio_history()
            steps.append(("drop", None, removed))
        hist = cache.history("blocks.0.attn")
        rows = np.zeros((0, 2), dtype=np.int64) if hist is None else hist.key[:, 0, :].numpy().astype(np.int64)
        steps[-1] = steps[-1] + (rows,)
    arrays = {"ops": np.array([s[0] for s in steps])}
    for i, (op, tags, extra, rows) in enumerate(steps):
        if tags is not None:
            arrays[f"tags_{i}"] = tags
        if op == "drop":
            arrays[f"removed_{i}"] = np.array(extra)
        arrays[f"rows_{i}"] = rows
    np.savez(path, **arrays)


def make_cache_f(path: Path) -> None:
    """The FL2AV cache (F/streaming/cache.py) through bounded commits, count-based retention,
    sink + recent retention and audio drop, with its strided attention history queried along
    the way. Its stage() accepts only CUDA bf16 K/V; the check is stubbed so the row
    bookkeeping runs on CPU (rows tagged by (commit serial, local row), exact in bf16)."""

    import torch
    import digitalhuman_h3.streaming.cache as fcache

    fcache._validate_av_pair = lambda pair, contract, *, layer: None
    layer = "blocks.0.attn"
    contract = fcache.KVContract(layer_names=(layer,), local_heads=1, head_dim=2)
    cache = fcache.CleanAVKVCache(contract)
    rng = np.random.default_rng(13)
    schedule = [("commit",), ("commit",), ("commit",), ("attn", 3, 1, 2, False),
                ("sink_recent", 1, True), ("commit",), ("attn", 3, 1, 3, True),
                ("bounded", 3), ("bounded", 3), ("retain_recent", 2), ("commit",),
                ("commit",), ("attn", 4, 2, 2, True), ("sink_recent", 2, False), ("drop",),
                ("commit",), ("attn", 3, 0, 4, False), ("bounded", 1), ("commit",)]
    arrays: dict[str, np.ndarray] = {}
    serial = 0
    for i, step in enumerate(schedule):
        op = step[0]
        if op in ("commit", "bounded"):
            audio = 2 * int(rng.integers(2, 5))
            video = int(rng.integers(6, 14))
            tags = np.array([1] * 3 + [2] * audio + [0] * video + [-1] * 2)
            commit = (tags == 0) | (tags == 2)
            ids = np.zeros((len(tags), 1, 2), dtype=np.float32)
            staged = np.nonzero(commit)[0]
            ids[staged, 0, 0] = serial
            ids[staged, 0, 1] = np.arange(staged.size)
            cache.begin_clean_commit(cache.committed_blocks)
            t = torch.from_numpy(ids).to(torch.bfloat16)
            cache.stage(layer, t, t.clone(), torch.from_numpy(tags), torch.from_numpy(commit))
            if op == "commit":
                cache.commit()
            else:
                cache.commit(retain_recent_commit_count=int(step[1]))
            arrays[f"tags_{i}"] = tags
            serial += 1
        elif op == "sink_recent":
            cache.retain_sink_and_recent_commits(int(step[1]), sink_video_only=bool(step[2]))
        elif op == "retain_recent":
            cache.retain_recent_commits(int(step[1]))
        elif op == "drop":
            arrays[f"removed_{i}"] = np.array(cache.drop_audio_history())
        elif op == "attn":
            sel = cache.attention_history(layer, count=int(step[1]), recent_full_blocks=int(step[2]),
                                          older_video_stride=int(step[3]),
                                          preserve_sink=bool(step[4]))
            arrays[f"attn_{i}"] = (np.zeros((0, 2), np.int64) if sel is None
                                   else sel.key[:, 0, :].float().numpy().astype(np.int64))
        hist = cache.history(layer)
        arrays[f"rows_{i}"] = (np.zeros((0, 2), np.int64) if hist is None
                               else hist.key[:, 0, :].float().numpy().astype(np.int64))
        arrays[f"counts_{i}"] = np.array(cache.commit_token_counts, dtype=np.int64)
        arrays[f"blocks_{i}"] = np.array(cache.committed_blocks)
    arrays["schedule"] = np.array(["|".join(str(x) for x in st) for st in schedule])
    np.savez(path, **arrays)


def make_topk(path: Path) -> None:
    """Six segmented-FP8 commits (2 heads of 128) with per-commit offsets, the key summaries
    the reference cache stores for them, then the same after retain_sink_and_recent_commits
    (which recomputes each kept block's summary over its kept rows). The selection is the
    expression of F/streaming/attention_hook.py:1271-1290 (inline in the hook, which needs
    CUDA) evaluated here on the reference's summaries. Its stage() accepts only CUDA bf16 K/V;
    that check is stubbed so the cache runs on CPU."""

    import math

    import torch
    import digitalhuman_h3.streaming.cache as fcache

    fcache._validate_av_pair = lambda pair, contract, *, layer: None
    layer = "blocks.0.attn"
    contract = fcache.KVContract(layer_names=(layer,), local_heads=2, head_dim=128)
    cache = fcache.CleanAVKVCache(contract, segmented_fp8_history=True)
    rng = np.random.default_rng(21)
    arrays: dict[str, np.ndarray] = {}
    for serial in range(6):
        audio = 2 * int(rng.integers(2, 5))
        video = int(rng.integers(12, 30))
        tags = np.array([1] * 3 + [2] * audio + [0] * video + [-1] * 2)
        commit = (tags == 0) | (tags == 2)
        offset = rng.standard_normal((1, 2, 128)).astype(np.float32)
        key = bf16(0.5 * rng.standard_normal((len(tags), 2, 128)).astype(np.float32) + offset)
        value = bf16(rng.standard_normal((len(tags), 2, 128)).astype(np.float32))
        cache.begin_clean_commit(cache.committed_blocks)
        cache.stage(layer, torch.from_numpy(key).to(torch.bfloat16),
                    torch.from_numpy(value).to(torch.bfloat16), torch.from_numpy(tags),
                    torch.from_numpy(commit))
        cache.commit()
        arrays[f"key_{serial}"] = key
        arrays[f"tags_{serial}"] = tags

    def select(stage: str, query: np.ndarray, density: float) -> None:
        blocks = cache.history_blocks(layer)
        summaries = torch.stack([pair.key_summary for pair in blocks], dim=0)
        arrays[f"summary_{stage}"] = summaries.numpy()
        q = torch.from_numpy(query).to(torch.bfloat16)
        count = max(1, min(len(blocks), math.ceil(len(blocks) * density)))
        scores = summaries.mul(q.float().mean(dim=0).unsqueeze(0)).sum(dim=-1).mean(dim=-1)
        arrays[f"scores_{stage}"] = scores.numpy()
        arrays[f"selected_{stage}"] = np.array(
            scores.topk(count, sorted=False).indices.sort().values.tolist(), dtype=np.int64)
        arrays[f"query_{stage}"] = query
        arrays[f"density_{stage}"] = np.array(density)

    select("full", bf16(rng.standard_normal((40, 2, 128)).astype(np.float32) + 0.3), 0.5)
    cache.retain_sink_and_recent_commits(3, sink_video_only=True)
    select("retained", bf16(rng.standard_normal((40, 2, 128)).astype(np.float32) - 0.2), 0.5)
    arrays["retained_counts"] = np.array(cache.commit_token_counts, dtype=np.int64)
    np.savez(path, **arrays)

def make_hook_f(path: Path) -> None:
    import torch
    import digitalhuman_h3.streaming.attention_hook as fhook
    import digitalhuman_h3.streaming.cache as fcache
    from inputs import HOOK_F_SCHEDULE, hook_f_inputs

    fcache._validate_av_pair = lambda pair, contract, *, layer: None
    fcache._validate_video_pair = lambda pair, contract, *, layer: None

    class CudaFlagged(torch.Tensor):
        """CPU tensor that answers is_cuda = True, so the hook's device checks pass."""

        @property
        def is_cuda(self):
            return True

    def t(x: np.ndarray, dtype=torch.bfloat16):
        return torch.from_numpy(x).to(dtype).as_subclass(CudaFlagged)

    class Attn:
        softmax_scale = 128 ** -0.5

    contract = fcache.KVContract(local_heads=2, head_dim=128)
    cache = fcache.CleanAVKVCache(contract)
    hook = fhook.H3StreamingAttentionHook(cache, attention_backend="sdpa")
    arrays: dict[str, np.ndarray] = {}
    prefix = None
    for step, (name, live, extra) in enumerate(HOOK_F_SCHEDULE):
        x = hook_f_inputs(step, live)
        kwargs = dict(extra)
        if name == "capture":
            hook.begin_full_prefix_capture(**kwargs)
        else:
            mode = {"clean_commit": fhook.HookMode.CLEAN_COMMIT,
                    "progress_commit": fhook.HookMode.PROGRESS_COMMIT,
                    "noisy_prefix": fhook.HookMode.NOISY, "noisy": fhook.HookMode.NOISY,
                    "fused_recent": fhook.HookMode.FUSED_PROGRESS_DENOISE,
                    "fused": fhook.HookMode.FUSED_PROGRESS_DENOISE}[name]
            kwargs["full_prefix"] = prefix if name in ("noisy_prefix", "fused_recent") else None
            if name == "fused_recent":
                kwargs["fused_previous_full_prefix"] = prefix
                # keep every block but mark the sink video-only: the fused current view then
                # drops the sink's audio once the pending block ages it out
                cache.retain_sink_and_recent_commits(cache.retained_blocks, sink_video_only=True)
            commit = mode in (fhook.HookMode.CLEAN_COMMIT, fhook.HookMode.PROGRESS_COMMIT,
                              fhook.HookMode.FUSED_PROGRESS_DENOISE)
            if commit:
                cache.begin_clean_commit(cache.committed_blocks)
            hook.activate(mode=mode, block_index=cache.committed_blocks, **kwargs)
        q, k, v = t(x["q"]), t(x["k"]), t(x["v"])
        tags = t(x["token_tags"], torch.int64)
        mask = t(x["commit_mask"], torch.bool)
        for layer in contract.layer_names:
            out = hook(attention=Attn(), layer_name=layer, query=q, key=k, value=v,
                       token_tags=tags, commit_mask=mask, cu_seqlens=None,
                       cu_seqlens_host=tuple(x["cu_seqlens"]), max_seqlen=64)
            if layer == contract.layer_names[0]:
                arrays[f"out_{step}"] = torch.Tensor(out).float().numpy()
        if name == "capture":
            prefix = hook.finish_full_prefix_capture()
            pair = prefix.get(contract.layer_names[0])
            arrays["prefix_key"] = torch.Tensor(pair.key).float().numpy()
            arrays["prefix_value"] = torch.Tensor(pair.value).float().numpy()
        else:
            hook.deactivate()
            if commit:
                cache.commit()
        arrays[f"counts_{step}"] = np.array(cache.commit_token_counts, dtype=np.int64)
        arrays[f"blocks_{step}"] = np.array(cache.committed_blocks)
    np.savez_compressed(path, **arrays)

def make_hook_f_policy(path: Path) -> None:
    """The FL2AV hook's history and current-video policies: strided older history
    (history_kv_older_video_stride, history_kv_recent_full_blocks), strided current video
    keys (current_video_kv_stride) through commits, noisy and fused calls; and the
    dense_current_document_when_empty rule on a first call with no history."""

    import torch
    import digitalhuman_h3.streaming.attention_hook as fhook
    import digitalhuman_h3.streaming.cache as fcache
    from inputs import HOOK_F_POLICY, HOOK_F_POLICY_SCHEDULE, hook_f_inputs

    fcache._validate_av_pair = lambda pair, contract, *, layer: None
    fcache._validate_video_pair = lambda pair, contract, *, layer: None

    class CudaFlagged(torch.Tensor):
        @property
        def is_cuda(self):
            return True

    def t(x: np.ndarray, dtype=torch.bfloat16):
        return torch.from_numpy(x).to(dtype).as_subclass(CudaFlagged)

    class Attn:
        softmax_scale = 128 ** -0.5

    modes = {"clean_commit": fhook.HookMode.CLEAN_COMMIT, "noisy": fhook.HookMode.NOISY,
             "fused": fhook.HookMode.FUSED_PROGRESS_DENOISE}
    contract = fcache.KVContract(local_heads=2, head_dim=128)
    arrays: dict[str, np.ndarray] = {}

    def run(hook, cache, step, name, live, extra, key):
        x = hook_f_inputs(100 + step, live)
        mode = modes[name]
        commit = mode is not fhook.HookMode.NOISY
        if commit:
            cache.begin_clean_commit(cache.committed_blocks)
        hook.activate(mode=mode, block_index=cache.committed_blocks, full_prefix=None, **extra)
        q, k, v = t(x["q"]), t(x["k"]), t(x["v"])
        tags, mask = t(x["token_tags"], torch.int64), t(x["commit_mask"], torch.bool)
        for layer in contract.layer_names:
            out = hook(attention=Attn(), layer_name=layer, query=q, key=k, value=v,
                       token_tags=tags, commit_mask=mask, cu_seqlens=None,
                       cu_seqlens_host=tuple(x["cu_seqlens"]), max_seqlen=64)
            if layer == contract.layer_names[0]:
                arrays[key] = torch.Tensor(out).float().numpy()
        hook.deactivate()
        if commit:
            cache.commit()

    cache = fcache.CleanAVKVCache(contract)
    hook = fhook.H3StreamingAttentionHook(cache, attention_backend="sdpa", **HOOK_F_POLICY)
    for step, (name, live, extra) in enumerate(HOOK_F_POLICY_SCHEDULE):
        run(hook, cache, step, name, live, extra, f"out_{step}")
        arrays[f"counts_{step}"] = np.array(cache.commit_token_counts, dtype=np.int64)
    cache = fcache.CleanAVKVCache(contract)
    hook = fhook.H3StreamingAttentionHook(cache, attention_backend="sdpa",
                                          dense_current_document_when_empty=True)
    run(hook, cache, 50, "noisy", 1, {}, "whole_out")
    np.savez_compressed(path, **arrays)


def make_hook_topk(path: Path) -> None:
    import torch
    import digitalhuman_h3.streaming.attention_hook as fhook
    import digitalhuman_h3.streaming.cache as fcache
    from inputs import hook_topk_inputs

    fcache._validate_av_pair = lambda pair, contract, *, layer: None

    class CudaFlagged(torch.Tensor):
        @property
        def is_cuda(self):
            return True

    def t(x: np.ndarray, dtype=torch.bfloat16):
        return torch.from_numpy(x).to(dtype).as_subclass(CudaFlagged)

    class Attn:
        softmax_scale = 128 ** -0.5

    contract = fcache.KVContract(local_heads=2, head_dim=128)
    cache = fcache.CleanAVKVCache(contract, segmented_fp8_history=True)
    hook = fhook.H3StreamingAttentionHook(cache, attention_backend="flash_attn3_fp8_segmented_topk",
                                          history_kv_dynamic_density=0.5)
    arrays: dict[str, np.ndarray] = {}
    for step in range(5):
        x = hook_topk_inputs(step)
        commit = step < 4
        if commit:
            cache.begin_clean_commit(cache.committed_blocks)
        mode = fhook.HookMode.CLEAN_COMMIT if commit else fhook.HookMode.NOISY
        hook.activate(mode=mode, block_index=cache.committed_blocks, full_prefix=None)
        q, k, v = t(x["q"]), t(x["k"]), t(x["v"])
        tags, mask = t(x["token_tags"], torch.int64), t(x["commit_mask"], torch.bool)
        for layer in contract.layer_names:
            out = hook(attention=Attn(), layer_name=layer, query=q, key=k, value=v,
                       token_tags=tags, commit_mask=mask, cu_seqlens=None,
                       cu_seqlens_host=tuple(x["cu_seqlens"]), max_seqlen=64)
            if layer == contract.layer_names[0]:
                arrays[f"out_{step}"] = torch.Tensor(out).float().numpy()
        hook.deactivate()
        if commit:
            cache.commit()
        arrays[f"selected_blocks_{step}"] = np.array(hook.dynamic_block_sparse_selected_blocks)
    np.savez_compressed(path, **arrays)

def make_w8a8(path: Path) -> None:
    import torch
    from taomate_h3.inference.w8a8 import _quantize_weight

    rng = np.random.default_rng(31)
    w = rng.standard_normal((96, 512)).astype(np.float32) * 0.02
    w[3, 17] = 0.9          # an outlier sets row 3's scale
    w[5] = 0.0              # all-zero row: the 1e-12 floor
    w[7] = np.linspace(-1.27, 1.27, 512, dtype=np.float32)  # exact multiples of the scale
    wb = bf16(w)
    q, scale = _quantize_weight(torch.from_numpy(wb).to(torch.bfloat16))
    np.savez(path, weight=wb, q=q.numpy(), scale=scale.numpy())

# ----------------------------------------------------------------------------- ulysses
def make_sol(path: Path) -> None:
    """The reference SOL-Attn adapter (F/inference/sol_attention.py:366-598) through Triton's
    CPU interpreter. The interpreter mishandles bf16 buffers, so the run keeps every buffer
    in float32 (torch.bfloat16 stands for float32 during the call): the summaries and the
    probabilities are not rounded to bf16, the output still is (its tl.bfloat16 cast)."""

    import subprocess

    code = (
        "import os, sys, numpy as np\n"
        "os.environ['TRITON_INTERPRET'] = '1'\n"
        f"sys.path.insert(0, {str(REF / 'src' / 'taomate-fl2av' / 'src')!r})\n"
        f"sys.path.insert(0, {str(HERE)!r})\n"
        "import torch\n"
        "from digitalhuman_h3.inference.sol_attention import sol_attn_rectangular\n"
        "from inputs import SOL_CASES, sol_inputs\n"
        "out = {}\n"
        "for c, (nq, nk, h, tau, sink) in enumerate(SOL_CASES):\n"
        "    q, k, v = (torch.from_numpy(a) for a in sol_inputs(c))\n"
        "    tel = torch.zeros(4, dtype=torch.int64)\n"
        "    saved, torch.bfloat16 = torch.bfloat16, torch.float32\n"
        "    try:\n"
        "        o = sol_attn_rectangular(q, k, v, scale=128 ** -0.5, tau=tau, sink_tokens=sink,\n"
        "                                 telemetry_counts=tel)\n"
        "    finally:\n"
        "        torch.bfloat16 = saved\n"
        "    out[f'out{c}'] = (o.numpy().view(np.uint32) >> 16).astype(np.uint16)  # bf16 bits\n"
        "    out[f'telemetry{c}'] = tel.numpy()\n"
        f"np.savez({str(path)!r}, **out)\n"
    )
    subprocess.run([sys.executable, "-c", code], check=True)


def make_hook_sol(path: Path) -> None:
    """The FL2AV hook's sol_attn backend (tests/golden/make_hook_sol.py, own process)."""

    import subprocess

    subprocess.run([sys.executable, str(HERE / "make_hook_sol.py"), str(path)], check=True,
                   cwd=HERE)


def _ulysses_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch
    import torch.distributed as dist
    from taomate_h3.distributed.parallel import ParallelContext
    from taomate_h3.distributed.ulysses import heads_to_sequence, merged_qkv_sequence_to_heads

    sys.path.insert(0, str(HERE))
    _import_reference()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    ctx = ParallelContext(1, 0, world, rank, dist.group.WORLD, dist.group.WORLD)
    tokens, heads, d = 6, 4, 16
    merged = ulysses_merged(rank, tokens, heads, d)
    q, k, v = merged_qkv_sequence_to_heads(torch.from_numpy(merged), num_heads=heads,
                                           head_dim=d, context=ctx)
    o = heads_to_sequence(q.contiguous(), context=ctx)
    np.savez(os.path.join(out_dir, f"ulysses_rank{rank}.npz"), q=q.numpy(),
             k=k.numpy(), v=v.numpy(), o=o.numpy())
    dist.destroy_process_group()


def make_ulysses(path: Path) -> None:
    import socket
    import tempfile

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_ulysses_worker, args=(2, port, tmp), nprocs=2, start_method="spawn")
        parts = [np.load(os.path.join(tmp, f"ulysses_rank{r}.npz")) for r in range(2)]
        np.savez(path, **{f"{key}{r}": parts[r][key] for r in range(2)
                          for key in ("q", "k", "v", "o")})


def _ulysses_pad_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    """The FL2AV exchange with heads not divisible by the world (3 heads over 2 ranks): the
    send side zero-pads to ceil(H/W) heads per rank, heads_to_sequence(num_heads=H) drops the
    padding again (F/distributed/ulysses.py:107-110, 150-156, 218-222)."""

    import datetime

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(HERE))
    _import_reference()
    from digitalhuman_h3.distributed.parallel import ParallelContext
    from digitalhuman_h3.distributed.ulysses import heads_to_sequence, merged_qkv_sequence_to_heads

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    ctx = ParallelContext(tp_world_size=1, tp_rank=0, ulysses_world_size=world,
                          ulysses_rank=rank, tp_group=dist.group.WORLD,
                          ulysses_group=dist.group.WORLD)
    tokens, heads, d = 6, 3, 16
    merged = ulysses_merged(rank, tokens, heads, d)
    q, k, v = merged_qkv_sequence_to_heads(torch.from_numpy(merged), num_heads=heads,
                                           head_dim=d, context=ctx)
    o = heads_to_sequence(q.contiguous(), context=ctx, num_heads=heads)
    np.savez(os.path.join(out_dir, f"ulysses_pad_rank{rank}.npz"), q=q.numpy(),
             k=k.numpy(), v=v.numpy(), o=o.numpy())
    dist.destroy_process_group()


def make_ulysses_pad(path: Path) -> None:
    import socket
    import tempfile

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_ulysses_pad_worker, args=(2, port, tmp), nprocs=2,
                           start_method="spawn")
        parts = [np.load(os.path.join(tmp, f"ulysses_pad_rank{r}.npz")) for r in range(2)]
        np.savez(path, **{f"{key}{r}": parts[r][key] for r in range(2)
                          for key in ("q", "k", "v", "o")})


def main() -> None:
    _import_reference()
    makers = {"prologue.npz": make_prologue, "hook_cpu.npz": make_hook, "fp8.npz": make_fp8,
              "mask.npz": make_mask, "cache.npz": make_cache, "ulysses.npz": make_ulysses,
              "ulysses_pad.npz": make_ulysses_pad, "cache_f.npz": make_cache_f,
              "topk.npz": make_topk, "hook_f.npz": make_hook_f,
              "hook_topk.npz": make_hook_topk, "w8a8.npz": make_w8a8, "sol.npz": make_sol,
              "hook_f_policy.npz": make_hook_f_policy, "hook_sol.npz": make_hook_sol}
    wanted = sys.argv[1:] or list(makers)  # optional: only the named fixtures
    for name, fn in makers.items():
        if name not in wanted:
            continue
        fn(HERE / name)
        print(f"wrote {name} ({(HERE / name).stat().st_size} bytes)")


if __name__ == "__main__":
    main()
