"""Host-side logic on CPU: C-ABI exports and validation, hook / cache / prologue errors.

Nothing here launches a kernel: every call either returns a validation status from the C
library before touching the device or raises in the Python layer before reaching it.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _lib():
    import h3sa._lib as lib

    return lib


def test_every_declared_symbol_is_exported() -> None:
    header = (ROOT / "include" / "h3sa.h").read_text()
    declared = re.findall(r"H3SA_API\s+[\w\s\*]+?\b(h3sa_\w+)\s*\(", header)
    assert len(declared) >= 12
    lib = ctypes.CDLL(str(_lib().library_path()))
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) <= set(_lib().SIGNATURES)


def test_abi_version_and_smem() -> None:
    lib = _lib()
    assert lib.LIB.h3sa_abi_version() == 1
    # two Q tiles + two K stages + two V stages of 128 x 128 bf16, plus barriers
    assert 6 * 32768 < lib.LIB.h3sa_attention_smem_bytes(0) <= 232_448
    assert lib.LIB.h3sa_attention_smem_bytes(1) < lib.LIB.h3sa_attention_smem_bytes(0)


def _attn(**over):
    lib = _lib()
    probs = (lib.Problem * 1)()
    probs[0].q_lo, probs[0].q_hi, probs[0].kv_lo, probs[0].kv_hi = 0, 128, 0, 128
    args = dict(query=16, out=32, rows=128, heads=2, head_dim=128, key=48, value=64, pages=1,
                table=80, blocks=1, probs=probs, n=1)
    args.update(over)
    return lib.LIB.h3sa_attention_fwd(args["query"], args["out"], args["rows"], args["heads"],
                                      args["head_dim"], args["key"], args["value"], args["pages"],
                                      args["table"], args["blocks"], args["probs"], args["n"],
                                      0.08, None, None, 0, 0, None, None)


def test_attention_argument_validation() -> None:
    lib = _lib()
    assert _attn(head_dim=64) == lib.H3SA_ERR_UNSUPPORTED
    assert "head_dim 128" in lib.last_error()
    assert _attn(query=None) == lib.H3SA_ERR_INVALID
    assert _attn(query=17) == lib.H3SA_ERR_INVALID and "16-byte aligned" in lib.last_error()
    assert _attn(n=5) == lib.H3SA_ERR_INVALID
    bad = (lib.Problem * 1)()
    bad[0].q_lo, bad[0].q_hi, bad[0].kv_lo, bad[0].kv_hi = 0, 129, 0, 128
    assert _attn(probs=bad) == lib.H3SA_ERR_INVALID and "query rows" in lib.last_error()
    bad[0].q_hi, bad[0].kv_hi = 128, 200
    assert _attn(probs=bad) == lib.H3SA_ERR_INVALID and "KV rows" in lib.last_error()
    bad[0].kv_hi, bad[0].sparse = 128, 1
    assert _attn(probs=bad) == lib.H3SA_ERR_INVALID and "block lists" in lib.last_error()


def test_attention_wrapper_argument_checks() -> None:
    """The wrapper rejects block lists and fp8 scales the kernel would read past their end,
    and mismatched pools, before anything reaches the C ABI (CPU tensors: shape checks only)."""

    from h3sa.kernels import _check_attention_args

    heads, rows, d = 3, 256, 128
    q = torch.zeros(rows, heads, d, dtype=torch.bfloat16)
    out = torch.zeros_like(q)
    kp = torch.zeros(heads, 1024, d, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    table = torch.zeros(8, dtype=torch.int32)
    num = torch.zeros(heads, 2, dtype=torch.int32)
    idx = torch.zeros(heads, 2, 8, dtype=torch.int32)
    s = torch.ones(heads, dtype=torch.float32)

    def check(**kw):
        args = dict(query=q, out=out, key_pool=kp, value_pool=vp, page_table=table,
                    kv_num_blocks=None, kv_indices=None, q_scale=None, k_scale=None, v_scale=None)
        args.update(kw)
        _check_attention_args(**args)

    check()
    check(kv_num_blocks=num, kv_indices=idx)
    check(kv_num_blocks=num.unsqueeze(0), kv_indices=idx.unsqueeze(0))  # flex [1, H, ...] layout
    check(q_scale=s, k_scale=s, v_scale=s)
    for bad, msg in [
        (dict(kv_num_blocks=num[:1], kv_indices=idx[:1]), "for every query head"),
        (dict(kv_num_blocks=num, kv_indices=idx[:, :1]), "for every query head"),
        (dict(kv_num_blocks=num), "both kv_num_blocks and kv_indices"),
        (dict(kv_num_blocks=num.long(), kv_indices=idx), "int32"),
        (dict(q_scale=s, k_scale=s), "q_scale, k_scale and v_scale"),
        (dict(q_scale=s[:2], k_scale=s, v_scale=s), "one value per head"),
        (dict(q_scale=s.half(), k_scale=s, v_scale=s), "one value per head"),
        (dict(value_pool=vp.float()), "same dtype"),
        (dict(value_pool=vp[:2]), "matching shapes"),
        (dict(out=out.float()), "bf16 with the query's shape"),
        (dict(page_table=table.long()), "int32"),
    ]:
        with pytest.raises(RuntimeError, match=msg):
            check(**bad)


def test_kv_copy_shape_checks() -> None:
    """kv_copy_rows addresses every tensor with the first source's heads and row size, so
    the wrapper refuses mixed shapes before launching (CPU tensors: shape checks only)."""

    from h3sa.kernels import _check_copy_args

    packed = torch.zeros(300, 3, 128, dtype=torch.bfloat16)
    pool = torch.zeros(3, 4 * 128, 128, dtype=torch.bfloat16)
    table = torch.zeros(4, dtype=torch.int32)
    assert _check_copy_args([packed], [pool], None, table) == (3, 256)
    assert _check_copy_args([pool, pool], [packed, packed], table, None) == (3, 256)
    pool8 = torch.zeros(3, 4 * 128, 128, dtype=torch.float8_e4m3fn)
    back8 = torch.zeros(128, 3, 128, dtype=torch.float8_e4m3fn)
    assert _check_copy_args([pool8], [back8], table, None) == (3, 128)
    for src, dst, st, dt in [
        ([packed], [pool[:2]], None, table),                       # fewer heads in dst
        ([packed], [pool.float()], None, table),                   # wider rows in dst
        ([packed], [torch.zeros(3, 4 * 128, 64, dtype=torch.bfloat16)], None, table),
        ([packed, packed[:, :2]], [pool, pool], None, table),      # second pair differs
        ([packed], [pool8], None, table),                          # bf16 rows into e4m3 pages
    ]:
        with pytest.raises(RuntimeError, match="same heads and row size"):
            _check_copy_args(src, dst, st, dt)
    with pytest.raises(RuntimeError, match="pages"):
        _check_copy_args([packed[0]], [pool], None, table)
    with pytest.raises(ValueError):
        _check_copy_args([packed, packed, packed], [pool, pool, pool], None, table)


def test_quantize_pool_checks() -> None:
    """The pool quantiser refuses an e4m3 pool or scale vector smaller than the bf16 pool."""

    from h3sa.kernels import _check_quant_pool_args

    pool = torch.zeros(3, 256, 128, dtype=torch.bfloat16)
    pool8 = torch.zeros_like(pool, dtype=torch.float8_e4m3fn)
    scale = torch.zeros(3, dtype=torch.float32)
    table = torch.zeros(2, dtype=torch.int32)
    _check_quant_pool_args(pool, pool8, scale, table)
    for args, msg in [
        ((pool, pool8[:, :128], scale, table), "bf16 pool's shape"),
        ((pool, pool.clone(), scale, table), "float8_e4m3fn"),
        ((pool, pool8, scale[:2], table), "one value per head"),
        ((pool, pool8, scale.double(), table), "one value per head"),
        ((pool.float(), pool8, scale, table), "bf16 pool"),
        ((pool, pool8, scale, table.long()), "int32"),
    ]:
        with pytest.raises(RuntimeError, match=msg):
            _check_quant_pool_args(*args)


def test_composite_mask_flag_lengths() -> None:
    """The composite mask refuses audio flag vectors shorter than its block counts."""

    import types

    from h3sa.block_sparse import composite_block_mask

    q = torch.zeros(300, 2, 128, dtype=torch.bfloat16)  # 3 query blocks
    paged = types.SimpleNamespace(key=torch.zeros(2, 1024, 128, dtype=torch.bfloat16),
                                  table=torch.zeros(8, dtype=torch.int32))
    kw = dict(q_lo=0, q_hi=300, n_hist=512, n_kv=812)  # 7 KV blocks
    with pytest.raises(ValueError, match="query block"):
        composite_block_mask(q, paged, q_block_audio=torch.zeros(2), kv_block_audio=torch.zeros(7),
                             **kw)
    with pytest.raises(ValueError, match="KV block"):
        composite_block_mask(q, paged, q_block_audio=torch.zeros(3), kv_block_audio=torch.zeros(6),
                             **kw)


def test_ulysses_layouts_stay_inside_their_buffers(monkeypatch) -> None:
    """The Ulysses pack/unpack layouts address exactly their buffers; a buffer one record too
    small is refused before launching (library call stubbed, CPU tensors)."""

    from h3sa import kernels, ulysses

    launched = []
    monkeypatch.setattr(kernels, "_require_cuda", lambda *t: None)
    monkeypatch.setattr(kernels, "call", lambda name, *a: launched.append(name))
    monkeypatch.setattr(kernels, "stream_handle", lambda s=None: 0)
    world, tokens, heads, d = 4, 37, 8, 128
    hl = heads // world
    merged = torch.zeros(tokens, 3 * heads * d, dtype=torch.bfloat16)
    send = torch.zeros(world, 3, tokens, hl, d, dtype=torch.bfloat16)
    ulysses.pack_qkv_send(merged, send, world=world, num_heads=heads, head_dim=d)
    out = torch.zeros(3, world * tokens, hl, d, dtype=torch.bfloat16)
    ulysses.unpack_qkv_recv(send, out, world=world, tokens=tokens, local_heads=hl, head_dim=d)
    orecv = torch.zeros(world, tokens, hl, d, dtype=torch.bfloat16)
    oseq = torch.zeros(tokens, world * hl, d, dtype=torch.bfloat16)
    ulysses.unpack_o_recv(orecv, oseq, world=world, tokens=tokens, local_heads=hl, head_dim=d)
    assert launched == ["h3sa_permute_rows"] * 3
    with pytest.raises(ValueError, match="destination"):
        short = torch.zeros(send.numel() - d, dtype=torch.bfloat16)  # one record short
        ulysses.pack_qkv_send(merged, short, world=world, num_heads=heads, head_dim=d)
    with pytest.raises(ValueError, match="source"):
        ulysses.unpack_qkv_recv(send[:, :, :-1], out, world=world, tokens=tokens, local_heads=hl,
                                head_dim=d)
    with pytest.raises(ValueError, match="destination"):
        ulysses.unpack_o_recv(orecv, oseq[:-1], world=world, tokens=tokens, local_heads=hl,
                              head_dim=d)


def test_other_entry_validation() -> None:
    lib = _lib()
    L = lib.LIB
    assert L.h3sa_quantize_fp8_per_head(16, 32, 48, 1, 10, 2, 64, None) == lib.H3SA_ERR_UNSUPPORTED
    assert L.h3sa_quantize_fp8_per_head(16, 32, 48, 0, 10, 2, 128, None) == lib.H3SA_ERR_INVALID
    rows = (lib.Rows * 3)()
    assert L.h3sa_kv_copy_rows(rows, rows, 3, None, 0, None, 0, 1, 1, 256, None, None) == lib.H3SA_ERR_INVALID
    assert L.h3sa_qkv_norm_rope(16, 32, 48, 64, 10, 7, 80, 4, 2, 128, 1e-5, None, None) == lib.H3SA_ERR_UNSUPPORTED
    assert "rotary" in lib.last_error()
    assert L.h3sa_qkv_norm_rope_pack(16, 32, 48, 64, 80, 10, 96, 96, 4, 6, 128, 4, 1e-5, None, None) == lib.H3SA_ERR_INVALID
    assert "divisible by Ulysses" in lib.last_error()
    pol = lib.MaskPolicy(mode=0, n_hist=1024, n_kv=2048, density=0.0)
    assert L.h3sa_block_mask(16, 128, 2, 128, 0, 128, 32, 16, 48, 16, pol, 64, 80, 16, None, None) == lib.H3SA_ERR_INVALID
    assert "density must be in (0, 1]" in lib.last_error()
    pol = lib.MaskPolicy(mode=0, n_hist=100, n_kv=2048, density=0.5)
    assert L.h3sa_block_mask(16, 128, 2, 128, 0, 128, 32, 16, 48, 16, pol, 64, 80, 16, None, None) == lib.H3SA_ERR_INVALID
    assert "no complete K/V block" in lib.last_error()
    dims = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    assert L.h3sa_permute_rows(16, 33, dims, dims, dims, 16, None) == lib.H3SA_ERR_INVALID


class _Attn:
    softmax_scale = 128 ** -0.5


def _hook_args(q, **over):
    args = dict(attention=_Attn(), layer_name="blocks.0.attn", query=q, key=q, value=q,
                token_tags=torch.zeros(q.shape[0], dtype=torch.long),
                commit_mask=torch.ones(q.shape[0], dtype=torch.bool), cu_seqlens_host=(0, q.shape[0]))
    args.update(over)
    return args


def test_hook_validation_messages_match_reference() -> None:
    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    hook = H3StreamingAttentionHook(CleanAVKVCache(KVContract(local_heads=2, head_dim=128)))
    q = torch.zeros(8, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="called while inactive"):
        hook(**_hook_args(q))
    hook.activate(HookMode.NOISY)
    with pytest.raises(RuntimeError, match="already active"):
        hook.activate(HookMode.NOISY)
    with pytest.raises(RuntimeError, match="requires cuda QKV"):
        hook(**_hook_args(q))
    with pytest.raises(RuntimeError, match="expected local attention tail"):
        hook(**_hook_args(torch.zeros(8, 3, 128, dtype=torch.bfloat16)))
    with pytest.raises(RuntimeError, match="requires torch.bfloat16 QKV"):
        hook(**_hook_args(torch.zeros(8, 2, 128)))
    hook.deactivate()
    with pytest.raises(ValueError, match="unsupported streaming hook mode"):
        hook.activate(HookMode.IDLE)
    with pytest.raises(ValueError, match="unsupported H3 streaming attention backend"):
        H3StreamingAttentionHook(hook.cache, backend="sage_attn")


def test_cache_transactions_match_reference() -> None:
    from h3sa.cache import CleanAVKVCache, KVContract

    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128))
    q = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    tags = torch.tensor([1, 2, 0, 0])
    mask = tags >= 0
    with pytest.raises(RuntimeError, match="begin_clean_commit"):
        cache.stage("blocks.0.attn", q, q, tags, mask)
    with pytest.raises(RuntimeError, match="no clean KV commit is active"):
        cache.commit()
    with pytest.raises(RuntimeError, match="expected clean chunk 0, got 3"):
        cache.begin_clean_commit(3)
    cache.begin_clean_commit(0)
    with pytest.raises(RuntimeError, match="already active"):
        cache.begin_clean_commit(0)
    with pytest.raises(KeyError, match="unexpected transformer layer"):
        cache.stage("blocks.50.attn", q, q, tags, mask)
    with pytest.raises(RuntimeError, match="matching rank-3 shapes"):
        cache.stage("blocks.0.attn", q[0], q[0], tags, mask)
    with pytest.raises(RuntimeError, match="packed metadata length"):
        cache.stage("blocks.0.attn", q, q, tags[:3], mask[:3])
    with pytest.raises(RuntimeError, match="cannot trim persistent KV"):
        cache.retain_sink_and_recent_commits()
    with pytest.raises(RuntimeError, match="cannot drop audio history"):
        cache.drop_audio_history()
    with pytest.raises(RuntimeError, match="missing 50 transformer layers"):
        cache.commit()
    cache.rollback()
    assert not cache.clean_commit_active and cache.committed_blocks == 0


def test_cache_retained_rows_match_oracle() -> None:
    from h3sa.cache import CleanAVKVCache, KVContract

    from oracle.cache_index import CacheIndexOracle

    cache = CleanAVKVCache(KVContract(local_heads=1, head_dim=8))
    oracle = CacheIndexOracle()
    for n_audio, n_video in ((4, 6), (2, 9), (6, 3), (4, 4)):
        tags = [2] * n_audio + [0] * n_video
        oracle.commit(tags, [True] * len(tags))
        cache._commit_token_counts.append(len(tags))
        cache._commit_token_tags.append(tuple(tags))
    sel = [(0, True), (2, False), (3, False)]
    rows, counts, kept = cache.retained_rows(sel)
    oracle._retain(sel)
    assert [divmod(r, 1) for r in rows] and len(rows) == oracle.history_tokens
    assert counts == oracle.counts and kept == oracle.tags


def test_prologue_validation_messages() -> None:
    from h3sa.prologue import fused_qkv_qk_norm_rope_

    w = torch.ones(128, dtype=torch.bfloat16)
    cs = torch.zeros(4, 96, dtype=torch.bfloat16)
    qkv = torch.zeros(4, 3 * 2 * 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="contiguous"):
        fused_qkv_qk_norm_rope_(qkv.t(), w, w, cs, torch.arange(4), 1e-5)
    with pytest.raises(ValueError, match="BF16"):
        fused_qkv_qk_norm_rope_(qkv.float(), w, w, cs, torch.arange(4), 1e-5)
    with pytest.raises(ValueError, match="three complete projections"):
        fused_qkv_qk_norm_rope_(torch.zeros(4, 700, dtype=torch.bfloat16), w, w, cs, torch.arange(4), 1e-5)
    with pytest.raises(ValueError, match="positions do not cover"):
        fused_qkv_qk_norm_rope_(qkv, w, w, cs, torch.arange(3), 1e-5)
    with pytest.raises(ValueError, match="cache span is invalid"):
        fused_qkv_qk_norm_rope_(qkv, w, w, torch.zeros(4, 97, dtype=torch.bfloat16), torch.arange(4), 1e-5)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_qkv_qk_norm_rope_(qkv, w, w, cs, torch.arange(4), 1e-5)


def test_parallel_context_validation() -> None:
    from h3sa.ulysses import ParallelContext

    with pytest.raises(ValueError, match="invalid ulysses topology"):
        ParallelContext(1, 0, 2, 2, object(), object())
    with pytest.raises(ValueError, match="process groups are required"):
        ParallelContext(1, 0, 2, 1, None, object())


def test_permute_rows_refuses_unaligned_records(monkeypatch) -> None:
    """The permute kernel moves 16-byte vectors: record sizes, strides and base pointers that
    are not 16-byte multiples are refused in the wrapper (library call stubbed, CPU tensors)."""

    from h3sa import kernels

    monkeypatch.setattr(kernels, "_require_cuda", lambda *t: None)
    monkeypatch.setattr(kernels, "call", lambda name, *a: None)
    monkeypatch.setattr(kernels, "stream_handle", lambda s=None: 0)
    src = torch.zeros(4096, dtype=torch.uint8)
    dst = torch.zeros(4096, dtype=torch.uint8)
    kernels.permute_rows(src, dst, (2, 2, 1, 1), (256, 128, 0, 0), (128, 256, 0, 0), 128)
    with pytest.raises(ValueError, match="multiples of 16"):
        kernels.permute_rows(src, dst, (2, 2, 1, 1), (256, 128, 0, 0), (128, 256, 0, 0), 120)
    with pytest.raises(ValueError, match="multiples of 16"):
        kernels.permute_rows(src, dst, (2, 2, 1, 1), (264, 128, 0, 0), (128, 256, 0, 0), 128)
    with pytest.raises(ValueError, match="16-byte boundary"):
        kernels.permute_rows(src[8:], dst, (2, 2, 1, 1), (256, 128, 0, 0), (128, 256, 0, 0), 128)


def test_peer_barrier_limit_validation() -> None:
    lib = _lib()
    L = lib.LIB
    for limit in (0, -5, 61_000_000_000):
        rc = L.h3sa_peer_barrier_limit(16, 2, 0, 1, limit, None, None)
        assert rc == lib.H3SA_ERR_INVALID and "wait limit" in lib.last_error()
    assert L.h3sa_peer_barrier_limit(16, 2, 2, 1, 1000, None, None) == lib.H3SA_ERR_INVALID


@pytest.mark.parametrize("heads,world", [(3, 2), (28, 8), (6, 4)])
def test_padded_ulysses_layouts_stay_inside_their_buffers(monkeypatch, heads: int, world: int) -> None:
    """Heads not divisible by the world: the pack and O-unpack layouts split into the ranks
    with full shards and the partial one, and every launch stays inside its buffers."""

    from h3sa import kernels, ulysses

    launched = []
    monkeypatch.setattr(kernels, "_require_cuda", lambda *t: None)
    monkeypatch.setattr(kernels, "call", lambda name, *a: launched.append(name))
    monkeypatch.setattr(kernels, "stream_handle", lambda s=None: 0)
    tokens, d = 5, 128
    hl = -(-heads // world)
    merged = torch.zeros(tokens, 3 * heads * d, dtype=torch.bfloat16)
    send = torch.zeros(world, 3, tokens, hl, d, dtype=torch.bfloat16)
    ulysses.pack_qkv_send(merged, send, world=world, num_heads=heads, head_dim=d)
    recv = torch.zeros(world, tokens, hl, d, dtype=torch.bfloat16)
    out = torch.zeros(tokens, heads, d, dtype=torch.bfloat16)
    ulysses.unpack_o_recv(recv, out, world=world, tokens=tokens, local_heads=hl, head_dim=d,
                          num_heads=heads)
    expect = (1 + (heads % hl != 0)) * 2
    assert len(launched) == expect


def test_cache_refuses_use_after_a_failed_commit() -> None:
    """A commit that fails half way (here: the e4m3 history quantiser cannot run on CPU
    tensors) leaves the cache invalid until clear(), as FL2AV's does
    (F/streaming/cache.py:766-778, 221-223)."""

    from h3sa.cache import CleanAVKVCache, KVContract

    cache = CleanAVKVCache(KVContract(local_heads=1, head_dim=128, device_type="cpu"),
                           layer_names=("blocks.0.attn",), device="cpu",
                           segmented_fp8_history=True)
    tags = torch.tensor([1, 2, 2, 0, 0, 0])
    commit = torch.tensor([False, True, True, True, True, True])
    kv = torch.zeros(6, 1, 128, dtype=torch.bfloat16)
    cache.layer("blocks.0.attn", torch.device("cpu"))  # the hook creates the layer first
    cache.begin_clean_commit(0)
    cache.stage_in_place("blocks.0.attn", kv, kv, tags, commit)
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.commit()
    for probe in (lambda: cache.committed_blocks, lambda: cache.history_tokens,
                  lambda: cache.history("blocks.0.attn"), lambda: cache.retain_recent_commits(1)):
        with pytest.raises(RuntimeError, match="invalid after a failed clean commit"):
            probe()
    cache.clear()
    assert cache.committed_blocks == 0 and cache.history_tokens == 0
    with pytest.raises(ValueError, match="bounded clean commit count must be positive"):
        cache.commit_bounded(0)
    with pytest.raises(ValueError, match="retained clean commit count"):
        cache.retain_recent_commits(0)
    with pytest.raises(ValueError, match="recent clean commit count must be non-negative"):
        cache.retain_sink_and_recent_commits(-1)


def test_live_document_hint_checks_match_reference() -> None:
    """FL2AV's live_documents_hint: same checks and messages as
    F/streaming/attention_hook.py:337-371; without a hint the commit mask decides."""

    from h3sa.hook import _live_documents_from_mask_or_hint as live

    bounds = ((0, 4), (4, 4), (4, 9))
    mask = torch.tensor([False, True, True, False, False, False, False, False, False])
    assert live(mask, bounds, None) == (0,)
    assert live(mask, bounds, (2,)) == (2,)
    with pytest.raises(TypeError, match="must be a tuple"):
        live(mask, bounds, [0])
    with pytest.raises(ValueError, match="invalid document index"):
        live(mask, bounds, (3,))
    with pytest.raises(ValueError, match="invalid document index"):
        live(mask, bounds, (True,))
    with pytest.raises(ValueError, match="sorted and unique"):
        live(mask, bounds, (2, 0))
    with pytest.raises(ValueError, match="empty document"):
        live(mask, bounds, (1,))


def test_snapshot_header_checks_run_before_device_work(tmp_path) -> None:
    """A snapshot file is validated on the host: wrong magic, another format version, a
    truncated or corrupted section and a contract mismatch are refused with ValueError."""

    import json
    import struct
    import zlib

    from h3sa import snapshot
    from h3sa.cache import KVContract

    data = bytes(range(256)) * 8
    header = {"format": snapshot.FORMAT_VERSION,
              "contract": {"local_heads": 2, "head_dim": 128, "dtype": "bfloat16",
                           "device_type": "cuda"},
              "layer_names": ["blocks.0.attn"], "segmented_fp8_history": False,
              "block_index": 1, "commit_token_counts": [8], "commit_token_tags": [[0] * 8],
              "layers": {}, "sections": [{"name": "blocks.0.attn/key", "offset": 0,
                                          "nbytes": len(data), "crc32": zlib.crc32(data),
                                          "dtype": "bfloat16", "shape": [4, 2, 128]}]}

    def write(name: str, hdr: dict, payload: bytes, magic: bytes = snapshot.MAGIC):
        head = json.dumps(hdr).encode()
        base = (len(magic) + 8 + len(head) + 4095) // 4096 * 4096
        p = tmp_path / name
        p.write_bytes(magic + struct.pack("<Q", len(head)) + head
                      + b"\0" * (base - len(magic) - 8 - len(head)) + payload)
        return p

    header_ok, base = snapshot.read_header(write("ok.h3kv", header, data))
    assert header_ok["block_index"] == 1 and base == 4096
    with pytest.raises(ValueError, match="not an H3 cache snapshot"):
        snapshot.read_header(write("magic.h3kv", header, data, magic=b"NOTACACH"))
    with pytest.raises(ValueError, match="format"):
        snapshot.read_header(write("ver.h3kv", dict(header, format=99), data))
    with pytest.raises(ValueError, match="truncated"):
        snapshot.load_cache(write("short.h3kv", header, data[:100]))
    corrupt = bytearray(data)
    corrupt[17] ^= 1
    with pytest.raises(ValueError, match="CRC-32"):
        snapshot.load_cache(write("crc.h3kv", header, bytes(corrupt)))
    with pytest.raises(ValueError, match="contract"):
        snapshot.load_cache(write("c.h3kv", header, data),
                            contract=KVContract(local_heads=4, head_dim=128))


def test_sol_history_modality_rows() -> None:
    """The SOL history split (F/streaming/cache.py:439-499) on the row bookkeeping alone: per
    selected block its audio rows, then its video rows; a fused current document's sink +
    recent window."""

    from h3sa.cache import CleanAVKVCache, KVContract

    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128), layer_names=("blocks.0.attn",))
    for tags in ((2, 2, 0, 0, 0), (0, 0, 0), (2, 0, 2, 0)):
        cache._commit_token_counts.append(len(tags))
        cache._commit_token_tags.append(tags)
    audio, video = cache.history_modality_parts_rows((0, 1, 2))
    assert audio == [[0, 1], [8, 10]]
    assert video == [[2, 3, 4], [5, 6, 7], [9, 11]]
    audio, video = cache.history_modality_parts_rows((0, 2))
    assert audio == [[0, 1], [8, 10]] and video == [[2, 3, 4], [9, 11]]


def test_sol_attention_argument_validation() -> None:
    """h3sa_sol_attention refuses bad sizes, scales and pointers before touching the device."""

    lib = _lib()
    L = lib.LIB
    A = 1 << 20  # a 16-byte aligned stand-in address, never dereferenced

    def call(**over):
        a = dict(q=A, nq=100, k=A, v=A, nk=1000, heads=2, hd=128, scale=0.088, tau=1.0, sink=64,
                 kc=A, vs=A, stats=A, mask=A, tele=None, out=A)
        a.update(over)
        return L.h3sa_sol_attention(a["q"], a["nq"], a["k"], a["v"], a["nk"], a["heads"], a["hd"],
                                    ctypes.c_float(a["scale"]), ctypes.c_float(a["tau"]), a["sink"],
                                    a["kc"], a["vs"], a["stats"], a["mask"], a["tele"], a["out"],
                                    None, None)

    assert call(hd=64) == lib.H3SA_ERR_UNSUPPORTED and "head_dim 128" in lib.last_error()
    assert call(nk=4096 * 64 + 1) == lib.H3SA_ERR_UNSUPPORTED and "exceed" in lib.last_error()
    for bad in (dict(nq=0), dict(nk=0), dict(heads=0), dict(sink=-1)):
        assert call(**bad) == lib.H3SA_ERR_INVALID, bad
    assert call(scale=0.0) == lib.H3SA_ERR_INVALID and "scale" in lib.last_error()
    assert call(tau=float("nan")) == lib.H3SA_ERR_INVALID
    assert call(kc=None) == lib.H3SA_ERR_INVALID and "null" in lib.last_error()
    assert call(out=A + 8) == lib.H3SA_ERR_INVALID and "aligned" in lib.last_error()


def test_hook_sol_dense_rules() -> None:
    """Which calls the sol_attn backend routes (F/streaming/attention_hook.py:909-929): none in
    the commit and capture modes, the first sol_attn_dense_layers layers or the first
    sol_attn_dense_denoise_steps denoise steps; in a fused forward the current document only."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128), layer_names=("blocks.0.attn",))
    hook = H3StreamingAttentionHook(cache, attention_backend="sol_attn", sol_attn_dense_layers=2,
                                    sol_attn_dense_denoise_steps=1)
    hook.activate(mode=HookMode.NOISY, block_index=0, full_prefix=None, denoise_step_index=1)
    assert hook._sol_documents("blocks.2.attn", False) == [0]
    assert hook._sol_documents("blocks.1.attn", False) == []
    hook.deactivate()
    hook.activate(mode=HookMode.NOISY, block_index=0, full_prefix=None, denoise_step_index=0)
    assert hook._sol_documents("blocks.9.attn", False) == []
    hook.deactivate()
    hook.activate(mode=HookMode.CLEAN_COMMIT, block_index=0, full_prefix=None)
    assert hook._sol_documents("blocks.9.attn", False) == []
    hook.deactivate()
    hook.activate(HookMode.NOISY)  # the T form: no denoise step index
    assert hook._sol_documents("blocks.9.attn", False) == [0]
    assert hook._sol_documents("blocks.9.attn", True) == [1]
    hook.deactivate()
    dense = H3StreamingAttentionHook(cache, attention_backend="sdpa")
    dense.activate(HookMode.NOISY)
    assert dense._sol_documents("blocks.9.attn", False) == [] and dense.sol_attn_receipt() is None
    with pytest.raises(ValueError, match="stride"):
        H3StreamingAttentionHook(cache, attention_backend="flash_attn3_fp8_dynamic",
                                 current_video_kv_stride=2)
    with pytest.raises(ValueError, match="SageAttention"):
        H3StreamingAttentionHook(cache, direct_sage_kv_workspace=True)
    with pytest.raises(ValueError, match="stride 1"):
        H3StreamingAttentionHook(cache, dense_current_document_when_empty=True,
                                 current_video_kv_stride=2)
