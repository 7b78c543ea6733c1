"""Segmented FP8 KV: per-part e4m3 quantisation and attention over parts with their own scales.

* ``quantize_fp8_rows`` quantises one part of a paged bf16 pool (any start row) into an e4m3
  pool starting on a block boundary, bit-exact against the oracle quantiser of that part,
  with the rest of the part's last block zeroed.
* ``attention_fwd_fp8_parts`` over parts quantised with different scales matches the
  reference's segmented backend (one FP8 attention per part, merged by log-sum-exp,
  F/streaming/attention_hook.py:1015-1066) restated in the oracle on the same bytes:
  relative L2 <= 3e-2 (FP8 tolerance), for the dense kernel and the block-sparse kernel
  (every block listed).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import fp8 as ofp8

pytestmark = pytest.mark.gpu
TOL = 3e-2


def _paged(rows: int, heads: int, dtype: torch.dtype, gen: np.random.Generator, extra: int = 3):
    from h3sa.kernels import PAGE_ROWS

    blocks = (rows + PAGE_ROWS - 1) // PAGE_ROWS
    pages = blocks + extra
    table = torch.from_numpy(gen.permutation(pages)[:blocks].astype(np.int32)).cuda()
    pool = torch.zeros(heads, pages * PAGE_ROWS, 128, dtype=dtype, device="cuda")
    return pool, table


def _phys(table: torch.Tensor, rows: np.ndarray) -> np.ndarray:
    tab = table.cpu().numpy()
    return tab[rows // 128] * 128 + rows % 128


def test_part_quantiser_bit_exact_with_zeroed_tail() -> None:
    from h3sa import kv_copy_rows
    from h3sa.kernels import quantize_fp8_rows

    gen = np.random.default_rng(3)
    heads, hist, start, count = 3, 2000, 333, 1100
    kb, tb = _paged(hist, heads, torch.bfloat16, gen)
    vb = torch.zeros_like(kb)
    k = torch.from_numpy(gen.standard_normal((hist, heads, 128)).astype(np.float32)).bfloat16().cuda()
    v = (torch.from_numpy(gen.standard_normal((hist, heads, 128)).astype(np.float32)) * 3).bfloat16().cuda()
    k[start + 7, 1, 5] = 60.0  # an outlier inside the part sets head 1's K scale
    kv_copy_rows([k, v], [kb, vb], count=hist, dst_table=tb)
    dst_start = 256
    k8, t8 = _paged(dst_start + count, heads, torch.float8_e4m3fn, gen)
    k8.view(torch.uint8).fill_(0x55)  # garbage the tail must overwrite
    v8 = torch.full_like(k8.view(torch.uint8), 0x55).view(torch.float8_e4m3fn)
    ks = torch.empty(heads, dtype=torch.float32, device="cuda")
    vs = torch.empty_like(ks)
    work = torch.empty(2 * heads, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the workspace is cleared by each call
        quantize_fp8_rows([kb, vb], [k8, v8], [ks, vs], work, count=count, src_start=start,
                          dst_start=dst_start, src_table=tb, dst_table=t8, zero_tail=True)
    torch.cuda.synchronize()
    logical = dst_start + np.arange(count)
    phys = _phys(t8, logical)
    end = dst_start + count
    tail = _phys(t8, np.arange(end, (end + 127) // 128 * 128))
    for src, q8, sc in ((k, k8, ks), (v, v8, vs)):
        ref_q, ref_s = ofp8.quantize_fp8_e4m3_per_head(src[start:start + count].float().cpu().numpy()[None])
        got = q8.view(torch.uint8).cpu().numpy()
        assert np.array_equal(sc.cpu().numpy(), ref_s[0])
        assert np.array_equal(got[:, phys].transpose(1, 0, 2), ref_q[0])
        assert np.all(got[:, tail] == 0)


def _parts_case(sizes: list[int], heads: int, nq: int, gen: np.random.Generator):
    """Parts of the given sizes, each quantised with its own scales into block-aligned pages
    of one e4m3 pool, plus e4m3 Q; returns device tensors and the oracle's part tuples."""

    from h3sa.kernels import PAGE_ROWS, quantize_fp8_e4m3_per_head, quantize_fp8_rows

    starts, cursor = [], 0
    for n in sizes:
        starts.append(cursor)
        cursor = (cursor + n + PAGE_ROWS - 1) // PAGE_ROWS * PAGE_ROWS
    k8, table = _paged(cursor, heads, torch.float8_e4m3fn, gen)
    v8 = torch.zeros_like(k8)
    n_blocks = int(table.numel())
    block_part = np.zeros(n_blocks, dtype=np.int32)
    kscale = torch.empty(len(sizes), heads, dtype=torch.float32, device="cuda")
    vscale = torch.empty_like(kscale)
    work = torch.empty(2 * heads, dtype=torch.int32, device="cuda")
    oracle_parts = []
    for i, (n, s0) in enumerate(zip(sizes, starts)):
        amp = 1.0 + 2.0 * i  # parts with clearly different scales
        k = (torch.from_numpy(gen.standard_normal((n, heads, 128)).astype(np.float32)) * amp).bfloat16().cuda()
        v = (torch.from_numpy(gen.standard_normal((n, heads, 128)).astype(np.float32)) / amp).bfloat16().cuda()
        quantize_fp8_rows([k, v], [k8, v8], [kscale[i], vscale[i]], work, count=n, dst_start=s0,
                          dst_table=table, zero_tail=True)
        for b in range(s0 // PAGE_ROWS, (s0 + n + PAGE_ROWS - 1) // PAGE_ROWS):
            block_part[b] = i | (min(PAGE_ROWS, s0 + n - b * PAGE_ROWS) << 16)
        torch.cuda.synchronize()
        phys = _phys(table, s0 + np.arange(n))
        oracle_parts.append((k8.view(torch.uint8).cpu().numpy()[:, phys].transpose(1, 0, 2),
                             v8.view(torch.uint8).cpu().numpy()[:, phys].transpose(1, 0, 2),
                             kscale[i].cpu().numpy(), vscale[i].cpu().numpy()))
    q = torch.from_numpy(gen.standard_normal((nq, heads, 128)).astype(np.float32)).bfloat16()
    q8, qs = quantize_fp8_e4m3_per_head(q.cuda().unsqueeze(0))
    return {"q": q, "q8": q8[0], "qs": qs.reshape(-1).contiguous(), "k8": k8, "v8": v8,
            "table": table, "block_part": torch.from_numpy(block_part).cuda(), "kscale": kscale,
            "vscale": vscale, "oracle_parts": oracle_parts, "n_kv": cursor}


@pytest.mark.parametrize("sparse", [False, True])
def test_attention_over_parts_matches_segmented_oracle(sparse: bool) -> None:
    from h3sa import AttentionProblem
    from h3sa.kernels import PAGE_ROWS, attention_fwd_fp8_parts

    gen = np.random.default_rng(5 + sparse)
    heads, nq, scale = 2, 700, 128 ** -0.5
    c = _parts_case([300, 1000, 257, 64], heads, nq, gen)
    out = torch.zeros(nq, heads, 128, dtype=torch.bfloat16, device="cuda")
    lists = {}
    if sparse:
        qb, kb = (nq + PAGE_ROWS - 1) // PAGE_ROWS, c["n_kv"] // PAGE_ROWS
        lists["kv_num_blocks"] = torch.full((heads, qb), kb, dtype=torch.int32, device="cuda")
        lists["kv_indices"] = torch.arange(kb, dtype=torch.int32, device="cuda").repeat(heads, qb, 1)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    attention_fwd_fp8_parts(c["q8"], out, c["k8"], c["v8"], c["table"],
                            [AttentionProblem(0, nq, 0, c["n_kv"], sparse=sparse)], scale,
                            q_scale=c["qs"], block_part=c["block_part"], part_k_scale=c["kscale"],
                            part_v_scale=c["vscale"], device_error=err, **lists)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = oatt.segmented_fp8_attention(c["q"], c["oracle_parts"], scale)
    rel = float((out.float().cpu() - ref).norm() / ref.norm())
    assert rel <= TOL, f"segmented FP8 attention rel L2 {rel:.3e}"


@pytest.mark.parametrize("paged", [False, True])
def test_segment_row_means_and_commit_scores_match_oracle(paged: bool) -> None:
    """Column means of bf16 row segments (sizes around the 256-row chunk) are bit-exact
    against the oracle's fp64 mean rounded to fp32; the commit scores agree to fp64
    rounding."""

    from h3sa.kernels import commit_scores, kv_copy_rows, segment_row_means
    from oracle import commit_topk as otopk

    gen = np.random.default_rng(5)
    heads, rows = 3, 1700
    x = (gen.standard_normal((rows, heads, 128)) * 2 + 0.5).astype(np.float32)
    xt = torch.from_numpy(x).bfloat16().cuda()
    xb = xt.float().cpu().numpy()
    segments = [(0, 1), (1, 255), (256, 256), (512, 257), (769, 700), (1469, 231), (5, 0)]
    if paged:
        pool, table = _paged(rows, heads, torch.bfloat16, gen)
        kv_copy_rows([xt], [pool], count=rows, dst_table=table)
        means = segment_row_means(pool, segments, src_table=table)
    else:
        means = segment_row_means(xt, segments)
    torch.cuda.synchronize()
    for i, (a, n) in enumerate(segments):
        if n == 0:
            assert torch.count_nonzero(means[i]) == 0
            continue
        ref = otopk.key_summary(xb[a:a + n])
        assert np.array_equal(means[i].cpu().numpy(), ref), i
    summaries = means[:6].contiguous()
    q_mean = segment_row_means(xt, [(100, 900)])[0]
    scores = commit_scores(summaries, q_mean).cpu().numpy()
    ref = otopk.commit_scores(summaries.cpu().numpy(), q_mean.cpu().numpy())
    np.testing.assert_allclose(scores, ref, rtol=1e-12, atol=1e-12)


def test_cache_key_summaries_match_reference_golden() -> None:
    """The segmented cache's per-part key summaries through the reference's own schedule
    (tests/golden/topk.npz: six commits, then sink + recent retention that keeps block 0's
    video rows): within an fp32 ulp of the reference cache's key.float().mean(dim=0)."""

    from pathlib import Path

    from h3sa.cache import CleanAVKVCache, KVContract

    g = np.load(Path(__file__).resolve().parent / "golden" / "topk.npz")
    layer = "blocks.0.attn"
    cache = CleanAVKVCache(KVContract(local_heads=2, head_dim=128), layer_names=(layer,),
                           segmented_fp8_history=True)
    for i in range(6):
        tags = torch.from_numpy(g[f"tags_{i}"]).cuda()
        key = torch.from_numpy(g[f"key_{i}"]).bfloat16().cuda()
        cache.begin_clean_commit(cache.committed_blocks)
        cache.stage(layer, key, key.clone(), tags, (tags == 0) | (tags == 2))
        cache.commit()

    def check(stage: str) -> None:
        got = cache.layer(layer).fp8.key_summary.cpu().numpy()
        ref = g[f"summary_{stage}"]
        assert got.shape == ref.shape, stage
        assert np.all(np.abs(got - ref) <= np.spacing(np.abs(ref))), stage

    check("full")
    cache.retain_sink_and_recent_commits(3, sink_video_only=True)
    assert list(cache.commit_token_counts) == list(g["retained_counts"])
    check("retained")
