"""GPU parity of the feeding kernels against the oracle and the reference golden vectors.

Bit-exact: e4m3 quantiser, block masks, Ulysses layouts, KV row copies, prologue (against
the oracle, which follows the same exact arithmetic); the prologue against the reference's
own CPU path is held to the same agreement as the oracle (<= 1 bf16 ulp, >= 99.9% exact).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from inputs import fp8_input, mask_inputs, prologue_inputs  # noqa: E402

from oracle import block_mask as omask  # noqa: E402
from oracle import fp8 as ofp8  # noqa: E402
from oracle import prologue as opro  # noqa: E402
from oracle import ulysses as ouly  # noqa: E402

pytestmark = pytest.mark.gpu


def _g(name: str) -> dict:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


def _bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _cuda_bf16(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).cuda()


def test_fp8_quantiser_bit_exact_vs_reference() -> None:
    import h3sa

    g = _g("fp8.npz")
    x = _cuda_bf16(fp8_input(int(g["seed"])))
    q, s = h3sa.quantize_fp8_e4m3_per_head(x)
    torch.cuda.synchronize()
    assert np.array_equal(s.cpu().numpy(), g["scale"])
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g["q"])


@pytest.mark.parametrize("shape", [(2, 1, 5, 128), (1, 1000, 7, 128), (1, 257, 3, 128)])
def test_fp8_quantiser_vs_oracle(shape: tuple[int, ...]) -> None:
    import h3sa

    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal(shape).astype(np.float32) * 3
    xb = _cuda_bf16(x)
    q, s = h3sa.quantize_fp8_e4m3_per_head(xb)
    oq, os_ = ofp8.quantize_fp8_e4m3_per_head(xb.float().cpu().numpy())
    assert np.array_equal(s.cpu().numpy(), os_)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), oq)


def test_fp8_pool_quantiser_matches_packed() -> None:
    """Quantising logical rows through a shuffled page table == quantising the packed rows."""

    import h3sa

    rng = np.random.default_rng(4)
    rows, heads = 1000, 3
    x = _cuda_bf16(rng.standard_normal((rows, heads, 128)).astype(np.float32))
    pages = 12
    table = torch.randperm(pages)[:8].to(torch.int32).cuda()
    pool = torch.zeros(heads, pages * 128, 128, dtype=torch.bfloat16, device="cuda")
    h3sa.kv_copy_rows([x], [pool], count=rows, dst_table=table)
    pool8 = torch.zeros_like(pool, dtype=torch.float8_e4m3fn)
    scale = torch.empty(heads, dtype=torch.float32, device="cuda")
    h3sa.quantize_fp8_pool(pool, pool8, scale, table, rows)
    back = torch.empty(rows, heads, 128, dtype=torch.float8_e4m3fn, device="cuda")
    h3sa.kv_copy_rows([pool8], [back], count=rows, src_table=table)
    q, s = h3sa.quantize_fp8_e4m3_per_head(x.unsqueeze(0))
    assert torch.equal(scale, s.reshape(-1))
    assert torch.equal(back.view(torch.uint8), q.squeeze(0).view(torch.uint8))


def _paged(keys: np.ndarray, shuffle: bool = True):
    """Logical rows [N, H, d] into a paged pool object with key/table attributes."""

    import h3sa

    n, heads, _ = keys.shape
    blocks = (n + 127) // 128
    pages = blocks + 3
    table = (torch.randperm(pages)[:blocks] if shuffle else torch.arange(blocks)).to(torch.int32).cuda()
    pool = torch.zeros(heads, pages * 128, 128, dtype=torch.bfloat16, device="cuda")
    h3sa.kv_copy_rows([_cuda_bf16(keys)], [pool], count=n, dst_table=table)

    class P:
        key = pool
        value = pool

    P.table = table
    return P


def test_history_mask_matches_reference_golden() -> None:
    from h3sa.block_sparse import history_block_mask

    g = _g("mask.npz")
    q, hk = mask_inputs(int(g["seed"]), int(g["heads"]), int(g["nq"]), int(g["nh"]))
    nq, nh, total = int(g["nq"]), int(g["nh"]), int(g["total"])
    extra = np.random.default_rng(0).standard_normal((int(g["heads"]), total - nh, 128)).astype(np.float32)
    keys = np.concatenate([hk[0], extra], axis=1).transpose(1, 0, 2)       # [N, H, d]
    paged = _paged(keys)
    query = _cuda_bf16(q[0].transpose(1, 0, 2))                            # [nq, H, d]
    num, idx = history_block_mask(query, paged, q_lo=0, q_hi=nq, n_hist=nh, n_kv=total,
                                  density=float(g["density"]))
    torch.cuda.synchronize()
    assert np.array_equal(num.cpu().numpy(), g["kv_num_blocks"][0])
    assert np.array_equal(idx.cpu().numpy(), g["kv_indices"][0])


@pytest.mark.parametrize("nq,nh,density", [(700, 1024, 0.25), (300, 1500, 0.5), (129, 2048, 0.1)])
def test_composite_mask_bit_exact_vs_oracle(nq: int, nh: int, density: float) -> None:
    from h3sa.block_sparse import block_flags, composite_block_mask

    rng = np.random.default_rng(nq + nh)
    heads = 3
    q = (rng.standard_normal((nq, heads, 128)) * 0.7).astype(np.float32)
    k = rng.standard_normal((nh + nq, heads, 128)).astype(np.float32)
    qb = torch.from_numpy(q).bfloat16().float().numpy()
    kb = torch.from_numpy(k).bfloat16().float().numpy()
    q_audio = np.zeros(nq, bool)
    q_audio[: min(40, nq)] = True
    k_audio = np.zeros(nh + nq, bool)
    k_audio[:20] = True
    k_audio[nh:nh + min(40, nq)] = True
    ref = omask.composite_mask(qb.transpose(1, 0, 2), kb.transpose(1, 0, 2), n_hist=nh,
                               q_audio=q_audio, k_audio=k_audio, density=density)
    paged = _paged(k)
    num, idx = composite_block_mask(
        _cuda_bf16(q), paged, q_lo=0, q_hi=nq, n_hist=nh, n_kv=nh + nq,
        q_block_audio=block_flags(torch.from_numpy(q_audio), nq),
        kv_block_audio=block_flags(torch.from_numpy(k_audio), nh + nq), density=density)
    torch.cuda.synchronize()
    assert np.array_equal(num.cpu().numpy(), ref["kv_num_blocks"])
    assert np.array_equal(idx.cpu().numpy(), ref["kv_indices"])


@pytest.mark.parametrize("nq,nh,density", [(512, 1280, 0.3), (1000, 3000, 0.5), (200, 4096, 0.05)])
def test_history_mask_bit_exact_vs_oracle(nq: int, nh: int, density: float) -> None:
    from h3sa.block_sparse import history_block_mask

    rng = np.random.default_rng(nq * 3 + nh)
    heads = 2
    q = torch.from_numpy(rng.standard_normal((nq, heads, 128)).astype(np.float32)).bfloat16().float().numpy()
    k = torch.from_numpy(rng.standard_normal((nh + nq + 64, heads, 128)).astype(np.float32)).bfloat16().float().numpy()
    ref = omask.dynamic_history_mask(q.transpose(1, 0, 2), k[:nh].transpose(1, 0, 2),
                                     k.shape[0], density)
    num, idx = history_block_mask(_cuda_bf16(q), _paged(k), q_lo=0, q_hi=nq, n_hist=nh,
                                  n_kv=k.shape[0], density=density)
    torch.cuda.synchronize()
    assert np.array_equal(num.cpu().numpy(), ref["kv_num_blocks"])
    assert np.array_equal(idx.cpu().numpy(), ref["kv_indices"])


def _prologue_case(seq: int, heads: int, seed: int = 11):
    inp = prologue_inputs(seed, seq, heads, 128)
    layout = opro.packed_layout(text_len=16, latent_t=2, latent_h=8, latent_w=12, audio_t=8)
    grid = layout["grid"][:seq] if seq <= layout["seq_len"] else np.resize(layout["grid"], (seq, 3))
    cs = opro.rope_cos_sin(grid, opro.default_inv_freq(16))
    return inp, cs


def test_prologue_bit_exact_vs_oracle_and_golden() -> None:
    from h3sa.prologue import fused_qkv_qk_norm_rope_

    g = _g("prologue.npz")
    seq, heads = int(g["seq"]), int(g["heads"])
    inp = prologue_inputs(int(g["seed"]), seq, heads, 128)
    cs = _bf16_bits_to_f32(g["cos_sin_bf16"])
    qkv = _cuda_bf16(inp["qkv"])
    fused_qkv_qk_norm_rope_(qkv, _cuda_bf16(inp["q_weight"]), _cuda_bf16(inp["k_weight"]),
                            _cuda_bf16(cs), torch.arange(seq, device="cuda"), 1e-5)
    out = qkv.float().cpu().numpy()
    ref = opro.qkv_norm_rope(inp["qkv"], inp["q_weight"], inp["k_weight"], cs, np.arange(seq),
                             heads, 128, 1e-5)
    assert np.array_equal(out, ref)
    view = out.reshape(seq, 3, heads, 128)
    for i, key in ((0, "q_bf16"), (1, "k_bf16")):
        gold = _bf16_bits_to_f32(g[key])
        diff = np.abs(view[:, i] - gold)
        assert (diff == 0).mean() > 0.999
        assert np.all(diff <= np.abs(gold) * 2.0 ** -7 + 1e-30)


def test_unmerged_qk_norm_rope_matches_oracle() -> None:
    """fused_qk_norm_rope (one of Q or K, out of place, per-token cos/sin with duplicated
    halves as the processor builds them) equals the oracle prologue's Q plane bit for bit,
    on a strided view of a merged projection."""

    from h3sa.prologue import fused_qk_norm_rope

    seq, heads = 200, 4
    inp, cs = _prologue_case(seq, heads, seed=17)
    pos = np.random.default_rng(2).integers(0, cs.shape[0], seq)
    half = cs.shape[1] // 2
    sel = cs[pos]
    cos = np.concatenate((sel[:, :half], sel[:, :half]), -1)
    sin = np.concatenate((sel[:, half:], sel[:, half:]), -1)
    merged = _cuda_bf16(inp["qkv"])
    q_view = merged.view(seq, 3, heads, 128)[:, 0]  # a strided view, as qkv.split gives
    out = fused_qk_norm_rope(q_view, _cuda_bf16(inp["q_weight"]), _cuda_bf16(cos), _cuda_bf16(sin),
                             1e-5)
    ref = opro.qkv_norm_rope(inp["qkv"], inp["q_weight"], inp["k_weight"], cs, pos, heads, 128,
                             1e-5).reshape(seq, 3, heads, 128)
    assert out.is_contiguous() and np.array_equal(out.float().cpu().numpy(), ref[:, 0])
    assert torch.equal(merged, _cuda_bf16(inp["qkv"]))  # the input is not modified


@pytest.mark.parametrize("world", [2, 4])
def test_prologue_pack_matches_oracle_send_layout(world: int) -> None:
    from h3sa.prologue import qkv_norm_rope_pack

    seq, heads = 96, 8
    inp, cs = _prologue_case(seq, heads, seed=3)
    pos = np.random.default_rng(1).integers(0, cs.shape[0], seq)
    send = qkv_norm_rope_pack(_cuda_bf16(inp["qkv"]), _cuda_bf16(inp["q_weight"]),
                              _cuda_bf16(inp["k_weight"]), _cuda_bf16(cs),
                              torch.from_numpy(pos).cuda(), 1e-5, world=world)
    ref = opro.qkv_norm_rope(inp["qkv"], inp["q_weight"], inp["k_weight"], cs, pos, heads, 128, 1e-5)
    expect = ref.reshape(seq, 3, world, heads // world, 128).transpose(2, 1, 0, 3, 4)
    assert np.array_equal(send.float().cpu().numpy(), expect)


@pytest.mark.parametrize("heads,world", [(16, 2), (16, 4), (16, 8), (3, 2), (28, 8), (6, 4)])
def test_ulysses_layouts_vs_oracle(heads: int, world: int) -> None:
    """Pack -> emulated all-to-all -> unpack on one GPU equals the oracle's every-rank view,
    including zero-padded head shards when the heads do not divide by the world."""

    from h3sa.ulysses import pack_qkv_send, unpack_o_recv, unpack_qkv_recv

    tokens, d = 10, 128
    hl = -(-heads // world)
    rng = np.random.default_rng(world)
    merged = [rng.standard_normal((tokens, 3 * heads * d)).astype(np.float32) for _ in range(world)]
    mb = [torch.from_numpy(m).bfloat16().float().numpy() for m in merged]
    sends = []
    for r in range(world):
        s = torch.full((world, 3, tokens, hl, d), 9.0, dtype=torch.bfloat16, device="cuda")
        pack_qkv_send(_cuda_bf16(mb[r]), s, world=world, num_heads=heads, head_dim=d)
        sends.append(s)
    expect = ouly.merged_qkv_sequence_to_heads(mb, heads, d)
    outs = []
    for r in range(world):
        recv = torch.stack([sends[s][r] for s in range(world)])
        out = torch.empty(3, world * tokens, hl, d, dtype=torch.bfloat16, device="cuda")
        unpack_qkv_recv(recv, out, world=world, tokens=tokens, local_heads=hl, head_dim=d)
        for i in range(3):
            assert np.array_equal(out[i].float().cpu().numpy(), expect[r][i])
        outs.append(out[0])
    expect_o = ouly.heads_to_sequence([e[0] for e in expect], num_heads=heads)
    for r in range(world):
        recv = torch.stack([outs[s].view(world, tokens, hl, d)[r] for s in range(world)])
        o = torch.empty(tokens, heads, d, dtype=torch.bfloat16, device="cuda")
        unpack_o_recv(recv, o, world=world, tokens=tokens, local_heads=hl, head_dim=d,
                      num_heads=heads)
        assert np.array_equal(o.float().cpu().numpy(), expect_o[r])
    # the FL2AV-named allocating forms of the same two layouts
    from h3sa.ulysses import attention_receive_layout, qkv_send_layout

    send0 = qkv_send_layout(_cuda_bf16(mb[0]), num_heads=heads, head_dim=d, world_size=world)
    padded = torch.zeros_like(sends[0])
    pack_qkv_send(_cuda_bf16(mb[0]), padded, world=world, num_heads=heads, head_dim=d)
    assert torch.equal(send0, padded)
    recv = torch.stack([outs[s].view(world, tokens, hl, d)[0] for s in range(world)])
    assert np.array_equal(attention_receive_layout(recv, num_heads=heads).float().cpu().numpy(),
                          expect_o[0])


def test_kv_copy_rows_index_and_bounds() -> None:
    import h3sa

    rows, heads = 300, 3
    x = torch.randn(rows, heads, 128, device="cuda").bfloat16()
    table = torch.tensor([5, 1, 4], dtype=torch.int32, device="cuda")
    pool = torch.zeros(heads, 6 * 128, 128, dtype=torch.bfloat16, device="cuda")
    idx = torch.randperm(rows)[:200].to(torch.int32).cuda()
    h3sa.kv_copy_rows([x], [pool], count=200, src_index=idx, dst_table=table, dst_start=50)
    back = torch.empty(200, heads, 128, dtype=torch.bfloat16, device="cuda")
    h3sa.kv_copy_rows([pool], [back], count=200, src_table=table, src_start=50)
    assert torch.equal(back, x[idx.long()])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    bad = torch.tensor([0, rows + 5], dtype=torch.int32, device="cuda")
    h3sa.kv_copy_rows([x], [pool], count=2, src_index=bad, dst_table=table, device_error=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 4


@pytest.mark.parametrize("seq,heads,dst_start", [(300, 8, 0), (1000, 24, 130), (37, 3, 1000)])
def test_prologue_scatter_into_cache_matches_oracle(seq: int, heads: int, dst_start: int) -> None:
    """The fused prologue + exchange + cache append on one GPU (world 1): Q rows in the plane,
    K/V rows in the paged pools through a shuffled page table, all bit-exact vs the oracle;
    pool rows outside the chunk untouched."""

    from h3sa.kernels import PAGE_ROWS
    from h3sa.peer import LocalBuffer
    from h3sa.prologue import qkv_norm_rope_scatter_paged

    inp, cs = _prologue_case(seq, heads, seed=5)
    rng = np.random.default_rng(2)
    pos = rng.integers(0, cs.shape[0], seq)
    blocks = (dst_start + seq + PAGE_ROWS - 1) // PAGE_ROWS
    pages = blocks + 3
    table = torch.from_numpy(rng.permutation(pages)[:blocks].astype(np.int32)).cuda()
    fill = 7.0
    kpool = torch.full((heads, pages * PAGE_ROWS, 128), fill, dtype=torch.bfloat16, device="cuda")
    vpool = torch.full_like(kpool, fill)
    q = torch.zeros(seq, heads, 128, dtype=torch.bfloat16, device="cuda")
    raw = _cuda_bf16(inp["qkv"])
    before = raw.clone()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    qkv_norm_rope_scatter_paged(raw, _cuda_bf16(inp["q_weight"]), _cuda_bf16(inp["k_weight"]),
                                _cuda_bf16(cs), torch.from_numpy(pos).cuda(), 1e-5,
                                q=LocalBuffer(q), key_pool=LocalBuffer(kpool),
                                value_pool=LocalBuffer(vpool), page_table=table,
                                dst_start=dst_start, device_error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(raw, before), "the merged input must be left as it was"
    ref = opro.qkv_norm_rope(inp["qkv"], inp["q_weight"], inp["k_weight"], cs, pos, heads, 128,
                             1e-5).reshape(seq, 3, heads, 128)
    assert np.array_equal(q.float().cpu().numpy(), ref[:, 0])
    tab = table.cpu().numpy()
    logical = dst_start + np.arange(seq)
    phys = tab[logical // PAGE_ROWS] * PAGE_ROWS + logical % PAGE_ROWS
    for pool, plane in ((kpool, 1), (vpool, 2)):
        host = pool.float().cpu().numpy()
        assert np.array_equal(host[:, phys].transpose(1, 0, 2), ref[:, plane])
        untouched = np.ones(pool.shape[1], dtype=bool)
        untouched[phys] = False
        assert np.all(host[:, untouched] == fill)


@pytest.mark.parametrize("seq,heads,dst_start,masked,unflagged_only",
                         [(300, 4, 0, False, False), (517, 6, 200, True, False),
                          (517, 6, 200, True, True)])
def test_prologue_scatter_fp8_matches_oracle(seq: int, heads: int, dst_start: int,
                                             masked: bool, unflagged_only: bool) -> None:
    """The fused RMSNorm + RoPE + e4m3 prologue (amax pass, then quantise-and-store) on one GPU:
    the scales and the e4m3 bytes of Q and of the K/V part (through a shuffled page table) are
    the oracle quantiser's on the oracle prologue's rows, the scales covering only the flagged
    rows; the optional bf16 rows equal the bf16 scatter's (only the unflagged ones, the flagged
    ones left untouched, when asked)."""

    from h3sa.kernels import PAGE_ROWS
    from h3sa.peer import LocalBuffer
    from h3sa.prologue import qkv_norm_rope_scatter_fp8
    from oracle import fp8 as ofp8

    inp, cs = _prologue_case(seq, heads, seed=9)
    rng = np.random.default_rng(4)
    pos = rng.integers(0, cs.shape[0], seq)
    flags = np.ones(seq, np.uint8)
    if masked:
        flags[:37] = 0        # e.g. text rows that the media part's scales do not cover
        flags[-11:] = 0
    blocks = (dst_start + seq + PAGE_ROWS - 1) // PAGE_ROWS
    pages = blocks + 2
    table = torch.from_numpy(rng.permutation(pages)[:blocks].astype(np.int32)).cuda()
    k8 = torch.zeros(heads, pages * PAGE_ROWS, 128, dtype=torch.float8_e4m3fn, device="cuda")
    v8 = torch.zeros_like(k8)
    q8 = torch.zeros(seq, heads, 128, dtype=torch.float8_e4m3fn, device="cuda")
    kpool = torch.zeros(heads, pages * PAGE_ROWS, 128, dtype=torch.bfloat16, device="cuda")
    vpool = torch.zeros_like(kpool)
    qbf = torch.zeros(seq, heads, 128, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    qs, ks, vs = qkv_norm_rope_scatter_fp8(
        _cuda_bf16(inp["qkv"]), _cuda_bf16(inp["q_weight"]), _cuda_bf16(inp["k_weight"]),
        _cuda_bf16(cs), torch.from_numpy(pos).cuda(), 1e-5, q8=LocalBuffer(q8),
        key_pool8=LocalBuffer(k8), value_pool8=LocalBuffer(v8), page_table8=table,
        dst8_start=dst_start, amax_rows=torch.from_numpy(flags).cuda(),
        q=LocalBuffer(qbf), key_pool=LocalBuffer(kpool), value_pool=LocalBuffer(vpool),
        page_table=table, dst_start=dst_start, bf16_unflagged_only=unflagged_only,
        device_error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = opro.qkv_norm_rope(inp["qkv"], inp["q_weight"], inp["k_weight"], cs, pos, heads, 128,
                             1e-5).reshape(seq, 3, heads, 128)
    sel = flags.astype(bool)
    bf16_rows = ~sel if unflagged_only else np.ones(seq, dtype=bool)
    host_q = qbf.float().cpu().numpy()
    assert np.array_equal(host_q[bf16_rows], ref[bf16_rows, 0])
    assert np.all(host_q[~bf16_rows] == 0)
    tab = table.cpu().numpy()
    logical = dst_start + np.arange(seq)
    phys = tab[logical // PAGE_ROWS] * PAGE_ROWS + logical % PAGE_ROWS
    for plane, got_scale, rows_of in ((0, qs, lambda: q8.view(torch.uint8).cpu().numpy()),
                                      (1, ks, lambda: k8.view(torch.uint8).cpu().numpy()[:, phys].transpose(1, 0, 2)),
                                      (2, vs, lambda: v8.view(torch.uint8).cpu().numpy()[:, phys].transpose(1, 0, 2))):
        _, scale = ofp8.quantize_fp8_e4m3_per_head(ref[sel, plane][None])
        assert np.array_equal(got_scale.cpu().numpy(), scale[0]), plane
        # every row is quantised with the flagged rows' scales
        y = np.clip(ref[:, plane] / scale[0][None, :, None], -448.0, 448.0).astype(np.float32)
        assert np.array_equal(rows_of(), ofp8.e4m3_encode(y)), plane
    for pool, plane in ((kpool, 1), (vpool, 2)):
        host = pool.float().cpu().numpy()[:, phys].transpose(1, 0, 2)
        assert np.array_equal(host[bf16_rows], ref[bf16_rows, plane])
        assert np.all(host[~bf16_rows] == 0)
