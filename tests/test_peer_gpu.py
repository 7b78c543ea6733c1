"""Fused Ulysses exchanges over peer memory against the NCCL all-to-all path (2+ GPUs).

Two ranks, one process per GPU (NCCL). Each rank holds a seeded post-prologue QKV shard;
the NCCL path (pack, all_to_all_single, unpack / attention / all_to_all_single, unpack) and
the fused path (scatter_qkv into peer q/k/v planes / attention storing into peer output
shards) must give bit-identical q/k/v planes and final outputs: both run the same kernels and
differ only in where the bytes go. scatter_qkv_paged, which writes K/V straight into the
owners' paged caches, must leave the same caches as the all-to-all plus kv_copy_rows. Skipped
with fewer than two GPUs.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _worker(rank: int, world: int, rendezvous: str) -> None:
    import datetime

    sys.path.insert(0, str(ROOT / "taomate-h3_b200"))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # file rendezvous: no port to race for
    torch.distributed.init_process_group("nccl", init_method=f"file://{rendezvous}", rank=rank,
                                         world_size=world, timeout=datetime.timedelta(seconds=60),
                                         device_id=dev)
    try:
        import h3sa
        from h3sa.kernels import PAGE_ROWS
        from h3sa.peer import PeerBarrier, PeerBuffer, attention_fwd_scatter, barrier, scatter_qkv
        from h3sa.ulysses import pack_qkv_send, unpack_o_recv, unpack_qkv_recv

        heads, d, tokens, hist = 4, 128, 300, 256
        hl, rows = heads // world, tokens * world
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        merged = torch.randn(tokens, 3 * heads * d, device=dev, generator=g).to(torch.bfloat16)
        hist_kv = torch.randn(hist, hl, d, device=dev,
                              generator=torch.Generator(device=dev).manual_seed(7 + rank)).to(torch.bfloat16)
        pages = (hist + rows + PAGE_ROWS - 1) // PAGE_ROWS
        table = torch.arange(pages, dtype=torch.int32, device=dev)
        scale = d ** -0.5
        probs = [h3sa.AttentionProblem(0, rows - 20, 0, hist + rows - 20),
                 h3sa.AttentionProblem(rows - 20, rows, hist + rows - 20, hist + rows)]

        def pools():
            kp = torch.zeros(hl, pages * PAGE_ROWS, d, dtype=torch.bfloat16, device=dev)
            vp = torch.zeros_like(kp)
            h3sa.kv_copy_rows([hist_kv, hist_kv], [kp, vp], count=hist, dst_table=table)
            return kp, vp

        # NCCL path
        send = torch.empty(world, 3, tokens, hl, d, dtype=torch.bfloat16, device=dev)
        recv = torch.empty_like(send)
        qkv_ref = torch.empty(3, rows, hl, d, dtype=torch.bfloat16, device=dev)
        pack_qkv_send(merged, send, world=world, num_heads=heads, head_dim=d)
        torch.distributed.all_to_all_single(recv, send)
        unpack_qkv_recv(recv, qkv_ref, world=world, tokens=tokens, local_heads=hl, head_dim=d)
        kp, vp = pools()
        h3sa.kv_copy_rows([qkv_ref[1], qkv_ref[2]], [kp, vp], count=rows, dst_table=table,
                          dst_start=hist)
        out = torch.empty(rows, hl, d, dtype=torch.bfloat16, device=dev)
        h3sa.attention_fwd(qkv_ref[0], out, kp, vp, table, probs, scale)
        orecv = torch.empty(world, tokens, hl, d, dtype=torch.bfloat16, device=dev)
        final_ref = torch.empty(tokens, heads, d, dtype=torch.bfloat16, device=dev)
        torch.distributed.all_to_all_single(orecv, out)
        unpack_o_recv(orecv, final_ref, world=world, tokens=tokens, local_heads=hl, head_dim=d)

        # fused path, twice (the second run overwrites buffers the first one filled)
        qkv_peer = PeerBuffer((3, rows, hl, d))
        out_peer = PeerBuffer((tokens, heads, d))
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        peer_barrier = PeerBarrier(device_error=err)
        for it in range(3):
            # the NCCL barrier and the peer-memory barrier order the same way
            sync = barrier if it == 0 else peer_barrier
            qkv_peer.tensor.zero_()
            out_peer.tensor.zero_()
            sync()
            scatter_qkv(merged, qkv_peer, num_heads=heads, head_dim=d)
            sync()
            assert torch.equal(qkv_peer.tensor, qkv_ref), "q/k/v planes differ"
            kp2, vp2 = pools()
            h3sa.kv_copy_rows([qkv_peer.tensor[1], qkv_peer.tensor[2]], [kp2, vp2], count=rows,
                              dst_table=table, dst_start=hist)
            attention_fwd_scatter(qkv_peer.tensor[0], kp2, vp2, table, probs, scale, out_peer,
                                  device_error=err)
            sync()
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            assert torch.equal(out_peer.tensor, final_ref), "final sequence shards differ"
        # Q to the owners' planes and K/V straight into the owners' paged caches
        from h3sa.peer import scatter_qkv_paged

        kp_ref, vp_ref = pools()
        h3sa.kv_copy_rows([qkv_ref[1], qkv_ref[2]], [kp_ref, vp_ref], count=rows, dst_table=table,
                          dst_start=hist)
        q_peer = PeerBuffer((rows, hl, d))
        k_peer = PeerBuffer((hl, pages * PAGE_ROWS, d))
        v_peer = PeerBuffer((hl, pages * PAGE_ROWS, d))
        for it in range(2):
            q_peer.tensor.zero_()
            kp3, vp3 = pools()
            k_peer.tensor.copy_(kp3)
            v_peer.tensor.copy_(vp3)
            peer_barrier()
            scatter_qkv_paged(merged, q_peer, k_peer, v_peer, table, dst_start=hist,
                              num_heads=heads, head_dim=d, device_error=err)
            peer_barrier()
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            assert torch.equal(q_peer.tensor, qkv_ref[0]), "q plane differs"
            assert torch.equal(k_peer.tensor, kp_ref), "key cache differs"
            assert torch.equal(v_peer.tensor, vp_ref), "value cache differs"
        # the prologue fused into the same exchange, from the raw projection: the same planes
        # and caches as the in-place prologue followed by scatter_qkv_paged
        from h3sa.prologue import fused_qkv_qk_norm_rope_, qkv_norm_rope_scatter_paged

        gp = torch.Generator(device=dev).manual_seed(55)  # same on every rank
        wq = (1 + 0.1 * torch.randn(d, device=dev, generator=gp)).to(torch.bfloat16)
        wk = (1 + 0.1 * torch.randn(d, device=dev, generator=gp)).to(torch.bfloat16)
        cos_sin = torch.randn(4096, 96, device=dev, generator=gp).to(torch.bfloat16)
        positions = torch.randint(0, 4096, (tokens,), device=dev, generator=g)
        post = merged.clone()
        fused_qkv_qk_norm_rope_(post, wq, wk, cos_sin, positions, 1e-5)
        kp_ref, vp_ref = pools()
        k_peer.tensor.copy_(kp_ref)
        v_peer.tensor.copy_(vp_ref)
        peer_barrier()
        scatter_qkv_paged(post, q_peer, k_peer, v_peer, table, dst_start=hist, num_heads=heads,
                          head_dim=d, device_error=err)
        peer_barrier()
        q_ref2, k_ref2, v_ref2 = (b.tensor.clone() for b in (q_peer, k_peer, v_peer))
        for it in range(2):
            q_peer.tensor.zero_()
            k_peer.tensor.copy_(kp_ref)
            v_peer.tensor.copy_(vp_ref)
            peer_barrier()
            qkv_norm_rope_scatter_paged(merged, wq, wk, cos_sin, positions, 1e-5, q=q_peer,
                                        key_pool=k_peer, value_pool=v_peer, page_table=table,
                                        dst_start=hist, device_error=err)
            peer_barrier()
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            assert torch.equal(q_peer.tensor, q_ref2), "fused prologue: q plane differs"
            assert torch.equal(k_peer.tensor, k_ref2), "fused prologue: key cache differs"
            assert torch.equal(v_peer.tensor, v_ref2), "fused prologue: value cache differs"
        # the e4m3 form: scales over the whole chunk (every rank's rows, maxima reduced over the
        # group), Q and the chunk's K/V as e4m3 into the owners' plane and caches
        from h3sa.prologue import qkv_norm_rope_scatter_fp8
        from oracle import fp8 as ofp8

        q8_peer = PeerBuffer((rows, hl, d // 2))
        k8_peer = PeerBuffer((hl, pages * PAGE_ROWS, d // 2))
        v8_peer = PeerBuffer((hl, pages * PAGE_ROWS, d // 2))
        for buf in (q8_peer, k8_peer, v8_peer):
            buf.tensor.zero_()
        peer_barrier()
        scales = qkv_norm_rope_scatter_fp8(merged, wq, wk, cos_sin, positions, 1e-5, q8=q8_peer,
                                           key_pool8=k8_peer, value_pool8=v8_peer,
                                           page_table8=table, dst8_start=hist, device_error=err)
        peer_barrier()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        chunk = slice(hist, hist + rows)
        for plane, ref_rows, buf in ((0, q_ref2, q8_peer),
                                     (1, k_ref2[:, chunk].transpose(0, 1), k8_peer),
                                     (2, v_ref2[:, chunk].transpose(0, 1), v8_peer)):
            want, scale = ofp8.quantize_fp8_e4m3_per_head(ref_rows.float().cpu().numpy()[None])
            assert np.array_equal(scales[plane].cpu().numpy(), scale[0]), plane
            got = buf.tensor.view(torch.uint8)
            if plane:
                got = got[:, chunk].transpose(0, 1)
            assert np.array_equal(got.cpu().numpy(), want[0]), plane
        # the group maximum over peer memory instead of NCCL, three calls (both slot sets and
        # a reuse): the same scales and bytes
        from h3sa.peer import PeerGroupMax

        group_max = PeerGroupMax(3 * heads, device_error=err)
        first = [b.tensor.clone() for b in (q8_peer, k8_peer, v8_peer)]
        for _ in range(3):
            for buf in (q8_peer, k8_peer, v8_peer):
                buf.tensor.zero_()
            peer_barrier()
            again = qkv_norm_rope_scatter_fp8(merged, wq, wk, cos_sin, positions, 1e-5,
                                              q8=q8_peer, key_pool8=k8_peer, value_pool8=v8_peer,
                                              page_table8=table, dst8_start=hist,
                                              peer_max=group_max, device_error=err)
            peer_barrier()
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            for a, b in zip(scales, again):
                assert torch.equal(a, b), "peer group max: scales differ"
            for a, b in zip(first, (q8_peer, k8_peer, v8_peer)):
                assert torch.equal(a, b.tensor), "peer group max: e4m3 bytes differ"
        barrier()
        torch.cuda.synchronize()
        for buf in (qkv_peer, out_peer, q_peer, k_peer, v_peer, q8_peer, k8_peer, v8_peer):
            buf.close()
        group_max.close()
        peer_barrier.close()
    finally:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def test_fused_exchanges_match_nccl_path(tmp_path: Path) -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, str(tmp_path / "rendezvous")), nprocs=2, join=True)
