"""The N > 1 exchange on two CPU ranks (gloo): the oracle's every-rank emulation of the
Ulysses all-to-all equals a real all_to_all_single of its send layouts, and the Ulysses
entry points validate their arguments under a live process group like the reference."""

from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _worker(rank: int, world: int, rendezvous: str, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "taomate-h3_b200"))
    from h3sa.ulysses import ParallelContext, merged_qkv_sequence_to_heads

    from oracle import ulysses as ouly

    dist.init_process_group("gloo", init_method=f"file://{rendezvous}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    tokens, heads, d = 5, 4, 8
    merged = [np.random.default_rng(50 + r).standard_normal((tokens, 3 * heads * d)).astype(np.float32)
              for r in range(world)]
    hl = heads // world
    send = torch.from_numpy(merged[rank].reshape(tokens, 3, world, hl, d)
                            .transpose(2, 1, 0, 3, 4).copy())
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)
    got = recv.permute(1, 0, 2, 3, 4).reshape(3, world * tokens, hl, d).numpy()
    expect = ouly.merged_qkv_sequence_to_heads(merged, heads, d)[rank]
    ok = all(np.array_equal(got[i], expect[i]) for i in range(3))
    # 3 heads over the ranks: zero-padded shards of ceil(3 / W) heads
    ph = 3
    pm = [np.random.default_rng(70 + r).standard_normal((tokens, 3 * ph * d)).astype(np.float32)
          for r in range(world)]
    phl = -(-ph // world)
    padded = np.zeros((tokens, 3, world * phl, d), np.float32)
    padded[:, :, :ph] = pm[rank].reshape(tokens, 3, ph, d)
    psend = torch.from_numpy(padded.reshape(tokens, 3, world, phl, d).transpose(2, 1, 0, 3, 4).copy())
    precv = torch.empty_like(psend)
    dist.all_to_all_single(precv, psend)
    pgot = precv.permute(1, 0, 2, 3, 4).reshape(3, world * tokens, phl, d).numpy()
    pexpect = ouly.merged_qkv_sequence_to_heads(pm, ph, d)[rank]
    ok = ok and all(np.array_equal(pgot[i], pexpect[i]) for i in range(3))
    # argument validation happens before any device work, under the live group
    ctx = ParallelContext(1, 0, world, rank, dist.group.WORLD, dist.group.WORLD)
    msg = ""
    try:
        merged_qkv_sequence_to_heads(torch.zeros(tokens, 7), num_heads=3, head_dim=d, context=ctx)
    except ValueError as exc:
        msg += "|" + str(exc)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([ok, t.item() == world], dtype=bool))
    with open(os.path.join(out_dir, f"m{rank}.txt"), "w") as f:
        f.write(msg)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_exchange_and_validation(tmp_path: Path) -> None:
    # file rendezvous: no port to race for
    mp.start_processes(_worker, args=(2, str(tmp_path / "rendezvous"), str(tmp_path)), nprocs=2,
                       start_method="spawn")
    for r in range(2):
        assert np.load(tmp_path / f"r{r}.npy").all()
        msg = (tmp_path / f"m{r}.txt").read_text()
        assert "merged QKV width differs" in msg


def _tp_sp_worker(rank: int, world: int, rendezvous: str, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "taomate-h3_b200"))
    from h3sa.ulysses import build_parallel_context

    from oracle import ulysses as ouly

    dist.init_process_group("gloo", init_method=f"file://{rendezvous}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    ctx = build_parallel_context(2, 2)
    ok = (ctx.tp_rank == rank % 2 and ctx.ulysses_rank == rank // 2
          and dist.get_process_group_ranks(ctx.tp_group) == [2 * (rank // 2), 2 * (rank // 2) + 1]
          and dist.get_process_group_ranks(ctx.ulysses_group) == [rank % 2, rank % 2 + 2])
    # the sequence -> heads exchange of this TP rank's 4 heads inside its Ulysses group only
    tokens, heads, d = 5, 4, 8
    sp = ctx.ulysses_world_size
    merged = {r: np.random.default_rng(90 + r).standard_normal((tokens, 3 * heads * d))
              .astype(np.float32) for r in range(world)}
    members = [rank % 2 + 2 * u for u in range(sp)]
    hl = heads // sp
    send = torch.from_numpy(merged[rank].reshape(tokens, 3, sp, hl, d)
                            .transpose(2, 1, 0, 3, 4).copy())
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=ctx.ulysses_group)
    got = recv.permute(1, 0, 2, 3, 4).reshape(3, sp * tokens, hl, d).numpy()
    expect = ouly.merged_qkv_sequence_to_heads([merged[m] for m in members], heads, d)[ctx.ulysses_rank]
    ok = ok and all(np.array_equal(got[i], expect[i]) for i in range(3))
    np.save(os.path.join(out_dir, f"tp{rank}.npy"), np.array([ok], dtype=bool))
    dist.barrier()
    dist.destroy_process_group()


def test_tp2_sp2_groups_follow_reference_layout(tmp_path: Path) -> None:
    """build_parallel_context on four CPU ranks: TP groups {0,1}, {2,3}, Ulysses groups
    {0,2}, {1,3} (T/runtime/direct.py:169-190), and each Ulysses group's exchange equals the
    oracle's over that group's members."""

    mp.start_processes(_tp_sp_worker, args=(4, str(tmp_path / "rendezvous"), str(tmp_path)),
                       nprocs=4, start_method="spawn")
    for r in range(4):
        assert np.load(tmp_path / f"tp{r}.npy").all(), r
