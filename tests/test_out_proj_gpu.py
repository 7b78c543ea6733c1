"""The row-parallel out_proj (bf16 tcgen05 GEMM) and its fused TP reduce.

* gemm_bf16 against the oracle's fp64 product rounded to bf16 (the fp32 tensor-core
  accumulation agrees up to one bf16 rounding) on ragged shapes;
* the GEMM's partial-slot epilogue plus tp_reduce on one GPU equals the plain GEMM bit for bit;
* tp_reduce bit-exact against the oracle (fp32 sum in rank order, one rounding);
* on two GPUs (TP=2): PeerRowParallelLinear (partials stored into the peers' slots by the GEMM
  epilogue, one peer barrier, reduce) is bit-identical to the same GEMM + NCCL all-reduce
  (the reference's structure) and within bf16 rounding of the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import out_proj as oop

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _close_bf16(got: np.ndarray, ref: np.ndarray, abs_sum: np.ndarray, k: int) -> None:
    """Within one bf16 step of the oracle plus the fp32 accumulation bound k * 2^-24 * sum|a b|
    (results that cancel to near zero carry the accumulation error of their large terms;
    cuBLAS on the same inputs shows the same elements)."""

    # bf16 step of the larger of the two values (a pair may straddle a power of two)
    ulp = np.spacing(np.maximum(np.abs(ref), np.abs(got)).astype(np.float32)) * 65536.0
    bound = ulp + k * 2.0 ** -24 * abs_sum
    bad = np.abs(got - ref) > bound
    assert not bad.any(), (int(bad.sum()), float(np.abs(got - ref).max()))
    assert np.mean(got == ref) > 0.99


@pytest.mark.parametrize("m,n,k", [(300, 520, 640), (128, 256, 64), (1, 8, 8), (1568, 5376, 1536)])
def test_gemm_bf16_vs_oracle(m: int, n: int, k: int) -> None:
    from h3sa.linear import gemm_bf16

    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
    b = (torch.randn(n, k, device="cuda", generator=gen) * 0.05).bfloat16()
    out = gemm_bf16(a, b)
    rows = slice(None) if m < 1000 else slice(0, m, 41)
    a_np, b_np = a[rows].float().cpu().numpy(), b.float().cpu().numpy()
    ref = oop.local_product(a_np, b_np)
    abs_sum = np.abs(a_np).astype(np.float64) @ np.abs(b_np).astype(np.float64).T
    _close_bf16(out[rows].float().cpu().numpy(), ref, abs_sum, k)


def test_partial_slots_and_reduce_on_one_gpu() -> None:
    from h3sa.linear import gemm_bf16, tp_reduce

    gen = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(200, 320, device="cuda", generator=gen).bfloat16()
    b = (torch.randn(264, 320, device="cuda", generator=gen) * 0.05).bfloat16()
    plain = gemm_bf16(a, b)
    slots = torch.full((1, 200, 264), float("nan"), dtype=torch.bfloat16, device="cuda")
    table = torch.tensor([slots.data_ptr()], dtype=torch.int64, device="cuda")
    gemm_bf16(a, b, None, partial_peers=table, ranks=1, slot=0)
    assert torch.equal(slots[0], plain)
    assert torch.equal(tp_reduce(slots), plain)
    three = (torch.randn(3, 77, 136, device="cuda", generator=gen) * 4).bfloat16()
    ref = oop.tp_reduce([t.float().cpu().numpy() for t in three])
    assert np.array_equal(tp_reduce(three).float().cpu().numpy(), ref)


def _tp2_worker(rank: int, world: int, rendezvous: str) -> None:
    import datetime

    sys.path.insert(0, str(ROOT / "taomate-h3_b200"))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.distributed.init_process_group("nccl", init_method=f"file://{rendezvous}", rank=rank,
                                         world_size=world, timeout=datetime.timedelta(seconds=60),
                                         device_id=dev)
    try:
        from h3sa.linear import PeerRowParallelLinear, row_parallel_linear

        rows, inner, hidden = 1568, 3072, 5376
        loc = inner // world
        g = torch.Generator(device=dev).manual_seed(10 + rank)
        x = torch.randn(rows, loc, device=dev, generator=g).bfloat16()
        gw = torch.Generator(device=dev).manual_seed(5)  # the full weight, same on every rank
        w_full = (torch.randn(hidden, inner, device=dev, generator=gw) * 0.02).bfloat16()
        w = w_full[:, rank * loc:(rank + 1) * loc].contiguous()
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        fused = PeerRowParallelLinear(w, rows, device_error=err)
        for it in range(3):  # both partial sets, then the first again
            got = fused(x)
            ref = row_parallel_linear(x, w, group=torch.distributed.group.WORLD)
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            assert torch.equal(got, ref), it
        xs = [torch.empty_like(x) for _ in range(world)]
        torch.distributed.all_gather(xs, x)
        sample = slice(0, rows, 53)
        want = oop.row_parallel([t[sample].float().cpu().numpy() for t in xs],
                                [w_full[:, r * loc:(r + 1) * loc].float().cpu().numpy()
                                 for r in range(world)])
        g_np = got[sample].float().cpu().numpy()
        # each partial may round one bf16 step apart from the oracle's; the sum stays close
        assert float(np.linalg.norm(g_np - want) / np.linalg.norm(want)) <= 5e-3
        torch.distributed.barrier()
        torch.cuda.synchronize()
        fused.close()
    finally:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def test_fused_tp2_out_proj_matches_nccl_all_reduce(tmp_path: Path) -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_tp2_worker, args=(2, str(tmp_path / "rendezvous")), nprocs=2, join=True)
