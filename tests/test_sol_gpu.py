"""Rectangular SOL-Attn (``h3sa_sol_attention``) against the CPU oracle.

The oracle (oracle/sol_attention.py) is pinned to the reference adapter run by Triton's CPU
interpreter (tests/test_oracle_golden.py). On the GPU:

* routing: the exact-block bitmask equals the oracle's except for decisions whose margin
  (mean proxy score - threshold, log2 units) is within 2e-3 of zero, where fp32 summation
  order may decide; the telemetry counts are the mask's;
* output: the oracle evaluated on the GPU's routing, rel-L2 <= 1e-2 (bf16 output, bf16
  probabilities in P V) and max error <= 2e-2 x the output's max;
* edges: a sink covering every key block is dense attention; a threshold nothing passes makes
  every block approximate; one query row; one key row; a partial last key block.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))

from inputs import SOL_CASES, sol_inputs  # noqa: E402

from oracle import sol_attention as osol  # noqa: E402

pytestmark = pytest.mark.gpu
SCALE = 128 ** -0.5


def _unpack(mask: torch.Tensor, kb: int) -> np.ndarray:
    """int32 [H, QB, words] -> bool [QB, H, KB]."""

    words = mask.cpu().numpy().view(np.uint32)
    bits = np.unpackbits(words.view(np.uint8), bitorder="little").reshape(*words.shape[:2], -1)
    return bits[:, :, :kb].astype(bool).transpose(1, 0, 2)


def _run(q: np.ndarray, k: np.ndarray, v: np.ndarray, tau: float, sink: int):
    from h3sa.sol_attention import sol_attn_rectangular

    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).cuda()  # noqa: E731
    nq, heads = q.shape[:2]
    kb = (k.shape[0] + 63) // 64
    mask = torch.full((heads, (nq + 63) // 64, (kb + 31) // 32), -1, dtype=torch.int32, device="cuda")
    tele = torch.zeros(4, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = sol_attn_rectangular(dev(q), dev(k), dev(v), scale=SCALE, tau=tau, sink_tokens=sink,
                               telemetry_counts=tele, exact_blocks=mask, device_error=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.float().cpu(), _unpack(mask, kb), tele.cpu().tolist()


def _check(q, k, v, tau, sink, *, max_flips: int = 0) -> np.ndarray:
    out, got_exact, tele = _run(q, k, v, tau, sink)
    tq, tk, tv = (torch.from_numpy(a) for a in (q, k, v))
    _, want_exact, margin, _ = osol.sol_attn_rectangular(tq, tk, tv, scale=SCALE, tau=tau,
                                                         sink_tokens=sink)
    flips = got_exact != want_exact.numpy()
    assert flips.sum() <= max_flips, int(flips.sum())
    assert np.all(np.abs(margin.numpy()[flips]) < 2e-3), margin.numpy()[flips]
    kb = got_exact.shape[2]
    sink_blocks = min(kb, (sink + 63) // 64)
    sel = got_exact[:, :, sink_blocks:].sum()
    cells = got_exact.shape[0] * got_exact.shape[1]
    assert tele == [int(sel), int(got_exact.sum()), cells * (kb - sink_blocks), cells * kb]
    ref, _, _, _ = osol.sol_attn_rectangular(tq, tk, tv, scale=SCALE, tau=tau, sink_tokens=sink,
                                             exact=torch.from_numpy(got_exact))
    err = (out - ref).norm() / ref.norm()
    assert err <= 1e-2, float(err)
    assert float((out - ref).abs().max()) <= 2e-2 * float(ref.abs().max())
    return got_exact


@pytest.mark.parametrize("case", range(len(SOL_CASES)))
def test_sol_matches_oracle_on_golden_cases(case: int) -> None:
    _, _, _, tau, sink = SOL_CASES[case]
    q, k, v = sol_inputs(case)
    exact = _check(q, k, v, tau, sink)
    assert exact.any() and not exact.all()  # some blocks approximate, some exact


def test_sol_larger_ragged() -> None:
    """More query tiles than query blocks pair up evenly (an odd query block count), 83 key
    blocks with a partial last one, three heads, a sink that ends inside a block."""

    rng = np.random.default_rng(21)
    nq, nk, heads = 1000, 5260, 3
    kb = (nk + 63) // 64
    centre = rng.standard_normal((kb, heads, 128)).astype(np.float32)
    k = 0.6 * rng.standard_normal((nk, heads, 128)).astype(np.float32)
    k += np.repeat(centre, 64, axis=0)[:nk]
    q = rng.standard_normal((nq, heads, 128)).astype(np.float32)
    v = rng.standard_normal((nk, heads, 128)).astype(np.float32)
    q, k, v = (torch.from_numpy(a).to(torch.bfloat16).float().numpy() for a in (q, k, v))
    exact = _check(q, k, v, 0.25, 1300, max_flips=4)
    assert exact[:, :, :21].all()  # the 21 sink blocks


def test_sol_full_sink_is_dense_attention() -> None:
    q, k, v = sol_inputs(0)
    out, exact, _ = _run(q, k, v, 0.5, k.shape[0])
    assert exact.all()
    tq, tk, tv = (torch.from_numpy(a) for a in (q, k, v))
    p = torch.softmax(torch.einsum("qhd,khd->hqk", tq, tk) * SCALE, -1)
    ref = torch.einsum("hqk,khd->qhd", p, tv)
    assert float((out - ref).norm() / ref.norm()) <= 1e-2


def test_sol_all_approximate() -> None:
    """tau so large that no block is routed and no sink: every block through its centroid."""

    q, k, v = sol_inputs(1)
    _, exact, tele = _run(q, k, v, 1e4, 0)
    assert not exact.any() and tele[0] == 0 and tele[1] == 0
    _check(q, k, v, 1e4, 0)


@pytest.mark.parametrize("nq,nk", [(1, 700), (150, 1), (64, 64)])
def test_sol_tiny_shapes(nq: int, nk: int) -> None:
    rng = np.random.default_rng(nq * 7 + nk)
    q, k, v = (torch.from_numpy(rng.standard_normal((n, 2, 128)).astype(np.float32))
               .to(torch.bfloat16).float().numpy() for n in (nq, nk, nk))
    _check(q, k, v, 0.0, 0, max_flips=1)


def test_sol_rejects_bad_arguments() -> None:
    from h3sa.sol_attention import sol_attn_rectangular

    q = torch.zeros(10, 2, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(4096 * 64 + 1, 2, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="exceed"):
        sol_attn_rectangular(q, k, k, scale=SCALE, tau=1.0, sink_tokens=0)
    with pytest.raises(RuntimeError, match="heads"):
        sol_attn_rectangular(q, k[:100, :1], k[:100, :1], scale=SCALE, tau=1.0, sink_tokens=0)
    with pytest.raises(RuntimeError, match="tau"):
        sol_attn_rectangular(q, k[:100], k[:100], scale=SCALE, tau=math.nan, sink_tokens=0)
