"""W8A8 projection kernels against the oracle, the reference's weight quantiser and vLLM.

* h3sa_quantize_int8_rows: the weight mode bit-exact against the reference's
  _quantize_weight (tests/golden/w8a8.npz) and the oracle; the per-token activation mode
  bit-exact against the oracle and, where vLLM's CUDA ops load, against scaled_int8_quant.
* h3sa_w8a8_gemm (tcgen05 kind::i8): bit-exact against the oracle's exact-integer GEMM and
  scale order on ragged shapes (M, N and K tails, an all-zero row); at the 768p projection
  shape against vLLM's cutlass_scaled_mm (the reference's call) where it loads.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import w8a8 as ow8

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _vllm_ops():
    try:
        import vllm._custom_ops as ops

        ops.scaled_int8_quant(torch.ones(1, 16, device="cuda", dtype=torch.bfloat16))
        return ops
    except Exception:  # noqa: BLE001 - vLLM's CUDA extension is optional on the box
        return None


def test_int8_row_quantisers_bit_exact() -> None:
    from h3sa.w8a8 import quantize_int8_rows, quantize_weight

    g = np.load(GOLDEN / "w8a8.npz")
    w = torch.from_numpy(g["weight"]).bfloat16().cuda()
    q, scale = quantize_weight(w)
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(scale.cpu().numpy(), g["scale"])
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((333, 776)) * 3).astype(np.float32)
    x[7] = 0.0
    x[9, 5] = 1000.0
    xb = torch.from_numpy(x).bfloat16()
    qa, sa = quantize_int8_rows(xb.cuda(), per_token=True)
    rq, rs = ow8.quantize_activation(xb.float().numpy())
    assert np.array_equal(qa.cpu().numpy(), rq) and np.array_equal(sa.cpu().numpy(), rs)
    ops = _vllm_ops()
    if ops is not None:
        vq, vs, _ = ops.scaled_int8_quant(xb.cuda())
        assert torch.equal(vq, qa) and torch.equal(vs.reshape(-1), sa.reshape(-1))


@pytest.mark.parametrize("m,n,k", [(300, 520, 640), (128, 256, 128), (1, 8, 16), (257, 1032, 1296)])
def test_w8a8_gemm_bit_exact_vs_oracle(m: int, n: int, k: int) -> None:
    from h3sa.w8a8 import w8a8_gemm

    rng = np.random.default_rng(m * 7 + n)
    qa = rng.integers(-128, 128, (m, k), dtype=np.int64).astype(np.int8)
    qb = rng.integers(-127, 128, (n, k), dtype=np.int64).astype(np.int8)
    if m > 3:
        qa[3] = 0
    sa = (rng.random((m, 1)) * 0.02 + 1e-4).astype(np.float32)
    sb = (rng.random((n, 1)) * 0.01 + 1e-4).astype(np.float32)
    out = w8a8_gemm(torch.from_numpy(qa).cuda(), torch.from_numpy(sa).cuda(),
                    torch.from_numpy(qb).cuda(), torch.from_numpy(sb).cuda())
    ref = ow8.scaled_mm(qa, sa, qb, sb)
    assert np.array_equal(out.float().cpu().numpy(), ref)


def test_w8a8_linear_projection_shape() -> None:
    """The 768p SP=8 QKV projection shape (1568 tokens x 5376 -> 9216): the drop-in
    cutlass_w8a8_linear against the oracle on sampled rows, and against vLLM's own
    scaled_int8_quant + cutlass_scaled_mm (the reference's path) where it loads."""

    from h3sa.w8a8 import cutlass_w8a8_linear, quantize_int8_rows, quantize_weight

    gen = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(1568, 5376, device="cuda", generator=gen).bfloat16()
    w = (torch.randn(9216, 5376, device="cuda", generator=gen) * 0.02).bfloat16()
    wq, ws = quantize_weight(w)
    out = cutlass_w8a8_linear(x, wq, ws, bias=None, workspace=None, weight_t=None,
                              weight_scale_t=None)
    qa, sa = quantize_int8_rows(x)
    rows = torch.arange(0, 1568, 97)
    ref = ow8.scaled_mm(qa[rows].cpu().numpy(), sa[rows].cpu().numpy(), wq.cpu().numpy(),
                        ws.cpu().numpy())
    assert np.array_equal(out[rows].float().cpu().numpy(), ref)
    ops = _vllm_ops()
    if ops is not None:
        vq, vs, _ = ops.scaled_int8_quant(x)
        assert torch.equal(vq, qa) and torch.equal(vs.reshape(-1), sa.reshape(-1))
        try:
            vout = ops.cutlass_scaled_mm(vq, wq.t(), vs, ws.t(), torch.bfloat16)
        except RuntimeError as exc:
            # vLLM's CUTLASS build refuses int8 on SM100 ("Int8 not supported on SM100"): the
            # reference's own W8A8 projection cannot run on B200 at all
            assert "not supported" in str(exc)
            return
        diff = (vout.float() - out.float()).abs()
        # the same products and scales; an epilogue that multiplies in another order differs
        # by at most one bf16 rounding
        assert float((diff / out.float().abs().clamp_min(1e-30)).max()) <= 2 ** -7
