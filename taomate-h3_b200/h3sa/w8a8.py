"""W8A8 projections on the sm_100a tensor cores (the reference's T/inference/w8a8.py).

The reference quantises the interior QKV / FC1 weights once to int8 with one scale per output
row (``_quantize_weight``, :56-63), quantises each call's activations per token
(vLLM ``scaled_int8_quant``) and multiplies with vLLM's CUTLASS ``cutlass_scaled_mm`` into bf16
(``cutlass_w8a8_linear``, :190-221). Here both quantisers and the GEMM are this library's own
kernels (``h3sa_quantize_int8_rows``, ``h3sa_w8a8_gemm``: tcgen05 kind::i8 with TMEM
accumulators), with the same call signature, so the projection in front of the attention
prologue runs without vLLM.
"""

from __future__ import annotations

import torch

from ._lib import call, ptr, stream_handle


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("W8A8 tensors must be CUDA tensors")


def quantize_int8_rows(x: torch.Tensor, *, per_token: bool = True,
                       stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``[rows, cols]`` -> (int8 ``[rows, cols]``, fp32 ``[rows, 1]``): the dynamic
    per-token activation quantiser (``per_token=True``) or the per-row weight quantiser."""

    _require_cuda(x)
    if x.ndim != 2 or x.dtype != torch.bfloat16:
        raise RuntimeError("quantize_int8_rows takes a bf16 [rows, cols] tensor")
    x = x.contiguous()
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    scale = torch.empty(int(x.shape[0]), 1, dtype=torch.float32, device=x.device)
    call("h3sa_quantize_int8_rows", ptr(x), ptr(q), ptr(scale), int(x.shape[0]), int(x.shape[1]),
         0 if per_token else 1, stream_handle(stream))
    return q, scale


def quantize_weight(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's ``_quantize_weight`` (T/inference/w8a8.py:56-63): int8 weight with one
    fp32 scale per output row, ``[N, 1]``."""

    return quantize_int8_rows(weight, per_token=False)


def w8a8_gemm(a: torch.Tensor, a_scale: torch.Tensor, b: torch.Tensor, b_scale: torch.Tensor,
              out: torch.Tensor | None = None, *, device_error: torch.Tensor | None = None,
              stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """bf16 ``[M, N]`` = a_scale * (b_scale * (a int8 ``[M, K]`` @ b int8 ``[N, K]``^T))."""

    _require_cuda(a, a_scale, b, b_scale, out, device_error)
    if a.dtype != torch.int8 or b.dtype != torch.int8 or a.ndim != 2 or b.ndim != 2:
        raise RuntimeError("w8a8_gemm takes int8 [M, K] activations and int8 [N, K] weights")
    m, k = (int(s) for s in a.shape)
    n = int(b.shape[0])
    if int(b.shape[1]) != k:
        raise RuntimeError(f"w8a8_gemm: K differs ({k} vs {int(b.shape[1])})")
    a_scale = a_scale.reshape(-1).contiguous()
    b_scale = b_scale.reshape(-1).contiguous()
    if (a_scale.dtype != torch.float32 or b_scale.dtype != torch.float32
            or a_scale.numel() != m or b_scale.numel() != n):
        raise RuntimeError("w8a8_gemm scales must be float32 with one value per row")
    a, b = a.contiguous(), b.contiguous()
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    if out.dtype != torch.bfloat16 or out.ndim != 2 or int(out.shape[0]) != m \
            or int(out.shape[1]) < n or out.stride(1) != 1:
        raise RuntimeError("w8a8_gemm output must be bf16 [M, >= N] with unit column stride")
    call("h3sa_w8a8_gemm", ptr(a), ptr(a_scale), ptr(b), ptr(b_scale), ptr(out), m, n, k,
         int(out.stride(0)), ptr(device_error), stream_handle(stream))
    return out


def cutlass_w8a8_linear(inputs: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                        *, bias: torch.Tensor | None = None, workspace=None,
                        weight_t: torch.Tensor | None = None,
                        weight_scale_t: torch.Tensor | None = None) -> torch.Tensor:
    """Drop-in for the reference's ``cutlass_w8a8_linear`` (T/inference/w8a8.py:190-221):
    ``inputs`` bf16 ``[..., K]``, ``weight`` int8 ``[N, K]``, ``weight_scale`` fp32 ``[N, 1]``;
    returns bf16 ``[..., N]``. ``workspace`` / ``weight_t`` / ``weight_scale_t`` are accepted
    for signature compatibility (the kernel reads the weight K-major as stored)."""

    del workspace, weight_t, weight_scale_t
    if bias is not None:
        raise RuntimeError("H3 W8A8 supports bias-free linears only")
    shape = (*inputs.shape[:-1], int(weight.shape[0]))
    flat = inputs.reshape(-1, int(inputs.shape[-1])).contiguous()
    q, scale = quantize_int8_rows(flat, per_token=True)
    return w8a8_gemm(q, scale, weight, weight_scale).reshape(shape)


__all__ = ["cutlass_w8a8_linear", "quantize_int8_rows", "quantize_weight", "w8a8_gemm"]
