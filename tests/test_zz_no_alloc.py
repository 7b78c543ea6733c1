"""The allocation-free quantiser entry point against the allocating one, through the C ABI.

h3sa_quantize_fp8_per_head_noalloc keeps its partial maxima in a fixed device array that
every call shares, so this file runs it twice in a row with different shapes (the second call
sees the first call's leftovers) and checks both results against h3sa_quantize_fp8_per_head
bit for bit: the quantiser is exact, so the tolerance is zero.
"""

from __future__ import annotations

import pytest
import torch

NOALLOC_SLOTS = 65536  # partial maxima the fixed scratch holds


def _lib():
    from h3sa import _lib

    return _lib


def _quantise(entry: str, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib()
    b, s, h, d = (int(v) for v in x.shape)
    y = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    scale = torch.full((b, h), float("nan"), dtype=torch.float32, device=x.device)
    rc = getattr(lib.LIB, entry)(lib.ptr(x), lib.ptr(y), lib.ptr(scale), b, s, h, d,
                                 lib.stream_handle(None))
    assert rc == 0, lib.last_error()
    return y, scale


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_on_consecutive_calls() -> None:
    gen = torch.Generator(device="cuda").manual_seed(7)
    shapes = [(2, 3000, 8, 128), (1, 700, 24, 128)]  # the second reuses slots the first wrote
    for i, shape in enumerate(shapes):
        x = (torch.randn(shape, device="cuda", generator=gen) * (1.0 + 3.0 * i)).bfloat16()
        x[0, 5, 0, 3] = 40.0 * (i + 1)  # one outlier sets head 0's scale
        y_ref, s_ref = _quantise("h3sa_quantize_fp8_per_head", x)
        y_new, s_new = _quantise("h3sa_quantize_fp8_per_head_noalloc", x)
        torch.cuda.synchronize()
        assert torch.equal(s_new, s_ref), (i, (s_new - s_ref).abs().max().item())
        assert torch.equal(y_new.view(torch.uint8), y_ref.view(torch.uint8)), i


@pytest.mark.gpu
def test_noalloc_leaves_the_stream_ordered_pool_untouched() -> None:
    """The allocating entry takes its scratch from the device's default stream-ordered pool;
    the no-allocation entry must not: the pool's used-memory high-water mark, reset before
    the call, stays at what was in use before it."""

    runtime = pytest.importorskip("cuda.bindings.runtime")
    driver = pytest.importorskip("cuda.bindings.driver")
    dev = torch.cuda.current_device()
    err, pool = runtime.cudaDeviceGetDefaultMemPool(dev)
    assert err == runtime.cudaError_t.cudaSuccess
    high = runtime.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh
    cur = runtime.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent

    def watermark(entry: str, x: torch.Tensor) -> tuple[int, int]:
        torch.cuda.synchronize()
        assert runtime.cudaMemPoolSetAttribute(pool, high, driver.cuuint64_t(0))[0] == \
            runtime.cudaError_t.cudaSuccess
        before = int(runtime.cudaMemPoolGetAttribute(pool, cur)[1])
        _quantise(entry, x)
        torch.cuda.synchronize()
        return before, int(runtime.cudaMemPoolGetAttribute(pool, high)[1])

    x = torch.randn(1, 4096, 8, 128, device="cuda").bfloat16()
    _quantise("h3sa_quantize_fp8_per_head_noalloc", x)  # first call: per-device set-up
    before, peak = watermark("h3sa_quantize_fp8_per_head_noalloc", x)
    assert peak == before, (before, peak)
    before, peak = watermark("h3sa_quantize_fp8_per_head", x)
    assert peak > before, "the allocating entry should show its scratch in the pool"


def test_noalloc_rejects_sizes_beyond_scratch() -> None:
    lib = _lib()
    seq = 256 * (NOALLOC_SLOTS // 4) + 1  # 4 heads of ceil(seq / 256) chunks: one slot too many
    rc = lib.LIB.h3sa_quantize_fp8_per_head_noalloc(16, 32, 48, 1, seq, 4, 128, None)
    assert rc == lib.H3SA_ERR_INVALID
    assert "exceeds the fixed scratch" in lib.last_error()
    # (batch, head) pairs run along the grid's y extent, at most 65535 of them; a single head
    # may have any number of 256-row chunks (they run along x)
    rc = lib.LIB.h3sa_quantize_fp8_per_head_noalloc(16, 32, 48, 1, 1, 65536, 128, None)
    assert rc == lib.H3SA_ERR_INVALID and "batch * heads" in lib.last_error()
    rc = lib.LIB.h3sa_quantize_fp8_per_head(16, 32, 48, 2, 1, 40000, 128, None)
    assert rc == lib.H3SA_ERR_INVALID and "batch * heads" in lib.last_error()
