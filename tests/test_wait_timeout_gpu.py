"""A bounded device wait that runs out: the peer barrier against a rank that never arrives.

One GPU, no second process. The barrier is called as rank 0 of a two-rank group whose flag
arrays are both this process's own buffer, so slot 1 (the absent rank's arrival) is never
written. The kernel must give up after the caller's limit, set H3SA_DEVERR_WAIT_TIMEOUT in
the device error word and return; the stream stays usable, and the streaming hook's error
check turns the word into an exception on the host. No fault, trap or endless loop is
involved: the wait is a bounded poll of a flag nobody sets.
"""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _barrier(flags: torch.Tensor, world: int, rank: int, epoch: int, limit_ns: int,
             err: torch.Tensor) -> None:
    from h3sa import _lib

    table = torch.tensor([flags.data_ptr()] * world, dtype=torch.int64, device=flags.device)
    _lib.call("h3sa_peer_barrier_limit", _lib.ptr(table), world, rank, ctypes.c_uint32(epoch),
              ctypes.c_int64(limit_ns), _lib.ptr(err), _lib.stream_handle(None))
    torch.cuda.synchronize()
    del table


def test_peer_barrier_gives_up_after_its_limit_and_reports_it() -> None:
    from h3sa import _lib
    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook

    dev = torch.device("cuda", torch.cuda.current_device())
    hook = H3StreamingAttentionHook(CleanAVKVCache(KVContract(local_heads=2), device=dev))
    err = hook.device_error(dev)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)

    # a one-rank group completes at once
    _barrier(flags, 1, 0, 1, 5_000_000, err)
    assert int(err.item()) == 0 and int(flags[0].item()) == 1

    # rank 1 never arrives: the wait ends after ~5 ms with the timeout bit
    flags.zero_()
    t0 = time.perf_counter()
    _barrier(flags, 2, 0, 1, 5_000_000, err)
    elapsed = time.perf_counter() - t0
    assert int(err.item()) & _lib.DEVERR_WAIT_TIMEOUT
    assert int(flags[0].item()) == 1 and int(flags[1].item()) == 0
    assert elapsed < 1.0, f"the 5 ms wait took {elapsed:.3f} s"
    with pytest.raises(RuntimeError, match="device error flags 0x1"):
        hook.check_device_error()

    # the context is intact: the next barrier, with the peer's slot now set, succeeds
    err.zero_()
    flags[1] = 2
    _barrier(flags, 2, 0, 2, 5_000_000, err)
    assert int(err.item()) == 0
    hook.check_device_error()
