"""One layer call end to end through the public drop-ins, against the oracle composed in the
reference's order (T/model/layers.py:376-442):

    merged QKV -> fused_qkv_qk_norm_rope_ -> merged_qkv_sequence_to_heads
               -> H3StreamingAttentionHook.__call__ -> heads_to_sequence

At SP=1 on one GPU, and at SP=2 on two GPUs (one process each) for both exchanges: NCCL
all-to-all (h3sa.ulysses) and peer stores over NVLink (h3sa.layer.PeerUlysses, attention
epilogue storing into the owners' shards). The oracle runs the whole sequence on the CPU;
each rank checks its own sequence shard. Tolerance: relative L2 <= 1e-2 (bf16); the two
exchanges must agree bit for bit (same kernels, only the bytes' route differs).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
HEADS, HD, HIST, EPS = 4, 128, 1000, 1e-5
TOL = 1e-2


class _Attn:
    softmax_scale = HD ** -0.5


def _inputs() -> dict:
    """Seeded merged QKV of a packed chunk (text | audio | video | pad), norm weights, the
    bf16 RoPE cache and a history, plus the oracle's output for the full sequence."""

    from oracle import attention as oatt
    from oracle import prologue as opro

    layout = opro.packed_layout(text_len=64, latent_t=3, latent_h=32, latent_w=32, audio_t=40)
    seq = layout["seq_len"]
    rng = np.random.default_rng(11)
    merged = opro.round_bf16(rng.standard_normal((seq, 3 * HEADS * HD)).astype(np.float32))
    wq = opro.round_bf16(1.0 + 0.1 * rng.standard_normal(HD).astype(np.float32))
    wk = opro.round_bf16(1.0 + 0.1 * rng.standard_normal(HD).astype(np.float32))
    cs = opro.rope_cos_sin(layout["grid"], opro.default_inv_freq(16))
    hist_k = opro.round_bf16(rng.standard_normal((HIST, HEADS, HD)).astype(np.float32))
    hist_v = opro.round_bf16(rng.standard_normal((HIST, HEADS, HD)).astype(np.float32))
    ref_qkv = opro.qkv_norm_rope(merged, wq, wk, cs, np.arange(seq), HEADS, HD, EPS)
    q, k, v = (torch.from_numpy(np.ascontiguousarray(t))
               for t in ref_qkv.reshape(seq, 3, HEADS, HD).transpose(1, 0, 2, 3))
    commit = torch.from_numpy(layout["commit_mask"])
    ref = oatt.streaming_hook_attention(q, k, v, commit, layout["cu_seqlens"],
                                        (torch.from_numpy(hist_k), torch.from_numpy(hist_v)),
                                        _Attn.softmax_scale)
    return {"layout": layout, "seq": seq, "merged": merged, "wq": wq, "wk": wk, "cs": cs,
            "hist_k": hist_k, "hist_v": hist_v, "ref": ref.reshape(seq, HEADS * HD)}


def _hook(inp: dict, dev: torch.device, head_lo: int, head_hi: int):
    """A NOISY-mode hook whose cache holds the history of heads [head_lo, head_hi)."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    hl = head_hi - head_lo
    cache = CleanAVKVCache(KVContract(local_heads=hl, head_dim=HD), layer_names=("blocks.0.attn",),
                           device=dev)
    paged = cache.layer("blocks.0.attn", dev)
    to = lambda x: torch.from_numpy(np.ascontiguousarray(x[:, head_lo:head_hi])).to(  # noqa: E731
        dev, torch.bfloat16)
    paged.write(to(inp["hist_k"]), to(inp["hist_v"]), start=0, count=HIST)
    paged.history_rows = HIST
    hook = H3StreamingAttentionHook(cache)
    hook.activate(HookMode.NOISY)
    return hook


def _call(inp: dict, dev: torch.device, hook, row_lo: int, row_hi: int, **ulysses) -> torch.Tensor:
    from h3sa.layer import attention_from_projection

    bf = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev, torch.bfloat16)  # noqa: E731
    layout = inp["layout"]
    qkv = bf(inp["merged"][row_lo:row_hi])
    positions = torch.arange(row_lo, row_hi, device=dev)
    out = attention_from_projection(
        qkv, q_weight=bf(inp["wq"]), k_weight=bf(inp["wk"]), rope_cache=(bf(inp["cs"]), positions),
        eps=EPS, num_heads=HEADS, head_dim=HD, hook=hook, attention=_Attn(),
        layer_name="blocks.0.attn", token_tags=torch.from_numpy(layout["token_tags"]).to(dev),
        commit_mask=torch.from_numpy(layout["commit_mask"]).to(dev),
        cu_seqlens_host=layout["cu_seqlens"], **ulysses)
    torch.cuda.synchronize()
    hook.check_device_error()
    return out.float().cpu()


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a - b).norm() / b.norm())


def test_layer_call_sp1_matches_composed_oracle() -> None:
    sys.path.insert(0, str(ROOT))
    inp = _inputs()
    dev = torch.device("cuda", torch.cuda.current_device())
    hook = _hook(inp, dev, 0, HEADS)
    out = _call(inp, dev, hook, 0, inp["seq"])
    err = _rel(out, inp["ref"])
    assert err <= TOL, f"layer output rel L2 {err:.3e}"
    # the call again (NOISY mode leaves the history as it was): same bits
    assert torch.equal(_call(inp, dev, hook, 0, inp["seq"]), out)


def _worker(rank: int, world: int, rendezvous: str) -> None:
    import datetime

    sys.path.insert(0, str(ROOT / "taomate-h3_b200"))
    sys.path.insert(0, str(ROOT))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.distributed.init_process_group("nccl", init_method=f"file://{rendezvous}", rank=rank,
                                         world_size=world, timeout=datetime.timedelta(seconds=60),
                                         device_id=dev)
    try:
        from h3sa.layer import PeerUlysses
        from h3sa.ulysses import ParallelContext

        inp = _inputs()
        seq, hl = inp["seq"], HEADS // world
        tokens = seq // world
        lo, hi = rank * tokens, (rank + 1) * tokens
        group = torch.distributed.group.WORLD
        ctx = ParallelContext(tp_world_size=1, tp_rank=0, ulysses_world_size=world,
                              ulysses_rank=rank, tp_group=group, ulysses_group=group)
        hook = _hook(inp, dev, rank * hl, (rank + 1) * hl)
        out_nccl = _call(inp, dev, hook, lo, hi, context=ctx)
        err = _rel(out_nccl, inp["ref"][lo:hi])
        assert err <= TOL, f"rank {rank} NCCL path rel L2 {err:.3e}"
        exchange = PeerUlysses(tokens, HEADS, HD, device_error=hook.device_error(dev))
        for _ in range(2):  # the second call reuses the planes and shards the first filled
            out_peer = _call(inp, dev, hook, lo, hi, exchange=exchange)
            assert hook.last_output_exchanged, "the attention epilogue did not store the rows"
            assert torch.equal(out_peer, out_nccl), f"rank {rank}: peer and NCCL paths differ"
        torch.distributed.barrier()
        torch.cuda.synchronize()
        exchange.close()
    finally:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def test_layer_call_sp2_nccl_and_peer_match_oracle(tmp_path: Path) -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, str(tmp_path / "rendezvous")), nprocs=2, join=True)
