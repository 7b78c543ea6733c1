#!/usr/bin/env python
"""Benchmark: 768p streaming chunk attention (TaoMate-H3 hot path) on B200.

One step = one streaming-hook layer call of the 768p chunk on this rank: the seq->heads
exchange of the local merged QKV shard (SP > 1), the current chunk's K/V rows written into the
paged cache after the 16384-row history, attention of the 12509 media queries over
[history | current] (plus the pad document over itself), and the heads->seq exchange of O
(SP > 1). Ulysses SP = number of GPUs, heads 24 / SP per GPU. For SP > 1 the exchanges are
peer stores over NVLink by default: one kernel scatters Q to the owners' planes and K/V
straight into the owners' caches, and the attention epilogue stores O into the owners'
sequence shards. `--unfused` uses NCCL all-to-all with pack/unpack kernels and a separate
cache append instead (the reference's structure).

Prints one JSON line (rank 0). ``value`` = total attention TFLOP/s of the whole job
(4 * Nq * Nk * d * H per step / max-over-ranks device time). ``e2e`` repeats the step
through the public API with every step's input copied from pinned host memory and its output
copied back inside the timed region; the copies are double-buffered on their own streams, so
the upload and download of neighbouring steps overlap the compute of the current one.
``--impl reference`` times the reference's CPU attention (its PyTorch path restated in
oracle/) on this host's cores on a bounded query sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "taomate-h3_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

CFG = {
    "heads": 24,
    "head_dim": 128,
    "video": 12384,   # 3 latent frames x 48 x 86
    "audio": 125,
    "history": 16384,
    "align": 64,      # packed-sequence alignment (T/model/architecture.py:12)
}
METRIC = "chunk attention TFLOP/s (768p, Ulysses SP=N, bf16, 16k KV cache)"


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"bf16": float(data["bf16_tflops"]), "bf16_sustained": float(data["bf16_tflops_sustained"]),
                "hbm": float(data["hbm_gbs"]), "source": "measured"}
    return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


def _ncu_traffic() -> float | None:
    """DRAM bytes per attention launch from the committed ncu summary, if present."""

    path = ROOT / "profiles" / "attention_768p_sp1_ncu.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / power / throttle-reason sampling, kept only inside the timed window.

    Samples every 20 ms with their timestamps; `mark_start()` / `mark_stop()` bracket the timed
    region (host wall clock, after a device synchronize) and `summary()` reports the samples that
    fall between them (all samples, flagged, if the window caught none).
    """

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc: subprocess.Popen | None = None
        self.t0 = self.t1 = None

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def mark_start(self) -> None:
        self.t0 = time.time()

    def mark_stop(self) -> None:
        self.t1 = time.time()

    def __exit__(self, *exc: object) -> None:
        self.lines: list[str] = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    @staticmethod
    def _epoch(stamp: str) -> float | None:
        import datetime

        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.datetime.strptime(stamp.strip(), fmt).timestamp()
            except ValueError:
                continue
        return None

    def summary(self) -> dict:
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                rows.append((self._epoch(parts[0]), float(parts[2]), float(parts[3]),
                             float(parts[4]), parts[6:10]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        inside = [r for r in rows if r[0] is not None and self.t0 is not None and
                  self.t1 is not None and self.t0 <= r[0] <= self.t1]
        use = inside or rows
        reasons = sorted({n for r in use for n, f in zip(names, r[4]) if f.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in use),
                "sm_max_mhz": max(r[2] for r in use), "reasons": reasons,
                "power_w": statistics.median(r[3] for r in use), "samples": len(use),
                "window": "timed region" if inside else "whole run (no sample inside the timed region)"}


def _dist() -> tuple[int, int, int]:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not torch.distributed.is_initialized():
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def _geometry(world: int) -> dict:
    nq = CFG["video"] + CFG["audio"]
    align = CFG["align"] * world // _gcd(CFG["align"], world)
    rows = (nq + align - 1) // align * align
    return {"nq": nq, "rows": rows, "pad": rows - nq, "tokens": rows // world,
            "heads_local": CFG["heads"] // world, "nk": CFG["history"] + nq}


def _gcd(a: int, b: int) -> int:
    while b:
        a, b = b, a % b
    return a


def _cpu_baseline(seconds: float = 12.0) -> dict:
    """Oracle (reference CPU attention math) on a bounded query sample, all host threads."""

    from oracle.attention import attention_flops, time_cpu_attention

    threads = len(os.sched_getaffinity(0))
    g = torch.Generator().manual_seed(7)
    nk = CFG["history"] + CFG["video"] + CFG["audio"]
    heads, d = CFG["heads"], CFG["head_dim"]
    k = torch.randn(nk, heads, d, generator=g)
    v = torch.randn(nk, heads, d, generator=g)
    nq = 64
    total_t = total_f = 0.0
    calls = 0
    while total_t < seconds and calls < 64:
        q = torch.randn(nq, heads, d, generator=g)
        t = time_cpu_attention(q, k, v, d ** -0.5, threads)
        total_t += t
        total_f += attention_flops(nq, nk, heads, d)
        calls += 1
        if t < 0.5 and nq < 4096:
            nq *= 2
    return {"value": total_f / total_t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{calls} calls, up to {nq} query rows x {heads} heads x {nk} keys, fp32 "
                      f"torch CPU (oracle.attention.sdpa_from_kv_parts), {total_t:.1f} s"}


def run_reference(args: argparse.Namespace) -> None:
    world, rank, _ = (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    if rank != 0:
        return
    from oracle.attention import attention_flops, sdpa_from_kv_parts

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    geo = _geometry(world)
    heads, d, nk = CFG["heads"], CFG["head_dim"], geo["nk"]
    k = torch.randn(nk, heads, d, generator=g)
    v = torch.randn(nk, heads, d, generator=g)
    sample_q = 256
    q = torch.randn(sample_q, heads, d, generator=g)
    for _ in range(args.warmup):
        sdpa_from_kv_parts(q, [(k, v)], d ** -0.5)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        sdpa_from_kv_parts(q, [(k, v)], d ** -0.5)
        times.append(time.perf_counter() - t0)
    flops = attention_flops(sample_q, nk, heads, d)
    value = flops * len(times) / sum(times) / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "768p chunk attention, reference CPU path on a bounded sample",
                   "heads": heads, "head_dim": d, "queries": geo["nq"], "keys": nk,
                   "sample_queries_per_step": sample_q},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{sample_q} query rows x {heads} heads x {nk} keys per step, "
                                   "fp32 torch CPU (oracle restatement of the reference "
                                   "_sdpa_from_kv_parts; FlashAttention-3 is sm_90a-only)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class Step:
    """Device buffers and launches of one benchmark step on this rank."""

    def __init__(self, world: int, rank: int, device: torch.device, fused: bool = True) -> None:
        import h3sa
        from h3sa.kernels import PAGE_ROWS

        self.h3sa = h3sa
        self.world, self.rank, self.device = world, rank, device
        # SP > 1: the two Ulysses exchanges as peer stores (scatter kernel, attention epilogue)
        # over NVLink, or NCCL all-to-all with layout copies (the reference's structure)
        self.fused = fused and world > 1
        self.phases = self.PHASES_FUSED if self.fused else self.PHASES
        geo = _geometry(world)
        self.geo = geo
        heads, d = CFG["heads"], CFG["head_dim"]
        hl = geo["heads_local"]
        self.hl = hl
        g = torch.Generator(device=device).manual_seed(1000 + rank)
        # this rank's post-prologue merged QKV shard [T, 3*H*d] (q, k RMS-normalised ~ N(0,1))
        self.merged = torch.randn(geo["tokens"], 3 * heads * d, device=device, generator=g).to(torch.bfloat16)
        nh = CFG["history"]
        self.n_hist = nh
        total_rows = nh + geo["rows"]
        pages = (total_rows + PAGE_ROWS - 1) // PAGE_ROWS
        self.table = torch.arange(pages, dtype=torch.int32, device=device)
        rows, tokens = geo["rows"], geo["tokens"]
        if self.fused:
            # every rank maps every rank's Q plane, KV pools and output shard: the QKV scatter
            # writes the current chunk's K/V straight into the owners' pools
            from h3sa.peer import PeerBarrier, PeerBuffer

            self.kpool_peer = PeerBuffer((hl, pages * PAGE_ROWS, d))
            self.vpool_peer = PeerBuffer((hl, pages * PAGE_ROWS, d))
            self.kpool, self.vpool = self.kpool_peer.tensor, self.vpool_peer.tensor
            self.kpool.zero_()
            self.vpool.zero_()
            self.q_peer = PeerBuffer((rows, hl, d))
            self.out_peer = PeerBuffer((tokens, heads, d))
            self.peer_barrier = PeerBarrier(device_error=None)
            self.final = self.out_peer.tensor
        else:
            self.kpool = torch.zeros(hl, pages * PAGE_ROWS, d, dtype=torch.bfloat16, device=device)
            self.vpool = torch.zeros_like(self.kpool)
        hist = torch.randn(nh, hl, d, device=device, generator=g).to(torch.bfloat16)
        h3sa.kv_copy_rows([hist, hist], [self.kpool, self.vpool], count=nh, dst_table=self.table)
        if world > 1 and not self.fused:
            self.send = torch.empty(world, 3, tokens, hl, d, dtype=torch.bfloat16, device=device)
            self.recv = torch.empty_like(self.send)
            self.qkv = torch.empty(3, rows, hl, d, dtype=torch.bfloat16, device=device)
            self.orecv = torch.empty(world, tokens, hl, d, dtype=torch.bfloat16, device=device)
            self.final = torch.empty(tokens, heads, d, dtype=torch.bfloat16, device=device)
        elif world == 1:
            self.qkv = self.merged.view(rows, 3, heads, d).permute(1, 0, 2, 3).contiguous()
        self.out = torch.empty(rows, hl, d, dtype=torch.bfloat16, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        if self.fused:
            self.peer_barrier.err = self.err  # a barrier wait that gives up shows in device_error
        P = h3sa.AttentionProblem
        nq, pad = geo["nq"], geo["pad"]
        self.problems = [P(0, nq, 0, nh + nq)]
        if pad:
            self.problems.append(P(nq, rows, nh + nq, nh + rows))
        self.scale = d ** -0.5
        self.flops = 4.0 * nq * (nh + nq) * d * hl  # this rank's algorithmic FLOPs
        # h3sa kernels per step: SP=1 cache append + attention; NCCL path + pack, two unpacks;
        # peer path: scatter into the caches, barrier, attention, barrier
        self.launches_per_step = 4 if self.fused else 2 + (3 if world > 1 else 0)

    PHASES = ("pack", "qkv_all_to_all", "unpack", "cache_append", "attention", "o_all_to_all",
              "o_unpack")
    PHASES_FUSED = ("qkv_scatter_into_cache", "barrier_before_attention", "unused", "unused_append",
                    "attention_with_o_scatter", "barrier_after_attention", "unused2")
    EXCHANGE_PHASES = ("qkv_all_to_all", "o_all_to_all", "qkv_scatter_into_cache",
                       "barrier_before_attention", "barrier_after_attention")

    def run(self, attn_events: tuple[torch.cuda.Event, torch.cuda.Event] | None = None,
            merged: torch.Tensor | None = None,
            marks: list[torch.cuda.Event] | None = None) -> torch.Tensor:
        """One step; `marks` (len(PHASES) + 1 events) are recorded at the phase boundaries."""

        from h3sa.ulysses import pack_qkv_send, unpack_o_recv, unpack_qkv_recv

        h3sa, geo, hl = self.h3sa, self.geo, self.hl
        d, heads = CFG["head_dim"], CFG["heads"]
        src = self.merged if merged is None else merged

        def mark(i: int) -> None:
            if marks is not None:
                marks[i].record()

        mark(0)
        if self.fused:
            from h3sa.peer import attention_fwd_scatter, scatter_qkv_paged

            # Q to the owners' planes, K/V into the owners' caches after the history
            scatter_qkv_paged(src, self.q_peer, self.kpool_peer, self.vpool_peer, self.table,
                              dst_start=self.n_hist, num_heads=heads, head_dim=d,
                              device_error=self.err)
            mark(1)
            self.peer_barrier()
            mark(2)
            mark(3)
            mark(4)
            if attn_events is not None:
                attn_events[0].record()
            attention_fwd_scatter(self.q_peer.tensor, self.kpool, self.vpool, self.table,
                                  self.problems, self.scale,
                                  self.out_peer, device_error=self.err)
            if attn_events is not None:
                attn_events[1].record()
            mark(5)
            self.peer_barrier()
            mark(6)
            mark(7)
            return self.final
        if self.world > 1:
            pack_qkv_send(src, self.send, world=self.world, num_heads=heads, head_dim=d)
            mark(1)
            torch.distributed.all_to_all_single(self.recv, self.send)
            mark(2)
            unpack_qkv_recv(self.recv, self.qkv, world=self.world, tokens=geo["tokens"],
                            local_heads=hl, head_dim=d)
        elif merged is not None:
            self.qkv.copy_(merged.view(geo["rows"], 3, heads, d).permute(1, 0, 2, 3))
            mark(1)
            mark(2)
        else:
            mark(1)
            mark(2)
        mark(3)
        q, k, v = self.qkv[0], self.qkv[1], self.qkv[2]
        # current chunk's K/V rows (media + pad document) after the history
        h3sa.kv_copy_rows([k, v], [self.kpool, self.vpool], count=geo["rows"], dst_table=self.table,
                          dst_start=self.n_hist, device_error=self.err)
        mark(4)
        if attn_events is not None:
            attn_events[0].record()
        h3sa.attention_fwd(q, self.out, self.kpool, self.vpool, self.table, self.problems,
                           self.scale, device_error=self.err)
        if attn_events is not None:
            attn_events[1].record()
        mark(5)
        if self.world > 1:
            torch.distributed.all_to_all_single(self.orecv, self.out)
            mark(6)
            unpack_o_recv(self.orecv, self.final, world=self.world, tokens=geo["tokens"],
                          local_heads=hl, head_dim=d)
            mark(7)
            return self.final
        mark(6)
        mark(7)
        return self.out


def _time_launch(fn, iters: int) -> float:
    """Mean device time (ms) of `fn` over `iters` launches after two warm-up calls."""

    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


VARIANTS = ("fp8", "sparse", "480p")


def _variants(peaks: dict, iters: int = 10, only: str | None = None) -> dict:
    """Kernel-only timings of the path's other variants on this GPU (all, or `only` one).

    * fp8: the 1080p per-GPU problem of the TP2 x SP4 configuration (24 heads / TP 2 / SP 4 =
      3 heads; 24480 video + 125 audio queries over a 32768-row cache plus the chunk), e4m3
      Q/K/V with per-head scales, inputs N(0,1) with 1% outliers x8 (seeded).
    * sparse: the 768p per-GPU problem at SP=8 (3 heads; 12509 queries over 16384 + 12509
      keys) with the composite 128x128 block mask (audio blocks, 2 sinks, +-4-block band, top-k
      fill to 25% of blocks).
    * 480p: dense bf16 on one GPU (24 heads; 4985 queries over 19940 + 4985 keys).
    FLOPs count only the work the kernel must do (kept blocks for the sparse case). Each
    variant times `iters` launches after two warm-up launches.
    """

    import h3sa
    from h3sa.kernels import PAGE_ROWS

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(7)

    def pools(rows: int, heads: int, k: torch.Tensor, v: torch.Tensor):
        pages = (rows + PAGE_ROWS - 1) // PAGE_ROWS
        table = torch.arange(pages, dtype=torch.int32, device=dev)
        kp = torch.zeros(heads, pages * PAGE_ROWS, CFG["head_dim"], dtype=torch.bfloat16,
                         device=dev)
        vp = torch.zeros_like(kp)
        h3sa.kv_copy_rows([k, v], [kp, vp], count=rows, dst_table=table)
        return kp, vp, table

    out = {}
    for name, fn in (("fp8", _variant_fp8), ("sparse", _variant_sparse), ("480p", _variant_480p)):
        if only in (None, name):
            out.update(fn(peaks, iters, dev, g, pools))
            torch.cuda.empty_cache()
    return out


def _variant_fp8(peaks: dict, iters: int, dev: torch.device, g: torch.Generator, pools) -> dict:
    import h3sa

    d = CFG["head_dim"]
    out = {}
    heads, nq, nh = 3, 24480 + 125, 32768
    nk = nh + nq

    def outliers(x: torch.Tensor) -> torch.Tensor:
        mask = torch.rand(x.shape, device=dev, generator=g) < 0.01
        return torch.where(mask, x * 8, x)

    q = outliers(torch.randn(nq, heads, d, device=dev, generator=g)).to(torch.bfloat16)
    k = outliers(torch.randn(nk, heads, d, device=dev, generator=g)).to(torch.bfloat16)
    v = outliers(torch.randn(nk, heads, d, device=dev, generator=g)).to(torch.bfloat16)
    kp, vp, table = pools(nk, heads, k, v)
    k8 = torch.empty_like(kp, dtype=torch.float8_e4m3fn)
    v8 = torch.empty_like(vp, dtype=torch.float8_e4m3fn)
    ks = torch.empty(heads, dtype=torch.float32, device=dev)
    vs = torch.empty_like(ks)
    h3sa.quantize_fp8_pool(kp, k8, ks, table, nk)
    h3sa.quantize_fp8_pool(vp, v8, vs, table, nk)
    q8, qs = h3sa.quantize_fp8_e4m3_per_head(q.unsqueeze(0))
    o = torch.empty(nq, heads, d, dtype=torch.bfloat16, device=dev)
    probs = [h3sa.AttentionProblem(0, nq, 0, nk)]
    ms = _time_launch(lambda: h3sa.attention_fwd(q8[0], o, k8, v8, table, probs, d ** -0.5,
                                                 q_scale=qs[0], k_scale=ks, v_scale=vs), iters)
    tf = 4.0 * nq * nk * d * heads / (ms * 1e-3) / 1e12
    fp8_peak = 2.0 * peaks["bf16"]
    out["fp8_1080p_tp2sp4_per_gpu"] = {
        "ms": ms, "tflops": tf, "heads": heads, "queries": nq, "keys": nk,
        "roofline": {"bound": "tensor", "peak": fp8_peak, "frac": tf / fp8_peak,
                     "peak_source": "2 x measured bf16 burst (no measured e4m3 GEMM peak; "
                                    "nominal dense e4m3 is 4500)"}}
    return out


def _variant_sparse(peaks: dict, iters: int, dev: torch.device, g: torch.Generator,
                    pools) -> dict:
    import types

    import h3sa
    from h3sa.block_sparse import composite_block_mask
    from h3sa.kernels import PAGE_ROWS

    d = CFG["head_dim"]
    out = {}
    heads, nq, nh = 3, CFG["video"] + CFG["audio"], CFG["history"]
    nk = nh + nq
    q = torch.randn(nq, heads, d, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(nk, heads, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(nk, heads, d, device=dev, generator=g).to(torch.bfloat16)
    kp, vp, table = pools(nk, heads, k, v)
    qb, kb = (nq + PAGE_ROWS - 1) // PAGE_ROWS, (nk + PAGE_ROWS - 1) // PAGE_ROWS
    q_audio = torch.zeros(qb, dtype=torch.uint8, device=dev)
    q_audio[CFG["video"] // PAGE_ROWS:] = 1           # the chunk's audio rows follow its video
    kv_audio = torch.zeros(kb, dtype=torch.uint8, device=dev)
    kv_audio[(nh + CFG["video"]) // PAGE_ROWS:] = 1
    kv_audio[torch.arange(31, nh // PAGE_ROWS, 32, device=dev)] = 1  # one audio block per 4096 history rows
    paged = types.SimpleNamespace(key=kp, table=table)
    num, idx = composite_block_mask(q, paged, q_lo=0, q_hi=nq, n_hist=nh, n_kv=nk,
                                    q_block_audio=q_audio, kv_block_audio=kv_audio, density=0.25)
    o = torch.empty(nq, heads, d, dtype=torch.bfloat16, device=dev)
    probs = [h3sa.AttentionProblem(0, nq, 0, nk, sparse=True)]
    ms = _time_launch(lambda: h3sa.attention_fwd(q, o, kp, vp, table, probs, d ** -0.5,
                                                 kv_num_blocks=num, kv_indices=idx), iters)
    kept = int(num.sum().item())
    density = kept / (heads * qb * kb)
    flops = 4.0 * kept * PAGE_ROWS * PAGE_ROWS * d  # kept 128x128 blocks (tail blocks counted whole)
    tf = flops / (ms * 1e-3) / 1e12
    out["sparse_768p_sp8_per_gpu"] = {
        "ms": ms, "tflops_on_kept_blocks": tf, "kept_block_fraction": density, "heads": heads,
        "queries": nq, "keys": nk,
        "roofline": {"bound": "tensor", "peak": peaks["bf16"], "frac": tf / peaks["bf16"]}}
    return out


def _variant_480p(peaks: dict, iters: int, dev: torch.device, g: torch.Generator, pools) -> dict:
    import h3sa

    d = CFG["head_dim"]
    out = {}
    heads, nq, nh = 24, 4860 + 125, 19940
    nk = nh + nq
    q = torch.randn(nq, heads, d, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(nk, heads, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(nk, heads, d, device=dev, generator=g).to(torch.bfloat16)
    kp, vp, table = pools(nk, heads, k, v)
    o = torch.empty(nq, heads, d, dtype=torch.bfloat16, device=dev)
    probs = [h3sa.AttentionProblem(0, nq, 0, nk)]
    ms = _time_launch(lambda: h3sa.attention_fwd(q, o, kp, vp, table, probs, d ** -0.5), iters)
    tf = 4.0 * nq * nk * d * heads / (ms * 1e-3) / 1e12
    out["dense_480p_1gpu"] = {
        "ms": ms, "tflops": tf, "heads": heads, "queries": nq, "keys": nk,
        "roofline": {"bound": "tensor", "peak": peaks["bf16"], "frac": tf / peaks["bf16"]}}
    return out


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def _comparator_sdpa(step: Step, iters: int = 5) -> dict:
    """The reference FL2VA `sdpa` backend on this GPU: torch.cat of the K/V parts then
    torch SDPA (F/streaming/attention_hook.py:288-316), same shapes, one rank."""

    geo, hl, d = step.geo, step.hl, CFG["head_dim"]
    nh, nq = step.n_hist, geo["nq"]
    q = step.qkv[0][:nq]
    hist_k = step.kpool[:, :nh].transpose(0, 1).contiguous()
    hist_v = step.vpool[:, :nh].transpose(0, 1).contiguous()
    cur_k, cur_v = step.qkv[1][:nq], step.qkv[2][:nq]

    def call() -> torch.Tensor:
        key = torch.cat((hist_k, cur_k), dim=0)
        value = torch.cat((hist_v, cur_v), dim=0)
        out = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(0, 1).unsqueeze(0), key.transpose(0, 1).unsqueeze(0),
            value.transpose(0, 1).unsqueeze(0), dropout_p=0.0, is_causal=False, scale=step.scale)
        return out.squeeze(0).transpose(0, 1)

    for _ in range(2):
        call()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(iters):
        a.record()
        call()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return {"impl": "torch SDPA on this GPU via the reference's sdpa-backend call pattern "
                    "(cat K/V parts + F.scaled_dot_product_attention)",
            "ms_p50": statistics.median(times)}


def run_h3sa(args: argparse.Namespace) -> None:
    world, rank, local = _dist()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    step = Step(world, rank, device, fused=not args.unfused)
    peaks = _peaks()

    for _ in range(args.warmup):
        step.run()
    _barrier(world)
    attn_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    step_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    phase_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(step.phases) + 1)]
                for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        _barrier(world)
        torch.cuda.synchronize()
        clocks.mark_start()
        start.record()
        for i in range(args.steps):
            step_ev[i][0].record()
            step.run(attn_ev[i], marks=phase_ev[i])
            step_ev[i][1].record()
        stop.record()
        torch.cuda.synchronize()
        clocks.mark_stop()
        _barrier(world)
    total_ms = _max_over_ranks(start.elapsed_time(stop), world)
    attn_ms = [a.elapsed_time(b) for a, b in attn_ev]
    phases = {name: _max_over_ranks(statistics.median(ev[j].elapsed_time(ev[j + 1]) for ev in phase_ev),
                                    world)
              for j, name in enumerate(step.phases) if not name.startswith("unused")}
    step_ms = [a.elapsed_time(b) for a, b in step_ev]
    attn_avg = _max_over_ranks(sum(attn_ms) / len(attn_ms), world)
    p50 = _max_over_ranks(statistics.median(step_ms), world)
    p90 = _max_over_ranks(sorted(step_ms)[int(0.9 * (len(step_ms) - 1))], world)
    err = int(step.err.item())

    # e2e: public API with pinned host input / output each step. Copies run on their own
    # streams, double-buffered: the upload of step i + 1 and the download of step i - 1
    # overlap the compute of step i (two copy engines, one per direction).
    e2e = None
    if not args.no_e2e:
        host_in = step.merged.cpu().pin_memory()
        out_shape = step.final.shape if world > 1 else step.out.shape
        host_out = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        dev_in = [torch.empty_like(step.merged) for _ in range(2)]
        dev_out = [torch.empty(out_shape, dtype=torch.bfloat16, device=device) for _ in range(2)]
        comp = torch.cuda.current_stream()
        h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
        ev = {name: [torch.cuda.Event() for _ in range(2)]
              for name in ("in_ready", "in_free", "out_ready", "out_free")}

        def e2e_step(i: int) -> None:
            k = i % 2
            h2d.wait_event(ev["in_free"][k])      # compute of step i - 2 is done with dev_in[k]
            with torch.cuda.stream(h2d):
                dev_in[k].copy_(host_in, non_blocking=True)
                ev["in_ready"][k].record(h2d)
            comp.wait_event(ev["in_ready"][k])
            res = step.run(merged=dev_in[k])
            ev["in_free"][k].record(comp)
            comp.wait_event(ev["out_free"][k])    # download of step i - 2 is done with dev_out[k]
            dev_out[k].copy_(res, non_blocking=True)
            ev["out_ready"][k].record(comp)
            d2h.wait_event(ev["out_ready"][k])
            with torch.cuda.stream(d2h):
                host_out[k].copy_(dev_out[k], non_blocking=True)
                ev["out_free"][k].record(d2h)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        _barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(comp)
        h2d.wait_stream(comp)
        for i in range(args.steps):
            e2e_step(i)
        b.record(d2h)
        torch.cuda.synchronize()
        _barrier(world)
        e2e_ms = _max_over_ranks(a.elapsed_time(b), world) / args.steps
        total_flops = 4.0 * step.geo["nq"] * step.geo["nk"] * CFG["head_dim"] * CFG["heads"]
        e2e = {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
               "d2h_bytes_per_step": host_out[0].numel() * host_out[0].element_size(),
               "api": "h3sa.ulysses + h3sa.kv_copy_rows + h3sa.attention_fwd (C ABI via ctypes)",
               "copies": "pinned host buffers, double-buffered on separate H2D / D2H streams, "
                         "overlapping the compute of the neighbouring steps"}

    extra = {}
    if rank == 0 and world == 1 and not args.no_comparator:
        extra["comparator"] = _comparator_sdpa(step)
        extra["comparator"]["speedup_p50"] = extra["comparator"]["ms_p50"] / attn_avg
    if rank == 0 and world == 1 and not args.no_variants:
        extra["variants"] = _variants(peaks)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline()

    if rank != 0:
        return
    geo = step.geo
    total_flops = 4.0 * geo["nq"] * geo["nk"] * CFG["head_dim"] * CFG["heads"]
    value = total_flops * args.steps / (total_ms * 1e-3) / 1e12
    achieved = step.flops / (attn_avg * 1e-3) / 1e12
    traffic = _ncu_traffic()
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {
            "workload": "768p chunk: 12384 video + 125 audio queries x [16384 history + 12509 "
                        "current] keys, H=24, d=128, dense non-causal",
            "ulysses_sp": world, "heads_per_gpu": step.hl, "packed_rows": geo["rows"],
            "pad_rows": geo["pad"], "parallelism": f"sp{world}",
            "exchange": ("peer stores over NVLink (scatter kernel + attention epilogue)" if step.fused
                         else ("NCCL all_to_all_single + layout copies" if world > 1 else "none")),
            "l2": "inputs larger than L2 (Q 77 MB + K/V pool 355 MB at SP=1)",
        },
        "per_gpu_tflops": value / world,
        "tokens_per_s": geo["nq"] * args.steps / (total_ms * 1e-3),
        "latency_ms": {"p50": p50, "p90": p90, "attention_kernel_avg": attn_avg,
                       "phases_p50_max_over_ranks": phases,
                       "p50_without_exchanges": p50 - sum(v for k_, v in phases.items()
                                                          if k_ in Step.EXCHANGE_PHASES)},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16"],
                     "frac_of_sustained": achieved / peaks["bf16_sustained"],
                     "peak_source": peaks["source"] + " bf16 burst (MEASURED_PEAKS.json)",
                     "traffic": traffic},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": step.launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "device_error": err,
        **extra,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["h3sa", "reference"], default="h3sa")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-comparator", action="store_true")
    ap.add_argument("--unfused", action="store_true",
                    help="SP > 1: NCCL all-to-all + layout copies instead of peer stores")
    ap.add_argument("--no-variants", action="store_true",
                    help="skip the kernel-only FP8 1080p, block-sparse 768p and 480p timings")
    ap.add_argument("--variant", choices=VARIANTS,
                    help="time only this kernel-only variant on one GPU and print its JSON "
                         "(2 warm-up launches, then --steps launches)")
    args = ap.parse_args()
    if args.variant:
        torch.cuda.set_device(0)
        print(json.dumps(_variants(_peaks(), iters=args.steps, only=args.variant)), flush=True)
        return
    if args.warmup < 3 and args.impl == "h3sa":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_h3sa(args)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
