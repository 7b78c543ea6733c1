#!/usr/bin/env python
"""Benchmark: 768p streaming chunk attention (TaoMate-H3 hot path) on B200.

One step = one streaming layer call of the 768p chunk on this rank, from the raw merged QKV
projection shard to the attention output: the QK-RMSNorm + RoPE prologue, the seq->heads
exchange (SP > 1), the current chunk's K/V rows written into the paged cache after the
16384-row history, attention of the 12509 media queries over [history | current] (plus the
pad document over itself), and the heads->seq exchange of O (SP > 1). Ulysses SP = number of
GPUs, heads 24 / SP per GPU. By default the prologue, the exchange and the cache append are
one kernel storing Q into the owners' planes and K/V straight into the owners' caches (over
NVLink at SP > 1), and the attention epilogue stores O into the owners' sequence shards.
`--unfused` runs the reference's structure instead: prologue into a send buffer, NCCL
all-to-all, unpack, cache append, attention, NCCL all-to-all, unpack.

Prints one JSON line (rank 0). ``value`` = total attention TFLOP/s of the whole job
(4 * Nq * Nk * d * H per step / max-over-ranks device time). ``e2e`` runs the drop-in path a
maintainer installs (h3sa.layer.attention_from_projection through the streaming hook) with
every step's raw projection copied from pinned host memory and its output copied back inside
the timed region; ``e2e_kernel_path`` does the same around the timed step's own calls.
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


def _rope_cache(rows: int, rotary: int, device: torch.device) -> torch.Tensor:
    """Synthetic bf16 cos|sin cache [rows, rotary]: one position per packed row, the standard
    base-10000 frequencies (the model builds its 3-axis table the same size)."""

    half = rotary // 2
    inv = 10000.0 ** (-torch.arange(half, dtype=torch.float64, device=device) / half)
    ang = torch.arange(rows, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cat((ang.cos(), ang.sin()), dim=1).to(torch.bfloat16)


class Step:
    """Device buffers and launches of one benchmark step on this rank.

    Input: this rank's raw merged QKV projection shard [T, 3*H*d] (before the QK-RMSNorm /
    RoPE prologue). Fused path (default, any SP): one kernel normalises and rotates Q/K and
    stores Q into the owning rank's attention plane and K/V straight into the owner's paged
    cache after the history (local at SP=1); a peer barrier (SP>1); attention, whose
    epilogue stores each output row into the owner's sequence shard (SP>1); a peer barrier.
    Unfused path (--unfused, the reference's structure): prologue into the send layout, NCCL
    all-to-all, unpack, cache append, attention, NCCL all-to-all, unpack.
    """

    PHASES_FUSED = ("prologue_scatter_into_cache", "barrier_before_attention",
                    "attention_with_o_store", "barrier_after_attention")
    PHASES_NCCL = ("prologue_pack", "qkv_all_to_all", "unpack", "cache_append", "attention",
                   "o_all_to_all", "o_unpack")
    EXCHANGE_PHASES = ("qkv_all_to_all", "o_all_to_all", "barrier_before_attention",
                       "barrier_after_attention")

    def __init__(self, world: int, rank: int, device: torch.device, fused: bool = True) -> None:
        import h3sa
        from h3sa.kernels import PAGE_ROWS
        from h3sa.peer import LocalBuffer, PeerBarrier, PeerBuffer

        self.h3sa = h3sa
        self.world, self.rank, self.device = world, rank, device
        self.fused = fused or world == 1
        self.phases = self.PHASES_FUSED if self.fused else self.PHASES_NCCL
        geo = _geometry(world)
        self.geo = geo
        heads, d = CFG["heads"], CFG["head_dim"]
        hl = geo["heads_local"]
        self.hl = hl
        rows, tokens = geo["rows"], geo["tokens"]
        g = torch.Generator(device=device).manual_seed(1000 + rank)
        # this rank's raw merged QKV projection shard [T, 3*H*d] ~ N(0,1)
        self.merged = torch.randn(tokens, 3 * heads * d, device=device, generator=g).to(torch.bfloat16)
        gw = torch.Generator(device=device).manual_seed(99)  # weights: the same on every rank
        self.q_weight = (1 + 0.05 * torch.randn(d, device=device, generator=gw)).to(torch.bfloat16)
        self.k_weight = (1 + 0.05 * torch.randn(d, device=device, generator=gw)).to(torch.bfloat16)
        self.cos_sin = _rope_cache(CFG["history"] + rows, 96, device)
        self.positions = CFG["history"] + rank * tokens + torch.arange(tokens, device=device)
        nh = CFG["history"]
        self.n_hist = nh
        pages = (nh + rows + PAGE_ROWS - 1) // PAGE_ROWS
        self.table = torch.arange(pages, dtype=torch.int32, device=device)
        shape_pool = (hl, pages * PAGE_ROWS, d)
        if world > 1:
            # every rank maps every rank's Q plane, KV pools and output shard
            self.k_buf, self.v_buf = PeerBuffer(shape_pool), PeerBuffer(shape_pool)
            self.q_buf = PeerBuffer((rows, hl, d))
            self.out_buf = PeerBuffer((tokens, heads, d))
            self.peer_barrier = PeerBarrier(device_error=None)
        else:
            self.k_buf = LocalBuffer(torch.zeros(shape_pool, dtype=torch.bfloat16, device=device))
            self.v_buf = LocalBuffer(torch.zeros(shape_pool, dtype=torch.bfloat16, device=device))
            self.q_buf = LocalBuffer(torch.zeros(rows, hl, d, dtype=torch.bfloat16, device=device))
        self.kpool, self.vpool = self.k_buf.tensor, self.v_buf.tensor
        self.kpool.zero_()
        self.vpool.zero_()
        hist = torch.randn(nh, hl, d, device=device, generator=g).to(torch.bfloat16)
        h3sa.kv_copy_rows([hist, hist], [self.kpool, self.vpool], count=nh, dst_table=self.table)
        if not self.fused:
            self.send = torch.empty(world, 3, tokens, hl, d, dtype=torch.bfloat16, device=device)
            self.recv = torch.empty_like(self.send)
            self.qkv = torch.empty(3, rows, hl, d, dtype=torch.bfloat16, device=device)
            self.orecv = torch.empty(world, tokens, hl, d, dtype=torch.bfloat16, device=device)
            self.final = torch.empty(tokens, heads, d, dtype=torch.bfloat16, device=device)
        self.out = torch.empty(rows, hl, d, dtype=torch.bfloat16, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        if world > 1:
            self.peer_barrier.err = self.err  # a barrier wait that gives up shows in device_error
        P = h3sa.AttentionProblem
        nq, pad = geo["nq"], geo["pad"]
        self.problems = [P(0, nq, 0, nh + nq)]
        if pad:
            self.problems.append(P(nq, rows, nh + nq, nh + rows))
        self.scale = d ** -0.5
        self.flops = 4.0 * nq * (nh + nq) * d * hl  # this rank's algorithmic FLOPs
        # h3sa kernels per step: fused: prologue/scatter + attention (+ 2 barriers at SP>1);
        # NCCL: prologue pack + unpack + cache append + attention + unpack
        self.launches_per_step = (2 + (2 if world > 1 else 0)) if self.fused else 5

    def run(self, attn_events: tuple[torch.cuda.Event, torch.cuda.Event] | None = None,
            merged: torch.Tensor | None = None,
            marks: list[torch.cuda.Event] | None = None) -> torch.Tensor:
        """One step from the raw projection `merged` (default: the step's own); `marks`
        (len(phases) + 1 events) are recorded at the phase boundaries."""

        from h3sa.peer import attention_fwd_scatter
        from h3sa.prologue import qkv_norm_rope_pack, qkv_norm_rope_scatter_paged
        from h3sa.ulysses import unpack_o_recv, unpack_qkv_recv

        h3sa, geo, hl = self.h3sa, self.geo, self.hl
        d, heads = CFG["head_dim"], CFG["heads"]
        src = self.merged if merged is None else merged

        def mark(i: int) -> None:
            if marks is not None:
                marks[i].record()

        def attention(fn) -> None:
            if attn_events is not None:
                attn_events[0].record()
            fn()
            if attn_events is not None:
                attn_events[1].record()

        mark(0)
        if self.fused:
            # prologue + Q to the owners' planes + K/V into the owners' caches after the history
            qkv_norm_rope_scatter_paged(src, self.q_weight, self.k_weight, self.cos_sin,
                                        self.positions, 1e-5, q=self.q_buf, key_pool=self.k_buf,
                                        value_pool=self.v_buf, page_table=self.table,
                                        dst_start=self.n_hist, device_error=self.err)
            mark(1)
            if self.world > 1:
                self.peer_barrier()
            mark(2)
            if self.world > 1:
                attention(lambda: attention_fwd_scatter(
                    self.q_buf.tensor, self.kpool, self.vpool, self.table, self.problems,
                    self.scale, self.out_buf, device_error=self.err))
            else:
                attention(lambda: h3sa.attention_fwd(
                    self.q_buf.tensor, self.out, self.kpool, self.vpool, self.table,
                    self.problems, self.scale, device_error=self.err))
            mark(3)
            if self.world > 1:
                self.peer_barrier()
            mark(4)
            return self.out_buf.tensor if self.world > 1 else self.out
        qkv_norm_rope_pack(src, self.q_weight, self.k_weight, self.cos_sin, self.positions, 1e-5,
                           world=self.world, send=self.send)
        mark(1)
        torch.distributed.all_to_all_single(self.recv, self.send)
        mark(2)
        unpack_qkv_recv(self.recv, self.qkv, world=self.world, tokens=geo["tokens"],
                        local_heads=hl, head_dim=d)
        mark(3)
        q, k, v = self.qkv[0], self.qkv[1], self.qkv[2]
        # current chunk's K/V rows (media + pad document) after the history
        h3sa.kv_copy_rows([k, v], [self.kpool, self.vpool], count=geo["rows"],
                          dst_table=self.table, dst_start=self.n_hist, device_error=self.err)
        mark(4)
        attention(lambda: h3sa.attention_fwd(q, self.out, self.kpool, self.vpool, self.table,
                                             self.problems, self.scale, device_error=self.err))
        mark(5)
        torch.distributed.all_to_all_single(self.orecv, self.out)
        mark(6)
        unpack_o_recv(self.orecv, self.final, world=self.world, tokens=geo["tokens"],
                      local_heads=hl, head_dim=d)
        mark(7)
        return self.final

    def close(self) -> None:
        if self.world > 1:
            for b in (self.k_buf, self.v_buf, self.q_buf, self.out_buf):
                b.close()
            self.peer_barrier.close()


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


VARIANTS = ("fp8", "sparse", "480p", "feeders", "w8a8", "sol", "sol_hook")


def w8a8_projection(peaks: dict, iters: int = 20) -> dict:
    """The W8A8 QKV projection in front of the attention at the 768p SP=8 per-GPU shape: 1568
    tokens x 5376 hidden -> 9216 (3 x 24 heads x 128), the reference's int8 path
    (T/inference/w8a8.py:190-221): per-token activation quantisation + scaled int8 GEMM. Timed:
    the GEMM alone, the whole cutlass_w8a8_linear drop-in, and torch's bf16 matmul (cuBLAS)
    of the same shape for scale. Ops = 2 * M * N * K. Peak: 2 x the measured bf16 figure
    (no measured int8 peak; nominal dense int8 4.5 POPS)."""

    from h3sa.w8a8 import cutlass_w8a8_linear, quantize_int8_rows, quantize_weight, w8a8_gemm

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(13)
    m, k, n = 1568, 5376, 9216
    x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    wq, ws = quantize_weight(w)
    qa, sa = quantize_int8_rows(x)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ops = 2.0 * m * n * k
    ms_gemm = _time_launch(lambda: w8a8_gemm(qa, sa, wq, ws, out), iters)
    ms_linear = _time_launch(lambda: cutlass_w8a8_linear(x, wq, ws), iters)
    ms_quant = _time_launch(lambda: quantize_int8_rows(x), iters)
    wt = w.t()
    ms_bf16 = _time_launch(lambda: torch.matmul(x, wt), iters)
    peak = 2 * peaks["bf16"]
    tops = ops / (ms_gemm * 1e-3) / 1e12
    return {"w8a8_qkv_768p_sp8_per_gpu": {
        "m": m, "n": n, "k": k, "gemm_ms": ms_gemm, "gemm_tops": tops,
        "linear_ms": ms_linear, "activation_quant_ms": ms_quant,
        "cublas_bf16_ms": ms_bf16, "cublas_bf16_tflops": ops / (ms_bf16 * 1e-3) / 1e12,
        "speedup_vs_bf16": ms_bf16 / ms_linear,
        "roofline": {"bound": "tensor", "peak": peak, "frac": tops / peak,
                     "peak_source": "2 x measured bf16 burst (no measured int8 peak)"},
        "reference_path_on_b200": "vLLM cutlass_scaled_mm refuses int8 on SM100"}}


def feeders(peaks: dict, iters: int = 20) -> dict:
    """Device time and HBM throughput of the kernels that feed the attention, at the shapes
    of the benchmark's configurations (algorithmic bytes: every byte read and written once):

    * prologue_scatter_768p_sp1: the fused QK-RMSNorm + RoPE prologue storing Q into the
      attention plane and K/V into the paged cache, from the raw 12544-row x 24-head merged
      projection (read 231 MB, write 231 MB);
    * prologue_in_place_768p: the drop-in in-place prologue (Q/K read and written: 154 MB each);
    * cache_append_768p: the current chunk's K/V rows into the paged cache (154 MB each way);
    * fp8_parts_1080p: per-part e4m3 quantisation of the current chunk's K and V at the 1080p
      per-GPU shape (24605 rows x 3 heads; amax pass + quantise pass: read 2 x 37.8 MB,
      write 18.9 MB);
    * composite_mask_768p_sp8: the block-sparse mask for 3 heads of the 768p chunk (block
      means of Q and K, scores, selection)."""

    import h3sa
    from h3sa.block_sparse import composite_block_mask
    from h3sa.kernels import PAGE_ROWS, quantize_fp8_rows
    from h3sa.peer import LocalBuffer
    from h3sa.prologue import fused_qkv_qk_norm_rope_, qkv_norm_rope_scatter_paged

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(11)
    heads, d, nh = CFG["heads"], CFG["head_dim"], CFG["history"]
    geo = _geometry(1)
    rows = geo["rows"]
    hbm = peaks["hbm"]
    out = {}

    def entry(name: str, ms: float, nbytes: float, **extra) -> None:
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": ms, "bytes": nbytes, "gb_s": gbs, "frac_of_hbm": gbs / hbm, **extra}

    merged = torch.randn(rows, 3 * heads * d, device=dev, generator=g).to(torch.bfloat16)
    w = torch.ones(d, dtype=torch.bfloat16, device=dev)
    cs = _rope_cache(nh + rows, 96, dev)
    pos = nh + torch.arange(rows, device=dev)
    pages = (nh + rows + PAGE_ROWS - 1) // PAGE_ROWS
    table = torch.arange(pages, dtype=torch.int32, device=dev)
    kp = LocalBuffer(torch.zeros(heads, pages * PAGE_ROWS, d, dtype=torch.bfloat16, device=dev))
    vp = LocalBuffer(torch.zeros_like(kp.tensor))
    qb = LocalBuffer(torch.zeros(rows, heads, d, dtype=torch.bfloat16, device=dev))
    ms = _time_launch(lambda: qkv_norm_rope_scatter_paged(
        merged, w, w, cs, pos, 1e-5, q=qb, key_pool=kp, value_pool=vp, page_table=table,
        dst_start=nh), iters)
    entry("prologue_scatter_768p_sp1", ms, 2.0 * merged.numel() * 2)
    work = merged.clone()
    ms = _time_launch(lambda: fused_qkv_qk_norm_rope_(work, w, w, cs, pos, 1e-5), iters)
    entry("prologue_in_place_768p", ms, 2.0 * 2 * rows * heads * d * 2)
    k = torch.randn(rows, heads, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn_like(k)
    ms = _time_launch(lambda: h3sa.kv_copy_rows([k, v], [kp.tensor, vp.tensor], count=rows,
                                                dst_table=table, dst_start=nh), iters)
    entry("cache_append_768p", ms, 2.0 * 2 * k.numel() * 2)
    del merged, work, k, v, kp, vp, qb
    torch.cuda.empty_cache()

    n8, h8 = 24480 + 125, 3
    k = torch.randn(n8, h8, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn_like(k)
    p8 = (n8 + PAGE_ROWS - 1) // PAGE_ROWS
    t8 = torch.arange(p8, dtype=torch.int32, device=dev)
    k8 = torch.zeros(h8, p8 * PAGE_ROWS, d, dtype=torch.float8_e4m3fn, device=dev)
    v8 = torch.zeros_like(k8)
    sc = torch.empty(2, h8, dtype=torch.float32, device=dev)
    ws = torch.empty(2 * h8, dtype=torch.int32, device=dev)
    ms = _time_launch(lambda: quantize_fp8_rows([k, v], [k8, v8], [sc[0], sc[1]], ws, count=n8,
                                                dst_table=t8, zero_tail=True), iters)
    entry("fp8_parts_1080p", ms, 2.0 * k.numel() * 2 * 2 + 2.0 * k.numel())
    del k, v, k8, v8
    torch.cuda.empty_cache()

    import types

    h3, nq = 3, geo["nq"]
    nk = nh + nq
    q = torch.randn(nq, h3, d, device=dev, generator=g).to(torch.bfloat16)
    kk = torch.randn(nk, h3, d, device=dev, generator=g).to(torch.bfloat16)
    pk = (nk + PAGE_ROWS - 1) // PAGE_ROWS
    tk = torch.arange(pk, dtype=torch.int32, device=dev)
    kpool = torch.zeros(h3, pk * PAGE_ROWS, d, dtype=torch.bfloat16, device=dev)
    h3sa.kv_copy_rows([kk], [kpool], count=nk, dst_table=tk)
    qa = torch.zeros((nq + PAGE_ROWS - 1) // PAGE_ROWS, dtype=torch.uint8, device=dev)
    qa[CFG["video"] // PAGE_ROWS:] = 1
    ka = torch.zeros(pk, dtype=torch.uint8, device=dev)
    ka[(nh + CFG["video"]) // PAGE_ROWS:] = 1
    paged = types.SimpleNamespace(key=kpool, table=tk)
    ms = _time_launch(lambda: composite_block_mask(q, paged, q_lo=0, q_hi=nq, n_hist=nh, n_kv=nk,
                                                   q_block_audio=qa, kv_block_audio=ka,
                                                   density=0.25), iters)
    entry("composite_mask_768p_sp8", ms, float(q.numel() * 2 + nk * h3 * d * 2))
    return out


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
    if only == "feeders":
        return {"feeders": feeders(peaks, iters)}
    if only == "w8a8":
        return w8a8_projection(peaks, iters)
    if only == "sol":
        return _variant_sol(peaks, iters, dev, g)
    if only == "sol_hook":
        return {"sol_768p_hook_24h": _sol_hook(dev, g, iters)}
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
    out["fp8_segmented_step_1080p_per_gpu"] = _fp8_step(q, k, v, kp, vp, table, nh, iters, dev)
    return out


def _fp8_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kp: torch.Tensor,
              vp: torch.Tensor, table: torch.Tensor, nh: int, iters: int,
              dev: torch.device) -> dict:
    """One layer call of the segmented FP8 backend against the bf16 one at the same shape.

    The history is four committed chunks of nh / 4 rows, each an e4m3 part quantised once at
    commit with its own scales (not timed: it happens once per commit, not per call). Timed
    per call, FP8: the current chunk's K/V as a new part (amax + quantise into block-aligned
    e4m3 pages), Q quantised per head, one attention launch over the parts. bf16: the current
    K/V rows appended to the bf16 cache, one attention launch."""

    import h3sa
    from h3sa.kernels import PAGE_ROWS, attention_fwd_fp8_parts, quantize_fp8_rows

    d = CFG["head_dim"]
    nq, heads = int(q.shape[0]), int(q.shape[1])
    parts = [nh // 4] * 4 + [nq]
    starts, cursor = [], 0
    for n in parts:
        starts.append(cursor)
        cursor = (cursor + n + PAGE_ROWS - 1) // PAGE_ROWS * PAGE_ROWS
    pages8 = cursor // PAGE_ROWS
    t8 = torch.arange(pages8, dtype=torch.int32, device=dev)
    k8 = torch.zeros(heads, pages8 * PAGE_ROWS, d, dtype=torch.float8_e4m3fn, device=dev)
    v8 = torch.zeros_like(k8)
    ks = torch.empty(len(parts), heads, dtype=torch.float32, device=dev)
    vs = torch.empty_like(ks)
    work = torch.empty(2 * heads, dtype=torch.int32, device=dev)
    block_part = torch.zeros(pages8, dtype=torch.int32)
    for i, (s0, n) in enumerate(zip(starts, parts)):
        for b in range(s0 // PAGE_ROWS, (s0 + n + PAGE_ROWS - 1) // PAGE_ROWS):
            block_part[b] = i | (min(PAGE_ROWS, s0 + n - b * PAGE_ROWS) << 16)
    block_part = block_part.to(dev)
    for i in range(4):  # history parts, quantised at their commits
        quantize_fp8_rows([k, v], [k8, v8], [ks[i], vs[i]], work, count=parts[i],
                          src_start=i * (nh // 4), dst_start=starts[i],
                          dst_table=t8, zero_tail=True)
    cur_k, cur_v = k[nh:].contiguous(), v[nh:].contiguous()
    o = torch.empty(nq, heads, d, dtype=torch.bfloat16, device=dev)
    probs8 = [h3sa.AttentionProblem(0, nq, 0, starts[-1] + nq)]
    scale = d ** -0.5

    def fp8_call() -> None:
        quantize_fp8_rows([cur_k, cur_v], [k8, v8], [ks[4], vs[4]], work, count=nq,
                          dst_start=starts[4], dst_table=t8, zero_tail=True)
        q8, qs = h3sa.quantize_fp8_e4m3_per_head(q.unsqueeze(0))
        attention_fwd_fp8_parts(q8[0], o, k8, v8, t8, probs8, scale, q_scale=qs[0],
                                block_part=block_part, part_k_scale=ks, part_v_scale=vs)

    probs = [h3sa.AttentionProblem(0, nq, 0, nh + nq)]

    def bf16_call() -> None:
        h3sa.kv_copy_rows([cur_k, cur_v], [kp, vp], count=nq, dst_table=table, dst_start=nh)
        h3sa.attention_fwd(q, o, kp, vp, table, probs, scale)

    ms8 = _time_launch(fp8_call, iters)
    ms16 = _time_launch(bf16_call, iters)
    q8, qs = h3sa.quantize_fp8_e4m3_per_head(q.unsqueeze(0))
    ms_attn = _time_launch(lambda: attention_fwd_fp8_parts(
        q8[0], o, k8, v8, t8, probs8, scale, q_scale=qs[0], block_part=block_part,
        part_k_scale=ks, part_v_scale=vs), iters)
    ms_plain_same_data = _time_launch(lambda: h3sa.attention_fwd(
        q8[0], o, k8, v8, t8, probs8, scale, q_scale=qs[0], k_scale=ks[0].contiguous(),
        v_scale=vs[0].contiguous()), iters)
    ms_kv = _time_launch(lambda: quantize_fp8_rows([cur_k, cur_v], [k8, v8], [ks[4], vs[4]], work,
                                                   count=nq, dst_start=starts[4], dst_table=t8,
                                                   zero_tail=True), iters)
    ms_q = _time_launch(lambda: h3sa.quantize_fp8_e4m3_per_head(q.unsqueeze(0)), iters)
    flops = 4.0 * nq * (nh + nq) * d * heads
    return {"fp8_ms": ms8, "bf16_ms": ms16, "speedup": ms16 / ms8,
            "fp8_parts": {"attention_ms": ms_attn, "kv_part_quant_ms": ms_kv, "q_quant_ms": ms_q,
                          "one_scale_kernel_same_data_ms": ms_plain_same_data},
            "fp8_tflops": flops / (ms8 * 1e-3) / 1e12, "bf16_tflops": flops / (ms16 * 1e-3) / 1e12,
            "history_parts": 4, "queries": nq, "keys": nh + nq, "heads": heads}


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


def _variant_sol(peaks: dict, iters: int, dev: torch.device, g: torch.Generator) -> dict:
    """SOL-Attn at 768p (12509 media queries; keys = the chunk's 12509 rows as the exact sink,
    then 16384 history rows routed, tau 1.0 as the FL2AV runtime's default), for the SP=8
    per-GPU shape (3 heads) and one GPU (24 heads), against this repo's dense kernel over the
    same keys. Keys are drawn around per-64-row-block centres (N(0,1) centres, N(0, 0.6^2)
    rows) so that the routing has something to select. `mma_tflops` counts the tensor-core
    work the attention kernel issues (per item: S = Q K^T and O += P V at M = 128, N / K = 64);
    `dense_equiv_tflops` counts the dense attention the call replaces."""

    import h3sa
    from h3sa.kernels import PAGE_ROWS
    from h3sa.sol_attention import sol_attn_rectangular

    d = CFG["head_dim"]
    nq, nh = CFG["video"] + CFG["audio"], CFG["history"]
    nk = nq + nh
    kb = (nk + 63) // 64
    out = {}
    for heads in (3, 24):
        q = torch.randn(nq, heads, d, device=dev, generator=g).to(torch.bfloat16)
        centre = torch.randn(kb, heads, d, device=dev, generator=g)
        k = (0.6 * torch.randn(nk, heads, d, device=dev, generator=g)
             + centre.repeat_interleave(64, 0)[:nk]).to(torch.bfloat16)
        v = torch.randn(nk, heads, d, device=dev, generator=g).to(torch.bfloat16)
        qb = (nq + 63) // 64
        mask = torch.empty(heads, qb, (kb + 31) // 32, dtype=torch.int32, device=dev)
        tele = torch.zeros(4, dtype=torch.int64, device=dev)
        sol_attn_rectangular(q, k, v, scale=d ** -0.5, tau=1.0, sink_tokens=nq,
                             telemetry_counts=tele, exact_blocks=mask)
        ms = _time_launch(lambda: sol_attn_rectangular(q, k, v, scale=d ** -0.5, tau=1.0,
                                                       sink_tokens=nq, exact_blocks=mask), iters)
        # items per (128-row tile, head): chunks holding an approximate block for either half,
        # plus the union of the two halves' exact blocks
        bits = ((mask.view(torch.int32).unsqueeze(-1) >> torch.arange(32, device=dev)) & 1)
        bits = bits.reshape(heads, qb, -1)[:, :, :kb].bool()
        exist = torch.ones(heads, qb + qb % 2, 1, dtype=torch.bool, device=dev)
        if qb % 2:  # the last tile's second half has no query block: no items of its own
            bits = torch.cat((bits, torch.zeros_like(bits[:, :1])), 1)
            exist[:, -1] = False
        ex = bits.reshape(heads, -1, 2, kb)
        union = ex.any(2)
        approx_any = ((~ex) & exist.reshape(heads, -1, 2, 1)).any(2)
        chunks = torch.nn.functional.pad(approx_any, (0, (-kb) % 64)).reshape(heads, -1, (kb + 63) // 64, 64).any(-1)
        items = int(union.sum().item()) + int(chunks.sum().item())
        mma_flops = items * 4.0 * 128 * 64 * d
        dense_flops = 4.0 * nq * nk * d * heads
        t = tele.tolist()
        pages = (nk + PAGE_ROWS - 1) // PAGE_ROWS
        table = torch.arange(pages, dtype=torch.int32, device=dev)
        kp = torch.zeros(heads, pages * PAGE_ROWS, d, dtype=torch.bfloat16, device=dev)
        vp = torch.zeros_like(kp)
        h3sa.kv_copy_rows([k, v], [kp, vp], count=nk, dst_table=table)
        o = torch.empty(nq, heads, d, dtype=torch.bfloat16, device=dev)
        probs = [h3sa.AttentionProblem(0, nq, 0, nk)]
        dense_ms = _time_launch(lambda: h3sa.attention_fwd(q, o, kp, vp, table, probs, d ** -0.5),
                                iters)
        mma_tf = mma_flops / (ms * 1e-3) / 1e12
        out[f"sol_768p_{heads}h"] = {
            "ms": ms, "dense_kernel_ms": dense_ms, "speedup_vs_dense": dense_ms / ms,
            "routed_fraction": t[0] / max(1, t[2]), "exact_fraction": t[1] / max(1, t[3]),
            "items": items, "mma_tflops": mma_tf,
            "dense_equiv_tflops": dense_flops / (ms * 1e-3) / 1e12, "heads": heads,
            "queries": nq, "keys": nk, "sink_tokens": nq, "tau": 1.0,
            "roofline": {"bound": "tensor", "peak": peaks["bf16"], "frac": mma_tf / peaks["bf16"],
                         "note": "whole call (summaries, statistics, routing, attention)"}}
        del kp, vp, k, v, q
        torch.cuda.empty_cache()
    out["sol_768p_hook_24h"] = _sol_hook(dev, g, iters)
    return out


def _sol_hook(dev: torch.device, g: torch.Generator, iters: int) -> dict:
    """The drop-in path at 768p on one GPU (24 heads): a NOISY call of the hook at a routed
    layer with the `sol_attn` backend (K/V gathered in the reference's part order, SOL over
    the history video, condition rows dense) against the same call with the dense backend.
    History: 4 committed blocks of 125 audio + 3971 video rows; the call: 64 text, 125 audio,
    12384 video rows."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode

    heads, d, layer = 24, CFG["head_dim"], "blocks.2.attn"
    block_tags = tuple([2] * 125 + [0] * 3971)
    n_text, n_audio, n_video = 64, CFG["audio"], CFG["video"]
    seq = n_text + n_audio + n_video
    tags = torch.tensor([1] * n_text + [2] * n_audio + [0] * n_video, device=dev)
    commit = tags != 1
    q = torch.randn(seq, heads, d, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(seq, heads, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(seq, heads, d, device=dev, generator=g).to(torch.bfloat16)

    class Attn:
        softmax_scale = d ** -0.5

    res = {}
    for backend in ("sol_attn", "sdpa"):
        cache = CleanAVKVCache(KVContract(local_heads=heads, head_dim=d), layer_names=(layer,))
        paged = cache.layer(layer, dev)
        n_hist = 4 * len(block_tags)
        centre = torch.randn((n_hist + 63) // 64, heads, d, device=dev, generator=g)
        hk = (0.6 * torch.randn(n_hist, heads, d, device=dev, generator=g)
              + centre.repeat_interleave(64, 0)[:n_hist]).to(torch.bfloat16)
        hv = torch.randn(n_hist, heads, d, device=dev, generator=g).to(torch.bfloat16)
        paged.write(hk, hv, start=0, count=n_hist)
        paged.history_rows = n_hist
        for _ in range(4):
            cache._commit_token_counts.append(len(block_tags))
            cache._commit_token_tags.append(block_tags)
        hook = H3StreamingAttentionHook(cache, attention_backend=backend)
        hook.activate(HookMode.NOISY)
        call = lambda: hook(attention=Attn(), layer_name=layer, query=q, key=k, value=v,  # noqa: E731
                            token_tags=tags, commit_mask=commit, cu_seqlens_host=(0, seq))
        res[backend] = _time_launch(call, iters)
        hook.deactivate()
        hook.check_device_error()
        del cache, paged, hk, hv
        torch.cuda.empty_cache()
    return {"sol_ms": res["sol_attn"], "dense_ms": res["sdpa"],
            "speedup": res["sdpa"] / res["sol_attn"], "heads": heads, "queries": seq,
            "history": 4 * len(block_tags), "tau": 1.0,
            "note": "whole hook call: K/V gather, SOL (or dense) attention, condition rows"}


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
    q = step.q_buf.tensor[:nq]  # the step has run: Q and the chunk's K/V rows are in place
    hist_k = step.kpool[:, :nh].transpose(0, 1).contiguous()
    hist_v = step.vpool[:, :nh].transpose(0, 1).contiguous()
    cur_k = step.kpool[:, nh:nh + nq].transpose(0, 1).contiguous()
    cur_v = step.vpool[:, nh:nh + nq].transpose(0, 1).contiguous()

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


def _copy_loop_ms(run, host_in: torch.Tensor, out_shape, steps: int, world: int,
                  device: torch.device) -> float:
    """ms per step of `run(dev_in) -> result` with the step's input uploaded from pinned host
    memory and its result downloaded into pinned host memory every step, all inside the
    timed region. Copies run on their own streams, double-buffered: the upload of step i + 1
    and the download of step i - 1 overlap the compute of step i."""

    host_out = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev_in = [torch.empty(host_in.shape, dtype=host_in.dtype, device=device) for _ in range(2)]
    dev_out = [torch.empty(out_shape, dtype=torch.bfloat16, device=device) for _ in range(2)]
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = {name: [torch.cuda.Event() for _ in range(2)]
          for name in ("in_ready", "in_free", "out_ready", "out_free")}

    def one(i: int) -> None:
        k = i % 2
        h2d.wait_event(ev["in_free"][k])      # compute of step i - 2 is done with dev_in[k]
        with torch.cuda.stream(h2d):
            dev_in[k].copy_(host_in, non_blocking=True)
            ev["in_ready"][k].record(h2d)
        comp.wait_event(ev["in_ready"][k])
        res = run(dev_in[k])
        ev["in_free"][k].record(comp)
        comp.wait_event(ev["out_free"][k])    # download of step i - 2 is done with dev_out[k]
        dev_out[k].copy_(res.reshape(out_shape), non_blocking=True)
        ev["out_ready"][k].record(comp)
        d2h.wait_event(ev["out_ready"][k])
        with torch.cuda.stream(d2h):
            host_out[k].copy_(dev_out[k], non_blocking=True)
            ev["out_free"][k].record(d2h)

    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    _barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(comp)
    h2d.wait_stream(comp)
    for i in range(steps):
        one(i)
    b.record(d2h)
    torch.cuda.synchronize()
    _barrier(world)
    return _max_over_ranks(a.elapsed_time(b), world) / steps


TEXT_ROWS = 64  # the live document's text condition rows (the hook protocol requires some)


def _e2e_hook(step: Step, steps: int, world: int, rank: int, device: torch.device) -> dict:
    """The drop-in path a maintainer installs, end to end: this rank's raw QKV projection shard
    from pinned host memory -> h3sa.layer.attention_from_projection (fused_qkv_qk_norm_rope_,
    Ulysses sequence -> heads, H3StreamingAttentionHook.__call__ writing the chunk into its
    paged cache and attending, heads -> sequence) -> the out_proj input back to pinned host
    memory. Packed sequence [64 text | 12384 video + 125 audio | pad]: the hook's live
    document needs condition rows."""

    from h3sa.cache import CleanAVKVCache, KVContract
    from h3sa.hook import H3StreamingAttentionHook, HookMode
    from h3sa.layer import PeerUlysses, attention_from_projection
    from h3sa.ulysses import ParallelContext

    heads, d, nh = CFG["heads"], CFG["head_dim"], CFG["history"]
    hl = heads // world
    nq = CFG["video"] + CFG["audio"]
    used = TEXT_ROWS + nq
    align = CFG["align"] * world // _gcd(CFG["align"], world)
    rows = (used + align - 1) // align * align
    tokens = rows // world
    g = torch.Generator(device=device).manual_seed(2000 + rank)
    merged = torch.randn(tokens, 3 * heads * d, device=device, generator=g).to(torch.bfloat16)
    host_in = merged.cpu().pin_memory()
    cos_sin = _rope_cache(nh + rows, 96, device)
    positions = nh + rank * tokens + torch.arange(tokens, device=device)
    tags = torch.zeros(rows, dtype=torch.long, device=device)
    tags[:TEXT_ROWS] = 1
    tags[TEXT_ROWS + CFG["video"]:used] = 2
    tags[used:] = -1
    commit = torch.zeros(rows, dtype=torch.bool, device=device)
    commit[TEXT_ROWS:used] = True
    cu = (0, used, rows)
    cache = CleanAVKVCache(KVContract(local_heads=hl, head_dim=d), layer_names=("blocks.0.attn",),
                           device=device)
    paged = cache.layer("blocks.0.attn", device)
    hist = torch.randn(nh, hl, d, device=device, generator=g).to(torch.bfloat16)
    paged.write(hist, hist, start=0, count=nh)
    paged.history_rows = nh
    hook = H3StreamingAttentionHook(cache)
    hook.activate(HookMode.NOISY)

    class Attn:
        softmax_scale = d ** -0.5

    ulysses: dict = {}
    exchange = None
    if world > 1:
        exchange = PeerUlysses(tokens, heads, d, device_error=hook.device_error(device))
        ulysses["exchange"] = exchange

    def run(x: torch.Tensor) -> torch.Tensor:
        return attention_from_projection(
            x, q_weight=step.q_weight, k_weight=step.k_weight, rope_cache=(cos_sin, positions),
            eps=1e-5, num_heads=heads, head_dim=d, hook=hook, attention=Attn(),
            layer_name="blocks.0.attn", token_tags=tags, commit_mask=commit, cu_seqlens_host=cu,
            **ulysses)

    ms = _copy_loop_ms(run, host_in, (tokens, heads * d), steps, world, device)
    hook.check_device_error()
    if exchange is not None:
        exchange.close()
    flops = 4.0 * d * heads * (nq * (nh + nq + TEXT_ROWS) + TEXT_ROWS ** 2 + (rows - used) ** 2)
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
            "d2h_bytes_per_step": tokens * heads * d * 2,
            "api": "h3sa.layer.attention_from_projection: fused_qkv_qk_norm_rope_ -> Ulysses "
                   + ("peer exchange" if world > 1 else "(SP=1: none)")
                   + " -> H3StreamingAttentionHook.__call__ -> heads_to_sequence",
            "workload": f"{TEXT_ROWS} text + {nq} media queries per layer call (media over "
                        f"[{nh} history | media | text] keys), raw QKV projection in, out_proj "
                        "input out",
            "copies": "pinned host buffers, double-buffered on separate H2D / D2H streams"}


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
              for j, name in enumerate(step.phases)}
    step_ms = [a.elapsed_time(b) for a, b in step_ev]
    attn_avg = _max_over_ranks(sum(attn_ms) / len(attn_ms), world)
    p50 = _max_over_ranks(statistics.median(step_ms), world)
    p90 = _max_over_ranks(sorted(step_ms)[int(0.9 * (len(step_ms) - 1))], world)
    err = int(step.err.item())

    # e2e: the drop-in hook path with host buffers (headline), and the kernel-level step of
    # the timed region with the same copies
    e2e = e2e_kernels = None
    if not args.no_e2e:
        e2e = _e2e_hook(step, args.steps, world, rank, device)
        host_in = step.merged.cpu().pin_memory()
        res = step.run()
        ms = _copy_loop_ms(lambda x: step.run(merged=x), host_in, tuple(res.shape), args.steps,
                           world, device)
        total_flops = 4.0 * step.geo["nq"] * step.geo["nk"] * CFG["head_dim"] * CFG["heads"]
        e2e_kernels = {"value": total_flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                       "ms_per_step": ms,
                       "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
                       "d2h_bytes_per_step": res.numel() * res.element_size(),
                       "api": "the timed step's C-ABI calls (fused prologue/exchange/cache "
                              "append, attention) with host buffers"}

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
    clk = clocks.summary()
    if clk.get("sm_mhz"):
        # time x clock: a kernel bound by the SM clock keeps this product as the clock moves
        clk["attention_ms_x_sm_mhz"] = attn_avg * clk["sm_mhz"]
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
                        "current] keys, H=24, d=128, dense non-causal; each step starts from "
                        "the raw merged QKV projection (QK-RMSNorm + RoPE prologue included)",
            "ulysses_sp": world, "heads_per_gpu": step.hl, "packed_rows": geo["rows"],
            "pad_rows": geo["pad"], "parallelism": f"sp{world}",
            "exchange": ("peer stores over NVLink (prologue kernel storing Q and K/V into "
                         "the owners' planes and caches, attention epilogue storing O)"
                         if step.fused and world > 1
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
        "e2e_kernel_path": e2e_kernels,
        "gpu_launches": step.launches_per_step * args.steps,
        "clocks": clk,
        "device_error": err,
        **extra,
    }
    print(json.dumps(line), flush=True)


def run_tp2sp4(args: argparse.Namespace) -> None:
    """The 1080p FP8 configuration in its TP2 x SP4 layout on 8 GPUs (T/runtime/direct.py:
    169-190): TP rank t owns 12 of the 24 heads; its Ulysses group {t, t+2, t+4, t+6} trades
    sequence rows for heads, 3 heads per GPU. Per step and rank: the fused RMSNorm + RoPE +
    e4m3 prologue (an amax pass over the media rows, the maxima reduced over the group, then Q
    and the chunk's K/V stored as e4m3 into the owners' plane and stores over NVLink, where
    the chunk's K/V form one part with its own per-head scales after the four history parts
    quantised at their commits; bf16 rows kept for the pad document); a peer barrier; one
    attention launch over the parts (the 35-row pad document attends to itself in bf16); the
    output all-to-all inside the group (NCCL) and its unpack. Timed with CUDA events, max over
    the 8 ranks. FLOPs: 4 * Nq * (Nh + Nq) * 128 per head."""

    import h3sa
    from h3sa.kernels import PAGE_ROWS, attention_fwd_fp8_parts, quantize_fp8_rows
    from h3sa.peer import PeerBarrier, PeerBuffer, PeerGroupMax
    from h3sa.prologue import qkv_norm_rope_scatter_fp8
    from h3sa.ulysses import build_parallel_context, unpack_o_recv

    world, rank, local = _dist()
    if world != 8:
        raise SystemExit("--layout tp2sp4 runs on 8 GPUs (torchrun --nproc-per-node 8)")
    dev = torch.device("cuda", local)
    ctx = build_parallel_context(2, 4)
    group, sp, ur = ctx.ulysses_group, ctx.ulysses_world_size, ctx.ulysses_rank
    d, heads_tp, nh, nq = 128, 12, 32768, 24480 + 125
    hl = heads_tp // sp
    align = 64 * sp // _gcd(64, sp)
    rows = (nq + align - 1) // align * align
    tokens = rows // sp
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    merged = torch.randn(tokens, 3 * heads_tp * d, device=dev, generator=g).to(torch.bfloat16)
    gw = torch.Generator(device=dev).manual_seed(99)
    wq = (1 + 0.05 * torch.randn(d, device=dev, generator=gw)).to(torch.bfloat16)
    wk = (1 + 0.05 * torch.randn(d, device=dev, generator=gw)).to(torch.bfloat16)
    cos_sin = _rope_cache(nh + rows, 96, dev)
    positions = nh + ur * tokens + torch.arange(tokens, device=dev)
    pages = rows // PAGE_ROWS + 1
    table = torch.arange(pages, dtype=torch.int32, device=dev)
    q_buf = PeerBuffer((rows, hl, d), group)
    k_buf = PeerBuffer((hl, pages * PAGE_ROWS, d), group)
    v_buf = PeerBuffer((hl, pages * PAGE_ROWS, d), group)
    k_buf.tensor.zero_()
    v_buf.tensor.zero_()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    peer_barrier = PeerBarrier(group, device_error=err)
    group_max = PeerGroupMax(3 * heads_tp, group, device_error=err)
    # e4m3 store: four committed history parts of nh / 4 rows, then the chunk's part
    parts = [nh // 4] * 4 + [nq]
    starts, cursor = [], 0
    for n in parts:
        starts.append(cursor)
        cursor = (cursor + n + PAGE_ROWS - 1) // PAGE_ROWS * PAGE_ROWS
    t8 = torch.arange(cursor // PAGE_ROWS, dtype=torch.int32, device=dev)
    # e4m3 stores of every rank of the group (the chunk's part is written by its owner's peers)
    k8_buf = PeerBuffer((hl, cursor, d // 2), group)
    v8_buf = PeerBuffer((hl, cursor, d // 2), group)
    q8_buf = PeerBuffer((rows, hl, d // 2), group)
    for buf in (k8_buf, v8_buf, q8_buf):
        buf.tensor.zero_()
    k8 = k8_buf.tensor.view(torch.float8_e4m3fn)
    v8 = v8_buf.tensor.view(torch.float8_e4m3fn)
    q8_plane = q8_buf.tensor.view(torch.float8_e4m3fn)
    # the scales cover the chunk's media rows, not the pad rows after them
    amax_rows = ((ur * tokens + torch.arange(tokens, device=dev)) < nq).to(torch.uint8)
    ks = torch.empty(len(parts), hl, dtype=torch.float32, device=dev)
    vs = torch.empty_like(ks)
    work = torch.empty(2 * hl, dtype=torch.int32, device=dev)
    block_part = torch.zeros(cursor // PAGE_ROWS, dtype=torch.int32)
    for i, (s0, n) in enumerate(zip(starts, parts)):
        for b in range(s0 // PAGE_ROWS, (s0 + n + PAGE_ROWS - 1) // PAGE_ROWS):
            block_part[b] = i | (min(PAGE_ROWS, s0 + n - b * PAGE_ROWS) << 16)
    block_part = block_part.to(dev)
    for i in range(4):
        hk = torch.randn(parts[i], hl, d, device=dev, generator=g).to(torch.bfloat16)
        hv = torch.randn(parts[i], hl, d, device=dev, generator=g).to(torch.bfloat16)
        quantize_fp8_rows([hk, hv], [k8, v8], [ks[i], vs[i]], work, count=parts[i],
                          dst_start=starts[i], dst_table=t8, zero_tail=True)
    out = torch.empty(rows, hl, d, dtype=torch.bfloat16, device=dev)
    orecv = torch.empty(sp, tokens, hl, d, dtype=torch.bfloat16, device=dev)
    final = torch.empty(tokens, heads_tp, d, dtype=torch.bfloat16, device=dev)
    P = h3sa.AttentionProblem
    scale = d ** -0.5
    phases = ("prologue_fp8_scatter", "barrier", "attention", "o_all_to_all", "o_unpack")

    def step(marks=None) -> None:
        def mark(i):
            if marks is not None:
                marks[i].record()

        mark(0)
        # RMSNorm + RoPE + e4m3: amax pass, group max over peer memory, then Q and the chunk's
        # K/V part as e4m3 into the owners' plane and stores (bf16 rows only for the pad
        # document, the rows the scales do not cover)
        qs, ks_c, vs_c = qkv_norm_rope_scatter_fp8(
            merged, wq, wk, cos_sin, positions, 1e-5, q8=q8_buf, key_pool8=k8_buf,
            value_pool8=v8_buf, page_table8=t8, dst8_start=starts[4], amax_rows=amax_rows,
            peer_max=group_max, q=q_buf, key_pool=k_buf, value_pool=v_buf, page_table=table,
            dst_start=0, bf16_unflagged_only=True, device_error=err)
        ks[4].copy_(ks_c)
        vs[4].copy_(vs_c)
        mark(1)
        peer_barrier()
        mark(2)
        attention_fwd_fp8_parts(q8_plane[:nq], out[:nq], k8, v8, t8, [P(0, nq, 0, starts[4] + nq)],
                                scale, q_scale=qs, block_part=block_part, part_k_scale=ks,
                                part_v_scale=vs, device_error=err)
        h3sa.attention_fwd(q_buf.tensor, out, k_buf.tensor, v_buf.tensor, table,
                           [P(nq, rows, nq, rows)], scale, device_error=err)
        mark(3)
        torch.distributed.all_to_all_single(orecv, out, group=group)
        mark(4)
        unpack_o_recv(orecv, final, world=sp, tokens=tokens, local_heads=hl, head_dim=d)
        mark(5)
        # no barrier before the next step's scatter into the peers' planes and pools: a rank
        # finishes its all-to-all only after every peer has sent, i.e. finished its attention

    for _ in range(args.warmup):
        step()
    t0, t1 = torch.cuda.Event(True), torch.cuda.Event(True)
    per = [[torch.cuda.Event(True) for _ in range(len(phases) + 1)] for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        _barrier(world)
        clocks.mark_start()
        t0.record()
        for i in range(args.steps):
            step(per[i])
        t1.record()
        _barrier(world)
        clocks.mark_stop()
    ms = _max_over_ranks(t0.elapsed_time(t1) / args.steps, world)
    phase_ms = {}
    for j, name in enumerate(phases):
        vals = sorted(per[i][j].elapsed_time(per[i][j + 1]) for i in range(args.steps))
        phase_ms[name] = _max_over_ranks(vals[len(vals) // 2], world)
    code = int(err.item())
    flops_gpu = 4.0 * nq * (nh + nq) * d * hl
    peaks = _peaks()
    attn_tf = flops_gpu / (phase_ms["attention"] * 1e-3) / 1e12
    torch.cuda.synchronize()
    _barrier(world)
    for b in (q_buf, k_buf, v_buf, q8_buf, k8_buf, v8_buf):
        b.close()
    group_max.close()
    peer_barrier.close()
    if rank == 0:
        line = {
            "metric": "chunk attention TFLOP/s (1080p FP8 e4m3, TP2 x SP4, 32k KV cache)",
            "value": flops_gpu * world / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic",
            "config": {"workload": "1080p FP8 chunk: 24480 video + 125 audio queries x [32768 "
                                   "history (4 e4m3 parts) + 24605 current] keys, 24 heads",
                       "parallelism": "tp2sp4", "heads_per_gpu": hl, "packed_rows": rows},
            "per_gpu_tflops": flops_gpu / (ms * 1e-3) / 1e12,
            "phases_p50_max_over_ranks_ms": phase_ms,
            "attention_tflops_per_gpu": attn_tf,
            "roofline": {"bound": "tensor", "peak": 2 * peaks["bf16"],
                         "frac": attn_tf / (2 * peaks["bf16"]),
                         "peak_source": "2 x measured bf16 burst (no measured e4m3 GEMM peak)"},
            "clocks": clocks.summary(),
            "device_error": code,
        }
        print(json.dumps(line), flush=True)


def run_out_proj(args: argparse.Namespace) -> None:
    """The attention's row-parallel out_proj over TP = world ranks (T/model/layers.py:441-443,
    T/distributed/linear.py:186-191) at the 768p TP2 x SP4 per-rank shape: 3136 sequence rows
    x (inner 3072 / TP) -> hidden 5376, bias-free. Three forms, each timed over --steps calls
    after --warmup (CUDA events, max over ranks): the fused PeerRowParallelLinear (partials
    stored into the peers' slots by the GEMM epilogue, peer barrier, slot reduce); the same
    tcgen05 GEMM + NCCL all-reduce; cuBLAS (torch.matmul) + NCCL all-reduce, the reference's
    structure. FLOPs per rank: 2 * rows * hidden * inner / TP."""

    from h3sa.linear import PeerRowParallelLinear, gemm_bf16

    world, rank, local = _dist()
    if world < 2:
        raise SystemExit("--layout out_proj runs on 2 or more GPUs (torchrun)")
    dev = torch.device("cuda", local)
    rows, inner, hidden = 3136, 3072, 5376
    loc = inner // world
    g = torch.Generator(device=dev).manual_seed(10 + rank)
    x = torch.randn(rows, loc, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(hidden, loc, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    fused = PeerRowParallelLinear(w, rows, device_error=err)
    wt = w.t()
    group = torch.distributed.group.WORLD

    def nccl_ours():
        out = gemm_bf16(x, w)
        torch.distributed.all_reduce(out, group=group)

    def nccl_cublas():
        out = torch.matmul(x, wt)
        torch.distributed.all_reduce(out, group=group)

    def timed(fn) -> float:
        for _ in range(args.warmup):
            fn()
        _barrier(world)
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        _barrier(world)
        return _max_over_ranks(a.elapsed_time(b) / args.steps, world)

    ms_fused = timed(lambda: fused(x))
    ms_ours = timed(nccl_ours)
    ms_cublas = timed(nccl_cublas)
    ms_gemm = timed(lambda: gemm_bf16(x, w))
    code = int(err.item())
    torch.cuda.synchronize()
    _barrier(world)
    fused.close()
    flops = 2.0 * rows * hidden * loc
    if rank == 0:
        peaks = _peaks()
        print(json.dumps({
            "metric": "row-parallel out_proj with TP all-reduce (768p TP2 x SP4 rank shape)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
            "config": {"rows": rows, "inner_per_rank": loc, "hidden": hidden, "tp": world},
            "ms": {"fused_peer_reduce": ms_fused, "tcgen05_gemm_plus_nccl": ms_ours,
                   "cublas_plus_nccl": ms_cublas, "gemm_alone": ms_gemm},
            "speedup_vs_cublas_nccl": ms_cublas / ms_fused,
            "gemm_tflops": flops / (ms_gemm * 1e-3) / 1e12,
            "gemm_frac_of_bf16_peak": flops / (ms_gemm * 1e-3) / 1e12 / peaks["bf16"],
            "nvlink_bytes_per_rank": rows * hidden * 2 * (world - 1),
            "device_error": code}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["h3sa", "reference"], default="h3sa")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-comparator", action="store_true")
    ap.add_argument("--unfused", action="store_true",
                    help="SP > 1: NCCL all-to-all + layout copies instead of peer stores")
    ap.add_argument("--no-variants", action="store_true",
                    help="skip the kernel-only FP8 1080p, block-sparse 768p and 480p timings")
    ap.add_argument("--layout", choices=["sp", "tp2sp4", "out_proj"], default="sp",
                    help="tp2sp4: the 1080p FP8 configuration in its TP2 x SP4 layout (8 GPUs); "
                         "out_proj: the row-parallel out_proj with its TP all-reduce (TP = GPUs)")
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
    elif args.layout == "tp2sp4":
        run_tp2sp4(args)
    elif args.layout == "out_proj":
        run_out_proj(args)
    else:
        run_h3sa(args)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
