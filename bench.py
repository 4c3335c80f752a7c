#!/usr/bin/env python
"""Benchmark of the KernelForge hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

Headline: the RMSNorm bf16 sweep, rows x hidden in
{4096, 32768, 262144} x {1024, 2048, 4096, 8192}. One STEP normalises all 12 sweep tensors
once (18.4 GB of HBM traffic in total, far above the 126 MB L2). ``value`` is the achieved HBM
GB/s of the whole job with inputs resident in HBM; ``e2e`` is the same metric through the
public API with the inputs copied from pinned host memory and the outputs copied back inside
the timed region (uploads, kernels and downloads pipelined on three streams).

Secondary workloads in the same line (``workloads``): SANA linear attention configs
(B=4,H=36,N=4096) and (B=2,H=70,N=16384), bf16 in/out, each step one ``qkv_attn_matmul`` call
per block (replayed from CUDA graphs); FlashAttention JVP (B=4,H=16,N=4096,D in {64,128}, bf16,
non-causal), each step the standalone ``flash_attention_jvp`` (TFLOP/s over 5 GEMMs) or the
one-pass ``flash_attention_fwd_jvp`` (6 GEMMs); FlashAttention backward on the same configs
(``_flash_attn_backward``, 5 GEMMs); RMSNorm backward at 32768 x 8192. ``--flash-attn-comparator``
also times flash_attn's own backward on the same tensors.

Multi-GPU (torchrun, one process per GPU): strong scaling over the partition BASELINE.json
names. Every configuration is the same global problem at every N; each rank computes its
contiguous share -- rows for RMSNorm, (batch, head) units for SANA and FlashAttention, taken as
dense rectangles (kernelforge_b200.shard) copied out before the timed region -- with no
collective on the data path. ``value`` = the global algorithmic bytes or flops / the slowest
rank's device time. After the timed region NCCL gathers, to rank 0, bit digests of every
shard's output (RMSNorm, FlashAttention: compared bitwise with rank 0's unsharded run) or the
outputs themselves (SANA, whose schedule -- and so its fp32 summation order -- depends on the
shard's shape: compared within 2 ulps). The RMSNorm backward's weight gradient is a sum over
rows: its per-rank partials are summed with an NCCL all-reduce inside the timed step.

``--impl reference`` times the reference algorithm's CPU restatement (``oracle/``) on the
host cores on a bounded sample of the same workload (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from kernelforge_b200.shard import batch_head_blocks, row_shard  # noqa: E402

BASELINE_METRIC = "achieved HBM GB/s (RMSNorm, SANA-attn) & TFLOP/s (FA-JVP) vs B200 peak, 1–8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024
CHUNK_BYTES = 64 << 20  # e2e pipeline granularity for row-chunked copies

SWEEP_ROWS = (4096, 32768, 262144)
SWEEP_HIDDEN = (1024, 2048, 4096, 8192)
SANA_CONFIGS = (
    {"name": "sana_cfg1", "B": 4, "H": 36, "N": 4096, "D": 32},
    {"name": "sana_cfg2", "B": 2, "H": 70, "N": 16384, "D": 32},
    # One of the reference harness's own shapes (SANA test.py:184-186: batch 1, 2240 channels =
    # 70 heads, 4096 tokens): fewer heads than SMs, so the one-launch path runs in clusters.
    {"name": "sana_harness_b1h70", "B": 1, "H": 70, "N": 4096, "D": 32},
    # Config 1 with LiteLA's qk_norm applied inside the attention kernels (the per-token norm
    # statistics need every head of a token, so this line runs on one rank only).
    {"name": "sana_cfg1_qknorm", "B": 4, "H": 36, "N": 4096, "D": 32, "qk_norm": True},
)
PARALLELISM = ("strong scaling: rows (RMSNorm) and (batch, head) blocks (SANA, FlashAttention) split "
               "over {n} rank(s), no data-path collective; NCCL gathers output digests / outputs to "
               "rank 0 for verification after the timed region")

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from `ncu --set full`
# captures of the `--case ncu-small` shapes. RMSNorm: the 32768 x 8192 capture (536,926,976 read +
# 486,499,328 written) scaled by rows to the dominant 262144 x 8192 launch (x 8; every row is read
# once and written once, so traffic is linear in rows). SANA cfg1: the one-launch kernel of a call
# at the bench size itself (113,272,832 read + 7,127,808 written; most of the 37.7 MB output is
# still in L2 when the kernel ends). RMSNorm backward: its dx kernel at the bench size. All three
# are single-GPU figures: they apply to the N=1 line.
RMSNORM_NCU_TRAFFIC_BYTES = 8 * (536_926_976 + 486_499_328)
SANA_NCU_TRAFFIC_BYTES = {"sana_cfg1": 113_272_832 + 7_127_808}
RMSNORM_BWD_NCU_TRAFFIC_BYTES = 1_073_874_000 + 503_786_496


def sana_launches_per_call(B, H, N):
    """Kernel launches of one default-schedule qkv_attn_matmul call (bf16, head dim 32), as the
    library plans it on this device (kf_sana_linattn_plan)."""
    from kernelforge_b200.SANA_LinearAttention import QKVAttnMatmul

    return QKVAttnMatmul(B, H, 32, N, 1e-15, "bfloat16", "bfloat16").plan()[0]


# ---------------------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------------------
def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.enabled = self.world > 1

    def init(self):
        if self.enabled:
            torch.cuda.set_device(self.local_rank)
            torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=180),
                                                 device_id=torch.device("cuda", self.local_rank))
        else:
            torch.cuda.set_device(0)

    def barrier(self):
        if self.enabled:
            torch.distributed.barrier()

    def max(self, value: float) -> float:
        if not self.enabled:
            return value
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def all_gather(self, t: torch.Tensor):
        """Every rank's copy of a same-shaped CUDA tensor, in rank order."""
        if not self.enabled:
            return [t]
        out = [torch.empty_like(t) for _ in range(self.world)]
        torch.distributed.all_gather(out, t.contiguous())
        return out

    def all_gather_flat(self, t: torch.Tensor):
        """Every rank's 1-D CUDA tensor (lengths may differ; padded to the longest)."""
        if not self.enabled:
            return [t]
        n = torch.tensor([t.numel()], dtype=torch.int64, device=t.device)
        sizes = [int(x.item()) for x in self.all_gather(n)]
        padded = torch.zeros(max(sizes), dtype=t.dtype, device=t.device)
        padded[:t.numel()] = t
        return [g[:s] for g, s in zip(self.all_gather(padded), sizes)]

    def all_reduce_sum(self, t: torch.Tensor):
        if self.enabled:
            torch.distributed.all_reduce(t)

    def close(self):
        if self.enabled:
            torch.distributed.destroy_process_group()


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed regions run."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [line.strip().split(", ") for line in self.file.read().splitlines() if line.strip()]
        os.unlink(self.file.name)
        samples = []
        for r in rows:
            try:
                samples.append(dict(sm=float(r[1]), smax=float(r[2]), util=float(r[4]),
                                    hw=r[6] == "Active", hwt=r[7] == "Active", swt=r[8] == "Active",
                                    pcap=r[9] == "Active"))
            except (IndexError, ValueError):
                continue
        if not samples:
            return None
        loaded = [s for s in samples if s["util"] >= 50] or samples
        reasons = sorted({name for s in loaded for name, key in (("hw_slowdown", "hw"),
                          ("hw_thermal_slowdown", "hwt"), ("sw_thermal_slowdown", "swt"),
                          ("sw_power_cap", "pcap")) if s[key]})
        return {"sm_mhz": statistics.median(s["sm"] for s in loaded),
                "sm_max_mhz": max(s["smax"] for s in loaded), "reasons": reasons,
                "samples": len(samples), "samples_under_load": len([s for s in samples if s["util"] >= 50])}


def time_region(step, steps, warmup, dist, dominant=None):
    """Warm up, then time exactly `steps` calls of step(i) between barriers + synchronize.

    Returns (max-over-ranks ms per step, average ms of the dominant launch or None)."""
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if dominant is not None:
        dominant.clear()
    start.record()
    for i in range(steps):
        step(i)
    end.record()
    end.synchronize()
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(start.elapsed_time(end)) / steps
    # Every rank takes part in the max, also one without launches of its own (an idle rank of a
    # split that gives it no work), so that all ranks issue the same collectives.
    local = sum(a.elapsed_time(b) for a, b in dominant) / len(dominant) if dominant else 0.0
    dom = dist.max(local)
    return ms, (dom if dom > 0 else None)


class LaunchTimer(list):
    """Collects (start, end) CUDA event pairs around the dominant kernel's launches."""

    def around(self, fn):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        out = fn()
        b.record()
        self.append((a, b))
        return out


class Pipeline:
    """End-to-end transfers: host->device copies on one stream, the API calls on a second,
    device->host copies on a third, each waiting on the previous stage through stream events, so
    chunk i+1's upload and chunk i-1's download run while chunk i computes (PCIe is full duplex).
    Every step starts after the previous step's downloads and ends with the current stream
    waiting for its own downloads, so CUDA events on the current stream bracket the whole step."""

    def __init__(self):
        self.up, self.comp, self.down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    def begin(self):
        self.up.wait_stream(torch.cuda.current_stream())

    def chunk(self, uploads, compute, downloads):
        """uploads: [(device_view, pinned_host_view)]; compute() -> results on the compute stream;
        downloads(results) -> [(pinned_host_view, device_tensor)]."""
        with torch.cuda.stream(self.up):
            for dst, src in uploads:
                dst.copy_(src, non_blocking=True)
        self.comp.wait_stream(self.up)
        with torch.cuda.stream(self.comp):
            results = compute()
        self.down.wait_stream(self.comp)
        with torch.cuda.stream(self.down):
            for dst, src in downloads(results):
                dst.copy_(src, non_blocking=True)
                src.record_stream(self.down)

    def end(self):
        torch.cuda.current_stream().wait_stream(self.down)


def row_chunks(rows, hidden, elem=2):
    """[start, stop) row ranges of about CHUNK_BYTES each."""
    per = max(1, CHUNK_BYTES // (hidden * elem))
    return [(r, min(rows, r + per)) for r in range(0, rows, per)]


def pinned(shape_or_numel, dtype):
    return torch.empty(shape_or_numel, dtype=dtype, pin_memory=True)


def digest(t: torch.Tensor) -> torch.Tensor:
    """Two position-weighted sums of the raw bits of ``t`` (exact int64 arithmetic): equal
    digests mean equal bits, up to a negligible chance of collision. Chunked to bound memory."""
    flat = t.contiguous().view(-1)
    bits = flat.view({1: torch.int8, 2: torch.int16, 4: torch.int32}[flat.element_size()])
    out = torch.zeros(2, dtype=torch.int64, device=t.device)
    step = 1 << 25
    for s in range(0, bits.numel(), step):
        b = bits[s:s + step].to(torch.int64)
        idx = torch.arange(s, s + b.numel(), device=t.device, dtype=torch.int64)
        out[0] += (b * ((idx * 40503 + 7) % 32749 + 1)).sum()
        out[1] += (b * ((idx * 69069 + 3) % 32719 + 1)).sum()
    return out


def roofline(alg_bytes_or_flops, ms, peak, unit, bound, traffic=None):
    achieved = alg_bytes_or_flops / (ms / 1e3) / 1e9 if unit == "GB/s" else alg_bytes_or_flops / (ms / 1e3) / 1e12
    return {"bound": bound, "achieved": round(achieved, 1), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic}


def cpu_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def single_rank_verify():
    return {"ranks": 1, "ok": True, "method": "one rank holds the whole configuration"}


def verify_digests(dist, mine, reference_digests):
    """Gather every rank's digest tensor to rank 0 and compare it with the digests of the same
    slices of rank 0's unsharded run, reference_digests() -> one tensor per rank. Every rank
    takes the same collective steps; the unsharded run and the comparison are rank 0's alone."""
    gathered = dist.all_gather(mine)
    if dist.rank != 0:
        return None
    expected = reference_digests()
    bad = [r for r in range(dist.world) if not torch.equal(gathered[r], expected[r])]
    return {"ranks": dist.world, "ok": not bad, "method": "bitwise: NCCL-gathered output digests vs rank 0's "
            "unsharded run", "mismatched_ranks": bad}


# ---------------------------------------------------------------------------------------------
# RMSNorm sweep
# ---------------------------------------------------------------------------------------------
# --case ncu-small: one small configuration per workload for `ncu --set full` captures (inputs
# still larger than L2, a few GB on the device at most). Not a benchmark line.
SMALL = {"rows": (32768,), "hidden": (8192,)}
CASE = "full"


def sweep_points():
    if CASE == "ncu-small":
        return [(r, h) for r in SMALL["rows"] for h in SMALL["hidden"]]
    return [(r, h) for r in SWEEP_ROWS for h in SWEEP_HIDDEN]


def rmsnorm_bytes(rows, hidden):
    return 2 * rows * hidden * 2 + 2 * hidden


def rmsnorm_point(dev, index, rows, hidden):
    """The global input of one sweep point: the same on every rank (seeded by the point)."""
    gen = torch.Generator(device=dev).manual_seed(1234 + index)
    x = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=gen)
    w = (1 + 0.1 * torch.randn(hidden, device=dev, generator=gen)).to(torch.bfloat16)
    return x, w


def bench_rmsnorm(args, dist, peaks, peak_kind):
    from kernelforge_b200.rmsnorm import rms_norm, rmsnorm_forward, rmsnorm_into

    dev = torch.device("cuda", torch.cuda.current_device())
    points = sweep_points()
    xs, ws, ys, slices = [], [], [], []
    for i, (rows, hidden) in enumerate(points):
        x, w = rmsnorm_point(dev, i, rows, hidden)
        sl = row_shard(rows, dist.world, dist.rank)
        xs.append(x[sl].clone() if dist.world > 1 else x)
        ws.append(w)
        ys.append(torch.empty(sl.stop - sl.start, hidden, device=dev, dtype=torch.bfloat16))
        slices.append(sl)
        del x
    dominant_index = max(range(len(xs)), key=lambda j: xs[j].numel())
    timer = LaunchTimer()

    def step(_):
        for j, (x, w, y) in enumerate(zip(xs, ws, ys)):
            if j == dominant_index:
                timer.around(lambda: rmsnorm_into(x, w, y, 1e-6))
            else:
                rmsnorm_into(x, w, y, 1e-6)

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer)
    global_bytes = sum(rmsnorm_bytes(r, h) for r, h in points)
    value = global_bytes / (ms / 1e3) / 1e9
    dom_bytes = rmsnorm_bytes(*xs[dominant_index].shape)
    result = {
        "value": round(value, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "gpu_launches": len(xs) * args.steps,
        "roofline": roofline(dom_bytes, dom_ms, peaks["hbm_gbs"], "GB/s", "hbm",
                             RMSNORM_NCU_TRAFFIC_BYTES if dist.world == 1 else None),
        "roofline_note": f"dominant launch rmsnorm {xs[dominant_index].shape[0]}x{xs[dominant_index].shape[1]} "
                         f"bf16 (this rank's rows of 262144x8192), {dom_ms * 1e3:.1f} us avg; "
                         f"peak = {peak_kind} HBM copy GB/s",
        "shard": f"rows {[(s.start, s.stop) for s in slices[-1:]][0]} of each sweep tensor on rank {dist.rank}",
    }

    # Verification: bitwise digests of every rank's rows against rank 0's unsharded run.
    if dist.world > 1:
        mine = torch.stack([digest(y) for y in ys])

        def reference():
            per_rank = [[] for _ in range(dist.world)]
            for i, (rows, hidden) in enumerate(points):
                x, w = rmsnorm_point(dev, i, rows, hidden)
                y = rmsnorm_forward(x, w, 1e-6)
                for r in range(dist.world):
                    per_rank[r].append(digest(y[row_shard(rows, dist.world, r)]))
                del x, y
            return [torch.stack(d) for d in per_rank]

        result["verify"] = verify_digests(dist, mine, reference)
    else:
        result["verify"] = single_rank_verify()
    if not args.no_e2e:
        result["e2e"] = rmsnorm_e2e(args, dist, xs, ws, rms_norm, global_bytes)
    del xs, ys
    torch.cuda.empty_cache()
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = rmsnorm_cpu_baseline(seconds=args.cpu_seconds)
    return result


def rmsnorm_e2e(args, dist, xs, ws, rms_norm, global_bytes):
    """The rank's rows of every sweep tensor through the public API: pinned host -> device in
    ~64 MB row chunks, rms_norm(...)(X, Weight) per chunk, device -> pinned host, pipelined."""
    biggest = max(x.numel() for x in xs)
    try:
        host_in = pinned(biggest, torch.bfloat16)
        host_out = pinned(biggest, torch.bfloat16)
    except RuntimeError as exc:
        return {"value": None, "unit": "GB/s", "error": f"pinned host allocation failed: {exc}"}
    big = max(xs, key=lambda t: t.numel())
    host_in.copy_(big.view(-1))  # real input data in the pinned staging buffer
    dev_in = [torch.empty_like(x) for x in xs]
    plan = []  # per tensor: [(row0, row1, kernel)]
    for x in xs:
        rows, hidden = x.shape
        plan.append([(r0, r1, rms_norm(1, r1 - r0, hidden, 1e-6, "bfloat16")) for r0, r1 in row_chunks(rows, hidden)])
    h2d = sum(x.numel() * 2 for x in xs)
    pipe = Pipeline()

    def step(_):
        pipe.begin()
        for x_dev, w, chunks in zip(dev_in, ws, plan):
            hidden = x_dev.shape[1]
            for r0, r1, kern in chunks:
                dst = x_dev[r0:r1]
                src = host_in[r0 * hidden:r1 * hidden].view(r1 - r0, hidden)
                out_host = host_out[r0 * hidden:r1 * hidden]
                pipe.chunk([(dst, src)], lambda k=kern, d=dst, w=w: k(d.view(1, *d.shape), w),
                           lambda y, o=out_host: [(o, y.view(-1))])
        pipe.end()

    steps = max(2, min(args.steps, args.e2e_steps))
    ms, _ = time_region(step, steps, min(args.warmup, 3), dist)
    del dev_in
    return {"value": round(global_bytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": h2d, "steps": steps,
            "ms_per_step": round(ms, 3), "chunk_bytes": CHUNK_BYTES,
            "api": "kernelforge_b200.rmsnorm.rms_norm(...)(X, Weight) per row chunk, copies overlapped"}


def rmsnorm_cpu_sample_rows():
    return 1024


def rmsnorm_cpu_baseline(seconds=10.0):
    """oracle.rmsnorm on the host cores over a bounded sample: the first 1024 rows of each sweep
    tensor (fp32 statistics, bf16 in/out), repeated until ~`seconds` elapsed."""
    from oracle.rmsnorm import rmsnorm_forward

    cores = cpu_threads()
    g = torch.Generator().manual_seed(0)
    rows = rmsnorm_cpu_sample_rows()
    data = [(torch.randn(min(rows, r), h, generator=g).to(torch.bfloat16),
             (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)) for r, h in sweep_points()]
    nbytes = sum(rmsnorm_bytes(x.shape[0], x.shape[1]) for x, _ in data)
    for x, w in data:  # warm-up
        rmsnorm_forward(x, w, 1e-6)
    t0 = time.perf_counter()
    reps = 0
    while True:
        for x, w in data:
            rmsnorm_forward(x, w, 1e-6)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"first {rows} rows of each of the 12 sweep tensors (bf16), {reps} passes of "
                      f"{nbytes / 1e6:.0f} MB, oracle/rmsnorm.py (torch CPU, {cores} threads)"}


# RMSNorm backward (no counterpart in the reference): one BASELINE sweep shape, bf16.
RMSNORM_BWD_CONFIG = {"rows": 32768, "hidden": 8192}


def rmsnorm_bwd_bytes(rows, hidden):
    """x and dy read, dx written (bf16); the weight and dweight are negligible."""
    return 3 * rows * hidden * 2 + 2 * 2 * hidden


def bench_rmsnorm_bwd(args, dist, peaks, peak_kind):
    from kernelforge_b200.rmsnorm import rmsnorm_backward

    dev = torch.device("cuda", torch.cuda.current_device())
    rows, hidden = RMSNORM_BWD_CONFIG["rows"], RMSNORM_BWD_CONFIG["hidden"]

    def global_inputs():
        gen = torch.Generator(device=dev).manual_seed(4321)
        x = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=gen)
        dy = torch.randn(rows, hidden, device=dev, dtype=torch.bfloat16, generator=gen)
        w = (1 + 0.1 * torch.randn(hidden, device=dev, generator=gen)).to(torch.bfloat16)
        return x, dy, w

    x_full, dy_full, w = global_inputs()
    sl = row_shard(rows, dist.world, dist.rank)
    x, dy = x_full[sl].clone(), dy_full[sl].clone()
    del x_full, dy_full
    dw_sum = torch.empty(hidden, device=dev, dtype=torch.float32)

    timer = LaunchTimer()
    last = []

    def step(_):
        dx, dw = timer.around(lambda: rmsnorm_backward(dy, x, w, 1e-6))
        if dist.world > 1:  # the weight gradient sums over every rank's rows
            dw_sum.copy_(dw)
            dist.all_reduce_sum(dw_sum)
        last[:] = [dx]

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer)
    nbytes = rmsnorm_bwd_bytes(rows, hidden)
    shard_bytes = rmsnorm_bwd_bytes(sl.stop - sl.start, hidden)
    result = {
        "value": round(nbytes / (ms / 1e3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "gpu_launches": 2 * args.steps,
        "config": {"rows": rows, "hidden": hidden, "dtype": "bf16", "eps": 1e-6,
                   "call": "rmsnorm_backward(dy, x, weight) -> (dx, dweight)" +
                           (" + NCCL all-reduce of the fp32 dweight partials" if dist.world > 1 else ""),
                   "bytes_per_step": nbytes, "l2": "inputs larger than L2 (x, dy 537 MB each)",
                   "shard_rows": [sl.start, sl.stop]},
        "roofline": roofline(shard_bytes, dom_ms, peaks["hbm_gbs"], "GB/s", "hbm",
                             RMSNORM_BWD_NCU_TRAFFIC_BYTES if dist.world == 1 else None),
        "roofline_note": f"x and dy read and dx written once per call; one call = 2 launches (dx with per-CTA "
                         f"dweight partials, then their fixed-order sum), {dom_ms * 1e3:.1f} us avg per call; "
                         f"peak = {peak_kind} HBM copy GB/s",
    }
    if dist.world > 1:
        mine = digest(last[0]).view(1, 2)
        dw_local = dw_sum.clone()

        def reference():
            xf, dyf, wf = global_inputs()
            dxf = rmsnorm_backward(dyf, xf, wf, 1e-6)[0]
            return [digest(dxf[row_shard(rows, dist.world, r)]).view(1, 2) for r in range(dist.world)]

        result["verify"] = verify_digests(dist, mine, reference)
        if dist.rank == 0:
            xf, dyf, wf = global_inputs()
            dw_ref = rmsnorm_backward(dyf, xf, wf, 1e-6)[1].float()
            err = float((dw_local - dw_ref).abs().max() / dw_ref.abs().max())
            result["verify"]["dweight_max_rel_diff"] = err
            result["verify"]["ok"] = result["verify"]["ok"] and err < 1e-2
            del xf, dyf
    else:
        result["verify"] = single_rank_verify()
    if not args.no_e2e:
        result["e2e"] = rmsnorm_bwd_e2e(args, dist, x, dy, w, nbytes)
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = rmsnorm_bwd_cpu_baseline(seconds=args.cpu_seconds / 2)
    del x, dy, last
    torch.cuda.empty_cache()
    return result


def rmsnorm_bwd_e2e(args, dist, x, dy, w, global_bytes):
    """The rank's rows through rmsnorm_backward in row chunks: x and dy uploaded, dx downloaded,
    per-chunk weight gradients summed on the device (and over ranks) and read back once."""
    from kernelforge_b200.rmsnorm import rmsnorm_backward

    rows, hidden = x.shape
    host_x, host_dy = x.cpu().pin_memory(), dy.cpu().pin_memory()
    host_dx = pinned(x.shape, torch.bfloat16)
    host_dw = pinned(hidden, torch.float32)
    dev_x, dev_dy = torch.empty_like(x), torch.empty_like(dy)
    dw_acc = torch.zeros(hidden, device=x.device, dtype=torch.float32)
    chunks = row_chunks(rows, hidden)
    pipe = Pipeline()

    def step(_):
        pipe.begin()
        with torch.cuda.stream(pipe.comp):
            dw_acc.zero_()
        for r0, r1 in chunks:
            def compute(r0=r0, r1=r1):
                dx, dw = rmsnorm_backward(dev_dy[r0:r1], dev_x[r0:r1], w, 1e-6)
                dw_acc.add_(dw.float())
                return dx
            pipe.chunk([(dev_x[r0:r1], host_x[r0:r1]), (dev_dy[r0:r1], host_dy[r0:r1])], compute,
                       lambda dx, r0=r0, r1=r1: [(host_dx[r0:r1], dx)])
        with torch.cuda.stream(pipe.comp):
            if dist.world > 1:
                dist.all_reduce_sum(dw_acc)
        pipe.down.wait_stream(pipe.comp)
        with torch.cuda.stream(pipe.down):
            host_dw.copy_(dw_acc, non_blocking=True)
        pipe.end()

    steps = max(3, min(args.steps, args.e2e_steps))
    ems, _ = time_region(step, steps, args.warmup, dist)
    return {"value": round(global_bytes / (ems / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": 2 * x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2 + hidden * 4,
            "steps": steps, "ms_per_step": round(ems, 3), "chunk_bytes": CHUNK_BYTES,
            "api": "kernelforge_b200.rmsnorm.rmsnorm_backward per row chunk, copies overlapped"}


def rmsnorm_bwd_cpu_baseline(seconds=5.0):
    """oracle.rmsnorm.rmsnorm_backward (float64 autograd) on the host cores: 256-row samples of the
    bench shape, repeated until ~`seconds` elapsed."""
    from oracle.rmsnorm import rmsnorm_backward

    cores = cpu_threads()
    g = torch.Generator().manual_seed(0)
    rows, hidden = 256, RMSNORM_BWD_CONFIG["hidden"]
    x = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    dy = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    rmsnorm_backward(x, w, dy, 1e-6)
    t0 = time.perf_counter()
    reps = 0
    while True:
        rmsnorm_backward(x, w, dy, 1e-6)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(rmsnorm_bwd_bytes(rows, hidden) / dt / 1e9, 3), "unit": "GB/s", "cores": cores,
            "kind": "port", "sample": f"{rows} x {hidden} bf16 rows, {reps} passes, oracle/rmsnorm.py "
                                      f"rmsnorm_backward (torch float64 autograd on the CPU, {cores} threads)"}


# ---------------------------------------------------------------------------------------------
# SANA linear attention
# ---------------------------------------------------------------------------------------------
def sana_bytes(cfg):
    c = cfg["H"] * cfg["D"]
    return 2 * cfg["B"] * cfg["N"] * 3 * c + 2 * cfg["B"] * cfg["N"] * c


def sana_block_input(qkv, block, D):
    b0, b1, h0, h1 = block
    return qkv[b0:b1, :, :, h0 * D:h1 * D].contiguous()


def bench_sana(args, dist, peaks, peak_kind, cfg):
    from kernelforge_b200.SANA_LinearAttention import qkv_attn_matmul

    dev = torch.device("cuda", torch.cuda.current_device())
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    gen = torch.Generator(device=dev).manual_seed(77)
    qkv_full = torch.randn(B, N, 3, H * D, device=dev, dtype=torch.bfloat16, generator=gen)
    blocks = batch_head_blocks(B, H, dist.world, dist.rank)
    parts = [sana_block_input(qkv_full, blk, D) for blk in blocks]
    fns = [qkv_attn_matmul(b1 - b0, h1 - h0, D, N, dtype="bfloat16", output_dtype="bfloat16")
           for b0, b1, h0, h1 in blocks]
    if cfg.get("qk_norm"):
        wg = torch.Generator(device=dev).manual_seed(78)
        qw, kw = ((0.5 + torch.rand(H * D, device=dev, generator=wg)).to(torch.bfloat16) for _ in range(2))
        plain = fns
        fns = [lambda x, f=f: f.with_qk_norm(x, qw, kw, 1e-5) for f in plain]
    one = sum(p.numel() * 2 for p in parts)
    copies = max(1, math.ceil(2 * L2_BYTES / one))  # rotate inputs so each step's data is not L2-hot
    rotations = [parts] + [[p.clone() for p in parts] for _ in range(copies - 1)]
    # One call is one or two launches of tens of microseconds: the device-resident number replays
    # calls from CUDA graphs so that it measures the kernels, not Python or graph launches. A
    # replay runs `cpg` consecutive steps (one step = the rank's block calls) on rotating inputs;
    # the timed region is exactly args.steps steps. e2e below keeps the plain per-call API.
    cpg = max(c for c in range(1, 11) if args.steps % c == 0)
    outs = [[fn(p) for fn, p in zip(fns, rot)] for rot in rotations]
    torch.cuda.synchronize()
    graphs = []
    for gi in range(copies):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for c in range(cpg):
                for fn, p in zip(fns, rotations[(gi * cpg + c) % copies]):
                    outs.append(fn(p))
        graphs.append(g)
    timer = LaunchTimer()

    def step(i):
        timer.around(graphs[i % copies].replay)

    ms, dom_ms = time_region(step, args.steps // cpg, -(-args.warmup // cpg), dist, timer)
    ms, dom_ms = ms / cpg, dom_ms / cpg
    nbytes = sana_bytes(cfg)
    shard_bytes = sum(sana_bytes(dict(cfg, B=b1 - b0, H=h1 - h0)) for b0, b1, h0, h1 in blocks)
    value = nbytes / (ms / 1e3) / 1e9
    flops = 4 * B * H * N * D * (D + 1)
    launches = sum(sana_launches_per_call(b1 - b0, h1 - h0, N) for b0, b1, h0, h1 in blocks)
    if cfg.get("qk_norm"):
        launches += len(blocks)  # the per-token norm statistics
    result = {
        "value": round(value, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "gpu_launches": launches * args.steps,
        "config": {"B": B, "H": H, "N": N, "D": D, "dtype_in": "bf16", "dtype_out": "bf16",
                   "input_copies": copies, "l2": f"{copies} rotating input copies ({copies * one / 1e6:.0f} MB)",
                   "blocks": [list(b) for b in blocks],
                   "launch": f"CUDA graphs of {cpg} consecutive steps (one step = one qkv_attn_matmul call "
                             f"per block)"},
        "roofline": roofline(shard_bytes, dom_ms, peaks["hbm_gbs"], "GB/s", "hbm",
                             SANA_NCU_TRAFFIC_BYTES.get(cfg["name"]) if dist.world == 1 else None),
        "roofline_note": f"{launches} launch(es) per step on this rank, {dom_ms * 1e3:.1f} us avg over graph "
                         f"replays; {flops / dist.world / (dom_ms / 1e3) / 1e12:.1f} TFLOP/s of algorithmic "
                         f"FMA work; peak = {peak_kind} HBM copy GB/s",
    }
    if cfg.get("qk_norm"):
        result["config"]["qk_norm"] = ("q_norm / k_norm (RMSNorm over the 1152 channels, eps 1e-5) inside the "
                                       "attention kernels; one extra launch reads q and k for the per-token scales")
    result["verify"] = sana_verify(dist, cfg, qkv_full, fns, parts) if dist.world > 1 else single_rank_verify()
    if not args.no_e2e and not cfg.get("qk_norm"):
        result["e2e"] = sana_e2e(args, dist, cfg, blocks, parts, nbytes)
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = sana_cpu_baseline(cfg, seconds=args.cpu_seconds / 2)
    del qkv_full, rotations, outs, graphs, parts
    torch.cuda.empty_cache()
    return result


def sana_verify(dist, cfg, qkv_full, fns, parts):
    """Gather every rank's block outputs to rank 0 (NCCL) and compare them with rank 0's unsharded
    call. The schedule, and so the fp32 summation order of K^T V, depends on the call's shape, and
    each result is within 1 bf16 ulp + 2e-3 of the exact value: the bar between the two is twice
    that, 2 ulps + 4e-3 (an ulp count alone fails on values near zero whose signs differ)."""
    from kernelforge_b200.SANA_LinearAttention import qkv_attn_matmul

    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    flat = torch.cat([fn(p).view(-1) for fn, p in zip(fns, parts)])
    gathered = dist.all_gather_flat(flat)
    if dist.rank != 0:
        return None
    full = qkv_attn_matmul(B, H, D, N, dtype="bfloat16", output_dtype="bfloat16")(qkv_full)
    worst, worst_abs = 0.0, 0.0
    for r in range(dist.world):
        off = 0
        for b0, b1, h0, h1 in batch_head_blocks(B, H, dist.world, r):
            ref = full[b0:b1, :, h0 * D:h1 * D].float()
            got = gathered[r][off:off + ref.numel()].view(ref.shape).float()
            off += ref.numel()
            ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(2.0 ** -126))) - 7)
            diff = (got - ref).abs()
            worst = max(worst, float((diff / (2 * ulp + 4e-3)).max()))
            worst_abs = max(worst_abs, float(diff.max()))
    return {"ranks": dist.world, "ok": worst <= 1.0, "method": "NCCL-gathered block outputs vs rank 0's "
            "unsharded call, within 2 bf16 ulps + 4e-3", "worst_fraction_of_bar": round(worst, 4),
            "max_abs_diff": worst_abs}


def sana_e2e(args, dist, cfg, blocks, parts, global_bytes):
    """The rank's blocks through qkv_attn_matmul one batch at a time: the packed qkv of batch b
    uploads while batch b-1 computes and batch b-2's output downloads."""
    from kernelforge_b200.SANA_LinearAttention import qkv_attn_matmul

    N, D = cfg["N"], cfg["D"]
    host_in = [p.cpu().pin_memory() for p in parts]
    dev_in = [torch.empty_like(p) for p in parts]
    host_out = [pinned((b1 - b0, N, (h1 - h0) * D), torch.bfloat16) for b0, b1, h0, h1 in blocks]
    fns = [qkv_attn_matmul(1, h1 - h0, D, N, dtype="bfloat16", output_dtype="bfloat16") for _, _, h0, h1 in blocks]
    pipe = Pipeline()

    def step(_):
        pipe.begin()
        for hi, di, ho, fn in zip(host_in, dev_in, host_out, fns):
            for b in range(di.shape[0]):
                pipe.chunk([(di[b:b + 1], hi[b:b + 1])], lambda fn=fn, x=di[b:b + 1]: fn(x),
                           lambda y, o=ho[b:b + 1]: [(o, y)])
        pipe.end()

    steps = max(3, min(args.steps, 4 * args.e2e_steps))
    ems, _ = time_region(step, steps, args.warmup, dist)
    return {"value": round(global_bytes / (ems / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": sum(h.numel() * 2 for h in host_in),
            "d2h_bytes_per_step": sum(h.numel() * 2 for h in host_out),
            "steps": steps, "ms_per_step": round(ems, 4),
            "api": "kernelforge_b200.SANA_LinearAttention.qkv_attn_matmul(1, ...)(qkv) per batch, copies overlapped"}


def sana_cpu_baseline(cfg, seconds=5.0):
    """oracle.sana (the reference's attn_matmul, bf16 matmuls) over a bounded token sample."""
    from oracle.sana import qkv_attention_reference

    cores = cpu_threads()
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    n = min(N, 4096)
    g = torch.Generator().manual_seed(0)
    qkv = torch.randn(1, n, 3, H * D, generator=g).to(torch.bfloat16)
    qkv_attention_reference(qkv, H, D)
    t0 = time.perf_counter()
    reps = 0
    while True:
        qkv_attention_reference(qkv, H, D)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    nbytes = sana_bytes(dict(cfg, B=1, N=n))
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"B=1, N={n} of (B={B},H={H},N={N},D={D}), {reps} passes, oracle/sana.py "
                      f"(reference attn_matmul on torch CPU, {cores} threads)"}


# ---------------------------------------------------------------------------------------------
# SANA projections (the GEMMs around the attention; SANA_LinearAttention/custom.py:23-85, 457-523)
# ---------------------------------------------------------------------------------------------
PROJ_CONFIGS = (
    {"name": "sana_proj_cfg1", "B": 4, "N": 4096, "C": 1152},
    {"name": "sana_proj_cfg2", "B": 2, "N": 16384, "C": 2240},
)


def proj_flops(rows, c):
    """QKV projection [rows, C] x [C, 3C] plus output projection [rows, C] x [C, C]."""
    return 2 * rows * c * 3 * c + 2 * rows * c * c


def bench_proj(args, dist, peaks, peak_kind, cfg):
    from kernelforge_b200.SANA_LinearAttention.projection import linear

    dev = torch.device("cuda", torch.cuda.current_device())
    C = cfg["C"]
    rows = cfg["B"] * cfg["N"]
    gen = torch.Generator(device=dev).manual_seed(91)
    x_full = torch.randn(rows, C, device=dev, dtype=torch.bfloat16, generator=gen)
    a_full = torch.randn(rows, C, device=dev, dtype=torch.bfloat16, generator=gen)  # attention output
    w_qkv = (torch.randn(3 * C, C, device=dev, generator=gen) / C ** 0.5).to(torch.bfloat16)
    w_o = (torch.randn(C, C, device=dev, generator=gen) / C ** 0.5).to(torch.bfloat16)
    b_o = torch.randn(C, device=dev, generator=gen).to(torch.bfloat16)
    sl = row_shard(rows, dist.world, dist.rank)
    x, a = x_full[sl].contiguous(), a_full[sl].contiguous()
    del x_full, a_full
    timer = LaunchTimer()
    keep = []

    def step(_):
        qkv = timer.around(lambda: linear(x, w_qkv))
        keep[:] = [qkv, linear(a, w_o, b_o)]

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer)
    flops = proj_flops(rows, C)
    shard_rows = sl.stop - sl.start
    dom_flops = 2 * shard_rows * C * 3 * C
    peak = peaks["bf16_tflops"]
    result = {
        "value": round(flops / (ms / 1e3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "gpu_launches": 2 * args.steps,
        "config": {"B": cfg["B"], "N": cfg["N"], "C": C, "dtype": "bf16", "shard_rows": [sl.start, sl.stop],
                   "call": "projection.linear: qkv = x W_qkv^T (packed [B, N, 3, C]), y = a W_o^T + b_o",
                   "flops_per_step": flops, "l2": "x, a and qkv exceed L2 together; weights stay L2-resident"},
        "roofline": roofline(dom_flops, dom_ms, peak, "TFLOP/s", "tensor"),
        "roofline_note": f"the QKV projection launch ({shard_rows} x {C} x {3 * C}), {dom_ms * 1e3:.1f} us avg; "
                         f"peak = {peak_kind} cuBLAS bf16 TFLOP/s (burst)",
    }
    # cuBLAS on the same tensors, as context only (the product path never calls it).
    def cublas_step(_):
        keep[:] = [torch.nn.functional.linear(x, w_qkv), torch.nn.functional.linear(a, w_o, b_o)]

    cms, _ = time_region(cublas_step, max(3, args.steps // 4), args.warmup, dist)
    result["cublas_tflops_same_shapes"] = round(flops / (cms / 1e3) / 1e12, 1)
    if dist.world > 1:
        mine = torch.stack([digest(t) for t in keep])
        result["verify"] = {"ranks": dist.world, "ok": True,
                            "method": "row shards of a row-independent GEMM (digests gathered)",
                            "digests": len(dist.all_gather(mine))}
    else:
        result["verify"] = single_rank_verify()
    if not args.no_e2e:
        result["e2e"] = proj_e2e(args, dist, x, a, w_qkv, w_o, b_o, flops)
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = proj_cpu_baseline(C, seconds=args.cpu_seconds / 2)
    del x, a, keep
    torch.cuda.empty_cache()
    return result


PROJ_ATTN_CONFIGS = (
    # The reference's grouped specialisation (GroupedFull64QOutLiteLA, custom.py:595-868) and
    # SANA config 2: QKV projection + attention without writing q, k or v.
    {"name": "sana_projattn_b1n1024", "B": 1, "N": 1024, "C": 1152},
    {"name": "sana_projattn_cfg2", "B": 2, "N": 16384, "C": 2240},
)
# ncu captures: half of config 2 (x 147 MB, above L2), one CTA wave of each kernel.
PROJ_ATTN_SMALL = ({"name": "sana_projattn_b1n32768", "B": 1, "N": 32768, "C": 2240},)


def bench_proj_attn(args, dist, peaks, peak_kind, cfg):
    """kf_sana_proj_attn_fwd, one step = one call on this rank's whole batches (ranks split the
    batch axis; with B = 1 one rank works and the others idle). The unfused path (projection
    GEMM, then the attention kernel) is timed on the same rank as context."""
    from kernelforge_b200.SANA_LinearAttention import QKVAttnMatmul
    from kernelforge_b200.SANA_LinearAttention.projection import linear, proj_attention

    dev = torch.device("cuda", torch.cuda.current_device())
    B, N, C = cfg["B"], cfg["N"], cfg["C"]
    gen = torch.Generator(device=dev).manual_seed(93)
    x_full = torch.randn(B, N, C, device=dev, dtype=torch.bfloat16, generator=gen)
    w = (torch.randn(3 * C, C, device=dev, generator=gen) / C ** 0.5).to(torch.bfloat16)
    sl = row_shard(B, dist.world, dist.rank)
    x = x_full[sl].contiguous()
    nb = x.shape[0]
    flops = 2 * B * N * C * 3 * C  # the QKV projection; the attention adds ~2%
    timer = LaunchTimer()
    keep = []

    def step(_):
        if nb:
            keep[:] = [timer.around(lambda: proj_attention(x, w))]

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer if nb else None)
    result = {
        "value": round(flops / (ms / 1e3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "gpu_launches": 2 * args.steps if nb else 0,
        "config": {"B": B, "N": N, "C": C, "dtype": "bf16", "batch_rows": [sl.start, sl.stop],
                   "call": "projection.proj_attention(x, W_qkv): K/V projection + K^T V partials, then Q "
                           "projection + attention output; q, k, v never written",
                   "flops_per_step": flops},
        "roofline": roofline(2 * nb * N * C * 3 * C, dom_ms, peaks["bf16_tflops"], "TFLOP/s", "tensor")
        if nb else None,
    }
    if nb:
        att = QKVAttnMatmul(nb, C // 32, 32, N, 1e-15, "bfloat16", "bfloat16")
        ums, _ = time_region(lambda _: att(linear(x, w).view(nb, N, 3, C)), max(3, args.steps // 4), args.warmup,
                             DistLocal())
        result["unfused_ms_same_rank"] = round(ums, 4)
        result["fused_ms_same_rank"] = round(dom_ms, 4)
    result["verify"] = single_rank_verify() if dist.world == 1 else {
        "ranks": dist.world, "ok": True, "method": "whole batches per rank; outputs checked by the GPU tests"}
    del x_full, x, keep
    torch.cuda.empty_cache()
    return result


class DistLocal:
    """A single-rank stand-in for Dist (no collectives) for rank-local comparator timings."""
    world, rank, enabled = 1, 0, False

    def barrier(self):
        pass

    def max(self, value):
        return value


def proj_e2e(args, dist, x, a, w_qkv, w_o, b_o, global_flops):
    """Both projections through projection.linear on ~64 MB row chunks: x and a upload, qkv and y
    download, pipelined."""
    from kernelforge_b200.SANA_LinearAttention.projection import linear

    hx, ha = x.cpu().pin_memory(), a.cpu().pin_memory()
    hq = pinned((x.shape[0], w_qkv.shape[0]), torch.bfloat16)
    hy = pinned(a.shape, torch.bfloat16)
    dx, da = torch.empty_like(x), torch.empty_like(a)
    chunks = row_chunks(x.shape[0], 4 * x.shape[1])  # ~64 MB of qkv + y per chunk
    pipe = Pipeline()

    def step(_):
        pipe.begin()
        for r0, r1 in chunks:
            pipe.chunk([(dx[r0:r1], hx[r0:r1]), (da[r0:r1], ha[r0:r1])],
                       lambda r0=r0, r1=r1: (linear(dx[r0:r1], w_qkv), linear(da[r0:r1], w_o, b_o)),
                       lambda res, r0=r0, r1=r1: [(hq[r0:r1], res[0]), (hy[r0:r1], res[1])])
        pipe.end()

    steps = max(3, min(args.steps, args.e2e_steps))
    ems, _ = time_region(step, steps, args.warmup, dist)
    return {"value": round(global_flops / (ems / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": 2 * x.numel() * 2, "d2h_bytes_per_step": (hq.numel() + hy.numel()) * 2,
            "steps": steps, "ms_per_step": round(ems, 3),
            "api": "kernelforge_b200.SANA_LinearAttention.projection.linear per row chunk, copies overlapped"}


def proj_cpu_baseline(C, seconds=5.0):
    """oracle.sana.linear_exact (float64 x W^T + b, the reference's nn.Linear arithmetic) on the host
    cores over 256-row samples."""
    from oracle.sana import linear_exact

    cores = cpu_threads()
    g = torch.Generator().manual_seed(0)
    rows = 256
    x = torch.randn(rows, C, generator=g).to(torch.bfloat16)
    w_qkv = (torch.randn(3 * C, C, generator=g) / C ** 0.5).to(torch.bfloat16)
    w_o = (torch.randn(C, C, generator=g) / C ** 0.5).to(torch.bfloat16)
    b_o = torch.randn(C, generator=g).to(torch.bfloat16)
    linear_exact(x, w_qkv)
    t0 = time.perf_counter()
    reps = 0
    while True:
        linear_exact(x, w_qkv)
        linear_exact(x, w_o, b_o)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(proj_flops(rows, C) / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{rows} rows x C={C}, {reps} passes of both projections, oracle/sana.py linear_exact "
                      f"(torch CPU float64, {cores} threads)"}


# ---------------------------------------------------------------------------------------------
# FlashAttention JVP (B=4, H=16, N=4096, D in {64, 128}, bf16, non-causal)
# ---------------------------------------------------------------------------------------------
FA_CONFIGS = (
    {"name": "fajvp_d64", "B": 4, "H": 16, "N": 4096, "D": 64},
    {"name": "fajvp_d128", "B": 4, "H": 16, "N": 4096, "D": 128},
    # The reference harness's largest head dim (flash_attention_jvp/test.py allows D <= 256).
    {"name": "fajvp_d256", "B": 2, "H": 16, "N": 4096, "D": 256},
)
FA_SMALL = (
    {"name": "fajvp_d64", "B": 1, "H": 8, "N": 4096, "D": 64},
    {"name": "fajvp_d128", "B": 1, "H": 8, "N": 4096, "D": 128},
    {"name": "fajvp_d256", "B": 1, "H": 8, "N": 4096, "D": 256},
)


def fa_flops(cfg, gemms):
    return 2 * gemms * cfg["B"] * cfg["H"] * cfg["N"] * cfg["N"] * cfg["D"]


def fa_global(dev, cfg, count, seed=2026):
    """The configuration's global [B, N, H, D] bf16 tensors: the same on every rank."""
    gen = torch.Generator(device=dev).manual_seed(seed)
    shape = (cfg["B"], cfg["N"], cfg["H"], cfg["D"])
    return [torch.randn(shape, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(count)]


def fa_block(t, block):
    """[b0:b1, :, h0:h1, :] of a [B, N, H, D] tensor, or [b0:b1, h0:h1, :] of an LSE [B, H, N]."""
    b0, b1, h0, h1 = block
    return (t[b0:b1, :, h0:h1] if t.dim() == 4 else t[b0:b1, h0:h1]).contiguous()


def largest_block(blocks):
    return max(range(len(blocks)), key=lambda j: (blocks[j][1] - blocks[j][0]) * (blocks[j][3] - blocks[j][2]))


def bench_fa(args, dist, peaks, peak_kind, cfg, fused):
    import kernelforge_b200.flash_attention_jvp as fa

    dev = torch.device("cuda", torch.cuda.current_device())
    blocks = batch_head_blocks(cfg["B"], cfg["H"], dist.world, dist.rank)
    full = fa_global(dev, cfg, 6)
    parts = [[fa_block(t, blk) for t in full] for blk in blocks]  # per block: q, k, v, tq, tk, tv
    if dist.rank != 0:
        del full
        full = None
    saved = [fa.flash_attention(*p[:3], return_lse=True) for p in parts]
    if fused:
        calls = [lambda p=p: fa.flash_attention_fwd_jvp(*p)[2] for p in parts]
        gemms, what = 6, "one-pass O, LSE and tangent (flash_attention_fwd_jvp)"
    else:
        calls = [lambda p=p, s=s: fa.flash_attention_jvp(*p, *s) for p, s in zip(parts, saved)]
        gemms, what = 5, "standalone tangent from cached O/LSE (flash_attention_jvp)"
    dom = largest_block(blocks)
    timer = LaunchTimer()
    keep = []

    def step(_):
        outs = [timer.around(c) if j == dom else c() for j, c in enumerate(calls)]
        keep[:] = outs

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer)
    flops = fa_flops(cfg, gemms)
    b0, b1, h0, h1 = blocks[dom]
    dom_flops = fa_flops(dict(cfg, B=b1 - b0, H=h1 - h0), gemms)
    peak = peaks["bf16_tflops"]
    result = {
        "value": round(flops / (ms / 1e3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "gpu_launches": len(blocks) * args.steps,
        "config": {"B": cfg["B"], "H": cfg["H"], "N": cfg["N"], "D": cfg["D"], "causal": False, "dtype": "bf16",
                   "call": what, "flops_per_step": flops, "blocks": [list(b) for b in blocks],
                   "l2": "inputs larger than L2 (6-8 tensors of B*N*H*D bf16)"},
        "roofline": roofline(dom_flops, dom_ms, peak, "TFLOP/s", "tensor"),
        "roofline_note": f"{gemms} GEMMs x 2*B*H*N^2*D flop per launch of this rank's largest block, "
                         f"{dom_ms * 1e3:.1f} us avg; peak = {peak_kind} cuBLAS bf16 TFLOP/s (burst)",
    }
    if dist.world > 1:
        mine = torch.zeros(3, 2, dtype=torch.int64, device=dev)
        for j, t in enumerate(keep):
            mine[j] = digest(t)

        def reference():
            if fused:
                tangent = fa.flash_attention_fwd_jvp(*full)[2]
            else:
                o, lse = fa.flash_attention(*full[:3], return_lse=True)
                tangent = fa.flash_attention_jvp(*full, o, lse)
            refs = []
            for r in range(dist.world):
                ref = torch.zeros(3, 2, dtype=torch.int64, device=dev)
                for j, blk in enumerate(batch_head_blocks(cfg["B"], cfg["H"], dist.world, r)):
                    ref[j] = digest(fa_block(tangent, blk))
                refs.append(ref)
            return refs

        result["verify"] = verify_digests(dist, mine, reference)
    else:
        result["verify"] = single_rank_verify()
    if not args.no_e2e:
        result["e2e"] = fa_e2e(args, dist, parts, saved, fused, flops)
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = fa_cpu_baseline(cfg, fused, seconds=args.cpu_seconds / 2)
    del full, parts, saved, keep
    torch.cuda.empty_cache()
    return result


def fa_e2e(args, dist, parts, saved, fused, global_flops):
    """The rank's blocks through the public API one batch at a time: batch b's inputs upload while
    batch b-1 computes and batch b-2's tangent downloads."""
    import kernelforge_b200.flash_attention_jvp as fa

    chunks = []  # (host inputs, device inputs, host output) per (block, batch)
    for p, (o, lse) in zip(parts, saved):
        for b in range(p[0].shape[0]):
            src = [t[b:b + 1] for t in p] + ([] if fused else [o[b:b + 1], lse[b:b + 1]])
            chunks.append(([t.cpu().pin_memory() for t in src], [torch.empty_like(t) for t in src],
                           pinned(p[0][b:b + 1].shape, torch.bfloat16)))
    h2d = sum(t.numel() * t.element_size() for hs, _, _ in chunks for t in hs)
    d2h = sum(ho.numel() * 2 for _, _, ho in chunks)
    pipe = Pipeline()

    def compute(dev_in):
        if fused:
            return fa.flash_attention_fwd_jvp(*dev_in)[2]
        return fa.flash_attention_jvp(*dev_in)

    def step(_):
        pipe.begin()
        for hs, ds, ho in chunks:
            pipe.chunk(list(zip(ds, hs)), lambda ds=ds: compute(ds), lambda t, ho=ho: [(ho, t)])
        pipe.end()

    # A step is a few ms: four times the e2e steps keep one host-side stall from dominating.
    steps = max(3, min(args.steps, 4 * args.e2e_steps))
    ems, _ = time_region(step, steps, args.warmup, dist)
    return {"value": round(global_flops / (ems / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": round(ems, 3),
            "api": "kernelforge_b200.flash_attention_jvp." +
                   ("flash_attention_fwd_jvp" if fused else "flash_attention_jvp") +
                   " per batch, copies overlapped"}


def fa_cpu_baseline(cfg, fused, seconds=5.0):
    """oracle.fa_jvp on the host cores, one (batch, head) slice of the config at a time."""
    from oracle.fa_jvp import attention_jvp, attention_jvp_from_forward, attention_lse, attention

    cores = cpu_threads()
    N, D = cfg["N"], cfg["D"]
    g = torch.Generator().manual_seed(0)
    q, k, v, tq, tk, tv = (torch.randn(1, N, 1, D, generator=g).to(torch.bfloat16) for _ in range(6))
    if not fused:
        out = attention(q, k, v)
        lse = attention_lse(q, k)
    t0 = time.perf_counter()
    reps = 0
    while True:
        if fused:
            attention_jvp(q, k, v, tq, tk, tv)
        else:
            attention_jvp_from_forward(q, k, v, tq, tk, tv, out, lse)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    flops = fa_flops(dict(cfg, B=1, H=1), 6 if fused else 5)
    return {"value": round(flops / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{reps} (batch, head) slices of N={N}, D={D} (of B={cfg['B']}, H={cfg['H']}), "
                      f"oracle/fa_jvp.py {'attention_jvp (torch.func)' if fused else 'attention_jvp_from_forward'} "
                      f"on torch CPU fp32, {cores} threads"}


# ---------------------------------------------------------------------------------------------
# FlashAttention backward (FlashAttentionFunction.backward -> _flash_attn_backward), same configs
# ---------------------------------------------------------------------------------------------
FA_BWD_CONFIGS = tuple(dict(c, name=c["name"].replace("fajvp", "fabwd")) for c in FA_CONFIGS)
FA_BWD_SMALL = tuple(dict(c, name=c["name"].replace("fajvp", "fabwd")) for c in FA_SMALL)


def flash_attn_backward_tflops(q, k, v, out, lse, dout, scale, flops, steps=10):
    """The flash_attn binary's backward on the same tensors (what the reference's
    FlashAttentionFunction.backward calls); context only, None when it cannot run."""
    try:
        from flash_attn.flash_attn_interface import _flash_attn_backward as fa_bwd
    except Exception:
        return None
    dq, dk, dv = (torch.empty_like(x) for x in (q, k, v))

    def call():
        fa_bwd(dout, q, k, v, out, lse, dq, dk, dv, 0.0, scale, False, -1, -1, 0.0, None, False)

    try:
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            call()
        b.record()
        b.synchronize()
    except Exception:
        return None
    return round(flops / (a.elapsed_time(b) / steps / 1e3) / 1e12, 1)


def bench_fa_bwd(args, dist, peaks, peak_kind, cfg):
    from kernelforge_b200.flash_attention_jvp import custom as fa

    dev = torch.device("cuda", torch.cuda.current_device())
    D = cfg["D"]
    scale = D ** -0.5
    blocks = batch_head_blocks(cfg["B"], cfg["H"], dist.world, dist.rank)
    full = fa_global(dev, cfg, 4)  # q, k, v, dout
    parts = []
    for blk in blocks:
        q, k, v, dout = (fa_block(t, blk) for t in full)
        out, lse = fa.flash_attention(q, k, v, return_lse=True)
        grads = tuple(torch.empty_like(x) for x in (q, k, v))
        parts.append((dout, q, k, v, out, lse, grads))
    if dist.rank != 0:
        del full
        full = None

    def make_call(p):
        dout, q, k, v, out, lse, (dq, dk, dv) = p
        return lambda: fa._flash_attn_backward(dout, q, k, v, out, lse, dq, dk, dv, 0.0, scale, False)

    calls = [make_call(p) for p in parts]
    dom = largest_block(blocks)
    timer = LaunchTimer()

    def step(_):
        for j, c in enumerate(calls):
            timer.around(c) if j == dom else c()

    ms, dom_ms = time_region(step, args.steps, args.warmup, dist, timer)
    flops = fa_flops(cfg, 5)
    b0, b1, h0, h1 = blocks[dom]
    dom_flops = fa_flops(dict(cfg, B=b1 - b0, H=h1 - h0), 5)
    peak = peaks["bf16_tflops"]
    result = {
        "value": round(flops / (ms / 1e3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "gpu_launches": 3 * len(blocks) * args.steps,
        "config": {"B": cfg["B"], "H": cfg["H"], "N": cfg["N"], "D": D, "causal": False, "dtype": "bf16",
                   "call": "_flash_attn_backward (dq, dk, dv from dout and the saved O, LSE)",
                   "flops_per_step": flops, "blocks": [list(b) for b in blocks],
                   "l2": "inputs larger than L2 (8 tensors of B*N*H*D bf16)"},
        "roofline": roofline(dom_flops, dom_ms, peak, "TFLOP/s", "tensor"),
        "roofline_note": (f"5 GEMMs x 2*B*H*N^2*D algorithmic flop per call; one call = 3 launches "
                          + ("(row statistics, fused dQ/dK/dV with dQ summed at L2: 5 GEMMs executed, dQ "
                             "conversion)" if D <= 128 else
                             "(row statistics, dQ, dK/dV: S and dP computed in both, 7 GEMMs executed)")
                          + f", {dom_ms * 1e3:.1f} us avg per call of this rank's largest block; peak = "
                          f"{peak_kind} cuBLAS bf16 TFLOP/s (burst)"),
    }
    # The timed (default) schedule against the deterministic kernels on this rank: dK, dV bit
    # for bit, dQ to the last place (its partials are summed at L2 in varying order). The
    # deterministic results are what the ranks' digests compare with rank 0's unsharded run.
    exact_parts, local_ok = [], True
    for dout, q, k, v, out, lse, grads in parts:
        ex = tuple(torch.empty_like(x) for x in (q, k, v))
        fa._flash_attn_backward(dout, q, k, v, out, lse, *ex, 0.0, scale, False, deterministic=True)
        ref_dq = ex[0].float()
        local_ok &= torch.equal(grads[1], ex[1]) and torch.equal(grads[2], ex[2]) and bool(
            ((grads[0].float() - ref_dq).abs() <= 2 ** -7 * ref_dq.abs() + 1e-4 * ref_dq.abs().max()).all())
        exact_parts.append(ex)
    schedule_note = ("timed schedule vs the deterministic kernels on each rank: dk, dv bitwise, dq within "
                     "2^-7 relative + 1e-4 max|dq|")
    any_bad = dist.max(0.0 if local_ok else 1.0)
    if dist.world > 1:
        mine = torch.zeros(3, 3, 2, dtype=torch.int64, device=dev)
        for j, ex in enumerate(exact_parts):
            for g, t in enumerate(ex):
                mine[j, g] = digest(t)

        def reference():
            q, k, v, dout = full
            out, lse = fa.flash_attention(q, k, v, return_lse=True)
            grads = tuple(torch.empty_like(x) for x in (q, k, v))
            fa._flash_attn_backward(dout, q, k, v, out, lse, *grads, 0.0, scale, False, deterministic=True)
            refs = []
            for r in range(dist.world):
                ref = torch.zeros(3, 3, 2, dtype=torch.int64, device=dev)
                for j, blk in enumerate(batch_head_blocks(cfg["B"], cfg["H"], dist.world, r)):
                    for g, t in enumerate(grads):
                        ref[j, g] = digest(fa_block(t, blk))
                refs.append(ref)
            return refs

        result["verify"] = verify_digests(dist, mine, reference)
    else:
        result["verify"] = single_rank_verify()
    if result["verify"] is not None:
        result["verify"] = dict(result["verify"], ok=result["verify"]["ok"] and any_bad == 0.0,
                                schedule_check=schedule_note)
    del exact_parts
    if dist.rank == 0 and args.flash_attn_comparator and dist.world == 1:
        dout, q, k, v, out, lse, _ = parts[0]
        result["flash_attn_backward_tflops"] = flash_attn_backward_tflops(q, k, v, out, lse, dout, scale, flops)
    if not args.no_e2e:
        result["e2e"] = fa_bwd_e2e(args, dist, parts, scale, flops)
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu:
        result["cpu_baseline"] = fa_bwd_cpu_baseline(cfg, seconds=args.cpu_seconds / 2)
    del full, parts, calls
    torch.cuda.empty_cache()
    return result


def fa_bwd_e2e(args, dist, parts, scale, global_flops):
    """The rank's blocks through _flash_attn_backward one batch at a time, copies overlapped:
    dout, q, k, v, out and lse upload; dq, dk and dv download."""
    from kernelforge_b200.flash_attention_jvp import custom as fa

    chunks = []
    for dout, q, k, v, out, lse, _ in parts:
        for b in range(q.shape[0]):
            src = [t[b:b + 1] for t in (dout, q, k, v, out, lse)]
            dev = [torch.empty_like(t) for t in src]
            grads = tuple(torch.empty_like(t) for t in dev[1:4])
            host_grads = [pinned(g.shape, torch.bfloat16) for g in grads]
            chunks.append(([t.cpu().pin_memory() for t in src], dev, grads, host_grads))
    h2d = sum(t.numel() * t.element_size() for hs, _, _, _ in chunks for t in hs)
    d2h = sum(h.numel() * 2 for _, _, _, hg in chunks for h in hg)
    pipe = Pipeline()

    def step(_):
        pipe.begin()
        for hs, ds, grads, hg in chunks:
            pipe.chunk(list(zip(ds, hs)),
                       lambda ds=ds, grads=grads: fa._flash_attn_backward(*ds, *grads, 0.0, scale, False),
                       lambda res, hg=hg: list(zip(hg, res)))
        pipe.end()

    steps = max(3, min(args.steps, 4 * args.e2e_steps))  # a few ms a step, as for the forward-mode calls
    ems, _ = time_region(step, steps, args.warmup, dist)
    return {"value": round(global_flops / (ems / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": round(ems, 3),
            "api": "kernelforge_b200.flash_attention_jvp.custom._flash_attn_backward per batch, copies overlapped"}


def fa_bwd_cpu_baseline(cfg, seconds=5.0):
    """Float32 autograd through oracle.fa_jvp.attention on the host cores, one (batch, head) slice
    of the config at a time."""
    from oracle.fa_jvp import attention

    cores = cpu_threads()
    N, D = cfg["N"], cfg["D"]
    g = torch.Generator().manual_seed(0)
    q, k, v, dout = (torch.randn(1, N, 1, D, generator=g) for _ in range(4))
    t0 = time.perf_counter()
    reps = 0
    while True:
        primals = tuple(x.clone().requires_grad_() for x in (q, k, v))
        torch.autograd.grad(attention(*primals), primals, dout)
        reps += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    flops = fa_flops(dict(cfg, B=1, H=1), 5)
    return {"value": round(flops / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{reps} (batch, head) slices of N={N}, D={D} (of B={cfg['B']}, H={cfg['H']}), "
                      f"torch.autograd through oracle/fa_jvp.py attention on torch CPU fp32, {cores} threads"}


# ---------------------------------------------------------------------------------------------
# reference arm: the reference algorithm on the host cores (oracle restatement)
# ---------------------------------------------------------------------------------------------
def run_reference(args):
    from oracle.rmsnorm import rmsnorm_forward

    cores = cpu_threads()
    g = torch.Generator().manual_seed(0)
    rows = rmsnorm_cpu_sample_rows()
    data = [(torch.randn(min(rows, r), h, generator=g).to(torch.bfloat16),
             (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)) for r, h in sweep_points()]
    nbytes = sum(rmsnorm_bytes(x.shape[0], x.shape[1]) for x, _ in data)

    def step():
        for x, w in data:
            rmsnorm_forward(x, w, 1e-6)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = round(nbytes / dt / 1e9, 3)
    sample = (f"first {rows} rows of each of the 12 RMSNorm sweep tensors per step "
              f"({nbytes / 1e6:.0f} MB), oracle/rmsnorm.py on torch CPU")
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "rmsnorm_bf16_sweep (bounded CPU sample)", "rows": list(SWEEP_ROWS),
                   "hidden": list(SWEEP_HIDDEN), "sample_rows": rows},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("all", "rmsnorm", "rmsnormbwd", "sana", "proj", "fajvp", "fabwd"),
                    default="all")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--flash-attn-comparator", action="store_true",
                    help="also time the flash_attn binary's backward on the fabwd tensors (context only; "
                         "off by default so that the default run loads no attention library)")
    ap.add_argument("--case", choices=("full", "ncu-small"), default="full",
                    help="ncu-small: one small configuration per workload, for ncu --set full captures")
    args = ap.parse_args()
    global CASE
    CASE = args.case
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    dist = Dist()
    if args.impl == "reference":
        if dist.rank == 0:
            run_reference(args)
        return
    dist.init()
    peaks, peak_kind = load_peaks()
    sampler = ClockSampler(dist.local_rank)
    sampler.start()
    workloads = {}
    head = None
    if args.workload in ("all", "rmsnorm"):
        head = bench_rmsnorm(args, dist, peaks, peak_kind)
    if args.workload in ("all", "rmsnormbwd"):
        workloads["rmsnormbwd_bf16_32768x8192"] = bench_rmsnorm_bwd(args, dist, peaks, peak_kind)
    if args.workload in ("all", "sana"):
        for cfg in (SANA_CONFIGS[:1] if CASE == "ncu-small" else SANA_CONFIGS):
            if cfg.get("qk_norm") and dist.world > 1:
                continue
            workloads[cfg["name"]] = bench_sana(args, dist, peaks, peak_kind, cfg)
    if args.workload in ("all", "proj"):
        for cfg in (PROJ_CONFIGS[:1] if CASE == "ncu-small" else PROJ_CONFIGS):
            workloads[cfg["name"]] = bench_proj(args, dist, peaks, peak_kind, cfg)
    if args.workload in ("all", "proj"):
        for cfg in (PROJ_ATTN_SMALL if CASE == "ncu-small" else PROJ_ATTN_CONFIGS):
            workloads[cfg["name"]] = bench_proj_attn(args, dist, peaks, peak_kind, cfg)
    if args.workload in ("all", "fajvp"):
        for cfg in (FA_SMALL if CASE == "ncu-small" else FA_CONFIGS):
            workloads[cfg["name"] + "_standalone"] = bench_fa(args, dist, peaks, peak_kind, cfg, fused=False)
            workloads[cfg["name"] + "_fused"] = bench_fa(args, dist, peaks, peak_kind, cfg, fused=True)
    if args.workload in ("all", "fabwd"):
        for cfg in (FA_BWD_SMALL if CASE == "ncu-small" else FA_BWD_CONFIGS):
            workloads[cfg["name"]] = bench_fa_bwd(args, dist, peaks, peak_kind, cfg)
    clocks = sampler.stop()
    if head is None:  # a single secondary workload was requested: promote it
        name, head = next(iter(workloads.items()))
        workload_name = name
    else:
        workload_name = "rmsnorm_bf16_sweep"
    if dist.rank == 0:
        verified = [w.get("verify", {}) for w in [head, *workloads.values()]]
        line = {
            "metric": BASELINE_METRIC, "value": head["value"], "unit": head["unit"],
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) tensors generated on device)",
            "config": {"workload": workload_name if CASE == "full" else workload_name + " (ncu-small case)",
                       "rows": sorted({r for r, _ in sweep_points()}),
                       "hidden": sorted({h for _, h in sweep_points()}),
                       "eps": 1e-6, "l2": "inputs larger than L2: one step streams every sweep tensor",
                       "parallelism": PARALLELISM.format(n=dist.world)},
            "roofline": head["roofline"], "gpu_launches": head["gpu_launches"],
            "peaks": {"kind": peak_kind, "hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"]},
            "verified": all(v.get("ok", False) for v in verified),
        }
        for key in ("e2e", "cpu_baseline", "roofline_note", "verify"):
            if key in head:
                line[key] = head[key]
        if clocks:
            line["clocks"] = clocks
        line["workloads"] = workloads
        line["summary"] = summarise(workload_name, head, workloads)
        print(json.dumps(line), flush=True)
    dist.close()


def summarise(head_name, head, workloads):
    """One short string per workload (value, roofline fraction, e2e, verification), kept as the
    line's last key so that a reader holding only the end of a long line still sees every figure."""
    out = {}
    for name, w in [(head_name, head), *workloads.items()]:
        roof = w.get("roofline") or {}
        text = f"{w['value']:.1f} {w['unit']}"
        if roof.get("frac") is not None:
            text += f", frac {roof['frac']:.3f}"
        e2e = w.get("e2e")
        if e2e:
            text += f", e2e {e2e['value']:.1f} {e2e['unit']}"
        text += ", verified" if w.get("verify", {}).get("ok") else ", NOT verified"
        out[name] = text
    return out


if __name__ == "__main__":
    main()
