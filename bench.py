#!/usr/bin/env python3
"""Benchmark of Kernix's dense matmul path on B200.

Default workload (the headline configuration): f32 GEMM M=N=K=8192 where A is a
non-contiguous strided slice (row stride 8704) of an 8192 x 8704 buffer, entries
uniform[-1,1] from SplitMix64 seeds 5 (A buffer) and 6 (B).  Rows of M are
sharded block-cyclically over the GPUs and the output is all-gathered over
NVLink, so ``scaling`` is strong (fixed total work).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under ``python -m torch.distributed.run --nproc-per-node N``.  Rank 0
prints one JSON line.  After the headline, the line carries ``per_config``: c1
and c2 (one GPU only: replicas) and c3 and c4 (their batch split over the
ranks), each timed on device-resident seeded inputs with its own clock record,
a parity check of the timed output against the oracle and a CPU baseline of
the reference's path on a bounded sample.
``--workload c1|c2|c3|c4`` measures one of them alone and prints its own line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEEDS = {"c1": (0,), "c2": (1,), "c3": (2,), "c4": (3, 4), "c5": (5, 6)}
CONFIG_TEXT = {
    "c1": "f32 GEMM 512^3, row-major contiguous",
    "c2": "f64 GEMM 4096^3, B a transposed (column-major) view",
    "c3": "batched f32 attention products 16x32 heads, seq 2048, d 128: S=QK^T, softmax(S/sqrt(128)), PV "
          "(one fused call)",
    "c4": "f32 conv2d NCHW 64x128x56x56, 3x3, 256 out, stride 1, pad 1 (implicit GEMM)",
    "c5": "f32 GEMM 8192^3, A strided slice (row stride 8704), rows sharded, output all-gathered",
}
METRIC = "GEMM TFLOP/s (f32, f64) at 1/2/4/8 B200 and % of pipe peak vs host-CPU ref"


def _rng():
    """The seeded input generator (kernix_b200/rng.py, plain numpy), loaded by
    path: the reference arm must not load the product library, which importing
    the package would do."""
    import importlib.util
    mod = sys.modules.get("_kx_rng")
    if mod is None:
        spec = importlib.util.spec_from_file_location("_kx_rng", ROOT / "kernix_b200" / "rng.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules["_kx_rng"] = mod
    return mod


def err_metrics(got, want, absum) -> dict:
    """Error of computed outputs ``got`` against the compensated oracle
    ``want`` (both float64 arrays of the same outputs; ``absum`` = sum |a b|
    per output): the scaled form |x - y| / sum|a b| (small_matmul_tests.rs:
    153-186), the elementwise |x - y| / (1 + |y|) (native_kernel_tests.rs:
    139-181) and the normwise max|x - y| / max|y|."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    d = np.abs(got - want)
    return {"max_err_over_sum_abs": float(np.max(d / np.maximum(absum, 1e-300))),
            "max_rel_err_elementwise": float(np.max(d / (1.0 + np.abs(want)))),
            "normwise": float(np.max(d) / max(float(np.max(np.abs(want))), 1e-300))}


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}, \
        "fallback"


def pipe_peak(pipe: str, peaks: dict, sm_mhz: float) -> tuple[float, str]:
    """Peak of the pipe the dominant kernel runs on, in TFLOP/s.

    FP32 SIMT and FP64 are derived from the SM clock (148 SMs x 128 FP32 or 64
    FP64 lanes x 2 flops); TF32 tensor is half the measured dense bf16 rate and
    3xTF32 a third of that."""
    if pipe == "fp32-simt":
        return 148 * 128 * 2 * sm_mhz * 1e6 / 1e12, f"derived: 148 SM x 128 FP32 lanes x 2 x {sm_mhz:.0f} MHz"
    if pipe == "fp64":
        return 148 * 64 * 2 * sm_mhz * 1e6 / 1e12, f"derived: 148 SM x 64 FP64 lanes x 2 x {sm_mhz:.0f} MHz"
    if pipe == "3xtf32":
        return peaks["bf16_tflops"] / 2 / 3, "measured bf16 dense / 2 (tf32) / 3 (three products)"
    raise ValueError(pipe)


# ---------------------------------------------------------------------------
# clocks (NVML reads only; no setting is changed)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period: float = 0.02):
        self.samples, self.reasons = [], set()
        self.period = period
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.dev = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.dev, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.dev, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.dev)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons)}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workload: c5 (headline)
# ---------------------------------------------------------------------------
M = N = K = 8192
ROW_STRIDE = 8704


def a_rows(rows: list[int], out: np.ndarray) -> np.ndarray:
    """Rows of the seed-5 8192 x 8704 buffer, in the given order, written into
    ``out`` (the stream is counter-based: runs of rows generate directly)."""
    rng = _rng()
    i = 0
    while i < len(rows):
        j = i
        while j + 1 < len(rows) and rows[j + 1] == rows[j] + 1:
            j += 1
        r0, cnt = rows[i], j - i + 1
        rng.uniform(SEEDS["c5"][0], cnt * ROW_STRIDE, -1.0, 1.0, np.float32,
                    out=out[i * ROW_STRIDE:(i + cnt) * ROW_STRIDE], start=r0 * ROW_STRIDE)
        i = j + 1
    return out


def run_ours(args, rank, world, local):
    import torch
    import torch.distributed as dist
    import kernix_b200 as kx
    rng = _rng()
    from kernix_b200.sharded import (PeerOutput, ReplicatedOutput, plan_rows, sharded_matmul, sharded_matmul_push,
                                     sharded_matmul_push_mc, sharded_matmul_replicated)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    h = kx.handle(local)
    group = dist.group.WORLD if world > 1 else None
    gather = args.gather if world > 1 else "none"
    rep = None
    if gather in ("auto", "nvls", "p2p-nvls"):
        # symmetric memory bound to an NVLink multicast object
        rep = ReplicatedOutput(M, N, torch.float32, group, local)
        if not rep.available:
            if gather != "auto":
                raise RuntimeError("no NVLink multicast (NVLS) on this node")
            rep.close()
            rep = None
        if gather == "auto":
            gather = "p2p-nvls" if rep is not None else "p2p"
    if gather == "nvls":
        plan = plan_rows(M, world, target_piece=args.piece or M // world)
    else:
        plan = plan_rows(M, world, target_piece=(args.piece or 512) if world > 1 else M)
    my_rows = plan.local_rows(rank)
    # Host inputs (pinned): this rank's rows of the A buffer, and B.
    a_host = torch.empty(len(my_rows) * ROW_STRIDE, dtype=torch.float32, pin_memory=True)
    a_rows(my_rows, a_host.numpy())
    b_host = torch.empty(K * N, dtype=torch.float32, pin_memory=True)
    rng.uniform(SEEDS["c5"][1], K * N, -1.0, 1.0, np.float32, out=b_host.numpy())
    a_buf = a_host.to(dev)
    b = b_host.to(dev).view(K, N)
    push = gather == "p2p"
    push_mc = gather == "p2p-nvls"
    peer_out = PeerOutput(M, N, torch.float32, group, local) if push else None
    if rep is not None:
        c = rep.tensor
    else:
        c = peer_out.tensor if push else torch.empty(M, N, dtype=torch.float32, device=dev)
    # piece i of this rank: rows [i*piece, (i+1)*piece) of the local buffer,
    # viewed with the 8704 row stride (first 8192 columns)
    pieces = [kx.TensorView(a_buf, (plan.piece, K), (ROW_STRIDE, 1), i * plan.piece * ROW_STRIDE)
              for i in range(plan.pieces)]
    scratch = [torch.empty(plan.piece, N, dtype=torch.float32, device=dev) for _ in range(plan.pieces)] \
        if gather == "nccl" else None
    streams = (torch.cuda.current_stream(dev), torch.cuda.Stream(dev)) if gather == "nccl" else None
    push_streams = None
    if push or push_mc:
        push_streams = {"comm": torch.cuda.Stream(dev)}

    # this rank's rows of A in piece order (the local buffer, row stride 8704)
    a_local = kx.TensorView(a_buf, (plan.pieces * plan.piece, K), (ROW_STRIDE, 1), 0)

    def step():
        if push_mc:
            sharded_matmul_push_mc(a_local, b, rep, plan, rank, group, streams=push_streams)
        elif rep is not None:
            sharded_matmul_replicated(pieces, b, rep, plan, rank, group)
        elif push:
            sharded_matmul_push(a_local, b, peer_out, plan, rank, group, streams=push_streams)
        else:
            sharded_matmul(pieces, b, c, plan, rank, group, streams=streams, scratch=scratch)

    step.a_dev, step.b_dev = a_buf, b

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    # warm-up
    for _ in range(args.warmup):
        step()
    barrier()
    # kernel-only timing of one GEMM launch (dominant kernel) for the roofline
    if rep is not None and not push_mc:
        s0, e0 = plan.rows_of(rank, 0)
        launch = lambda: kx.matmul_into_replicated(pieces[0], b, c[s0:e0], rep.mc + s0 * rep.row_bytes)  # noqa: E731
    else:
        launch = lambda: kx.matmul_into(pieces[0], b, c[:plan.piece])  # noqa: E731
    kern_ms = time_dominant_kernel(launch, dev)
    step_kernel = h.last_kernel     # the family the timed GEMM launches use
    barrier()
    launches0 = h.launches
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        barrier()
    launches = h.launches - launches0
    h.synchronize()   # raises DeviceTimeout if any bounded device wait expired
    elapsed = start.elapsed_time(end) / 1e3
    t = torch.tensor([elapsed], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed = float(t.item())
    flops = 2.0 * M * N * K
    value = flops * args.steps / elapsed / 1e12

    # end-to-end through the public API with host buffers
    e2e = None if args.no_e2e else e2e_run(args, rank, world, local, a_host, b_host, plan, kx, dist, group,
                                           step_fn=step, c=c)
    # correctness of the timed output: rows against the compensated oracle on
    # rank 0, and (N > 1) every gathered row equal to what its owner computed
    check = spot_check(c, a_host, b_host, plan, rank) if rank == 0 else None
    gathered = gather_check(c, plan, rank, world, group) if world > 1 else None
    if rank == 0 and gathered is not None:
        check["gathered_rows_equal_owner"] = gathered
        check["pass"] = check["pass"] and gathered
    if peer_out is not None:
        peer_out.close()
    if rep is not None:
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[local])
        rep.close()

    result = None
    if rank == 0:
        peaks, peak_src = measured_peaks()
        clocks = clk.summary()
        pipe = "fp32-simt"
        kname = step_kernel
        if "tf32" in kname:
            pipe = "3xtf32"
        sm_max = clocks.get("sm_max_mhz") or peaks.get("sm_max_mhz", 1965.0)
        peak, basis = pipe_peak(pipe, peaks, float(sm_max))
        per_launch_flops = 2.0 * plan.piece * N * K
        achieved = per_launch_flops / (kern_ms / 1e3) / 1e12
        traffic = load_traffic(kname, plan.piece)
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed * 1e3 / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (SplitMix64 seeds 5, 6)",
            "config": {"workload": "c5: " + CONFIG_TEXT["c5"], "M": M, "N": N, "K": K, "a_row_stride": ROW_STRIDE,
                       "parallelism": f"rows{world} block-cyclic piece={plan.piece}" + {
                           "none": "", "nvls": " + NVLS multicast stores from the GEMM epilogue",
                           "p2p-nvls": " + copy-engine push to peers, NVLS multicast store of the last piece",
                           "p2p": " + push to peers over CUDA IPC (copy engines, all-SM kernel for the last piece)",
                           "nccl": " + NCCL all-gather"}[gather],
                       "l2": "inputs larger than L2 (A span 285 MB, B 268 MB)", "kernel": kname},
            "e2e": e2e,
            "gpu_launches": launches,
            "roofline": {"bound": "tensor", "pipe": pipe, "achieved": round(achieved, 3), "peak": round(peak, 3),
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_basis": basis + (" (of measured)" if pipe == "3xtf32" and peak_src == "measured"
                                                else ""),
                         "kernel": kname, "kernel_ms": round(kern_ms, 4),
                         "launch_flops": per_launch_flops},
            "clocks": clocks,
            "check": check,
        }
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_seconds)
    return result


def time_dominant_kernel(launch, dev, reps=5):
    """Average duration of one GEMM launch (one piece, as the step issues it)
    with CUDA events on the stream the kernel runs on."""
    import torch
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launch()
    torch.cuda.synchronize(dev)
    s.record()
    for _ in range(reps):
        launch()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / reps


class SharedHostBuffer:
    """``nbytes`` of host memory shared by the ranks of one node (a /dev/shm
    file that rank 0 creates and every rank maps), page-locked in each
    process with cudaHostRegister so device copies into it are DMA."""

    def __init__(self, nbytes: int, rank: int, world: int, dist, dev):
        import mmap
        import torch
        tag = torch.tensor([os.getpid() if rank == 0 else 0], dtype=torch.int64, device=dev)
        dist.broadcast(tag, 0)
        self.path = f"/dev/shm/kx_bench_e2e_{int(tag.item())}"
        self.rank = rank
        if rank == 0:
            with open(self.path, "wb") as f:
                f.truncate(nbytes)
        dist.barrier(device_ids=[dev.index])
        self.fd = os.open(self.path, os.O_RDWR)
        self.map = mmap.mmap(self.fd, nbytes)
        self.view = memoryview(self.map)
        self.ptr = np.frombuffer(self.view, dtype=np.uint8).ctypes.data
        rt = torch.cuda.cudart()
        rc = rt.cudaHostRegister(self.ptr, nbytes, 0)
        if int(rc) != 0:
            raise RuntimeError(f"cudaHostRegister failed ({rc})")
        self.dist, self.dev = dist, dev

    def close(self):
        import torch
        torch.cuda.synchronize(self.dev)
        torch.cuda.cudart().cudaHostUnregister(self.ptr)
        self.view.release()
        self.map.close()
        os.close(self.fd)
        self.dist.barrier(device_ids=[self.dev.index])
        if self.rank == 0:
            os.unlink(self.path)


def e2e_run(args, rank, world, local, a_host, b_host, plan, kx, dist, group, step_fn=None, c=None):
    """Same metric measured through the public API from pinned host buffers.

    N=1: ``try_strided_matmul`` -- the reference-facing MatmulElement hook --
    on the host A view (row stride 8704) and B, result read back to host.
    N>1: host->device copy of this rank's A rows and its 1/N slice of B, an
    NCCL all-gather of B, the sharded matmul with its gather (``step_fn`` on
    the device buffers it was built on), and every rank reading its own rows
    of C into one shared host buffer."""
    import torch
    dev = torch.device("cuda", local)
    steps = max(1, min(args.steps, 5))
    if world == 1:
        a_np, b_np = a_host.numpy(), b_host.numpy()
        out = torch.empty(M * N, dtype=torch.float32, pin_memory=True).numpy()
        ma = kx.MatrixInput(a_np, [M, K], [ROW_STRIDE, 1], 0)
        mb = kx.MatrixInput(b_np, [K, N], [N, 1], 0)
        assert kx.try_strided_matmul(ma, mb, out)   # warm (allocates staging)
        t0 = time.perf_counter()
        for _ in range(steps):
            ok = kx.try_strided_matmul(ma, mb, out)
            assert ok
        dt = (time.perf_counter() - t0) / steps
        h2d = ((M - 1) * ROW_STRIDE + K) * 4 + K * N * 4
        d2h = M * N * 4
    else:
        # Inputs: this rank's A rows and 1/N of B's rows go up over this GPU's
        # own PCIe link; NCCL all-gathers B over NVLink.  Result: each rank
        # reads its own rows of the gathered C into one host buffer that all
        # ranks share (a /dev/shm mapping, page-locked in every process).
        a_dev, b_dev = step_fn.a_dev, step_fn.b_dev
        kb = K // world
        b_mine = b_host[rank * kb * N:(rank + 1) * kb * N]
        b_slice = torch.empty(kb * N, dtype=torch.float32, device=dev)
        shared = SharedHostBuffer(M * N * 4, rank, world, dist, dev)
        c_host = torch.from_numpy(np.frombuffer(shared.view, dtype=np.float32).reshape(M, N))
        my_ranges = [plan.rows_of(rank, i) for i in range(plan.pieces)]

        def one():
            a_dev.copy_(a_host, non_blocking=True)
            b_slice.copy_(b_mine, non_blocking=True)
            dist.all_gather_into_tensor(b_dev.view(-1), b_slice, group=group)
            step_fn()
            for s0, e0 in my_ranges:
                c_host[s0:e0].copy_(c[s0:e0], non_blocking=True)
            torch.cuda.synchronize(dev)
        one()
        dist.barrier(device_ids=[local])
        t0 = time.perf_counter()
        for _ in range(steps):
            one()
        dist.barrier(device_ids=[local])
        dt = (time.perf_counter() - t0) / steps
        t = torch.tensor([dt], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
        # the host buffer holds every rank's rows: compare one row per rank
        ok = True
        if rank == 0:
            for r in range(world):
                s0, _ = plan.rows_of(r, 0)
                ok = ok and bool(torch.equal(c_host[s0], c[s0].cpu()))
        del c_host
        shared.close()
        h2d = a_host.numel() * 4 * world + K * N * 4
        d2h = M * N * 4
        if rank == 0 and not ok:
            raise RuntimeError("e2e: host copy of C differs from the gathered device C")
    return {"value": round(2.0 * M * N * K / dt / 1e12, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": round(dt * 1e3, 3), "steps": steps,
            "api": "try_strided_matmul (C-ABI hook)" if world == 1 else
            "per rank: H2D of its A rows and 1/N of B, NCCL all-gather of B, sharded matmul + gather, D2H of its "
            "rows of C into one shared pinned host buffer"}


def gather_check(c, plan, rank, world, group):
    """Every rank's rows, as rank 0 holds them after the gather, must equal
    (bit for bit: the gather copies bytes) what the owning rank computed:
    compared through per-row float64 sums, all-gathered from the owners."""
    import torch
    import torch.distributed as dist
    mine = torch.cat([c[s:e] for s, e in (plan.rows_of(rank, i) for i in range(plan.pieces))]).double().sum(dim=1)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine, group=group)
    if rank != 0:
        return None
    ok = True
    for r in range(world):
        held = torch.cat([c[s:e] for s, e in (plan.rows_of(r, i) for i in range(plan.pieces))]).double().sum(dim=1)
        ok = ok and bool(torch.equal(held, every[r]))
    return ok


def check_rows(m: int, count: int = 64) -> list[int]:
    """``count`` rows spread over all 128-row tiles of an m-row output (one
    per tile when m = 128 * count), at varying offsets inside the tile."""
    tiles = max(1, m // 128)
    rows = []
    for i in range(count):
        t = i * tiles // count
        rows.append(min(m - 1, t * 128 + (i * 53 + 7) % 128))
    return sorted(set(rows))


def spot_check(c, a_host, b_host, plan, rank):
    """Check of the timed (gathered) output on rank 0: 64 rows spread over
    every row tile (any rank's rows: the seeded A rows are regenerated here)
    against the compensated oracle.  Reports the gate used throughout,
    |x - y| <= 2e-6 sum|a b| (small_matmul_tests.rs:153-186), the elementwise
    |x - y| / (1 + |y|) and normwise errors, and the same metrics for the
    blocked fp32 CPU engine restatement (the engine Kernix calls) on the same
    rows."""
    import oracle
    b = b_host.numpy().reshape(K, N)
    rows = check_rows(M)
    a = np.empty(len(rows) * ROW_STRIDE, dtype=np.float32)
    a_rows(rows, a)
    va = oracle.View(a, (len(rows), K), (ROW_STRIDE, 1))
    want, ab = oracle.gemm_dot2(va, oracle.View.of(b))
    got = c[rows].cpu().numpy().astype(np.float64)
    ours = err_metrics(got, want, ab)
    engine = err_metrics(oracle.engine_gemm(va, oracle.View.of(b), threads=oracle.THREADS), want, ab)
    ok = ours["max_err_over_sum_abs"] <= 2e-6 and ours["normwise"] <= 1e-5
    return {"rows_checked": len(rows), **ours, "bound": 2e-6, "normwise_bound": 1e-5,
            "elementwise_target": 1e-5, "elementwise_meets_target": ours["max_rel_err_elementwise"] <= 1e-5,
            "cpu_fp32_engine": {**engine, "what": "blocked fp32 FMA engine restatement (gemm-f32 / "
                                                  "matrixmultiply loop nest), same rows"},
            "pass": ok}


def load_traffic(kernel: str, piece_rows: int):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (scaled to this launch's rows when captured on a smaller case)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    e = d.get(kernel)
    if not e:
        return None
    return int(e["dram_bytes_per_row"] * piece_rows) if "dram_bytes_per_row" in e else e.get("dram_bytes")


# ---------------------------------------------------------------------------
# CPU baseline: restatements of Kernix's CPU path, timed on the host cores
# ---------------------------------------------------------------------------
ENGINE_SAMPLE_TEXT = ("blocked fp32 engine restatement (oracle/kx_engine.c: the BLIS loop nest of gemm-f32 0.19.0 / "
                      "matrixmultiply 0.3.11, AVX2 FMA micro-tiles, strided A read while packing), output rows "
                      "chunked over host threads like CpuExecutor::matmul_into (execution.rs:188-233)")


def _c5_b() -> np.ndarray:
    b = np.empty(K * N, dtype=np.float32)
    _rng().uniform(SEEDS["c5"][1], K * N, -1.0, 1.0, np.float32, out=b)
    return b.reshape(K, N)


def _engine_rows_sized(b, threads: int, seconds: float, cap: int):
    """Rows of c5's A for which the engine takes about ``seconds`` (a probe
    of 256 rows first), with the A rows already generated."""
    import oracle
    probe = 256
    a = np.empty(cap * ROW_STRIDE, dtype=np.float32)
    a_rows(list(range(probe)), a[:probe * ROW_STRIDE])
    va = oracle.View(a, (probe, K), (ROW_STRIDE, 1))
    t0 = time.perf_counter()
    oracle.engine_gemm(va, oracle.View.of(b), threads=threads)
    t = time.perf_counter() - t0
    rows = int(min(cap, max(probe, probe * seconds / max(t, 1e-3))))
    rows = max(64, rows // 64 * 64)
    a_rows(list(range(rows)), a[:rows * ROW_STRIDE])
    return a, rows


def cpu_baseline(budget_s: float = 12.0, threads: int | None = None):
    """The reference path's CPU throughput on c5, restated: the blocked engine
    on all host threads (the headline figure), beside the ordered port
    (matmul_reference's arithmetic, linalg.rs:236-316) and a labelled stand-in
    (torch's CPU sgemm at 1 and all threads) for the third-party engines."""
    import oracle
    threads = threads or oracle.THREADS
    b = _c5_b()
    a, rows = _engine_rows_sized(b, threads, budget_s, M)
    va = oracle.View(a, (rows, K), (ROW_STRIDE, 1))
    t0 = time.perf_counter()
    oracle.engine_gemm(va, oracle.View.of(b), threads=threads)
    t = time.perf_counter() - t0
    value = 2.0 * rows * N * K / t / 1e12
    # the ordered port on a few rows
    orows = max(threads, 16)
    vo = oracle.View(a, (orows, K), (ROW_STRIDE, 1))
    t0 = time.perf_counter()
    oracle.gemm_ordered_par(vo, oracle.View.of(b), threads=threads)
    to = time.perf_counter() - t0
    standin = {}
    try:
        import torch
        prev = torch.get_num_threads()
        srows = min(rows, 1024)
        ta = torch.from_numpy(a[:srows * ROW_STRIDE].reshape(srows, ROW_STRIDE))[:, :K]
        tb = torch.from_numpy(b)
        for nt in (1, threads):
            torch.set_num_threads(nt)
            torch.matmul(ta[:64], tb)
            t0 = time.perf_counter()
            torch.matmul(ta, tb)
            standin[f"threads_{nt}"] = round(2.0 * srows * N * K / (time.perf_counter() - t0) / 1e12, 5)
        torch.set_num_threads(prev)
        standin["what"] = (f"torch CPU sgemm on {srows} rows: a labelled stand-in for gemm-f32 / matrixmultiply "
                           "(may use AVX-512, which Kernix's V3 build does not)")
    except Exception as e:  # pragma: no cover - torch is plumbing only
        standin = {"unavailable": str(e)}
    return {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of 8192 rows of the c5 GEMM (strided A, K=N=8192), {t:.1f} s; " + ENGINE_SAMPLE_TEXT,
            "ordered_port": {"value": round(2.0 * orows * N * K / to / 1e12, 6), "cores": threads,
                             "sample": f"{orows} rows; oracle port of matmul_reference's ordered recurrence "
                                       "(linalg.rs:236-316), row-split over host threads"},
            "engine_standin": standin}


def run_reference(args, rank, world):
    """Reference arm: Kernix's CPU path for c5 restated (the blocked engine on
    all host threads, rows chunked like CpuExecutor::matmul_into), timed on the
    host cores.  Rank 0 only; it never loads the product library."""
    if rank != 0:
        return None
    import oracle
    threads = oracle.THREADS
    per_step = max(1.0, min(6.0, 120.0 / max(1, args.steps + args.warmup)))
    b = _c5_b()
    a, rows = _engine_rows_sized(b, threads, per_step, M)
    va = oracle.View(a, (rows, K), (ROW_STRIDE, 1))

    def run():
        t0 = time.perf_counter()
        oracle.engine_gemm(va, oracle.View.of(b), threads=threads)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        run()
    times = [run() for _ in range(args.steps)]
    tot = sum(times)
    value = 2.0 * rows * N * K * args.steps / tot / 1e12
    return {"metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(tot / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (SplitMix64 seeds 5, 6)",
            "config": {"workload": "c5: " + CONFIG_TEXT["c5"], "M": M, "N": N, "K": K, "a_row_stride": ROW_STRIDE,
                       "parallelism": f"{threads} host threads"},
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"{rows} of 8192 rows per step; " + ENGINE_SAMPLE_TEXT},
            "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# the other workloads: c1, c2 (one GPU), c3, c4 (batch split over the ranks)
# ---------------------------------------------------------------------------
def _timed(fn, steps, warmup, dev, world=1, handle=None):
    """Average ms per call over ``steps`` after ``warmup`` calls, CUDA events
    on the current stream, with the clock record of the timed region and the
    number of kernels ``handle`` launched in it; with several ranks the region
    is bracketed by barriers and the time is the maximum over ranks."""
    import torch
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize(dev)
    for _ in range(warmup):
        fn()
    barrier()
    launches0 = handle.launches if handle is not None else 0
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clk:
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        barrier()
    ms = s.elapsed_time(e) / steps
    launches = handle.launches - launches0 if handle is not None else None
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, clk.summary(), launches


def _max_over_ranks(values: list[float], world: int, dev) -> list[float]:
    if world == 1:
        return values
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def _pipe_of(kernel: str) -> str:
    if "tf32" in kernel:
        return "3xtf32"
    if "dmma" in kernel or kernel.endswith("f64"):
        return "fp64"
    return "fp32-simt"


def _im2col(x: np.ndarray, kh: int, kw: int, pad: int) -> np.ndarray:
    """[n, c, h, w] -> [c*kh*kw, n*oh*ow] for stride 1, dilation 1 (the
    (ci, ky, kx) row order of neural.rs:212-302)."""
    n, c, h, w = x.shape
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    oh, ow = h + 2 * pad - kh + 1, w + 2 * pad - kw + 1
    cols = np.empty((c, kh, kw, n, oh, ow), dtype=x.dtype)
    for ky in range(kh):
        for kx_ in range(kw):
            cols[:, ky, kx_] = xp[:, :, ky:ky + oh, kx_:kx_ + ow].transpose(1, 0, 2, 3)
    return cols.reshape(c * kh * kw, n * oh * ow)


def _cpu_line(flops, seconds, cores, sample):
    """The host-CPU restatement of the reference's path for one configuration,
    timed on a bounded sample (kind "port": the oracle's C restatements)."""
    return {"value": round(flops / max(seconds, 1e-9) / 1e12, 6), "unit": "TFLOP/s", "cores": int(cores),
            "kind": "port", "sample": sample}


def run_workload(w, steps, warmup, rank=0, world=1, local=0, batch=0, size=0):
    """Measure one of c1..c4 and check the timed output against the oracle.

    c1 and c2 run on one GPU (replicas only). c3 and c4 shard their batch
    across the ranks (contiguous images, or (batch, head) units in whole
    batches), every rank generating its own window of the seeded stream; no
    collective touches the data, the time is the maximum over ranks and the
    value the whole job's FLOPs over it (strong scaling).  Every check reports
    the scaled, elementwise and normwise errors against the compensated oracle
    and, for the GEMM-shaped outputs, the same errors of the blocked CPU
    engine restatement on the same outputs."""
    import torch
    import kernix_b200 as kx
    import oracle
    rng = _rng()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    h = kx.handle(local)
    peaks, peak_src = measured_peaks()
    if world > 1 and w in ("c1", "c2"):
        raise SystemExit(f"{w} is a single-GPU workload (replicas only): run it with one process")
    res = {"metric": METRIC, "workload": f"{w}: {CONFIG_TEXT[w]}", "n_gpus": world, "steps": steps,
           "warmup": warmup, "data": f"synthetic (SplitMix64 seed(s) {SEEDS[w]})"}
    threads = oracle.THREADS
    if w == "c1":
        v = rng.uniform(SEEDS["c1"][0], 2 * 512 * 512, -1.0, 1.0, np.float32)
        a_np, b_np = v[:512 * 512].reshape(512, 512), v[512 * 512:].reshape(512, 512)
        a, b = torch.from_numpy(a_np).to(dev), torch.from_numpy(b_np).to(dev)
        c = torch.empty(512, 512, device=dev)
        ms, clocks, launches = _timed(lambda: kx.matmul_into(a, b, c), steps, warmup, dev, 1, h)
        flops = 2.0 * 512 ** 3
        # the same calls captured once in a CUDA graph and replayed: device time
        # per product without the per-call host path (ctypes, validation, launch)
        graph_calls = 50
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                kx.matmul_into(a, b, c)             # workspace grown before capture
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(graph_calls):
                kx.matmul_into(a, b, c)
        g_ms, _, _ = _timed(g.replay, max(1, steps // graph_calls), 2, dev, 1, None)
        graph_us = 1000.0 * g_ms / graph_calls
        va, vb = oracle.View.of(a_np), oracle.View.of(b_np)
        exp, ab = oracle.gemm_dot2(va, vb)
        ours = err_metrics(c.cpu().numpy(), exp, ab)
        t0 = time.perf_counter()
        eng_c = oracle.engine_gemm(va, vb, threads=1)
        res["cpu_baseline"] = _cpu_line(flops, time.perf_counter() - t0, 1,
                                        "the whole product, blocked fp32 engine restatement on one thread "
                                        "(Kernix's default Parallelism::None; stand-in for gemm-f32)")
        eng = err_metrics(eng_c, exp, ab)
        check = {"outputs_checked": 512 * 512, **ours, "bound": 2e-6, "normwise_bound": 1e-5,
                 "elementwise_target": 1e-5, "cpu_fp32_engine": eng,
                 "pass": ours["max_err_over_sum_abs"] <= 2e-6 and ours["normwise"] <= 1e-5}
        res.update(dtype="f32", config={"workload": "c1", "M": 512, "N": 512, "K": 512,
                                        "l2": "inputs (3 MB) stay L2-resident: latency-bound"},
                   cuda_graph={"us_per_product": round(graph_us, 3),
                               "tflops": round(flops / graph_us / 1e6, 3), "products_per_graph": graph_calls,
                               "what": "the same matmul_into calls captured in one CUDA graph and replayed: "
                                       "device time per product without the host call path"})
    elif w == "c2":
        n = size or 4096
        v = rng.normal(SEEDS["c2"][0], 2 * n * n, 1.0, np.float64)
        a_np, bt_np = v[:n * n].reshape(n, n), v[n * n:].reshape(n, n)
        a, bt = torch.from_numpy(a_np).to(dev), torch.from_numpy(bt_np).to(dev)
        c = torch.empty(n, n, dtype=torch.float64, device=dev)
        ms, clocks, launches = _timed(lambda: kx.matmul_into(a, bt.t(), c), steps, warmup, dev, 1, h)
        flops = 2.0 * n ** 3
        rows = check_rows(n)
        sub = np.ascontiguousarray(a_np[rows])
        va, vb = oracle.View.of(sub), oracle.View(bt_np, (n, n), (1, n))
        exp, ab = oracle.gemm_dot2(va, vb)
        ours = err_metrics(c[rows].cpu().numpy(), exp, ab)
        t0 = time.perf_counter()
        eng_c = oracle.engine_gemm(va, vb, threads=threads)
        res["cpu_baseline"] = _cpu_line(2.0 * len(rows) * n * n, time.perf_counter() - t0, threads,
                                        f"{len(rows)} rows of C, blocked f64 engine restatement with B read "
                                        "through its transposed view (stand-in for matrixmultiply)")
        eng = err_metrics(eng_c, exp, ab)
        check = {"rows_checked": len(rows), **ours, "bound": 1e-13, "elementwise_target": 1e-12,
                 "cpu_f64_engine": eng,
                 "pass": ours["max_err_over_sum_abs"] <= 1e-13 and ours["max_rel_err_elementwise"] <= 1e-12}
        res.update(dtype="f64", config={"workload": "c2", "M": n, "N": n, "K": n, "b_layout": "transposed view",
                                        "l2": "inputs larger than L2 (134 MB each, C 134 MB)"})
    elif w == "c3":
        total = batch or 16
        from kernix_b200.sharded import shard_window
        b0, nb = shard_window(total, rank, world)       # this rank's batches (library plan)
        shape = (nb, 32, 2048, 128)
        cnt = int(np.prod(shape))
        unit = 32 * 2048 * 128
        # Q, K and V are consecutive windows of one stream of total * 32 * 2048 * 128
        # values each; this rank's batches start at b0 * unit inside each
        host = torch.empty(3 * cnt, dtype=torch.float32, pin_memory=True)
        hv = host.numpy()
        for j in range(3):
            rng.normal(SEEDS["c3"][0], cnt, 1.0, np.float32, out=hv[j * cnt:(j + 1) * cnt],
                       start=j * total * unit + b0 * unit)
        q = host[:cnt].view(shape).to(dev)
        k_ = host[cnt:2 * cnt].view(shape).to(dev)
        v_ = host[2 * cnt:].view(shape).to(dev)
        del host, hv
        t = math.sqrt(128.0)
        o = torch.empty(shape, device=dev)
        kt = k_.transpose(2, 3)

        def step():
            kx.attention_into(q, kt, v_, t, o)
        ms, clocks, launches = _timed(step, steps, warmup, dev, world, h)
        fused_kernel = h.last_kernel
        flops = 2.0 * 2 * total * 32 * 2048 * 2048 * 128
        # the composed path (S and P through HBM) on the same inputs, for comparison
        sc = torch.empty(nb, 32, 2048, 2048, device=dev)
        pr = torch.empty_like(sc)
        oc = torch.empty(shape, device=dev)
        qk_ms, _, _ = _timed(lambda: kx.matmul_into(q, kt, sc), 3, 1, dev, world)
        qk_kernel = h.last_kernel
        sm_ms, _, _ = _timed(lambda: kx.softmax_temperature_into(sc, -1, t, pr), 3, 1, dev, world)
        pv_ms, _, _ = _timed(lambda: kx.matmul_into(pr, v_, oc), 3, 1, dev, world)
        pv_kernel = h.last_kernel
        del sc, pr
        # parity: four heads of this rank, sixteen rows each, against the exact
        # attention of the same inputs (compensated scores, long-double softmax)
        heads = sorted({(0, 0), (nb // 3, 11), ((2 * nb) // 3, 22), (nb - 1, 31)})
        rows = check_rows(2048, 16)
        ours, comp, eng = [], [], []
        tol_scale = 0.0
        for bi, hi in heads:
            qh, kh, vh = (x[bi, hi].cpu().numpy()[None] for x in (q, k_, v_))
            truth, absv, sabs = oracle.attention_truth(qh, kh, vh, t, rows)
            # the f32 bound on P v plus the score bound carried through the softmax
            tol_scale = max(tol_scale, float((2e-6 + 4e-6 * sabs / t).max()))
            ours.append(err_metrics(o[bi, hi, rows].cpu().numpy()[None], truth, absv))
            comp.append(err_metrics(oc[bi, hi, rows].cpu().numpy()[None], truth, absv))
            # the reference's composition on the CPU: blocked fp32 engine, f32 softmax, engine
            s32 = oracle.engine_gemm(oracle.View.of(np.ascontiguousarray(qh[0][rows])),
                                     oracle.View(kh[0], (128, 2048), (1, 128)), threads=threads)
            p32 = oracle.softmax_temperature(s32, -1, t)
            e32 = oracle.engine_gemm(oracle.View.of(p32), oracle.View.of(vh[0]), threads=threads)
            eng.append(err_metrics(e32[None], truth, absv))
        del oc

        if rank == 0:
            # the reference's path for one (batch, head) pair, timed and scaled
            # to the whole job: S through the ordered general fallback (K^T is
            # a view), softmax_temperature, P V through the blocked engine
            try:
                qh, kh, vh = (x[0, 0].cpu().numpy() for x in (q, k_, v_))
                t0 = time.perf_counter()
                s_ref = oracle.matmul_reference(oracle.View.of(qh), oracle.View(kh, (128, 2048), (1, 128)))
                p_ref = oracle.softmax_temperature(s_ref, -1, t)
                oracle.engine_gemm(oracle.View.of(p_ref), oracle.View.of(vh), threads=1)
                pair_s = time.perf_counter() - t0
                res["cpu_baseline"] = _cpu_line(
                    flops, pair_s * total * 32, 1,
                    f"one (batch, head) pair in {pair_s:.2f} s, extrapolated x{total * 32}: S by the ordered "
                    "general-fallback restatement (linalg.rs:176-213), softmax_temperature, P V by the blocked "
                    "engine (stand-in for gemm-f32)")
            except Exception as e:      # a baseline, never a reason to lose the line
                res["cpu_baseline"] = {"unavailable": f"{type(e).__name__}: {e}"}

        def worst(lst):
            return {kk: max(e[kk] for e in lst) for kk in lst[0]}
        wo, wc, we = worst(ours), worst(comp), worst(eng)
        keys = list(wo)
        flat = _max_over_ranks([wo[kk] for kk in keys] + [wc[kk] for kk in keys], world, dev)
        wo, wc = dict(zip(keys, flat[:3])), dict(zip(keys, flat[3:]))
        check = {"heads_checked": len(heads) * world, "rows_per_head": len(rows),
                 "against": "exact attention of the same inputs (compensated S, long-double softmax); "
                            "max_err_over_sum_abs is |x - y| / sum_j p_j |v_j|",
                 "O": wo, "composed_gpu_O": wc, "cpu_fp32_composition_O": we,
                 "bound": round(tol_scale, 9),
                 "bound_is": "(2e-6 + 2 * 2e-6 * max_j sum|q k_j| / T): the f32 bound on P v plus the f32 score "
                             "bound carried through the softmax",
                 "elementwise_target": 1e-5, "pass": wo["max_err_over_sum_abs"] <= tol_scale}
        sm_bytes = 2.0 * nb * 32 * 2048 * 2048 * 4 * world
        res["parts"] = {"fused_kernel": fused_kernel,
                        "composed_ms": round(qk_ms + sm_ms + pv_ms, 3),
                        "composed_tflops": round(flops / (qk_ms + sm_ms + pv_ms) / 1e9, 2),
                        "qk_ms": round(qk_ms, 3), "qk_tflops": round(flops / 2 / qk_ms / 1e9, 2), "qk_kernel": qk_kernel,
                        "softmax_ms": round(sm_ms, 3), "softmax_gbs": round(sm_bytes / sm_ms / 1e6, 1),
                        "softmax_frac_of_hbm": round(sm_bytes / world / sm_ms / 1e6 / peaks["hbm_gbs"], 3),
                        "pv_ms": round(pv_ms, 3), "pv_tflops": round(flops / 2 / pv_ms / 1e9, 2),
                        "pv_kernel": pv_kernel}
        res.update(dtype="f32", config={"workload": "c3", "batch": total, "heads": 32, "seq": 2048, "d": 128,
                                        "parallelism": f"batch{world}: {nb} batches x 32 heads per rank, "
                                                       "no collective" if world > 1 else "one GPU",
                                        "l2": "inputs larger than L2 (S and P 8.6 GB at batch 16)"})
        del o, q, k_, v_
    elif w == "c4":
        total = batch or 64
        from kernix_b200.sharded import shard_window
        i0, nb = shard_window(total, rank, world)       # this rank's images (library plan)
        xn = nb * 128 * 56 * 56
        # this rank's images: a window of the input stream; weights on every rank
        x_np = rng.uniform(SEEDS["c4"][0], xn, -1.0, 1.0, np.float32,
                           start=i0 * 128 * 56 * 56).reshape(nb, 128, 56, 56)
        w_np = rng.normal(SEEDS["c4"][1], 256 * 128 * 9, math.sqrt(2.0 / 1152.0), np.float32).reshape(256, 128, 3, 3)
        x, wt = torch.from_numpy(x_np).to(dev), torch.from_numpy(w_np).to(dev)
        opts = kx.Conv2dOptions(padding=(1, 1))
        y = kx.conv2d(x, wt, opts)
        ms, clocks, launches = _timed(lambda: kx.conv2d_into(x, wt, y, opts), steps, warmup, dev, world, h)
        flops = 2.0 * 256 * 1152 * total * 56 * 56
        # parity: two images of this rank, every output channel and pixel
        imgs = [0, nb - 1] if nb > 1 else [0]
        xs = np.ascontiguousarray(x_np[imgs])
        d2, ab = oracle.conv2d_dot2(oracle.View.of(xs), oracle.View.of(w_np), padding=(1, 1))
        got = y[imgs].cpu().numpy()
        ours = err_metrics(got, d2, ab)
        # the reference's lowering on the CPU: im2col, then the blocked engine
        t0 = time.perf_counter()
        cols = _im2col(xs, 3, 3, 1)
        eng = oracle.engine_gemm(oracle.View.of(w_np.reshape(256, 1152)), oracle.View.of(cols), threads=threads)
        res["cpu_baseline"] = _cpu_line(2.0 * 256 * 1152 * len(imgs) * 56 * 56, time.perf_counter() - t0, threads,
                                        f"{len(imgs)} images: im2col then the blocked fp32 engine restatement "
                                        "(neural.rs:212-302 lowering; stand-in for gemm-f32)")
        eng = eng.reshape(256, len(imgs), 56, 56).transpose(1, 0, 2, 3)
        eng_err = err_metrics(eng, d2, ab)
        vals = _max_over_ranks([ours[k] for k in ours], world, dev)
        ours = dict(zip(list(ours), vals))
        check = {"outputs_checked": int(got.size) * world, **ours, "bound": 2e-6, "elementwise_target": 1e-5,
                 "cpu_fp32_engine": {**eng_err, "what": "im2col + blocked fp32 engine (neural.rs:212-302 lowering)"},
                 "pass": ours["max_err_over_sum_abs"] <= 2e-6 and ours["normwise"] <= 1e-5}
        res.update(dtype="f32", config={"workload": "c4", "batch": total, "c_in": 128, "hw": 56, "c_out": 256,
                                        "parallelism": f"batch{world}: {nb} images per rank, weights on every "
                                                       "rank, no collective" if world > 1 else "one GPU",
                                        "kernel_hw": 3, "stride": 1, "pad": 1,
                                        "l2": "x 103 MB + y 206 MB at batch 64: larger than L2"})
        del x, wt, y
    else:
        raise ValueError(w)
    kernel = h.last_kernel if w != "c3" else res["parts"]["fused_kernel"]
    h.synchronize()
    tflops = flops / ms / 1e9
    pipe = _pipe_of(kernel if w != "c3" else res["parts"]["fused_kernel"])
    sm_max = clocks.get("sm_max_mhz") or peaks.get("sm_max_mhz", 1965.0)
    peak, basis = pipe_peak(pipe, peaks, float(sm_max))
    res.update(value=round(tflops, 3), unit="TFLOP/s", ms_per_step=round(ms, 4), higher_is_better=True,
               scaling="strong", vs_baseline=None, gpu_launches=launches,
               kernel=kernel, clocks=clocks, check=check,
               roofline={"bound": "tensor" if pipe != "fp32-simt" else "fp32 pipe", "pipe": pipe,
                         "achieved": round(tflops / world, 3), "peak": round(peak, 3), "unit": "TFLOP/s",
                         "frac": round(tflops / world / peak, 4), "per": "GPU",
                         "peak_basis": basis + (" (of measured)" if peak_src == "measured" else "")})
    torch.cuda.empty_cache()
    return res if rank == 0 else None


# (warm-up, timed steps) of the c1..c4 measurements attached to the headline line
# c1's calls take ~17 us: 4000 of them keep its timed region (~70 ms) long
# against the clock sampler's start-up inside it
PER_CONFIG_STEPS = {"c1": (50, 4000), "c2": (3, 5), "c3": (3, 5), "c4": (3, 5)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--piece", type=int, default=0, help="rows per sharded piece (0: 512 when sharded)")
    ap.add_argument("--gather", choices=["auto", "p2p", "p2p-nvls", "nvls", "nccl"], default="auto",
                    help="gathered output: the library's row-sharded product pushing into peers' C (copy "
                         "engines while a piece computes, an all-SM kernel for the last piece; p2p-nvls: an "
                         "NVLS multicast store for the last piece), NVLS multicast stores from the GEMM "
                         "epilogue, or NCCL all-gather; auto = p2p-nvls where the node has NVLink "
                         "multicast, else p2p")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--workload", choices=["c5", "c1", "c2", "c3", "c4"], default="c5",
                    help="c5 is the headline (this bench line); c1..c4 print their own measurement (c3 and c4 "
                         "split their batch over the ranks under torchrun)")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the c1..c4 measurements attached to the c5 line as per_config")
    ap.add_argument("--batch", type=int, default=0, help="c3/c4: batch size (default: the workload's)")
    ap.add_argument("--size", type=int, default=8192,
                    help="profiling aid: M=N=K=size with row stride size+512 (8192 is the workload)")
    args = ap.parse_args()
    global M, N, K, ROW_STRIDE
    if args.size != 8192:
        M = N = K = args.size
        ROW_STRIDE = args.size + 512
    rank, world, local = env_rank()
    if args.workload != "c5":
        if args.size == 8192:
            args.size = 0
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "workload": args.workload,
                                  "unavailable": "the reference arm times the headline workload (c5) only"}))
            return
        import torch
        import torch.distributed as dist
        if world > 1:
            from datetime import timedelta
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        try:
            res = run_workload(args.workload, args.steps, args.warmup, rank, world, local, args.batch, args.size)
            if res is not None:
                print(json.dumps(res), flush=True)
        finally:
            if world > 1:
                dist.barrier(device_ids=[local])
                dist.destroy_process_group()
        return
    if world != args.gpus:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    try:
        res = run_ours(args, rank, world, local)
        if not args.no_per_config and args.size == 8192:
            per = {}
            for w, (wu, st) in PER_CONFIG_STEPS.items():
                if world > 1 and w in ("c1", "c2"):
                    continue        # single-GPU configurations: replicas only
                r = run_workload(w, st, wu, rank, world, local)
                if r is not None:
                    per[w] = {k: r[k] for k in ("value", "unit", "ms_per_step", "steps", "warmup", "dtype", "kernel",
                                                "gpu_launches", "check", "roofline", "clocks", "config")}
                    for extra in ("parts", "cuda_graph", "cpu_baseline"):
                        if extra in r:
                            per[w][extra] = r[extra]
            if res is not None:
                res["per_config"] = per
        if res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.barrier(device_ids=[local])
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
