"""Benchmark of the fused RMSNorm -> FP8 path (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload NAME] [--threads-per-row T]

A step is one pass of the path over one batch of the workload. The default
workload is g128_sharded_262144x8192 (x bf16 [262144, 8192] with outlier
channels, 1x128 groups, fp32 column-major scales, no residual), the one
configuration defined at 1, 2, 4 and 8 GPUs: under torchrun (N > 1) the
262144 rows are split evenly by rows over the ranks (strong scaling), every
rank processing its own contiguous shard on its own GPU with no data-path
collective (NCCL carries only the barrier and the max-over-ranks time). At
N = 1 the same line also carries, under "secondary", the device-timed
measurement of g128_16384x7168 (the DeepSeek-V3 shape, 16384 rows). Other
workloads (--workload) run as weak scaling: every rank its own full batch.

value: algorithmic HBM bytes of all ranks / max-over-ranks device time of K
steps with inputs resident in HBM; consecutive steps rotate through enough
workspaces that the data touched by a step is never resident in L2.
e2e: the same metric through the host-buffer API (thingy_b200.host), with
the H2D copy of x and the D2H copy of q and scales inside the timed region.
roofline: bytes per launch / mean per-launch device time (CUDA events on the
launch stream) against MEASURED_PEAKS.json's HBM copy bandwidth.
cpu_baseline / --impl reference: the reference's PyTorch path (restated in
oracle/reference.py) on the host cores, on a bounded row sample; this arm
imports no module that loads the CUDA library.
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

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "fused RMSNorm+FP8 quant HBM GB/s & % of B200 peak; tokens/s at 1/2/4/8 GPU"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
DEFAULT_WORKLOAD = "g128_sharded_262144x8192"  # BASELINE config 5, defined at 1/2/4/8 GPUs
SECONDARY_WORKLOAD = "g128_16384x7168"         # BASELINE config 2, device-timed at N = 1



def _kernel_name(w, threads_per_row) -> str:
    """The kernel that carries the timed step (the launch shape rules of csrc/capi.cu)."""
    if w.kind == "rms_f32":
        return "rmsnorm_f32_kernel"
    if w.kind == "rms_bf16":  # the fused kernels without quantization
        return ("rowstage_rmsnorm_fp8_kernel" if w.M >= 4096 and w.H <= 8192
                else "pipe_rmsnorm_fp8_kernel")
    if w.kind == "bwd":  # rows of up to 16384 take the bulk-copy ring variant
        return "rmsnorm_backward_ring_kernel" if w.H <= 16384 else "rmsnorm_backward_kernel"
    if w.kind == "prologue":
        return "gemm_rmsnorm_mxfp8_kernel"
    if threads_per_row == 32:
        return "rowwarp_rmsnorm_fp8_kernel"
    if (not threads_per_row and not w.residual and w.M >= 4096 and w.H <= 8192
            and w.group_size in (None, 128)):
        return "rowstage_rmsnorm_fp8_kernel"  # one warp a row, the row in registers
    if w.group_size is None:  # per-token scaling: the single-pass kernel
        return "fused_rmsnorm_fp8_kernel"
    return "pipe_rmsnorm_fp8_kernel"

def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default=None,
                    help=f"default {DEFAULT_WORKLOAD} (strong scaling over the ranks)")
    ap.add_argument("--threads-per-row", type=int, default=0)
    ap.add_argument("--rows", type=int, default=0,
                    help="rows a rank processes (0: the workload's own split); a smaller "
                         "case of the same kernel for profiling")
    ap.add_argument("--e2e-steps", type=int, default=0, help="0: min(steps, 20)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--graph", action="store_true",
                    help="capture the K timed launches in one CUDA graph and replay it")
    ap.add_argument("--no-clocks", action="store_true",
                    help="skip clock sampling and its soak (profiling runs)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target CPU work for the cpu_baseline sample")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.steps < 1:
        ap.error("--steps must be >= 1")
    args.secondary = args.workload is None
    args.workload = args.workload or DEFAULT_WORKLOAD
    return args


def measured_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(p.read_text())["hbm_gbs"])
        return v, "measured (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s, earlier measurement on this pool)"


def ncu_traffic(workload: str):
    """DRAM bytes per launch from the committed ncu summary of this workload, if any."""
    p = REPO / "profiles" / "dram_traffic.txt"
    try:
        for line in p.read_text().splitlines():
            parts = line.split()
            if parts and not line.startswith("#") and parts[0] == workload:
                return int(parts[1]), parts[2] if len(parts) > 2 else None
    except Exception:
        pass
    return None, None


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples: list[tuple[int, int]] = []
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None
        self.error = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                    uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report the gap instead of guessing
            self.nvml = None
            self.error = f"nvml unavailable: {e}"

    def _read(self):
        n = self.nvml
        mhz = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
        try:
            reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception:
            reasons = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
        return mhz, reasons

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._read())
            except Exception as e:
                self.error = str(e)
                return
            time.sleep(self.period)

    def start(self):
        if self.nvml is not None:
            self._stop.clear()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            self._thread = None

    def summary(self, window: str) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0, "window": window, "note": self.error or "no samples"}
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [name for bit, name in self.REASONS.items() if mask & bit and bit != 0x1]
        return {
            "sm_mhz": statistics.median(m for m, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(self.samples),
            "window": window,
        }


# --------------------------------------------------------------------------- workloads


def workload_rows(w, world: int, rank: int):
    """(rows this rank processes, scaling) for the workload."""
    from thingy_b200.shard import shard_rows

    if w.name == "g128_sharded_262144x8192":
        return shard_rows(w.M, world, rank).rows, "strong"
    return w.M, "weak"


def rows_override(args, w, M: int, scaling: str):
    """--rows R: R rows a rank, weak scaling (a smaller case of the same kernel)."""
    if args.rows <= 0:
        return M, scaling
    return args.rows, "weak"


def n_workspaces(w, M) -> int:
    """Workspaces rotated between steps so a step never finds its data in L2."""
    return max(2, math.ceil(3 * L2_BYTES / w.bytes_moved(M)))


def bench_config(args, w, M: int, world: int, scaling: str) -> dict:
    """The `config` object of the JSON line; both arms emit exactly this."""
    bytes_step = w.bytes_moved(M)
    n_ws = n_workspaces(w, M)
    return {
        "workload": w.name,
        "rows_per_gpu": M,
        "rows_total": w.M if scaling == "strong" else world * M,
        "H": w.H,
        "group_size": w.group_size or "per-token",
        "scale_format": w.scale_format,
        "scale_layout": w.scale_layout,
        "residual": w.residual,
        "parallelism": (f"row shards, dp{world}, "
                        + ("one batch split by rows" if scaling == "strong"
                           else "a full batch per rank") + ", no data-path collective"),
        "l2": f"rotating {n_ws} workspaces of {bytes_step / 1e6:.1f} MB "
              f"({n_ws * bytes_step / 1e6:.0f} MB > L2 {L2_BYTES / 1e6:.0f} MB)",
        **({"N": w.N} if w.kind == "prologue" else {}),
        "threads_per_row": args.threads_per_row or "auto",
        "launch": "one CUDA graph of the K launches" if args.graph else "eager launches",
    }


def dtype_of(w) -> str:
    if w.kind == "rms_bf16":
        return "bf16 in, fp32 statistics, bf16 out"
    if w.kind == "rms_f32":
        return "fp32"
    if w.kind == "prologue":
        return "bf16 in, fp32 statistics, e4m3 x e4m3 MXFP8 MMA, fp32 accumulate, bf16 out"
    return ("bf16 gradients, fp32 sums, e4m3 dx" if w.kind == "bwd"
            else "bf16 in, fp32 statistics, e4m3 out")


class Workspace:
    """One set of device inputs and outputs for a step."""

    def __init__(self, w, M, src, device):
        import thingy_b200 as tb

        if w.kind in ("rms_f32", "rms_bf16"):
            self.x = src["x"].clone()
            self.out = torch.empty_like(self.x)
            self.res = None
            return
        if w.kind == "prologue":
            from thingy_b200.ops import launch_rms_norm_fp8

            # each workspace has its own copy of the GEMM weight, so a step
            # never finds it in L2 (a decode step reads a new layer's weight)
            self.x = src["x"].clone()
            self.d = torch.empty(M, w.N, dtype=torch.bfloat16, device=device)
            self.qb = torch.empty(w.N, w.H, dtype=torch.float8_e4m3fn, device=device)
            self.sb = tb.empty_scale(w.N, w.H, 32, "e8m0", "mx", device)
            launch_rms_norm_fp8(src["gemm_weight"], None, 0.0, q=self.qb, scale=self.sb,
                                group_size=32, scale_format="e8m0", scale_layout="mx",
                                normalize=False)
            # the two-kernel path's intermediate (only the unfused comparison uses it)
            self.q = torch.empty(M, w.H, dtype=torch.float8_e4m3fn, device=device)
            self.scale = tb.empty_scale(M, w.H, 32, "e8m0", "mx", device)
            return
        if w.kind == "bwd":
            from thingy_b200.ops import backward_workspace_bytes

            self.dn = src["d_normalized"].clone()
            self.r = src["r"].clone()
            self.dro = src["d_residual_out"].clone() if "d_residual_out" in src else None
            self.dx = torch.empty_like(self.r)
            self.dw = torch.empty(w.H, dtype=torch.bfloat16, device=device)
            self.ws = torch.empty(backward_workspace_bytes(M, w.H, device), dtype=torch.uint8,
                                  device=device)
            self.q = (torch.empty(M, w.H, dtype=torch.float8_e4m3fn, device=device)
                      if w.group_size else None)
            self.scale = (tb.empty_scale(M, w.H, 128, w.scale_format, w.scale_layout, device)
                          if w.group_size else None)
            return
        self.x = src["x"].clone()
        self.res = src["residual"].clone() if "residual" in src else None
        self.q = torch.empty(M, w.H, dtype=torch.float8_e4m3fn, device=device)
        self.scale = tb.empty_scale(M, w.H, w.group_size, w.scale_format, w.scale_layout, device)
        self.res_out = torch.empty_like(self.x) if self.res is not None else None


def device_run(args, w, M, src, device, local_rank, world, K, unfused=False):
    """W warm-up steps, then K timed steps (CUDA events on the launch stream).

    unfused (prologue workloads): the two-kernel path instead of the fused
    kernel, for comparison. Returns (per-step ms of this rank, clock summary or None)."""
    from thingy_b200.gemm import mxfp8_gemm, rms_norm_mxfp8_gemm
    from thingy_b200.ops import launch_rms_norm, launch_rms_norm_backward, launch_rms_norm_fp8

    import torch.distributed as dist

    weight = src["weight"]
    n_ws = n_workspaces(w, M)
    ws = [Workspace(w, M, src, device) for _ in range(n_ws)]
    stream = torch.cuda.current_stream(device)

    def step(i):  # one launch on the current stream
        s = ws[i % n_ws]
        if w.kind in ("rms_f32", "rms_bf16"):
            launch_rms_norm(s.x, weight, w.eps, s.out, threads_per_row=args.threads_per_row)
            return
        if w.kind == "prologue":
            if unfused:  # RMSNorm + MXFP8 to HBM, then the GEMM reads it back
                launch_rms_norm_fp8(s.x, weight, w.eps, q=s.q, scale=s.scale, group_size=32,
                                    scale_format="e8m0", scale_layout="mx")
                mxfp8_gemm(s.q, s.scale, s.qb, s.sb, out=s.d)
            else:
                rms_norm_mxfp8_gemm(s.x, weight, w.eps, s.qb, s.sb, out=s.d, fused=True)
            return
        if w.kind == "bwd":  # backward: two kernels (rows, then the d_weight reduction)
            launch_rms_norm_backward(
                s.dn, s.r, weight, w.eps, dx=s.dx, d_residual_out=s.dro, d_weight=s.dw,
                workspace=s.ws, q=s.q, scale=s.scale, scale_format=w.scale_format,
                scale_layout=w.scale_layout)
            return
        launch_rms_norm_fp8(
            s.x, weight, w.eps, residual=s.res, q=s.q, scale=s.scale, residual_out=s.res_out,
            group_size=w.group_size, scale_format=w.scale_format, scale_layout=w.scale_layout,
            threads_per_row=args.threads_per_row,
        )

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(device)

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    graph = None
    if args.graph:
        # the same K launches recorded once; timed by events around the replay
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(K):
                step(i)
        torch.cuda.synchronize(device)
    clocks = ClockSampler(local_rank) if not args.no_clocks else None
    barrier()
    torch.cuda.synchronize(device)
    if clocks:
        clocks.start()
    # K launches back to back (no event between them, so a launch's prologue
    # may overlap the previous one's tail through programmatic dependent
    # launch); the mean launch is the timed region over K.
    start.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for i in range(K):
            step(i)
    end.record(stream)
    torch.cuda.synchronize(device)
    if clocks:
        clocks.stop()
    barrier()
    total_ms = start.elapsed_time(end)
    window = "timed"
    if clocks and len(clocks.samples) < 5:
        # The timed region was too short for the sampler: keep the same launches
        # running for ~1 s more (untimed) so the clock record covers the load.
        # Every rank soaks for the same wall time and meets at the barrier.
        t_end = time.monotonic() + 1.0
        clocks.start()
        i = 0
        while time.monotonic() < t_end:
            for _ in range(64):
                step(i)
                i += 1
            torch.cuda.synchronize(device)
        clocks.stop()
        window = "timed+1s untimed soak (timed region shorter than the sampler period)"
    barrier()
    del graph, ws
    return total_ms / K, (clocks.summary(window) if clocks else None)


def roofline(w, bytes_step, launch_ms, threads_per_row, M=None) -> dict:
    peak, peak_src = measured_peak()
    achieved = bytes_step / (launch_ms * 1e-3) / 1e9
    traffic, traffic_src = ncu_traffic(w.name)
    if traffic is not None and M is not None and M != w.M:
        traffic = round(traffic * M / w.M)  # DRAM bytes grow with the rows a launch processes
    return {
        "bound": "hbm",
        "achieved": round(achieved, 2),
        "peak": peak,
        "unit": "GB/s",
        "frac": round(achieved / peak, 4),
        "traffic": traffic,
        "traffic_source": traffic_src,
        "peak_source": peak_src,
        "kernel": _kernel_name(w, threads_per_row),
        "bytes_per_launch": bytes_step,
        "mean_launch_ms": round(launch_ms, 5),
    }


def run_ours(args, rank, world, local_rank):
    import thingy_b200 as tb
    from thingy_b200 import _lib
    from thingy_b200.host import rms_norm_fp8_host
    from thingy_b200.shard import max_over_ranks
    from thingy_b200.workloads import WORKLOADS, make_inputs

    import torch.distributed as dist

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _lib.load()
    w = WORKLOADS[args.workload]
    M, scaling = rows_override(args, w, *workload_rows(w, world, rank))
    src = make_inputs(w, M, device=device, seed=0, row_offset=rank)
    weight = src["weight"]
    bytes_step = w.bytes_moved(M)
    K = args.steps
    step_ms, clocks = device_run(args, w, M, src, device, local_rank, world, K)
    t_step_ms = max_over_ranks(step_ms, device) if world > 1 else step_ms
    unfused = None
    if w.kind == "prologue":  # the same step as two kernels, for comparison
        u_ms, _ = device_run(args, w, M, src, device, local_rank, world, K, unfused=True)
        u_ms = max_over_ranks(u_ms, device) if world > 1 else u_ms
        unfused = {
            "ms_per_step": round(u_ms, 5),
            "launches_per_step": 2,
            "path": "cutie_rms_norm_fp8 (1x32, e8m0, swizzled) to HBM, then cutie_gemm_mxfp8",
            "fused_speedup": round(u_ms / t_step_ms, 3),
        }

    # all ranks' algorithmic bytes (strong scaling: the whole batch, plus one
    # weight read per extra rank) over the slowest rank's step time
    total_bytes = world * bytes_step if scaling == "weak" else (
        w.bytes_moved() + 2 * w.H * (world - 1))
    value = total_bytes / (t_step_ms * 1e-3) / 1e9
    rows_total = world * M if scaling == "weak" else w.M
    peak, _ = measured_peak()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # e2e through the host-buffer API: pinned host x in, q + scales out
    e2e = None
    if not args.no_e2e and w.kind == "fused":
        K2 = args.e2e_steps or min(K, 20)
        xh = src["x"].cpu().pin_memory()
        rh = src["residual"].cpu().pin_memory() if "residual" in src else None
        qh = torch.empty(M, w.H, dtype=torch.float8_e4m3fn).pin_memory()
        sh = tb.empty_scale(M, w.H, w.group_size, w.scale_format, w.scale_layout, "cpu")
        sh = sh.pin_memory() if sh.is_contiguous() else sh.t().contiguous().pin_memory().t()
        roh = torch.empty_like(xh).pin_memory() if rh is not None else None
        pipe = None
        chunk = 2048
        stream = torch.cuda.current_stream(device)

        def e2e_step():
            nonlocal pipe
            pipe = rms_norm_fp8_host(
                xh, weight, w.eps, residual=rh, out=qh, scale=sh, residual_out=roh,
                group_size=w.group_size, scale_format=w.scale_format,
                scale_layout=w.scale_layout, pipeline=pipe, chunk_rows=chunk)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(device)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(K2):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / K2
        e2e_ms = max_over_ranks(e2e_ms, device) if world > 1 else e2e_ms
        h2d = xh.numel() * 2 + (rh.numel() * 2 if rh is not None else 0)
        d2h = qh.numel() + sh.numel() * sh.element_size() + (
            roh.numel() * 2 if roh is not None else 0)
        e2e = {
            "value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 3),
            "unit": "GB/s",
            "ms_per_step": round(e2e_ms, 4),
            "steps": K2,
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "thingy_b200.host.rms_norm_fp8_host (pinned host buffers, "
                   f"{chunk}-row chunks over 3 streams)",
        }
        del xh, rh, qh, sh, roh, pipe

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and w.kind == "fused":
        cpu = cpu_baseline(w, args.cpu_seconds)

    # N = 1 with the default workload: also time BASELINE config 2 (the
    # DeepSeek-V3 shape) on the device, same rules, so its roofline is on record
    secondary = None
    if args.secondary and world == 1:
        del src
        torch.cuda.empty_cache()
        w2 = WORKLOADS[SECONDARY_WORKLOAD]
        src2 = make_inputs(w2, device=device, seed=0)
        ms2, clocks2 = device_run(args, w2, w2.M, src2, device, local_rank, 1, K)
        del src2
        b2 = w2.bytes_moved()
        secondary = {
            "workload": w2.name,
            "value": round(b2 / (ms2 * 1e-3) / 1e9, 2),
            "unit": "GB/s",
            "ms_per_step": round(ms2, 5),
            "steps": K,
            "tokens_per_s": round(w2.M / (ms2 * 1e-3), 1),
            "config": bench_config(args, w2, w2.M, 1, "weak"),
            "roofline": roofline(w2, b2, ms2, args.threads_per_row),
            "clocks": clocks2,
        }

    result = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(t_step_ms, 5),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": dtype_of(w),
        "data": "synthetic (seeded; shapes and distributions of the workload)",
        "config": bench_config(args, w, M, world, scaling),
        "tokens_per_s": round(rows_total / (t_step_ms * 1e-3), 1),
        "pct_of_hbm_peak": round(100 * value / (peak * world), 2),
        "pct_of_8tbs": round(100 * value / (8000.0 * world), 2),
        "roofline": roofline(w, bytes_step, t_step_ms, args.threads_per_row, M),
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": K * (2 if w.kind == "bwd" else 1),
        "clocks": clocks,
    }
    if secondary is not None:
        result["secondary"] = secondary
    if unfused is not None:
        result["unfused"] = unfused
    if rank == 0:
        print(json.dumps(result), flush=True)


# --------------------------------------------------------------------------- CPU legs


def cpu_sample_rows(w, target_s: float, threads: int):
    """Rows of the workload whose oracle pass takes about target_s / 4 seconds."""
    from oracle import reference as ora
    from thingy_b200.workloads import make_inputs

    probe = min(w.M, 256)
    inp = make_inputs(w, probe, device="cpu", seed=0)
    t0 = time.perf_counter()
    ora.rms_norm_fp8(inp["x"], inp["weight"], w.eps, residual=inp.get("residual"),
                     group_size=w.group_size, scale_format=w.scale_format)
    dt = time.perf_counter() - t0
    rows = int(probe * (target_s / 4) / max(dt, 1e-6))
    return max(16, min(w.M, rows))


def time_oracle(w, rows: int, reps: int):
    from oracle import reference as ora
    from thingy_b200.workloads import make_inputs

    inp = make_inputs(w, rows, device="cpu", seed=0)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        if w.kind == "rms_bf16":
            ora.rms_norm_reference(inp["x"], inp["weight"], w.eps)
        elif w.kind == "rms_f32":
            ora.rms_norm_f32(inp["x"], inp["weight"], w.eps)
        else:
            q, s, _, _ = ora.rms_norm_fp8(inp["x"], inp["weight"], w.eps,
                                          residual=inp.get("residual"),
                                          group_size=w.group_size, scale_format=w.scale_format)
            if w.scale_layout != "row":
                ora.layout_scales(s, w.scale_layout)
        times.append(time.perf_counter() - t0)
    return times


def cpu_baseline(w, target_s: float) -> dict:
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = cpu_sample_rows(w, target_s, threads)
    times = time_oracle(w, rows, 4)
    t = statistics.median(times)
    return {
        "value": round(w.bytes_moved(rows) / t / 1e9, 4),
        "unit": "GB/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"{rows} of {w.M} rows of {w.name}, median of 4 passes "
                  f"({t:.3f} s each), torch CPU ops as in the reference's PyTorch path",
        "cpu": cpu_model(),
    }


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args, rank, world):
    """The reference's PyTorch path on the host cores (oracle/reference.py restates it).

    Imports only pure-Python modules of the package (workloads, shard): the
    CUDA library and the torch binding are never loaded by this arm."""
    if rank != 0:
        return
    from thingy_b200.workloads import WORKLOADS

    w = WORKLOADS[args.workload]
    M, scaling = rows_override(args, w, *workload_rows(w, world, rank))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # bounded sample per step so W + K steps finish in a few minutes
    per_step_s = min(2.0, 150.0 / max(1, args.steps + args.warmup))
    rows = min(M, cpu_sample_rows(w, 4 * per_step_s, threads))
    time_oracle(w, rows, args.warmup)
    times = time_oracle(w, rows, args.steps)
    t = sum(times) / len(times)
    value = w.bytes_moved(rows) / t / 1e9
    sample = (f"{rows} of the {M} rows of one rank of {w.name} per step, torch CPU ops "
              "as in the reference's PyTorch path (oracle/reference.py), rank 0 only")
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": dtype_of(w),
        "data": "synthetic (seeded; shapes and distributions of the workload)",
        "config": bench_config(args, w, M, world, scaling),
        "tokens_per_s": round(rows / t, 1),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse_args()
    from thingy_b200.shard import init_from_env

    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, rank, world_env)
        return
    if world_env != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world_env}: launch N>1 with torchrun")
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    rank, world, local_rank = init_from_env("nccl" if world_env > 1 else "gloo", timeout_s=300)
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
