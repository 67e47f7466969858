"""Benchmark of the B200-native NeRF hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload encode]

Workloads (BASELINE configurations, seeded synthetic inputs -- the reference's datasets are not
available here):
  encode  config 0: hash-grid encoding forward + backward, 2^18 points per GPU, L=16, F=2,
          log2 T=19, base 16, b=exp(ln(2048/16)/15).  One step = forward, zero the fp32 gradient
          table, backward (and, for N > 1, an NCCL all-reduce of the gradient table).

Timing: W untimed warm-up steps, then K steps each bracketed by CUDA events on the launching
stream; L2 is flushed (a 256 MB write) before every timed step, outside the events.  The whole
timed loop is bracketed by a barrier and a device synchronize; the max over ranks is reported.
`value` is the whole-job throughput (all ranks' points / max per-rank time).  `e2e` repeats the
step through the public API with host-resident (pinned) inputs copied in and the result copied
out inside the timed region.

--impl reference runs the reference's own CUDA build (oracle/_ref, compiled from the reference's
sources for sm_100a) on the same workload at the reference's layout (8 levels x 4 features, the
only one its kernels support), on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "instant-ngp_b200"))

L2_FLUSH_BYTES = 256 << 20


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region (200 ms period)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout: float = 5.0) -> None:
        """Block until nvidia-smi has produced its first sample, so the timed region is covered."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.05)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------
# distributed plumbing
# ------------------------------------------------------------------------------------------------
def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------------
# encode workload (config 0)
# ------------------------------------------------------------------------------------------------
ENCODE_N = 1 << 18


def time_steps(step_fn, steps: int, warmup: int, flush, stream, world: int, events_per_kernel=None):
    """Warm up, then time `steps` calls of step_fn, each between CUDA events on `stream` with an
    L2 flush before it (outside the events).  Returns per-step ms list (this rank)."""
    import torch

    for _ in range(warmup):
        step_fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        flush()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        step_fn()
        end.record(stream)
        end.synchronize()
        times.append(start.elapsed_time(end))
    torch.cuda.synchronize()
    barrier(world)
    return times


def bench_encode_ours(args, rank, world, local):
    import torch
    import ngp_b200 as ngp
    import workloads

    layout = ngp.config0_layout()
    L, F, n = 16, 2, ENCODE_N
    coords_h, table_h, dy_h = workloads.encode_inputs(n, layout.n_params, L, F, seed=1000 + rank)
    stream = torch.cuda.current_stream()
    coords = torch.from_numpy(coords_h).cuda()
    table = torch.from_numpy(table_h.view(np.int16)).cuda()
    dy = torch.from_numpy(dy_h).cuda()
    feats = torch.empty((L * F, n), dtype=torch.float16, device="cuda")
    grad = torch.empty(layout.n_params, dtype=torch.float32, device="cuda")
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    def flush():
        flush_buf.fill_(1.0)

    def step():
        ngp.encode_grid_forward(layout, coords, table, feats, stream=stream)
        grad.zero_()
        ngp.encode_grid_backward(layout, coords, dy, grad, stream=stream)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(grad)

    # per-kernel timing (for the roofline) on the same stream, L2 flushed before each launch
    def kernel_times(reps=20):
        fw, bw = [], []
        for _ in range(reps):
            for which, acc in (("f", fw), ("b", bw)):
                flush()
                if which == "b":
                    grad.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                if which == "f":
                    ngp.encode_grid_forward(layout, coords, table, feats, stream=stream)
                else:
                    ngp.encode_grid_backward(layout, coords, dy, grad, stream=stream)
                e.record(stream)
                e.synchronize()
                acc.append(s.elapsed_time(e))
        return statistics.median(fw), statistics.median(bw)

    with ClockSampler(local) as clocks:
        clocks.wait_first()
        times = time_steps(step, args.steps, args.warmup, flush, stream, world)
        time.sleep(0.25)
    ms = max_over_ranks(sum(times) / len(times), world)
    fwd_ms, bwd_ms = kernel_times() if not args.quick else (float("nan"), float("nan"))
    if args.quick:
        return {"metric": "hash-encode fwd+bwd Gpts/s (config 0)", "value": world * n / (ms * 1e-3) / 1e9, "quick": True}

    # e2e through the public API: pinned host inputs in, encoded features out, every step.
    coords_pin = torch.from_numpy(coords_h).pin_memory()
    dy_pin = torch.from_numpy(dy_h).pin_memory()
    feats_pin = torch.empty((L * F, n), dtype=torch.float16).pin_memory()

    def e2e_step():
        coords.copy_(coords_pin, non_blocking=True)
        dy.copy_(dy_pin, non_blocking=True)
        step()
        feats_pin.copy_(feats, non_blocking=True)

    e2e_times = time_steps(e2e_step, max(3, args.steps // 2), 2, flush, stream, world)
    e2e_ms = max_over_ranks(sum(e2e_times) / len(e2e_times), world)
    h2d = coords_h.nbytes + dy_h.nbytes
    d2h = feats.numel() * 2

    peaks = load_peaks()
    # algorithmic bytes per point (forward): 12 B coords + 64 B features out (HBM) + 8 corners x
    # 16 levels x 2 features x 2 B gathered from the table (served by L2 / L1).
    fwd_bytes_pt = 12 + L * F * 2 + L * 8 * F * 2
    bwd_bytes_pt = 12 + L * F * 2 + L * 8 * F * 4
    dom = "forward" if fwd_ms >= bwd_ms else "backward"
    dom_ms = max(fwd_ms, bwd_ms)
    dom_bytes = (fwd_bytes_pt if dom == "forward" else bwd_bytes_pt) * n
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    res = {
        "metric": "hash-encode fwd+bwd Gpts/s (config 0)",
        "value": round(world * n / (ms * 1e-3) / 1e9, 4),
        "unit": "Gpts/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16 table/features, fp32 accumulation and gradients",
        "data": "synthetic (seeded uniform points, U(+-1e-4) fp16 table, N(0,1) fp16 dL/dy)",
        "config": {"workload": "config0 hash-grid encode fwd+bwd", "points_per_gpu": n, "levels": L, "features": F,
                   "log2_hashmap_size": 19, "base_resolution": 16, "per_level_scale": round(2 ** (7 / 15), 6),
                   "parallelism": f"dp{world}", "l2": "flushed (256 MB write) before every timed step"},
        "kernels_ms": {"encode_forward": round(fwd_ms, 5), "encode_backward": round(bwd_ms, 5)},
        "roofline": {"kernel": f"encode_{dom}", "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": peaks["source"],
                     "note": "achieved counts HBM streams plus table bytes gathered (L2-served) per point"},
        "e2e": {"value": round(world * n / (e2e_ms * 1e-3) / 1e9, 4), "unit": "Gpts/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_encode(layout)
    return res


def cpu_baseline_encode(layout, budget_s: float = 12.0) -> dict:
    """The oracle (scalar C++ port of the reference math) on the host cores, bounded sample."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import workloads
    from oracle import Oracle

    ora = Oracle()
    cores = os.cpu_count() or 1
    lay = (np.array(layout.level_offsets(), np.uint32), np.array(layout.level_resolutions(), np.uint32),
           np.array(layout.level_scales(), np.float32))
    n = 1 << 15
    coords, table, dy = workloads.encode_inputs(n, layout.n_params, 16, 2, seed=7)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        ora.encode_forward(lay, coords, table, 2, mode=0, threads=cores)
        ora.encode_backward(lay, coords, dy, 2, threads=cores)
        done += n
    dt = time.perf_counter() - t0
    return {"value": round(done / dt / 1e9, 6), "unit": "Gpts/s", "cores": cores, "kind": "port",
            "sample": f"{done} points of config 0 (fwd+bwd, {n}-point batches) in {dt:.1f} s"}


def bench_encode_reference(args, rank, world, local):
    """The reference's own encode_grid_forward/backward kernels (its 8x4 layout) on one B200."""
    import torch

    sys.path.insert(0, str(ROOT / "oracle"))
    import workloads
    from oracle import RefLib

    ref = RefLib()
    total = int(ref.lib.ref_total_param_count())
    mlp = int(ref.lib.ref_mlp_param_count())
    n_grid = total - mlp
    n = ENCODE_N
    coords_h, table_h, dy_h = workloads.encode_inputs(n, n_grid, 8, 4, seed=1000, coord_stride=7)
    stream = torch.cuda.current_stream()
    coords = torch.from_numpy(coords_h).cuda()
    table = torch.from_numpy(table_h.view(np.int16)).cuda()
    dy = torch.from_numpy(dy_h).cuda()
    feats = torch.empty((32, n), dtype=torch.float16, device="cuda")
    grad = torch.empty(n_grid, dtype=torch.float16, device="cuda")
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    sp = ctypes.c_void_p(stream.cuda_stream)

    def step():
        ref.call("ref_encode_forward", ctypes.c_uint32(n), ctypes.c_void_p(coords.data_ptr()), ctypes.c_void_p(table.data_ptr()),
                 ctypes.c_void_p(feats.data_ptr()), sp)
        grad.zero_()
        ref.call("ref_encode_backward", ctypes.c_uint32(n), ctypes.c_void_p(coords.data_ptr()), ctypes.c_void_p(dy.data_ptr()),
                 ctypes.c_void_p(grad.data_ptr()), sp)

    with ClockSampler(local) as clocks:
        clocks.wait_first()
        times = time_steps(step, args.steps, args.warmup, lambda: flush_buf.fill_(1.0), stream, 1)
        time.sleep(0.25)
    ms = sum(times) / len(times)
    value = n / (ms * 1e-3) / 1e9
    return {
        "impl": "reference",
        "metric": "hash-encode fwd+bwd Gpts/s (config 0)",
        "value": round(value, 4), "unit": "Gpts/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 table/features, fp16 accumulation and gradients (reference)",
        "data": "synthetic (seeded)",
        "config": {"workload": "config0 hash-grid encode fwd+bwd", "points_per_gpu": n, "levels": 8, "features": 4,
                   "note": "reference kernels support only their compiled 8x4 layout (static_assert ngp.train.cu:58); "
                           "same 32 features and 512 gathered table bytes per point as config 0",
                   "parallelism": "dp1", "l2": "flushed (256 MB write) before every timed step"},
        "cpu_baseline": {"value": round(value, 4), "unit": "Gpts/s", "cores": 0, "kind": "reference",
                         "sample": "reference CUDA build (oracle/_ref) on one B200; the reference has no CPU implementation"},
        "e2e": {"value": round(value, 4), "unit": "Gpts/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "clocks": clocks.summary(),
    }


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["encode"], default="encode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="timed steps only (for profiler runs)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank, world, local = dist_setup()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(bench_encode_reference(args, rank, world, local)), flush=True)
        return 0
    res = bench_encode_ours(args, rank, world, local)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
