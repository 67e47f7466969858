"""Benchmark of the B200-native NeRF hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload train|encode|mlp|march|render]

Workloads (BASELINE configurations; seeded synthetic inputs stand in for the reference's
NeRF-synthetic datasets, which are not available here):
  train   config 3 (default): end-to-end NeRF training on the procedural 64-sphere scene, 100
          train / 20 test views of 800x800, config-0 hash grid + config-1 MLPs, batch 2^18
          samples per step per GPU with the adaptive ray count.  One step = the reference's
          step (density-grid update on its schedule, marching, inference pass, loss and
          compaction, backward, Adam); data parallel over N GPUs with one NCCL gradient
          all-reduce per step (weak scaling: 2^18 samples per GPU).
  encode  config 0: hash-grid encoding forward + backward, 2^18 points per GPU.
  mlp     config 1: fused density + colour MLPs forward + backward, 2^18 rows per GPU.
  march   config 2: density-grid update + marching of 2^18 rays per GPU.
  render  config 4: 1920x1080 novel views of a model trained with log2 T = 22.

Timing: W untimed warm-up steps, then K steps timed on the device with CUDA events on the
stream that runs them, bracketed by a barrier and a device synchronize; the max over ranks is
reported.  Training's working set (117 MB of samples, 268 MB of encodings, 256 MB dataset)
exceeds the 126 MB L2; the encode workload flushes L2 before every timed step.

--impl reference runs the reference's own CUDA build (oracle/_ref, compiled from the reference's
sources for sm_100a) on the same workload, on rank 0 only, at the reference's compiled grid
layout (8 levels x 4 features; its kernels support no other).
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
BATCH = 1 << 18


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
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout: float = 5.0) -> None:
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

    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def clocks_ok(c: dict) -> bool:
    return not any(r in c.get("reasons", []) for r in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"))


# ------------------------------------------------------------------------------------------------
# train workload (config 3)
# ------------------------------------------------------------------------------------------------
def make_dataset(args):
    import workloads

    return workloads.procedural_dataset(n_train=args.views, n_test=args.test_views, width=args.res, height=args.res, seed=3, device="cuda")


# FLOPs per row of the fused MLPs: forward 2*(32*64 + 64*16) + 2*(32*64 + 64*64 + 64*16) = 20,480;
# forward + backward (input gradients + weight gradients) = 61,440.
MLP_FWD_FLOP = 20480
MLP_FWDBWD_FLOP = 61440
DENSITY_FWD_FLOP = 6144
COMPACTED_ROWS = BATCH + 1024


# Algorithmic HBM bytes per unit of each training-step phase (inputs read once, outputs written
# once; table gathers and atomics are L1/L2-served and counted separately), and the DRAM bytes
# per unit that one ncu capture of the phase's main kernel measured (the profiles/ summaries of
# the config-3 step: DRAM read + write of that launch / units it processed).
PHASE_BYTES = {
    # per marched sample: its record is read once (28 B) to decide how far the ray keeps samples;
    # the densities evaluated (encoding 12 B in + 64 B out, density 64 B in + 2 B out) cover only the
    # samples in front of each ray's stopping point, and the kept ones are compacted (92 B each)
    "inference_compact": {"unit": "pre-compaction sample", "bytes": 28, "kernel": "encode_forward_points_kernel + mlp_forward_kernel<density> + keep/compact",
                          # DRAM read + write of the phase's launches in one ncu-captured step of
                          # 1,393,551 marched samples (two rounds of encode, density, keep and list
                          # kernels, then the compaction copy that the selection flow has since
                          # replaced; the selection flow's step in profiles/*__train_config3.md
                          # reads and writes 176 MB)
                          "ncu_dram_bytes_per_unit": 218.9e6 / 1393551},
    # 12 B rays in + 28 B records out per sample (dominant), 8 B per ray of counts
    "march": {"unit": "pre-compaction sample", "bytes": 28, "kernel": "march_count_kernel + march_write_kernel"},
    "encode_bwd": {"unit": "batch sample", "bytes": 12 + 64, "l2_atomic_bytes": 16 * 8 * 2 * 4, "kernel": "encode_backward_kernel"},
    "adam": {"unit": "parameter", "bytes": 40, "kernel": "adam_kernel"},
    "mlp_fwd_loss_pad": {"unit": "batch sample", "bytes": 64 + 32 + 28 + 32, "kernel": "mlp_forward_kernel + loss_compacted_kernel"},
    "grid_update": {"unit": "grid cell", "bytes": 16, "kernel": "density grid kernels"},
}


def phase_roofline(phases: dict, peaks: dict) -> dict:
    """Roofline of the dominant phase of the training step.  Phase durations come from CUDA events
    recorded on the trainer's stream between the phases of profiled steps (run right after the
    timed steps, on the same model); units per launch are the step's sample counts."""
    steps = max(phases["steps"], 1)
    ms = {k: v / steps for k, v in phases["ms"].items()}
    n_inf = phases["mean_inference_samples"]
    total = sum(ms.values())
    # the profiled steps march serially; in the timed steps the march runs on its own stream
    # during the previous step's backward pass, so the dominant phase is taken among the others
    dom = max((k for k in ms if k != "march"), key=ms.get)
    t = ms[dom] * 1e-3
    if dom == "mlp_bwd":
        flops = MLP_FWDBWD_FLOP * BATCH
        achieved = flops / t / 1e12
        return {"kernel": dom, "bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16_tflops_sustained"], 4), "traffic": None, "share": round(ms[dom] / total, 3),
                "peak_source": peaks["source"] + " (sustained dense bf16; fp16 has the same tensor rate)"}
    info = PHASE_BYTES.get(dom, {"unit": "?", "bytes": 0, "kernel": dom})
    units = {"pre-compaction sample": n_inf, "batch sample": BATCH, "parameter": 12_206_480, "grid cell": 128 ** 3 * 2}.get(info["unit"], 0)
    achieved = info["bytes"] * units / t / 1e9
    res = {"kernel": info["kernel"], "phase": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
           "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None, "share": round(ms[dom] / total, 3),
           "peak_source": peaks["source"] + " (HBM copy bandwidth)",
           "per_unit": f"{info['bytes']} algorithmic HBM bytes per {info['unit']}, {units:.0f} units per launch, {ms[dom] * 1e3:.1f} us per launch"}
    if "ncu_dram_bytes_per_unit" in info:
        res["traffic"] = round(info["ncu_dram_bytes_per_unit"] * units)
        res["traffic_note"] = "ncu DRAM read+write of one launch of this kernel in the config-3 step, per unit, times this launch's units"
    if "l2_gather_bytes" in info:
        res["l2_gather_GBps"] = round(info["l2_gather_bytes"] * units / t / 1e9, 1)
        res["note"] = ("the table (24 MB) is L2-resident: the kernel is bound by L1/L2 gather issue (16 levels x 8 corner loads per "
                       "sample), not by HBM; l2_gather_GBps counts the gathered table bytes")
    return res


def bench_train_ours(args, rank, world, local):
    import torch
    import ngp_b200 as ngp

    peaks = load_peaks()
    ds = make_dataset(args)
    model = ngp.InstantNGP(ds, ngp.config0_trainer_config())
    if world > 1:
        model.join_process_group()
    model.train(args.warmup)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        clocks.wait_first()
        launches0 = ngp.kernel_launch_count()
        stats = model.train(args.steps)
        launches = ngp.kernel_launch_count() - launches0
        time.sleep(0.25)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(stats["elapsed_ms"], world)
    # per-phase breakdown (separate, profiled steps; not part of the timed number)
    model.set_profiling(True)
    model.train(min(args.steps, 50))
    phases = model.phase_times()
    model.set_profiling(False)
    # e2e through the public API: one train(1) call per step (host round trip, counters and loss
    # read back every step), timed with events around the whole loop
    n_e2e = max(3, args.steps // 4)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    rays = 0
    for _ in range(n_e2e):
        st = model.train(1)
        rays = st["rays_per_batch"]
    e.record()
    e.synchronize()
    e2e_ms = max_over_ranks(s.elapsed_time(e) / n_e2e, world)
    psnr = model.test(count=min(4, args.test_views))["psnr"] if rank == 0 else None
    model.close()
    value = world * BATCH * args.steps / (ms * 1e-3)
    res = {
        "metric": "NeRF train samples/s (config 3)",
        "value": round(value, 1),
        "unit": "samples/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16 params/activations, fp32 accumulation, gradients and Adam",
        "data": "synthetic procedural scene (64 Lambert spheres, seeded), rendered on the device",
        "config": {"workload": "config3 end-to-end training", "views": args.views, "resolution": args.res, "batch_samples_per_gpu": BATCH,
                   "grid": "L=16 F=2 log2T=19 base 16 b=1.3819", "mlp": "density 32-64-16, colour 32-64-64-16",
                   "parallelism": f"dp{world} (NCCL all-reduce of the fp32 gradient per step)",
                   "l2": "working set > L2 (samples 117 MB, encodings 268 MB, dataset 256 MB); no flush",
                   "pre_compaction_samples_per_step": stats["measured_sample_count_before_compaction"],
                   "rays_per_batch": stats["rays_per_batch"], "test_psnr_after_run": psnr,
                   "steps_trained": args.warmup + args.steps},
        "phase_ms_per_step": {k: round(v / max(phases["steps"], 1), 4) for k, v in phases["ms"].items()},
        "roofline": phase_roofline(phases, peaks),
        "e2e": {"value": round(world * BATCH / (e2e_ms * 1e-3), 1), "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 12 + 4 * rays,
                "note": "InstantNGP.train(1) per step; the dataset is uploaded once at construction (as the reference does), each step "
                        "reads back its 3 counters and the per-ray loss"},
        "gpu_launches": None,
        "clocks": clocks.summary(),
    }
    res["gpu_launches"] = launches
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_train(args, int(stats["measured_sample_count_before_compaction"]))
    return res


def cpu_baseline_train(args, pre_compaction: int, budget_s: float = 4.0) -> dict:
    """The scalar C++ oracle (the reference's algorithm restated on the host) timed on bounded
    samples of each part of a config-3 training step, combined into the time of one step at this
    run's per-step counts: marching of every pre-compaction sample, the encoding + full network
    forward on all of them (the reference's inference pass), the encoding + network forward and
    backward of the 2^18-sample batch, and Adam over every parameter, each on all host cores."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import ngp_b200 as ngp
    import workloads
    from oracle import Oracle

    ora = Oracle()
    cores = os.cpu_count() or 1
    lay = ngp.config0_layout()
    layt = (np.array(lay.level_offsets(), np.uint32), np.array(lay.level_resolutions(), np.uint32), np.array(lay.level_scales(), np.float32))
    n = 1 << 13
    coords, table, dy_enc = workloads.encode_inputs(n, lay.n_params, 16, 2, seed=7, coord_stride=7)
    _, c2, dy = workloads.mlp_inputs(n, seed=8)
    coords[:, 4:7] = c2[:, 4:7]
    params = workloads.xavier_mlp_params(1)

    def rate(fn, units):
        done, t0 = 0, time.perf_counter()
        while True:
            fn()
            done += units
            dt = time.perf_counter() - t0
            if dt >= budget_s:
                return done / dt

    # encoding + full network forward (threaded oracle)
    fwd = rate(lambda: ora.mlp_forward(params, ora.encode_forward(layt, coords, table, 2, mode=0, threads=cores), coords, threads=cores), n)

    # network backward + encoding backward
    x = ora.encode_forward(layt, coords, table, 2, mode=0, threads=cores)
    mlp_bwd = rate(lambda: ora.mlp_backward(params, x, coords, dy, threads=cores), n)
    enc_bwd = rate(lambda: ora.encode_backward(layt, coords, dy_enc, 2, threads=cores), n)
    # marching, per emitted sample
    vals = workloads.blob_grid_values(workloads.gaussian_blob_density())
    bits = np.packbits((vals > 0.01).reshape(-1, 8), axis=1, bitorder="little").reshape(-1)
    rays = workloads.march_rays_config2(4096, seed=3)
    per_call = ora.march_rays_mt(rays, bits, cores)[2]
    march = rate(lambda: ora.march_rays_mt(rays, bits, cores), per_call)
    # Adam, every parameter touched
    m_p = 1 << 20
    master = np.random.default_rng(1).uniform(-1e-4, 1e-4, m_p).astype(np.float32)
    adam_state = [master, master.astype(np.float16), np.full(m_p, 1e-3, np.float32), np.zeros(m_p, np.float32), np.zeros(m_p, np.float32),
                  np.zeros(m_p, np.uint32)]
    adam = rate(lambda: ora.adam(10240, *adam_state, threads=cores), m_p)

    n_params = 12_206_480
    t_step = (pre_compaction / march + pre_compaction / fwd + BATCH / fwd + BATCH / mlp_bwd + BATCH / enc_bwd + n_params / adam)
    return {"value": round(BATCH / t_step, 1), "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": (f"one config-3 step ({pre_compaction} marched samples, {BATCH} batch samples, {n_params} parameters) timed part by "
                       f"part on bounded samples of the scalar oracle ({budget_s:.0f} s each): march {march / 1e6:.2f} M samples/s, "
                       f"encode + network forward {fwd / 1e6:.2f} M/s, network backward {mlp_bwd / 1e6:.2f} M/s, encode backward "
                       f"{enc_bwd / 1e6:.2f} M/s, Adam {adam / 1e6:.1f} M params/s; every part on {cores} host threads"),
            "step_s": round(t_step, 3)}


def bench_train_reference(args, rank, world, local):
    import torch

    sys.path.insert(0, str(ROOT / "oracle"))
    from oracle import RefLib

    ref = RefLib()
    ds = make_dataset(args)
    tr, te = ds["train"], ds["test"]
    px, cam = np.ascontiguousarray(tr["pixels"]), np.ascontiguousarray(tr["camera"])
    tpx, tcam = np.ascontiguousarray(te["pixels"]), np.ascontiguousarray(te["camera"])
    f = ref.lib
    f.ref_train_create.restype = ctypes.c_void_p
    h = f.ref_train_create(ctypes.c_void_p(px.ctypes.data), ctypes.c_size_t(px.nbytes), ctypes.c_void_p(cam.ctypes.data), ctypes.c_uint32(px.shape[0]),
                           ctypes.c_uint32(args.res), ctypes.c_uint32(args.res), ctypes.c_float(tr["focal"][0]), ctypes.c_float(tr["focal"][1]),
                           ctypes.c_float(tr["principal"][0]), ctypes.c_float(tr["principal"][1]), ctypes.c_void_p(tpx.ctypes.data),
                           ctypes.c_size_t(tpx.nbytes), ctypes.c_void_p(tcam.ctypes.data), ctypes.c_uint32(tpx.shape[0]))
    if not h:
        return {"impl": "reference", "unavailable": "reference trainer construction failed"}
    h = ctypes.c_void_p(h)
    out = (ctypes.c_float * 4)()
    if f.ref_train_steps(h, ctypes.c_int32(args.warmup), out) != 0:
        return {"impl": "reference", "unavailable": "reference training stopped during warm-up"}
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        clocks.wait_first()
        rc = f.ref_train_steps(h, ctypes.c_int32(args.steps), out)
        time.sleep(0.25)
    ms = float(out[0])
    sse = ctypes.c_double(0)
    f.ref_train_test_sse(h, ctypes.byref(sse))
    mse = sse.value / (args.test_views * args.res * args.res * 3.0)
    f.ref_train_destroy(h)
    value = BATCH * args.steps / (ms * 1e-3)
    return {
        "impl": "reference", "metric": "NeRF train samples/s (config 3)", "value": round(value, 1), "unit": "samples/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 params/activations and accumulation (reference)", "data": "synthetic procedural scene (seeded)",
        "config": {"workload": "config3 end-to-end training", "views": args.views, "resolution": args.res, "batch_samples_per_gpu": BATCH,
                   "grid": "reference compiled layout L=8 F=4 log2T=19 (its kernels support no other)", "parallelism": "dp1",
                   "pre_compaction_samples_per_step": int(out[2]), "rays_per_batch": int(out[3]),
                   "test_psnr_after_run": (-10 * math.log10(mse)) if mse > 0 else None, "steps_trained": args.warmup + args.steps,
                   "ok": rc == 0},
        "cpu_baseline": {"value": round(value, 1), "unit": "samples/s", "cores": 0, "kind": "reference",
                         "sample": "reference CUDA build (oracle/_ref: its own ngp::cuda step sequence) on one B200; the reference has "
                                   "no CPU implementation of this path"},
        "e2e": {"value": round(value, 1), "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 8},
        "clocks": clocks.summary(),
    }


# ------------------------------------------------------------------------------------------------
# encode workload (config 0)
# ------------------------------------------------------------------------------------------------
def time_steps(step_fn, steps: int, warmup: int, flush, stream, world: int):
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
    L, F, n = 16, 2, BATCH
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

    with ClockSampler(local) as clocks:
        clocks.wait_first()
        times = time_steps(step, args.steps, args.warmup, flush, stream, world)
        time.sleep(0.25)
    ms = max_over_ranks(sum(times) / len(times), world)
    fw, bw = [], []
    for _ in range(20):
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
    fwd_ms, bwd_ms = statistics.median(fw), statistics.median(bw)
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
    peaks = load_peaks()
    probe = probe_gather_scatter(stream)
    fwd_bytes_pt = 12 + L * F * 2 + L * 8 * F * 2
    bwd_bytes_pt = 12 + L * F * 2 + L * 8 * F * 4
    dom = "forward" if fwd_ms >= bwd_ms else "backward"
    dom_bytes = (fwd_bytes_pt if dom == "forward" else bwd_bytes_pt) * n
    achieved = dom_bytes / (max(fwd_ms, bwd_ms) * 1e-3) / 1e9
    return {
        "metric": "hash-encode fwd+bwd Gpts/s (config 0)", "value": round(world * n / (ms * 1e-3) / 1e9, 4), "unit": "Gpts/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 table/features, fp32 accumulation and gradients",
        "data": "synthetic (seeded uniform points, U(+-1e-4) fp16 table, N(0,1) fp16 dL/dy)",
        "config": {"workload": "config0 hash-grid encode fwd+bwd", "points_per_gpu": n, "levels": L, "features": F, "log2_hashmap_size": 19,
                   "base_resolution": 16, "per_level_scale": round(2 ** (7 / 15), 6), "parallelism": f"dp{world}",
                   "l2": "flushed (256 MB write) before every timed step"},
        "kernels_ms": {"encode_forward": round(fwd_ms, 5), "encode_backward": round(bwd_ms, 5)},
        "roofline": {"kernel": f"encode_{dom}", "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None, "peak_source": peaks["source"],
                     "note": "achieved counts HBM streams plus table bytes gathered (L2-served) per point; the L2-resident table makes "
                             "the kernels gather/atomic-bound: see l2_roofline"},
        "table_access": {
            "forward_Gaccess_s": round(n * L * 8 / (fwd_ms * 1e-3) / 1e9, 2), "backward_Gaccess_s": round(n * L * 8 / (bwd_ms * 1e-3) / 1e9, 2),
            "random_gather_Gaccess_s": probe["gather_G_s"], "random_float2_atomic_Gaccess_s": probe["scatter_G_s"],
            "note": "table corner accesses per second (8 corners x 16 levels per point) beside the measured rate of fully random "
                    "4-byte loads / float2 atomics on an L2-resident table (ngp_probe_gather / ngp_probe_scatter, run live).  The kernels "
                    "exceed the fully random rates because a cell's x-neighbour corners share sectors and the coarse levels stay L1-resident; "
                    "their bounding resource is L1 throughput (ncu l1tex__throughput 70-85 % of peak, "
                    "profiles/encode_forward_points_kernel__train_config3.md, profiles/encode_backward_kernel__train_config3.md)"},
        "e2e": {"value": round(world * n / (e2e_ms * 1e-3) / 1e9, 4), "unit": "Gpts/s", "h2d_bytes_per_step": coords_h.nbytes + dy_h.nbytes,
                "d2h_bytes_per_step": feats.numel() * 2},
        "gpu_launches": 2 * args.steps, "clocks": clocks.summary(),
    }


def probe_gather_scatter(stream) -> dict:
    """Measured rate of random 4-byte loads from a 32 MB table and of random float2 atomic adds
    into a 64 MB table (the L2-resident access patterns the encoding kernels are bound by)."""
    import torch
    import ngp_b200 as ngp

    lib = ngp.lib()
    threads, rounds = 1 << 20, 4
    tab = torch.ones(1 << 23, dtype=torch.int32, device="cuda")
    out = torch.empty(threads, dtype=torch.int32, device="cuda")
    acc = torch.zeros(1 << 24, dtype=torch.float32, device="cuda")
    s = ctypes.c_void_p(stream.cuda_stream)
    res = {}
    for name, call in (("gather_G_s", lambda: lib.ngp_probe_gather(ctypes.c_void_p(tab.data_ptr()), 23, threads, rounds, ctypes.c_void_p(out.data_ptr()), s)),
                       ("scatter_G_s", lambda: lib.ngp_probe_scatter(ctypes.c_void_p(acc.data_ptr()), 23, threads, rounds, s))):
        for _ in range(3):
            call()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record()
            for _ in range(10):
                if call() != 0:
                    raise RuntimeError(lib.ngp_last_error().decode())
            ev1.record()
        ev1.synchronize()
        res[name] = round(10 * threads * rounds * 16 / (ev0.elapsed_time(ev1) * 1e-3) / 1e9, 2)
    return res


def bench_encode_reference(args, rank, world, local):
    import torch

    sys.path.insert(0, str(ROOT / "oracle"))
    import workloads
    from oracle import RefLib

    ref = RefLib()
    n_grid = int(ref.lib.ref_total_param_count()) - int(ref.lib.ref_mlp_param_count())
    n = BATCH
    coords_h, table_h, dy_h = workloads.encode_inputs(n, n_grid, 8, 4, seed=1000, coord_stride=7)
    stream = torch.cuda.current_stream()
    coords, table, dy = (torch.from_numpy(a).cuda() for a in (coords_h, table_h.view(np.int16), dy_h))
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
        "impl": "reference", "metric": "hash-encode fwd+bwd Gpts/s (config 0)", "value": round(value, 4), "unit": "Gpts/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 table/features, fp16 accumulation and gradients (reference)", "data": "synthetic (seeded)",
        "config": {"workload": "config0 hash-grid encode fwd+bwd", "points_per_gpu": n, "levels": 8, "features": 4,
                   "note": "reference kernels support only their compiled 8x4 layout (static_assert ngp.train.cu:58)", "parallelism": "dp1"},
        "cpu_baseline": {"value": round(value, 4), "unit": "Gpts/s", "cores": 0, "kind": "reference",
                         "sample": "reference CUDA build (oracle/_ref) on one B200; the reference has no CPU implementation"},
        "e2e": {"value": round(value, 4), "unit": "Gpts/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "clocks": clocks.summary(),
    }


# ------------------------------------------------------------------------------------------------
# render workload (config 4): large table, novel 1920x1080 views partitioned across ranks
# ------------------------------------------------------------------------------------------------
def bench_mlp_ours(args, rank, world, local):
    """Config 1: the fused density + colour MLPs, forward + backward (input and weight gradients)
    over 2^18 rows per GPU; L2 flushed before every step."""
    import torch
    import ngp_b200 as ngp
    import workloads

    n = BATCH
    x_h, c_h, dy_h = workloads.mlp_inputs(n, seed=31 + rank)
    params = torch.from_numpy(workloads.xavier_mlp_params(1).view(np.int16)).cuda()
    x, coords, dy = torch.from_numpy(x_h).cuda(), torch.from_numpy(c_h).cuda(), torch.from_numpy(dy_h).cuda()
    out = torch.empty((n, 16), dtype=torch.float16, device="cuda")
    dx = torch.empty((32, n), dtype=torch.float16, device="cuda")
    dw = torch.empty(10240, dtype=torch.float32, device="cuda")
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    ngp.mlp_backward_scratch()

    def flush():
        flush_buf.fill_(1.0)

    def fwd():
        ngp.mlp_forward(params, x, coords, out, stream=stream)

    def bwd():
        ngp.mlp_backward(params, x, coords, dy, dx=dx, dw_f32=dw, stream=stream)

    def step():
        fwd()
        bwd()

    with ClockSampler(local) as clocks:
        clocks.wait_first()
        launches0 = ngp.kernel_launch_count()
        times = time_steps(step, args.steps, args.warmup, flush, stream, world)
        launches = ngp.kernel_launch_count() - launches0
        time.sleep(0.25)
    ms = max_over_ranks(sum(times) / len(times), world)
    fwd_ms = statistics.median(time_steps(fwd, 20, 2, flush, stream, 1))
    bwd_ms = statistics.median(time_steps(bwd, 20, 2, flush, stream, 1))
    # e2e: inputs from pinned host memory, outputs and weight gradients read back
    pins = [torch.from_numpy(a).pin_memory() for a in (x_h, c_h, dy_h)]
    out_h = torch.empty((n, 16), dtype=torch.float16).pin_memory()
    dw_h = torch.empty(10240, dtype=torch.float32).pin_memory()

    def e2e_step():
        for dst, src in zip((x, coords, dy), pins):
            dst.copy_(src, non_blocking=True)
        step()
        out_h.copy_(out, non_blocking=True)
        dw_h.copy_(dw, non_blocking=True)

    e2e_ms = max_over_ranks(statistics.mean(time_steps(e2e_step, max(3, args.steps // 4), 2, flush, stream, world)), world)
    peaks = load_peaks()
    tflops = MLP_FWDBWD_FLOP * n / (ms * 1e-3) / 1e12
    return {
        "metric": "fused MLP fwd+bwd rows/s (config 1)", "value": round(world * n / (ms * 1e-3), 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 weights/activations, fp32 accumulation (tcgen05 kind::f16)",
        "data": "synthetic (U(-1,1) fp16 inputs, directions uniform on S^2, N(0,1) dL/dy, Xavier weights; seeded)",
        "config": {"workload": "config1 fused MLP fwd+bwd", "rows_per_gpu": n, "density": "32-64-16", "colour": "32-64-64-16",
                   "parallelism": f"dp{world} (no collective)", "l2": "flushed (256 MB write) before every timed step"},
        "kernels_ms": {"mlp_forward": round(fwd_ms, 5), "mlp_backward": round(bwd_ms, 5)},
        "roofline": {"kernel": "mlp_forward_kernel + mlp_backward_kernel", "bound": "tensor", "achieved": round(tflops, 2),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4), "traffic": None,
                     "peak_source": peaks["source"] + " (dense bf16 burst; fp16 has the same tensor rate)",
                     "per_unit": f"{MLP_FWDBWD_FLOP} FLOP per row (forward 20,480, input gradients 20,480, weight gradients 20,480)"},
        "e2e": {"value": round(world * n / (e2e_ms * 1e-3), 1), "unit": "rows/s",
                "h2d_bytes_per_step": int(x_h.nbytes + c_h.nbytes + dy_h.nbytes), "d2h_bytes_per_step": n * 32 + 10240 * 4},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }


def bench_march_ours(args, rank, world, local):
    """Config 2: density-grid update (EMA, mean, bitfield) of the 128^3 grid with the blob
    field's optical thickness as the step's observations, then marching 2^18 rays through it
    (counts and sample records); L2 flushed before every step."""
    import torch
    import ngp_b200 as ngp
    import workloads

    n = 1 << 18
    obs = torch.from_numpy(workloads.blob_grid_values(workloads.gaussian_blob_density())).cuda()
    values = obs.clone()
    scratch = torch.zeros_like(obs)
    partial = torch.zeros(ngp.density_grid_partials(), dtype=torch.float32, device="cuda")
    mean = torch.zeros(1, dtype=torch.float32, device="cuda")
    bits = torch.zeros(128 ** 3 // 8, dtype=torch.uint8, device="cuda")
    occ = torch.zeros(1, dtype=torch.int32, device="cuda")
    rays = torch.from_numpy(workloads.march_rays_config2(n, seed=2 + rank)).cuda()
    limit = 1 << 26  # every ray's samples fit (about 43 M at this configuration)
    coords = torch.empty((limit, 7), dtype=torch.float32, device="cuda")
    numsteps = torch.empty((n, 2), dtype=torch.int32, device="cuda")
    msc = torch.empty(ngp.march_scratch_words(n), dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()

    def flush():
        flush_buf.fill_(1.0)
        scratch.copy_(obs)  # the step's observations (the splat's output)

    def grid():
        ngp.density_grid_update(values, scratch, partial, mean, bits, occ, stream=stream)

    def march():
        ngp.march_rays(rays, bits, coords, numsteps, msc, counter, sample_limit=limit, stream=stream)

    def step():
        grid()
        march()

    with ClockSampler(local) as clocks:
        clocks.wait_first()
        launches0 = ngp.kernel_launch_count()
        times = time_steps(step, args.steps, args.warmup, flush, stream, world)
        launches = ngp.kernel_launch_count() - launches0
        time.sleep(0.25)
    ms = max_over_ranks(sum(times) / len(times), world)
    grid_ms = statistics.median(time_steps(grid, 10, 2, flush, stream, 1))
    march_ms = statistics.median(time_steps(march, 10, 2, flush, stream, 1))
    samples = min(int(counter.item()), limit)
    # e2e: rays from pinned host memory, per-ray counts and the samples read back
    rays_pin = rays.cpu().pin_memory()
    ns_h = torch.empty((n, 2), dtype=torch.int32).pin_memory()
    co_h = torch.empty((samples, 7), dtype=torch.float32).pin_memory()

    def e2e_step():
        rays.copy_(rays_pin, non_blocking=True)
        step()
        ns_h.copy_(numsteps, non_blocking=True)
        co_h.copy_(coords[:samples], non_blocking=True)

    e2e_ms = max_over_ranks(statistics.mean(time_steps(e2e_step, max(3, args.steps // 4), 2, flush, stream, world)), world)
    peaks = load_peaks()
    march_bytes = n * (24 + 8) + samples * 28
    achieved = march_bytes / (march_ms * 1e-3) / 1e9
    return {
        "metric": "density-grid update + march rays/s (config 2)", "value": round(world * n / (ms * 1e-3), 1), "unit": "rays/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 positions, uint32 counts, uint8 bitfield",
        "data": "synthetic (8 seeded Gaussian blobs, rays from the radius-4 sphere aimed near the origin)",
        "config": {"workload": "config2 density-grid update + ray marching", "rays_per_gpu": n, "grid": "128^3, 1 cascade, EMA 0.95",
                   "samples_per_step": samples, "parallelism": f"dp{world} (no collective)", "l2": "flushed (256 MB write) before every timed step"},
        "kernels_ms": {"grid_update": round(grid_ms, 5), "march": round(march_ms, 5)},
        "samples_per_s": round(world * samples / (ms * 1e-3), 1),
        "roofline": {"kernel": "march_count_kernel + march_write_kernel", "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": peaks["source"] + " (HBM copy bandwidth)",
                     "per_unit": f"24 B in + 8 B counts per ray, 28 B per emitted sample; {n} rays, {samples} samples per launch"},
        "e2e": {"value": round(world * n / (e2e_ms * 1e-3), 1), "unit": "rays/s", "h2d_bytes_per_step": n * 24,
                "d2h_bytes_per_step": n * 8 + samples * 28},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }


def render_encode_roofline(ngp, workloads, peaks, n: int = 1 << 22) -> dict:
    """Config 4's encode HBM rate: the encoding forward over the config-4 table (log2 T = 22,
    finest resolution 4096; larger than L2) on n uniformly random points, the gather pattern with
    the least reuse, timed with CUDA events after an L2 flush."""
    import torch

    layout = ngp.grid_layout(16, 2, 22, 16, math.log2(4096.0 / 16.0) / 15.0)
    coords_h, table_h, _ = workloads.encode_inputs(n, layout.n_params, 16, 2, seed=77)
    coords = torch.from_numpy(coords_h).cuda()
    table = torch.from_numpy(table_h.view(np.int16)).cuda()
    feats = torch.empty((32, n), dtype=torch.float16, device="cuda")
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    times = []
    for k in range(8):
        flush_buf.fill_(1.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        ngp.encode_grid_forward(layout, coords, table, feats, stream=stream)
        e.record(stream)
        e.synchronize()
        if k >= 3:
            times.append(s.elapsed_time(e))
    t_ms = statistics.median(times)
    per_point = 12 + 64 + 16 * 8 * 4  # coordinates, features out, 8 corners x 16 levels x 2 fp16
    achieved = per_point * n / (t_ms * 1e-3) / 1e9
    return {"kernel": "encode_forward_points_kernel (config-4 table)", "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None, "peak_source": peaks["source"] + " (HBM copy bandwidth)",
            "per_unit": f"{per_point} algorithmic bytes per point (table bytes gathered, counted once), {n} random points per launch, "
                        f"{t_ms * 1e3:.1f} us per launch",
            "table_MB": round(layout.n_params * 2 / 1e6, 1),
            "note": "the coarse levels of the table stay L2-resident; the finer hashed levels miss L2 and are read from HBM"}


def bench_render_ours(args, rank, world, local):
    import torch
    import ngp_b200 as ngp
    import workloads

    peaks = load_peaks()
    ds = make_dataset(args)
    model = ngp.InstantNGP(ds, ngp.config4_trainer_config())
    model.train(args.train_steps)  # untimed: an occupancy grid and weights of a trained model
    poses = workloads.render_poses(max(64, args.steps * world))
    w, h = poses["width"], poses["height"]
    # step k renders view k * world + rank on this rank (no collective)
    views = [poses["camera"][k * world + rank] for k in range(args.steps)]
    out = torch.empty((h * w, 3), dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        model.render(views[0], w, h, poses["focal"], poses["principal"], out=out)
    barrier(world)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        clocks.wait_first()
        launches0 = ngp.kernel_launch_count()
        torch.cuda.nvtx.range_push("render")  # lets a profiler select the timed renders
        s.record()
        for v in views:
            model.render(v, w, h, poses["focal"], poses["principal"], out=out)
        e.record()
        torch.cuda.nvtx.range_pop()
        e.synchronize()
        launches = ngp.kernel_launch_count() - launches0
        time.sleep(0.25)
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e), world)
    # e2e: the same renders with each image read back to pinned host memory
    host = torch.empty((h * w, 3), dtype=torch.float32, pin_memory=True)
    n_e2e = max(2, args.steps // 2)
    barrier(world)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for v in views[:n_e2e]:
        model.render(v, w, h, poses["focal"], poses["principal"], out=out)
        host.copy_(out, non_blocking=True)
    e2.record()
    e2.synchronize()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / n_e2e, world)
    model.close()
    roofline = render_encode_roofline(ngp, workloads, peaks)
    rays = w * h
    value = world * rays * args.steps / (ms * 1e-3)
    return {
        "metric": "render rays/s (config 4)", "value": round(value, 1), "unit": "rays/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 params/activations, fp32 accumulation", "data": "synthetic procedural scene (64 Lambert spheres, seeded)",
        "config": {"workload": "config4 render 1920x1080 novel views after training", "table": "L=16 F=2 log2T=22 base 16 finest 4096",
                   "views_per_gpu": args.steps, "trained_steps": args.train_steps, "parallelism": f"views partitioned over {world} ranks, no collective",
                   "l2": "table 170 MB fp16 > L2; no flush"},
        "e2e": {"value": round(world * rays / (e2e_ms * 1e-3), 1), "unit": "rays/s", "h2d_bytes_per_step": 48,
                "d2h_bytes_per_step": rays * 12, "note": "InstantNGP.render per view with the image read back to pinned host memory"},
        "gpu_launches": launches, "clocks": clocks.summary(), "roofline": roofline,
    }


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["train", "encode", "mlp", "march", "render"], default="train")
    ap.add_argument("--train-steps", type=int, default=1000, help="render workload: untimed training steps before rendering")
    ap.add_argument("--views", type=int, default=100)
    ap.add_argument("--test-views", type=int, default=20)
    ap.add_argument("--res", type=int, default=800)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"train": 300, "encode": 500, "mlp": 200, "march": 100, "render": 8}[args.workload]
    if args.warmup is None:
        args.warmup = {"train": 300, "encode": 5, "mlp": 5, "march": 5, "render": 3}[args.workload]
    args.warmup = max(args.warmup, 3)

    rank, world, local = dist_setup()
    if args.impl == "reference":
        if rank == 0:
            if args.workload == "render":
                print(json.dumps({"impl": "reference", "unavailable": "the reference build's compiled grid (8x4, log2 T 19) cannot express config 4"}),
                      flush=True)
                return 0
            if args.workload in ("mlp", "march"):
                print(json.dumps({"impl": "reference", "unavailable": f"no reference arm for the {args.workload} workload; "
                                                                      "its kernels run inside the train workload's reference step"}), flush=True)
                return 0
            fn = bench_train_reference if args.workload == "train" else bench_encode_reference
            print(json.dumps(fn(args, rank, world, local)), flush=True)
        return 0
    fn = {"train": bench_train_ours, "encode": bench_encode_ours, "mlp": bench_mlp_ours, "march": bench_march_ours,
          "render": bench_render_ours}[args.workload]
    res = fn(args, rank, world, local)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
