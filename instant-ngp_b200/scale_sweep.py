"""Scene-scale sweep with the reference's benchmark flags, stages and CSV schema (benchmark.cpp).

    python instant-ngp_b200/scale_sweep.py --dataset <path> [--steps 10000] [--chunk-steps 1000]
        [--validation-interval 5000] [--coarse-scales 0.125,...,4] [--refine-count 9]
        [--output-csv scale-benchmark.csv]

Stage "coarse" trains one model per candidate scene scale (validating every interval and at the
end); stage "refine" places `--refine-count` log-spaced candidates between the best coarse
candidate's neighbours (candidates already run are reused).  The best candidate has the highest
final validation PSNR; PSNRs within 0.05 dB prefer the smaller scale.  One CSV row per candidate.
"""
from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

CSV_HEADER = ("stage,rank,scene_scale,status,error,final_step,best_validation_step,final_psnr,final_mse,best_psnr,best_mse,final_loss,"
              "occupancy_ratio,occupied_cells,average_samples,average_compacted,train_ms,validation_ms,steps_per_second")
DEFAULT_COARSE = "0.125,0.1767767,0.25,0.3535534,0.5,0.7071068,1,1.4142135,2,2.8284271,4"


def _same(a: float, b: float) -> bool:
    return abs(a - b) <= max(1.0, max(abs(a), abs(b))) * 1e-6


def parse_coarse(text: str) -> list[float]:
    """Comma-separated finite positive scales, at least two, no duplicates; sorted."""
    vals = []
    for tok in text.split(","):
        try:
            v = float(tok)
        except ValueError:
            v = float("nan")
        if tok == "" or not math.isfinite(v) or v <= 0.0:
            raise ValueError("--coarse-scales must contain finite positive scene_scale values.")
        vals.append(float(v))
    if len(vals) < 2:
        raise ValueError("--coarse-scales must contain at least two values.")
    vals.sort()
    if any(_same(vals[i], vals[i - 1]) for i in range(1, len(vals))):
        raise ValueError("--coarse-scales contains duplicate scene_scale values.")
    return vals


def best_index(results: list[dict], stage: str) -> int | None:
    """Highest final PSNR; within 0.05 dB the smaller scale."""
    best = None
    for i, r in enumerate(results):
        if r["stage"] != stage or r["failed"]:
            continue
        if best is None:
            best = i
            continue
        b = results[best]
        if r["final_psnr"] > b["final_psnr"] + 0.05 or (abs(r["final_psnr"] - b["final_psnr"]) <= 0.05 and r["scene_scale"] < b["scene_scale"]):
            best = i
    return best


def refine_candidates(coarse: list[float], best: float, refine_count: int) -> list[float]:
    """Log-spaced candidates between the best coarse scale's neighbours (benchmark.cpp)."""
    pos = next(i for i, c in enumerate(coarse) if _same(best, c))
    if pos == 0:
        lower, upper = best / (coarse[1] / coarse[0]), coarse[1]
    elif pos + 1 == len(coarse):
        lower, upper = coarse[pos - 1], best * (coarse[pos] / coarse[pos - 1])
    else:
        lower, upper = coarse[pos - 1], coarse[pos + 1]
    if not (math.isfinite(lower) and math.isfinite(upper) and 0.0 < lower < upper):
        raise ValueError("invalid refine bounds")
    half = refine_count // 2
    out = [math.exp(math.log(lower) * (1.0 - i / half) + math.log(best) * (i / half)) for i in range(half)]
    out.append(best)
    out += [math.exp(math.log(best) * (1.0 - i / half) + math.log(upper) * (i / half)) for i in range(1, half + 1)]
    return out


def run_candidate(root: Path, synthetic: bool, scale: float, steps: int, chunk: int, interval: int) -> dict:
    import ngp_b200
    import ngp_dataset

    r = {"final_step": 0, "best_validation_step": 0, "final_psnr": 0.0, "final_mse": 0.0, "best_psnr": 0.0, "best_mse": 0.0, "final_loss": 0.0,
         "occupancy_ratio": 0.0, "occupied_cells": 0, "average_samples": 0, "average_compacted": 0, "train_ms": 0.0, "validation_ms": 0.0,
         "steps_per_second": 0.0, "failed": False, "error": "", "scene_scale": scale}
    model = None
    try:
        ds = ngp_dataset.load_nerf_synthetic(root, scale) if synthetic else ngp_dataset.load_dd_nerf(root, scale)
        r["scene_scale"] = ds["scene_scale"]
        model = ngp_b200.InstantNGP(ds, ngp_b200.trainer_config())
        samples = compacted = chunks = 0
        trained, next_val = 0, interval
        r["final_psnr"] = float("nan")
        while trained < steps:
            n = min(chunk, steps - trained)
            st = model.train(n)
            r.update(final_loss=st["loss"], final_step=st["step"], occupied_cells=st["density_grid_occupied_cells"],
                     occupancy_ratio=st["density_grid_occupancy_ratio"])
            r["train_ms"] += st["elapsed_ms"]
            samples += st["measured_sample_count_before_compaction"]
            compacted += st["measured_sample_count"]
            chunks += 1
            trained += n
            if st["step"] >= next_val or st["step"] >= steps:
                import time

                t0 = time.perf_counter()
                v = model.validate()
                r["validation_ms"] += (time.perf_counter() - t0) * 1e3
                r["final_mse"], r["final_psnr"] = v["mse"], v["psnr"]
                if v["psnr"] > r["best_psnr"]:
                    r["best_psnr"], r["best_mse"], r["best_validation_step"] = v["psnr"], v["mse"], st["step"]
                while next_val <= st["step"]:
                    next_val += interval
        r["average_samples"] = samples // max(chunks, 1)
        r["average_compacted"] = compacted // max(chunks, 1)
        if r["train_ms"] > 0:
            r["steps_per_second"] = r["final_step"] * 1000.0 / r["train_ms"]
        if not math.isfinite(r["final_psnr"]):
            raise RuntimeError("benchmark did not produce final validation PSNR.")
    except Exception as e:  # a failed candidate is recorded, the sweep continues (benchmark.cpp)
        r["failed"], r["error"] = True, str(e)
    finally:
        if model is not None:
            model.close()
    return r


def csv_row(r: dict) -> str:
    err = r["error"].replace('"', '""')
    vals = [r["stage"], r["rank"], f"{r['scene_scale']:g}", "failed" if r["failed"] else "ok", f'"{err}"', r["final_step"],
            r["best_validation_step"], f"{r['final_psnr']:g}", f"{r['final_mse']:g}", f"{r['best_psnr']:g}", f"{r['best_mse']:g}",
            f"{r['final_loss']:g}", f"{r['occupancy_ratio']:g}", r["occupied_cells"], r["average_samples"], r["average_compacted"],
            f"{r['train_ms']:g}", f"{r['validation_ms']:g}", f"{r['steps_per_second']:g}"]
    return ",".join(str(v) for v in vals)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="scale-sweep")
    ap.add_argument("--dataset", required=True)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--chunk-steps", type=int, default=1000)
    ap.add_argument("--validation-interval", type=int, default=5000)
    ap.add_argument("--coarse-scales", default=DEFAULT_COARSE)
    ap.add_argument("--refine-count", type=int, default=9)
    ap.add_argument("--output-csv", default="scale-benchmark.csv")
    args = ap.parse_args(sys.argv[1:] if argv is None else argv)
    if min(args.steps, args.chunk_steps, args.validation_interval) <= 0:
        print("error: --steps, --chunk-steps and --validation-interval must be positive integers.")
        return 2
    if args.refine_count < 3 or args.refine_count % 2 == 0:
        print("error: --refine-count must be an odd integer >= 3.")
        return 2
    root, out = Path(args.dataset), Path(args.output_csv)
    if not root.is_dir():
        print(f"error: dataset path '{root}' is not a directory.")
        return 2
    if str(out.parent) not in ("", ".") and not out.parent.is_dir():
        print(f"error: output CSV parent directory '{out.parent}' does not exist.")
        return 2
    try:
        coarse = parse_coarse(args.coarse_scales)
    except ValueError as e:
        print(f"error: {e}")
        return 2
    synthetic = all((root / f"transforms_{s}.json").is_file() for s in ("train", "val", "test"))
    dd = (root / "cameras.json").is_file() and (root / "images").is_dir()
    if synthetic == dd:
        print(f"error: dataset path '{root}' must contain exactly one supported dataset marker set.")
        return 2
    results: list[dict] = []
    for stage in ("coarse", "refine"):
        if stage == "coarse":
            scales = coarse
        else:
            b = best_index(results, "coarse")
            if b is None:
                break
            try:
                scales = refine_candidates(coarse, results[b]["scene_scale"], args.refine_count)
            except ValueError:
                return 1
        for rank, scale in enumerate(scales):
            prev = next((r for r in results if _same(r["scene_scale"], scale)), None) if stage == "refine" else None
            r = dict(prev) if prev is not None else run_candidate(root, synthetic, scale, args.steps, args.chunk_steps, args.validation_interval)
            r.update(stage=stage, rank=rank)
            print(f"{stage:<7} rank={rank} scene_scale={r['scene_scale']:.7f} status={'failed' if r['failed'] else 'ok'} "
                  f"psnr={r['final_psnr']:.2f}", flush=True)
            results.append(r)
    out.write_text(CSV_HEADER + "\n" + "".join(csv_row(r) + "\n" for r in results))
    b = best_index(results, "refine")
    if b is None:
        print(f"BEST      no successful refined scene_scale candidates; csv={out}")
        return 1
    r = results[b]
    print(f"BEST      scene_scale={r['scene_scale']:.7f} final_psnr={r['final_psnr']:.2f} final_mse={r['final_mse']:.8f} "
          f"best_psnr={r['best_psnr']:.2f} best_step={r['best_validation_step']} occupancy={r['occupancy_ratio'] * 100:.2f}% csv={out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
