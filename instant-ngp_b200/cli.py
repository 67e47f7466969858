"""Command-line trainer with the reference application's flags and flow (main.cpp:19-372).

    python instant-ngp_b200/cli.py [dataset-path] [--dataset <path>] [--scene-scale <v>] [--steps <n>]
        [--chunk-steps <n>] [--validation-interval <n>] [--early-stop-patience <n>]
        [--early-stop-min-delta <mse>] [--load-weights <path>] [--export-weights <path>]

Loads a NeRF-synthetic or DD-NeRF scene (exactly one marker set must be present), optionally
loads safetensors weights, trains in chunks with a progress line per chunk, validates every
`--validation-interval` steps with early stopping after `--early-stop-patience` checks without an
MSE improvement of at least `--early-stop-min-delta`, writes the test comparison images to
test/test_NNNN.png with the test PSNR, and optionally exports the weights.  Exit status 0 on
success, 1 when the pipeline fails, 2 on invalid arguments, as the reference.
"""
from __future__ import annotations

import argparse
import datetime as _dt
import math
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))


def _now() -> str:
    return _dt.datetime.now().strftime("%Y-%m-%d %H:%M:%S")


def _log(tag: str, text: str) -> None:
    print(f"[{_now()}] {tag:<7} {text}", flush=True)


def _positive_int(name):
    def parse(v: str) -> int:
        try:
            x = int(v)
        except ValueError:
            x = 0
        if x <= 0:
            raise argparse.ArgumentTypeError(f"{name} must be a positive integer.")
        return x
    return parse


def _nonnegative_float(name):
    def parse(v: str) -> float:
        try:
            x = float(v)
        except ValueError:
            x = -1.0
        if not math.isfinite(x) or x < 0.0:
            raise argparse.ArgumentTypeError(f"{name} must be a finite non-negative number.")
        return x
    return parse


def parse_args(argv) -> argparse.Namespace:
    ap = argparse.ArgumentParser(prog="instant-ngp-b200", description="NeRF training on the B200-native hot path.")
    ap.add_argument("dataset_path", nargs="?", default=None, help="NeRF synthetic or DD-NeRF dataset root")
    ap.add_argument("--dataset", default=None, help="dataset root (default ../data/nerf-synthetic/lego)")
    ap.add_argument("--scene-scale", type=_nonnegative_float("--scene-scale"), default=0.33)
    ap.add_argument("--steps", type=_positive_int("--steps"), default=200000)
    ap.add_argument("--chunk-steps", type=_positive_int("--chunk-steps"), default=1000)
    ap.add_argument("--validation-interval", type=_positive_int("--validation-interval"), default=5000)
    ap.add_argument("--early-stop-patience", type=_positive_int("--early-stop-patience"), default=5)
    ap.add_argument("--early-stop-min-delta", type=_nonnegative_float("--early-stop-min-delta"), default=1e-6)
    ap.add_argument("--load-weights", default=None)
    ap.add_argument("--export-weights", default=None)
    args = ap.parse_args(argv)
    if args.dataset is not None and args.dataset_path is not None:
        ap.error("dataset path was provided more than once.")
    args.dataset = args.dataset or args.dataset_path or "../data/nerf-synthetic/lego"
    if args.scene_scale <= 0.0:
        ap.error("--scene-scale must be a finite positive number.")
    return args


def main(argv=None) -> int:
    args = parse_args(sys.argv[1:] if argv is None else argv)
    root = Path(args.dataset)
    if not root.is_dir():
        print(f"error: dataset path '{root}' is not a directory.")
        return 2
    if args.load_weights is not None and not Path(args.load_weights).is_file():
        print(f"error: weights file '{args.load_weights}' does not exist.")
        return 2
    if args.export_weights is not None and str(Path(args.export_weights).parent) not in ("", ".") and not Path(args.export_weights).parent.is_dir():
        print(f"error: weights export parent directory '{Path(args.export_weights).parent}' does not exist.")
        return 2
    import ngp_dataset as datasets

    synthetic = all((root / f"transforms_{s}.json").is_file() for s in ("train", "val", "test"))
    dd = (root / "cameras.json").is_file() and (root / "images").is_dir()
    if synthetic == dd:
        print(f"error: dataset path '{root}' must contain exactly one supported dataset marker set: NeRF synthetic transforms_*.json or "
              "DD-NeRF cameras.json + images/.")
        return 2
    _log("CONFIG", f"dataset={root} format={'nerf-synthetic' if synthetic else 'dd-nerf-dataset'} scene_scale={args.scene_scale} "
                   f"steps={args.steps} chunk={args.chunk_steps} validation_interval={args.validation_interval} "
                   f"patience={args.early_stop_patience} min_delta_mse={args.early_stop_min_delta} test_output=test "
                   f"load_weights={args.load_weights or 'none'} export_weights={args.export_weights or 'none'}")
    error = None
    try:
        import ngp_b200

        _log("INFO", "loading dataset")
        ds = datasets.load_nerf_synthetic(root, args.scene_scale) if synthetic else datasets.load_dd_nerf(root, args.scene_scale)
        model = ngp_b200.InstantNGP(ds, ngp_b200.trainer_config())
        if args.load_weights is not None:
            model.load_weights(args.load_weights)
            _log("WEIGHT", f"loaded={args.load_weights}")
        best_mse, best_psnr, best_step, bad_checks, stopped = math.inf, 0.0, 0, 0, False
        next_validation = args.validation_interval
        trained, first_loss, last_loss, train_ms = 0, None, None, 0.0
        while trained < args.steps:
            n = min(args.chunk_steps, args.steps - trained)
            st = model.train(n)
            trained += n
            first_loss = st["loss"] if first_loss is None else first_loss
            last_loss = st["loss"]
            train_ms += st["elapsed_ms"]
            _log("TRAIN", f"step={st['step']:>6}/{args.steps} loss={st['loss']:>10.6f} chunk={st['elapsed_ms']:>8.3f}ms "
                          f"grid={st['density_grid_update_ms']:>7.3f}ms rate={n / max(st['elapsed_ms'], 1e-9) * 1e3:>7.2f} step/s "
                          f"rays={st['rays_per_batch']:>6} samples={st['measured_sample_count']:>7}/{st['measured_sample_count_before_compaction']:<7} "
                          f"occupied={st['density_grid_occupied_cells']:>7} occupancy={st['density_grid_occupancy_ratio'] * 100:>6.2f}%")
            if st["step"] >= next_validation or st["step"] >= args.steps:
                if model.split_frames.get(1, 0) > 0:
                    v = model.validate()
                    if v["mse"] < best_mse - args.early_stop_min_delta:
                        best_mse, best_psnr, best_step, bad_checks = v["mse"], v["psnr"], st["step"], 0
                    else:
                        bad_checks += 1
                    _log("VALID", f"step={st['step']:>6} | MSE={v['mse']:.8f} PSNR={v['psnr']:>5.2f} | BEST={best_mse:.8f}@{best_step} | "
                                  f"patience={bad_checks}/{args.early_stop_patience}")
                    if bad_checks >= args.early_stop_patience:
                        stopped = True
                        break
                while next_validation <= st["step"]:
                    next_validation += args.validation_interval
        _log("SUMMARY", f"steps={model.step} stopped_early={str(stopped).lower()} first_loss={first_loss or 0:.6f} last_loss={last_loss or 0:.6f} "
                        f"train={train_ms / 1e3:.3f}s best_validation={best_mse:.8f}@{best_step} psnr={best_psnr:.2f}")
        if model.split_frames.get(2, 0) > 0:
            t = model.write_test_images("test")
            _log("TEST", f"step={model.step:>6} | MSE={t['mse']:.8f} PSNR={t['psnr']:>5.2f} | images={t['image_count']:>3} "
                         f"pixels={t['pixel_count']} output={t['output_dir']}")
        if args.export_weights is not None:
            model.export_weights(args.export_weights)
            _log("WEIGHT", f"exported={args.export_weights}")
        model.close()
    except Exception as e:  # the reference reports any pipeline error and exits 1
        error = str(e)
    if error is None:
        _log("DONE", "pipeline=succeeded")
        return 0
    _log("ERROR", f'pipeline=failed error="{error}"')
    return 1


if __name__ == "__main__":
    sys.exit(main())
