"""The command line end to end on a small NeRF-synthetic scene written here (64-sphere scene
renders as PNGs with their transforms.json), and the weights checkpoint through the trainer:
export after training, load into a fresh trainer, identical parameters."""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

import workloads

pytestmark = pytest.mark.gpu


def write_scene(root: Path, counts=(6, 2, 2), size=64, seed=3) -> None:
    from PIL import Image

    scene = workloads.sphere_scene(seed)
    rng = np.random.default_rng(seed + 1)
    fov = 0.69
    focal = 0.5 * size / math.tan(fov * 0.5)
    for split, count in zip(("train", "val", "test"), counts):
        frames = []
        pos = workloads.hemisphere_positions(count, 4.0, rng)
        for i in range(count):
            c2w = workloads.look_at_c2w(pos[i])
            img = workloads.render_spheres(scene, c2w, size, size, focal, "cuda")
            (root / split).mkdir(parents=True, exist_ok=True)
            Image.fromarray(img, "RGBA").save(root / split / f"r_{i}.png")
            frames.append({"file_path": f"./{split}/r_{i}", "transform_matrix": np.asarray(c2w).tolist()})
        (root / f"transforms_{split}.json").write_text(json.dumps({"camera_angle_x": fov, "frames": frames}))


def test_cli_trains_tests_and_exports(tmp_path, monkeypatch):
    import cli

    scene = tmp_path / "scene"
    write_scene(scene)
    monkeypatch.chdir(tmp_path)
    out = tmp_path / "w.safetensors"
    rc = cli.main([str(scene), "--steps", "60", "--chunk-steps", "20", "--validation-interval", "20", "--export-weights", str(out)])
    assert rc == 0
    assert sorted(p.name for p in (tmp_path / "test").iterdir()) == ["test_0000.png", "test_0001.png"]
    from PIL import Image

    with Image.open(tmp_path / "test" / "test_0000.png") as im:
        assert im.size == (128, 64) and im.mode == "RGB"
    assert out.is_file()
    assert cli.main([str(scene), "--steps", "1", "--load-weights", str(out)]) == 0


def test_weights_roundtrip_through_trainer(tmp_path):
    import ngp_b200 as ngp
    import ngp_dataset

    write_scene(tmp_path, counts=(4, 1, 1), size=48)
    ds = ngp_dataset.load_nerf_synthetic(tmp_path)
    a = ngp.InstantNGP(ds, ngp.trainer_config())
    a.train(20)
    a.export_weights(tmp_path / "w.safetensors")
    pa = a.get_params()
    a.close()
    b = ngp.InstantNGP(ds, ngp.trainer_config())
    b.load_weights(tmp_path / "w.safetensors")
    assert b.get_params().tobytes() == pa.tobytes()
    b.train(1)
    with pytest.raises(RuntimeError, match="before training"):
        b.load_weights(tmp_path / "w.safetensors")
    b.close()


def test_scale_sweep_runs_and_writes_csv(tmp_path):
    import scale_sweep

    scene = tmp_path / "scene"
    write_scene(scene, counts=(4, 1, 1), size=48)
    out = tmp_path / "sweep.csv"
    rc = scale_sweep.main(["--dataset", str(scene), "--steps", "20", "--chunk-steps", "10", "--validation-interval", "10",
                           "--coarse-scales", "0.25,0.33", "--refine-count", "3", "--output-csv", str(out)])
    lines = out.read_text().splitlines()
    assert lines[0] == scale_sweep.CSV_HEADER
    assert [ln.split(",")[0] for ln in lines[1:]] == ["coarse", "coarse", "refine", "refine", "refine"]
    assert rc == 0 and all(",ok," in ln for ln in lines[1:])
