"""The reference's own entry points on this build (drop-in for the PyOpenCL path): its
``ffnerf_cli.py`` ``inspect``, ``train`` (the unmodified ``run_ffnerf_OG.train`` loop: producer and
IO threads, pyopencl copies and events, periodic metrics, preview renders, checkpoints) and
``snapshot``, run through ``run_reference.py`` on a synthetic scene written in the reference's SfM
archive format, then the checkpoint it wrote loaded by this package's ``Nerf.load_latest``.

The reference's Python modules come from the git-ignored ``baseline/_ref`` (installed by
``oracle/ref_install.py``); the test is skipped where they are absent.

Contracts: every CLI call exits 0; inspect reports the 8 registered cameras; train writes a
checkpoint with steps_trained = the requested steps, a loss log whose mse falls over training, and
preview images; snapshot writes a non-empty PNG; the checkpoint loads and its parameters are finite.
"""
import csv
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
LAUNCHER = ROOT / "ffnerf-experimental_b200" / "run_reference.py"
STEPS = 300


def _cli(*args, timeout=600):
    env = dict(os.environ, PYTHONUNBUFFERED="1")
    r = subprocess.run([sys.executable, str(LAUNCHER), "--reference", str(REF), *args], capture_output=True,
                       text=True, timeout=timeout, env=env)
    assert r.returncode == 0, f"{args[0]} failed ({r.returncode}):\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    return r.stdout


def test_reference_cli_train_inspect_snapshot(tmp_path):
    if not (REF / "ffnerf_cli.py").exists():
        pytest.skip("the reference's modules are not installed in baseline/_ref (oracle/ref_install.py)")
    from synthetic_scene import BlobScene, cameras_sphere, intrinsics, write_sfm_archive
    W = H = 64
    scene_dir = tmp_path / "scene"
    npz = write_sfm_archive(scene_dir, BlobScene(0), cameras_sphere(8, 2.0, 0), intrinsics(W, H, 50.0), W, H)
    cfg = {
        "data": {"reconstruction": str(npz), "images_dir": "", "sfm_max_side": 1600, "max_side": 800},
        "scene": {"box_min": [-1.0, -1.0, -1.0], "box_max": [1.0, 1.0, 1.0], "near": 0.3},
        "training": {"directory": str(tmp_path / "training"), "model_id": "refcli", "steps": STEPS, "period": 50,
                     "batch_rays": 512, "samples_per_ray": 64, "lr": 0.0005, "lmd": 0.00013, "seed": 777},
        "preview": {"enabled": False, "host": "127.0.0.1", "port": 8080, "width": 64, "height": 64, "downscale": 2,
                    "samples_per_ray": 64, "views": [0, 1, 2], "save_seconds": 120, "image_seconds": 30},
        "viewer": {"width": 64, "height": 64, "block_size": 8, "samples_per_ray": 64, "camera": 0, "move_speed": 1.0},
    }
    cfg_path = tmp_path / "scene.json"
    cfg_path.write_text(json.dumps(cfg))

    out = _cli("inspect", "--config", str(cfg_path))
    assert "Registered cameras: 8" in out

    out = _cli("train", "--config", str(cfg_path), "--no-web")
    tdir = tmp_path / "training"
    ckpts = sorted(tdir.glob("refcli_weights_*.npz"))
    assert ckpts, out[-2000:]
    with np.load(tdir / "refcli_weights_latest.npz" if (tdir / "refcli_weights_latest.npz").exists() else ckpts[-1]) as z:
        assert int(z["steps_trained"]) == STEPS
    logs = sorted(tdir.glob("refcli_loss_*.csv"))
    assert logs
    rows = list(csv.DictReader(logs[-1].open()))
    assert len(rows) >= 3, rows
    mse = [float(r["mse"]) for r in rows]
    assert all(np.isfinite(mse)) and mse[-1] < mse[0], mse
    assert list(tdir.glob("refcli_preview_*_multiview.png"))

    snap = tmp_path / "snap.png"
    _cli("snapshot", "--config", str(cfg_path), "--output", str(snap))
    import cv2
    img = cv2.imread(str(snap))
    assert img is not None and img.shape == (H, W, 3) and img.max() > 0

    import ffnerf_tools as ft
    ctx = ft.Context([ft.Device(0)])
    q, _ = ft.make_queue(ctx)
    nerf = ft.Nerf(ctx, q, training_dir=tdir, model_id="refcli", load_id="refcli", verbose=False)
    assert nerf.steps_trained == STEPS
    blob = nerf._blob_from_state()
    assert np.isfinite(blob).all() and np.abs(blob).max() > 0
