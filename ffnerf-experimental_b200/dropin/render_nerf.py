"""Headless stand-in for the reference's ``render_nerf`` module (MolSzabi/ffnerf-experimental,
render_nerf.py), for the reference's trainer and CLI running on this build.

Kept: ``build_c2w_rt_yaw_pitch`` (render_nerf.py:108-147, imported by run_ffnerf_OG.py:22 for its
browser preview) and the ``snapshot`` path of ``main(config, output)`` (render_nerf.py:610-671):
load the model's latest checkpoint, render viewer.camera's pose at viewer.width x viewer.height and
write an 8-bit PNG -- here with the device ray generator and inference kernel (render_gpu).
Left out: the interactive pygame review window (``main`` without ``output``) and its IPC client,
which are not part of the training-step path; they raise a clear error.
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np


def build_c2w_rt_yaw_pitch(pos_xyz, yaw: float, pitch: float) -> np.ndarray:
    """Camera-to-world 4x4 for a camera at pos_xyz looking along (cos yaw cos pitch, sin yaw
    cos pitch, sin pitch), world up +Z; columns right, down, forward (OpenCV camera axes: the
    image's v axis points down), the position in the last column."""
    pos = np.asarray(pos_xyz, dtype=np.float32).reshape(3)
    fwd = np.array([math.cos(yaw) * math.cos(pitch), math.sin(yaw) * math.cos(pitch), math.sin(pitch)], np.float32)
    fwd /= np.linalg.norm(fwd) + 1e-12
    right = np.cross(fwd, np.array([0.0, 0.0, 1.0], np.float32)).astype(np.float32)
    n = np.linalg.norm(right)
    right = np.array([1.0, 0.0, 0.0], np.float32) if n < 1e-6 else right / (n + 1e-12)
    up = np.cross(right, fwd).astype(np.float32)
    up /= np.linalg.norm(up) + 1e-12
    rt = np.eye(4, dtype=np.float32)
    rt[:3, 0], rt[:3, 1], rt[:3, 2], rt[:3, 3] = right, -up, fwd, pos
    return rt


def main(config=None, output=None):
    """``ffnerf_cli.py snapshot``: renders the configured viewer camera of the model's latest
    checkpoint into ``output`` (PNG).  ``review`` (no output: the pygame window) is not available."""
    if output is None:
        raise RuntimeError("the interactive review window (pygame) is not part of this build; use "
                           "'ffnerf_cli.py snapshot' for a headless render")
    if config is None:
        raise ValueError("snapshot needs the loaded scene configuration")
    import ffnerf_tools as ft
    import render_gpu
    from sfm_data import image_geometry, read_scene, scaled_intrinsics
    paths, poses, K, _, _ = read_scene(config["data"])
    v, t = config["viewer"], config["training"]
    if not 0 <= v["camera"] < len(poses):
        raise ValueError("viewer.camera is outside the registered-camera list")
    first, _ = image_geometry(paths[v["camera"]], config["data"])
    W, H = int(v["width"]), int(v["height"])
    view_k = scaled_intrinsics(K, (first.shape[1], first.shape[0]), (W, H), config["data"]["sfm_max_side"])
    training_dir, model_id = Path(t["directory"]), t["model_id"]
    if not list(training_dir.glob(f"{model_id}_weights_*.npz")):
        raise FileNotFoundError(f"No checkpoints for {model_id} in {training_dir}")
    _, dev = ft.pick_first_device()
    ctx = ft.Context([dev])
    queue, _ = ft.make_queue(ctx, dev)
    nerf = ft.Nerf.from_kernels(ctx=ctx, queue=queue, background="black", training_dir=training_dir,
                                model_id=model_id, load_id=model_id, rng_seed=777)
    nerf.samples_per_ray = int(v["samples_per_ray"])
    out = render_gpu.snapshot(nerf, poses[v["camera"]], view_k, W, H, output)
    print(f"Saved snapshot: {Path(out).resolve()}")
    return out
