"""Headless view rendering (render_gpu.render_frame / snapshot; ffn_camera_rays + ffn_render) against
the host module's view rays and the CPU oracle's inference pass.

Contracts:
  * view rays equal rays_from_rt_indices (host mirror, golden-pinned) for every pixel: origin exact,
    direction within 1e-6 (K given and the fallback focal);
  * a frame rendered in chunks (ray ids = row-major pixel index) equals the oracle's inference
    forward (do_train = 0, black background) over the whole view within 1e-4 (fp32 MLP) / 1e-3
    (fp16 tensor-core MLP) per channel;
  * the snapshot PNG is clip(frame, 0, 1) * 255 truncated, in BGR order for cv2.
"""
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ffnerf_tools as ft
import render_gpu as rg
from oracle import OrcStep, make_orc_config

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("with_k", [True, False])
def test_view_rays_match_host(with_k):
    import ctypes as C
    import ffn_native as fn
    g = np.load(GOLD / "golden_rays.npz")
    c2w, K = g["c2w"][1], g["K"]
    W, H = 23, 17
    n = W * H
    rays = torch.empty((n, 8), device="cuda")
    lib = fn.load_library()
    Kp = K if with_k else None
    rc = lib.ffn_camera_rays(np.ascontiguousarray(c2w).ctypes.data_as(C.c_void_p),
                             None if Kp is None else np.ascontiguousarray(Kp).ctypes.data_as(C.c_void_p),
                             W, H, 0, n, C.c_void_p(rays.data_ptr()), None)
    assert rc == 0
    torch.cuda.synchronize()
    yy, xx = np.mgrid[0:H, 0:W]
    host = np.ascontiguousarray(ft.rays_from_rt_indices(c2w, xx.ravel(), yy.ravel(), W, H, K=Kp)).view(np.float32).reshape(-1, 8)
    r = rays.cpu().numpy()
    assert np.array_equal(r[:, :4], host[:, :4])
    assert np.abs(r[:, 4:] - host[:, 4:]).max() < 1e-6


def _nerf(tmp_path, prec):
    ctx = ft.Context([ft.Device(0)])
    queue = ft.CommandQueue(ctx)
    occ = ft.OccParams(G_occ=32, box_min=np.array([-1, -1, -1], np.float32), box_max=np.array([1, 1, 1], np.float32),
                       rho_min=np.float32(1.0), rho_max=np.float32(16.0)).finalize()
    nerf = ft.Nerf(ctx, queue, training_dir=tmp_path, model_id="r", transfer_fmt="fp32", table_size_entries=16 << 12,
                   f_per_level=2, occ=occ, rng_seed=3, background="black", finest_resolution=512.0, nd=1, nc=2,
                   mlp_precision=prec, verbose=False)
    rng = np.random.default_rng(2)
    nerf.state_i32["table"] = rng.uniform(-0.5, 0.5, nerf.state_i32["table"].size).astype(np.float32).view(np.int32)
    words = rng.integers(0, 2 ** 32, nerf.state_i32["occ_grid_in_u32"].size, dtype=np.uint64).astype(np.uint32)
    nerf.state_i32["occ_grid_in_u32"] = words.view(np.int32).copy()
    nerf.state_i32["occ_grid_st_u32"] = words.view(np.int32).copy()
    nerf.setup_buffers(64, 64, do_train=False)
    return nerf


@pytest.mark.parametrize("prec,tol", [("fp32", 1e-4), ("fp16", 1e-3)])
def test_frame_matches_oracle(oracle, tmp_path, prec, tol):
    nerf = _nerf(tmp_path, prec)
    c2w = np.eye(4, dtype=np.float32)
    c2w[:3, 3] = [0.0, 0.0, -2.5]
    W, H = 24, 16
    K = np.array([[20.0, 0, W / 2], [0, 20.0, H / 2], [0, 0, 1]], np.float32)
    frame = rg.render_frame(nerf, c2w, K, W, H, chunk_rays=64, rng_u32=77)
    nerf.queue.finish()
    yy, xx = np.mgrid[0:H, 0:W]
    rays = np.ascontiguousarray(ft.rays_from_rt_indices(c2w, xx.ravel(), yy.ravel(), W, H, K=K)).view(np.float32).reshape(-1, 8)
    nat = nerf.native
    blob = nat.tensor(ft.ffn_native.BUF_PARAMS).cpu().numpy()
    table = nat.tensor(ft.ffn_native.BUF_TABLE).cpu().numpy()
    occ = nat.tensor(ft.ffn_native.BUF_OCC_IN).cpu().numpy().view(np.uint32)
    out_o = np.zeros((W * H, 4), np.float32)
    oracle.forward_backward(make_orc_config(nerf.geometry(64)), OrcStep(0.0, 1.0, 0.0, 77, 0, 0), blob, table, occ.copy(),
                            occ.copy(), rays, np.zeros((W * H, 4), np.float32), out_o)
    got = frame.cpu().numpy().reshape(-1, 3)
    assert np.abs(got - out_o[:, :3]).max() < tol
    assert got.std() > 0.01                     # a non-trivial image
    # snapshot conversion
    import cv2
    path = rg.snapshot(nerf, c2w, K, W, H, tmp_path / "snap.png", chunk_rays=64, rng_u32=77)
    png = cv2.imread(str(path), cv2.IMREAD_COLOR)[:, :, ::-1]
    assert np.array_equal(png, (np.clip(frame.cpu().numpy(), 0, 1) * 255).astype(np.uint8))
