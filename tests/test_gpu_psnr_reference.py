"""End-of-training parity with the reference kernels.

The same 1,600 training steps of the synthetic cfg1 scene -- the same initial state (the reference's
init draws from one seed), the same batches (512 uniformly drawn pixels per step, host rays of
rays_targets_from_indices), the same schedules (run_ffnerf_OG.py:1356-1365, the occupancy updates
live after step 1,500 with decay every 32nd step) and the same per-step seeds -- are trained twice:
  * by the reference's own kernels compiled for the CPU (oracle/_ref: the fused training kernel with
    its Hogwild table updates over all host cores, weight_update.cl's Adam, the occupancy decay), the
    host steps of Nerf.step (ffnerf_tools.py:1357-1544) restated around them;
  * by the device through ffnerf_tools.Nerf.step (fp32 MLP, immediate table update).
Each model then renders the 8 training views with its own implementation (the reference kernel with
do_train = 0; the device inference kernel), and the PSNR over all pixels is compared.

Contract: |PSNR(device) - PSNR(reference)| <= 0.2 dB.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ffnerf_tools as ft
import schedules as sch
import trainer
from ffn_config import param_layout, param_shapes
from oracle import RefKernels

STEPS, RAYS, SPR = 1600, 512, 64


def _psnr(frames, images):
    se = sum(float(((np.clip(f, 0, 1) - im.astype(np.float32) / 255.0) ** 2).sum()) for f, im in zip(frames, images))
    return -10.0 * np.log10(se / sum(f.size for f in frames))


def test_psnr_matches_reference_after_training(tmp_path):
    try:
        ref = RefKernels("cfg1")
    except (FileNotFoundError, OSError) as e:
        pytest.skip(f"reference kernels for the CPU not built: {e}")
    images, cams, K, W, H = trainer.synthetic_scene_views("cfg1", 0)
    dev = trainer.synthetic_nerf("cfg1", "fp32", 0, str(tmp_path / "dev"))
    host = trainer.synthetic_nerf("cfg1", "fp32", 0, str(tmp_path / "ref"))   # init state + seed stream
    g = dev.geometry(SPR)
    cores = os.cpu_count() or 1

    # reference state from the same init draws
    blob = host._blob_from_state()
    lay, _ = param_layout(g["F"], g["ND"], g["NC"])
    shapes = param_shapes(g["F"], g["ND"], g["NC"])
    params = {n: (blob[o:o + s].view(np.int32).copy() if n in shapes else np.zeros(0, np.int32))
              for n, (o, s) in lay.items()}
    m = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
    v = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
    table = host.state_i32["table"].copy()
    occ_in = host.state_i32["occ_grid_in_u32"].view(np.uint32).copy()
    occ_st = host.state_i32["occ_grid_st_u32"].view(np.uint32).copy()
    scr = ref.alloc_scratch(RAYS * SPR)
    out = np.zeros((RAYS, 4), np.float32)

    io = ft.RayBatch.init(dev.ctx, dev.queue, RAYS, SPR)
    dev.setup_buffers(RAYS, SPR)
    lmbda = sch.lr_lambda(sch.LMBDA_BASE, RAYS, SPR)
    rng = np.random.default_rng(2024)
    for step in range(STEPS):
        im = rng.integers(0, images.shape[0], RAYS)
        u, vv = rng.integers(0, W, RAYS), rng.integers(0, H, RAYS)
        rays, tg = ft.rays_targets_from_indices(im, u, vv, images, cams, W, H, K)
        lr_f = float(sch.lr_schedule(step, 1e-3, lmbda, RAYS, SPR))
        sh = float(sch.sh_multiplier_function(step))
        crl = float(sch.color_MLP_rel_lr_function(step))
        occ_s = float(dev.occ.occ_update_strength0) * float(sch.occ_u_multiplier_function(step))
        # device
        io.upload_rays(rays)
        io.upload_targets(tg)
        dev.step(io, lr_f=lr_f, do_train=True, return_output=False, sh_multiplier=sh, color_MLP_rel_lr=crl,
                 occ_update_strength=occ_s)
        # reference, the host steps of Nerf.step around its kernels
        seed = int(host._get_rng_u32())
        host.steps_trained += 1
        ref.train(params, table, rays.view(np.float32).reshape(RAYS, 8), tg, out, scr, occ_in, occ_st, g,
                  lr_f, sh, occ_s, seed, True, cores)
        if host.maintenance_due(host.steps_trained, occ_s):
            ref.decay(occ_in, occ_st, host.decay_q24(occ_s), seed)
        ref.weight_update(params, m, v, scr, RAYS * SPR, float(host.lr_t(lr_f)), crl, float(host.ADAM_BETA1),
                          float(host.ADAM_BETA2), float(host.ADAM_EPS), cores)
    dev.queue.finish()
    assert dev.native.status() == 0

    # renders of the training views, each model by its own implementation
    from render_gpu import render_frame
    dev_frames = [render_frame(dev, c, K, W, H, rng_u32=i).cpu().numpy() for i, c in enumerate(cams)]
    rscr = ref.alloc_scratch(W * H * SPR)
    rout = np.zeros((W * H, 4), np.float32)
    zeros = np.zeros((W * H, 4), np.float32)
    ref_frames = []
    for i, c in enumerate(cams):
        uu, vv = np.meshgrid(np.arange(W), np.arange(H))
        rays = ft.rays_from_rt_indices(c, uu.ravel(), vv.ravel(), W, H, K)
        ref.train(params, table, rays.view(np.float32).reshape(-1, 8), zeros, rout, rscr, occ_in, occ_st.copy(), g,
                  0.0, 1.0, 0.0, i, False, cores)
        ref_frames.append(rout[:, :3].reshape(H, W, 3).copy())
    p_dev, p_ref = _psnr(dev_frames, images), _psnr(ref_frames, images)
    print(f"PSNR after {STEPS} steps: device {p_dev:.3f} dB, reference {p_ref:.3f} dB")
    assert p_ref > 12.0, p_ref                     # the reference learned the scene
    assert abs(p_dev - p_ref) <= 0.2, (p_dev, p_ref)
