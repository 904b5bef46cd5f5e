"""Device-resident training loop: the inner loop of the reference trainer (run_ffnerf_OG.py:974-1570)
with every per-step piece on the GPU.

Reference                                   here
batch_producer thread (numpy rejection,     GpuBatchProducer.next_batch: one kernel draws the batch
  rays_targets_from_indices, upload)          into the RayBatch's device buffers
Nerf.step with the schedules of             Nerf.step (libffnerf), the same schedules (schedules.py)
  run_ffnerf_OG.py:1356-1365
periodic metrics + pixel-weight feedback    batch_metrics / GpuBatchProducer.feedback on the device;
  (D2H of the output, numpy, :1368-1403)      the figures are read back only when reported
periodic save after queue.finish()          Nerf.save(async_write=True): training keeps running
  (:1508-1516)                                while the checkpoint is read back and written

The images stay in HBM; nothing per step crosses PCIe.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np

import schedules as sch
from batch_gpu import GpuBatchProducer, batch_metrics


@dataclass
class TrainConfig:
    steps: int = 20000
    batch_rays: int = 512
    samples_per_ray: int = 64
    lr: float = 1e-3                  # reference CLI default (run_ffnerf_OG.py:1603)
    lmbda_base: float = sch.LMBDA_BASE
    period: int = 100                 # metrics + weight-map feedback every `period` steps
    save_seconds: float = 0.0         # 0: no periodic checkpoint
    rng_seed: int = 0
    log: bool = True
    history: list = field(default_factory=list)


def train(nerf, producer: GpuBatchProducer, cfg: TrainConfig, start_step: int = 0):
    """Runs cfg.steps training steps of ``nerf`` (an ffnerf_tools.Nerf) on batches from
    ``producer``.  Returns the list of (step, mse, rmse, l2, lr_f) reported every cfg.period steps."""
    import ffnerf_tools as ft
    io = ft.RayBatch.init(nerf.ctx, nerf.queue, cfg.batch_rays, cfg.samples_per_ray)
    nerf.setup_buffers(cfg.batch_rays, cfg.samples_per_ray)
    lmbda = sch.lr_lambda(cfg.lmbda_base, cfg.batch_rays, cfg.samples_per_ray)
    pending = []
    last_save = time.time()
    t0 = time.time()
    for k in range(cfg.steps):
        step = start_step + k
        producer.next_batch(io.rays_buf, io.targets_buf, stream=nerf.queue.stream)
        lr_f = sch.lr_schedule(step, cfg.lr, lmbda, cfg.batch_rays, cfg.samples_per_ray)
        occ_s = float(nerf.occ.occ_update_strength0) * float(sch.occ_u_multiplier_function(step))
        nerf.step(io, lr_f=float(lr_f), do_train=True, return_output=False,
                  sh_multiplier=float(sch.sh_multiplier_function(step)),
                  color_MLP_rel_lr=float(sch.color_MLP_rel_lr_function(step)), occ_update_strength=occ_s)
        if cfg.period > 0 and step % cfg.period == 0:
            import torch
            with torch.cuda.stream(nerf.queue.stream):
                m = batch_metrics(io.out_buf, io.targets_buf, cfg.batch_rays, stream=nerf.queue.stream)
                producer.feedback(io.out_buf, io.targets_buf, stream=nerf.queue.stream)
            pending.append((step, m, float(lr_f)))
        if len(pending) > 4 or (pending and k == cfg.steps - 1):
            nerf.queue.finish()
            st = nerf.native.status()
            if st:
                raise RuntimeError(f"device status {st:#x} by step {step}: "
                                   + ("non-finite colours or gradients (the model diverged)" if st & 1
                                      else "a bounded wait ran out"))
            for s, m, lr in pending:
                mse, rmse, l2 = (float(v) for v in m.cpu().numpy())
                cfg.history.append((s, mse, rmse, l2, lr))
                if cfg.log:
                    psnr = -10.0 * np.log10(max(mse, 1e-12))
                    print(f"[step {s}] mse={mse:.5f} psnr={psnr:.2f} dB l2={l2:.4f} lr_f={lr:.3e} "
                          f"({time.time() - t0:.1f} s)", flush=True)
            pending.clear()
        if cfg.save_seconds > 0 and time.time() - last_save > cfg.save_seconds:
            nerf.save(min_new_file_seconds=300, async_write=True)
            last_save = time.time()
    nerf.queue.finish()
    nerf.wait_saved()
    return cfg.history


SYNTHETIC = {"cfg1": dict(n_cams=8, W=64, H=64, log2T=14, rmax=512.0, G=64),
             "cfg2": dict(n_cams=56, W=800, H=450, log2T=19, rmax=2048.0, G=128)}


def synthetic_scene_views(workload: str = "cfg1", seed: int = 0, device: str = "cuda"):
    """The seeded synthetic Gaussian-blob scene of the benchmark configurations (cfg1: 8 cameras
    at 64x64 on a radius-2 sphere; cfg2: 56 cameras at 450x800 on a ring), rendered analytically
    on `device` into 8-bit images (the reference's loader quantises too).
    Returns (images uint8 [n, H, W, 3], c2w [n, 4, 4], K [3, 3], W, H)."""
    import torch
    from synthetic_scene import BlobScene, cameras_ring, cameras_sphere, intrinsics, pixel_rays
    wl = SYNTHETIC[workload]
    scene = BlobScene(seed)
    cams = cameras_sphere(wl["n_cams"], 2.0, seed) if wl["n_cams"] <= 8 else cameras_ring(wl["n_cams"], 2.5, seed)
    K = intrinsics(wl["W"], wl["H"], 50.0)
    vv, uu = np.mgrid[0:wl["H"], 0:wl["W"]]
    images = []
    for c in cams:
        rgb = scene.render_torch(torch.from_numpy(pixel_rays(c, K, uu.ravel(), vv.ravel())).to(device), n_quad=192)
        images.append(torch.round(rgb.clamp(0, 1) * 255).to(torch.uint8).cpu().numpy().reshape(wl["H"], wl["W"], 3))
    return np.stack(images), np.asarray(cams, np.float32), K, wl["W"], wl["H"]


def synthetic_nerf(workload: str = "cfg1", mlp_precision: str = "fp16", seed: int = 0,
                   training_dir: str | None = None, table_update: str = "immediate", host_only: bool = False,
                   background: str = "random"):
    """A fresh ffnerf_tools.Nerf for the synthetic scene's geometry: hash L=16 F=2 (T and Rmax of
    the workload), ND=1, NC=2, `background` ("random" by default), box [-1, 1]^3, near clip 0.3, rng
    seed 777+seed.
    host_only: no device or queue (the host state, seeds and schedules only)."""
    import tempfile
    import ffnerf_tools as ft
    wl = SYNTHETIC[workload]
    ctx = None if host_only else ft.Context([ft.Device(0)])
    queue = None if host_only else ft.CommandQueue(ctx)
    occ = ft.OccParams(G_occ=wl["G"], box_min=np.array([-1, -1, -1], np.float32),
                       box_max=np.array([1, 1, 1], np.float32), rho_min=np.float32(1.0),
                       rho_max=np.float32(16.0), t_near_clip=np.float32(0.3)).finalize()
    tdir = training_dir or tempfile.mkdtemp(prefix="ffn_train_")
    return ft.Nerf(ctx, queue, training_dir=tdir, model_id=f"synthetic_{workload}", transfer_fmt="fp32",
                   table_size_entries=16 << wl["log2T"], f_per_level=2, occ=occ, rng_seed=777 + seed,
                   background=background, finest_resolution=wl["rmax"], nd=1, nc=2, mlp_precision=mlp_precision,
                   verbose=False, table_update=table_update)


def synthetic_run(workload: str = "cfg1", steps: int = 3000, mlp_precision: str = "fp16", seed: int = 0,
                  log: bool = True, training_dir: str | None = None):
    """Trains on the synthetic scene (synthetic_scene_views), 512 rays x 64 samples per step, with
    the device batch producer.  Returns (nerf, history, (images, c2w, K, W, H))."""
    data = synthetic_scene_views(workload, seed)
    images, cams, K, W, H = data
    nerf = synthetic_nerf(workload, mlp_precision, seed, training_dir)
    prod = GpuBatchProducer(images, cams, K, W, H, batch_rays=512, rng_seed=seed)
    cfg = TrainConfig(steps=steps, batch_rays=512, samples_per_ray=64, period=100, log=log, rng_seed=seed)
    hist = train(nerf, prod, cfg)
    return nerf, hist, data


def evaluate_psnr(nerf, images, cams, K, W: int, H: int) -> float:
    """PSNR (dB) of the model's renders of the training views against the 8-bit images, over all
    pixels of all views (inference rule, black background; render_gpu.render_frame)."""
    import torch
    from render_gpu import render_frame
    se, count = 0.0, 0
    for i, c in enumerate(cams):
        frame = render_frame(nerf, c, K, W, H, rng_u32=i)
        ref = torch.from_numpy(images[i].astype(np.float32) / 255.0).to(frame.device)
        se += float(((frame.clamp(0, 1) - ref) ** 2).sum())
        count += frame.numel()
    return -10.0 * np.log10(max(se / count, 1e-12))


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="train on the synthetic benchmark scene on the device")
    ap.add_argument("--workload", choices=["cfg1", "cfg2"], default="cfg1")
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--mlp", choices=["fp16", "fp32"], default="fp16")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    t = time.time()
    nerf, hist, data = synthetic_run(a.workload, a.steps, a.mlp, a.seed)
    print(f"{a.steps} steps in {time.time() - t:.1f} s; final batch mse {hist[-1][1]:.5f}; "
          f"PSNR of the training views {evaluate_psnr(nerf, *data):.2f} dB")


if __name__ == "__main__":
    main()
