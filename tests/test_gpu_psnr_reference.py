"""End-of-training parity with the reference's algorithm.

The same 1,600 training steps of the synthetic cfg1 scene -- the same initial state (the reference's
init draws from one seed), the same batches (512 uniformly drawn pixels per step, host rays of
rays_targets_from_indices), the same schedules (run_ffnerf_OG.py:1356-1365, the occupancy updates
live after step 1,500 with decay every 32nd step) and the same per-step seeds -- are trained by:
  * the device through ffnerf_tools.Nerf.step (fp32 MLP, immediate table update: in the split step
    every gather of a step precedes its scatters);
  * the oracle with the deferred table update (every ray of a step reads the step-start table: the
    schedule of a GPU that runs all of a step's rays at once) -- OracleModel;
  * the reference's own kernels compiled for the CPU (oracle/_ref) in two schedules -- RefModel:
    lockstep (every ray's work-group advances barrier interval by barrier interval with all the
    others, so every table read of a step precedes every in-kernel table update: the schedule of a
    GPU that holds the whole batch), and near-sequential (host threads each running one ray's
    work-group at a time, so each ray's Hogwild update is visible to nearly every later ray).
The host steps of Nerf.step (ffnerf_tools.py:1357-1544) are restated around the CPU kernels.  Each
model renders the 8 training views with its own renderer and the PSNR over all pixels is compared.

The table-update schedule moves the PSNR at this point of training: the oracle in its sequential
mode (rays applied in order) ends 0.29 dB above its deferred mode on this protocol (21.72 vs
21.43 dB), and the reference kernels' near-sequential runs end at 21.76-21.96 dB.  The 0.2 dB
contract therefore compares the device with the reference kernels under the device's schedule (the
lockstep run; tests/test_oracle_pin.py shows that one lockstep step is bit-identical to the deferred
oracle's), and with the deferred oracle; the near-sequential run is reported and held to 1 dB.

The device's side is the median of three runs: the immediate table update adds its float atomics in
a different order from run to run, and single device runs of this protocol have ended anywhere in
21.20-21.45 dB on B200s, which alone spans more than the contract's 0.2 dB.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import ffnerf_tools as ft
import schedules as sch
import trainer
from ffn_config import param_layout, param_shapes
from oracle import Oracle, OrcStep, RefKernels, make_orc_config

STEPS, RAYS, SPR = 1600, 512, 64
DEVICE_RUNS = 3


def psnr(frames, images):
    se = sum(float(((np.clip(f, 0, 1) - im.astype(np.float32) / 255.0) ** 2).sum()) for f, im in zip(frames, images))
    return -10.0 * np.log10(se / sum(f.size for f in frames))


def batches(images, cams, K, W, H, steps=STEPS, seed=2024):
    """Per step: 512 uniformly drawn (image, pixel) pairs, host rays and targets, and the schedules."""
    rng = np.random.default_rng(seed)
    lmbda = sch.lr_lambda(sch.LMBDA_BASE, RAYS, SPR)
    occ0 = float(ft.OCC_U_STR)
    for step in range(steps):
        im = rng.integers(0, images.shape[0], RAYS)
        u, v = rng.integers(0, W, RAYS), rng.integers(0, H, RAYS)
        rays, tg = ft.rays_targets_from_indices(im, u, v, images, cams, W, H, K)
        yield (rays, tg, float(sch.lr_schedule(step, 1e-3, lmbda, RAYS, SPR)), float(sch.sh_multiplier_function(step)),
               float(sch.color_MLP_rel_lr_function(step)), occ0 * float(sch.occ_u_multiplier_function(step)))


class RefModel:
    """A model trained by the reference kernels compiled for the CPU, with the host steps of
    Nerf.step around them: per-step seed from the model's numpy stream, occupancy decay every 32nd
    step once updates are live, Adam bias correction with t = steps trained."""

    def __init__(self, host, cores=None, lockstep=False):
        self.host = host                          # an ffnerf_tools.Nerf: init state, seeds, schedules
        self.lockstep = lockstep
        self.ref = RefKernels("cfg1")
        self.g = host.geometry(SPR)
        self.cores = cores or os.cpu_count() or 1
        g = self.g
        blob = host._blob_from_state()
        lay, _ = param_layout(g["F"], g["ND"], g["NC"])
        shapes = param_shapes(g["F"], g["ND"], g["NC"])
        self.params = {n: (blob[o:o + s].view(np.int32).copy() if n in shapes else np.zeros(0, np.int32))
                       for n, (o, s) in lay.items()}
        self.m = {k: np.zeros(v.size, np.float32) for k, v in self.params.items()}
        self.v = {k: np.zeros(v.size, np.float32) for k, v in self.params.items()}
        self.table = host.state_i32["table"].copy()
        self.occ_in = host.state_i32["occ_grid_in_u32"].view(np.uint32).copy()
        self.occ_st = host.state_i32["occ_grid_st_u32"].view(np.uint32).copy()
        self.scr = self.ref.alloc_scratch(RAYS * SPR)
        self.out = np.zeros((RAYS, 4), np.float32)

    def step(self, rays, tg, lr_f, sh, crl, occ_s):
        h = self.host
        seed = int(h._get_rng_u32())
        h.steps_trained += 1
        self.ref.train(self.params, self.table, np.ascontiguousarray(rays).view(np.float32).reshape(-1, 8), tg,
                       self.out, self.scr, self.occ_in, self.occ_st, self.g, lr_f, sh, occ_s, seed, True, self.cores,
                       lockstep=self.lockstep)
        if h.maintenance_due(h.steps_trained, occ_s):
            self.ref.decay(self.occ_in, self.occ_st, h.decay_q24(occ_s), seed)
        self.ref.weight_update(self.params, self.m, self.v, self.scr, RAYS * SPR, float(h.lr_t(lr_f)), crl,
                               float(h.ADAM_BETA1), float(h.ADAM_BETA2), float(h.ADAM_EPS), self.cores)

    def render(self, cams, K, W, H):
        """The views rendered by the reference kernel (do_train = 0), view i keyed with seed i."""
        scr = self.ref.alloc_scratch(W * H * SPR)
        out = np.zeros((W * H, 4), np.float32)
        zeros = np.zeros((W * H, 4), np.float32)
        uu, vv = np.meshgrid(np.arange(W), np.arange(H))
        frames = []
        for i, c in enumerate(cams):
            rays = np.ascontiguousarray(ft.rays_from_rt_indices(c, uu.ravel(), vv.ravel(), W, H, K))
            self.ref.train(self.params, self.table, rays.view(np.float32).reshape(-1, 8), zeros, out, scr, self.occ_in,
                           self.occ_st.copy(), self.g, 0.0, 1.0, 0.0, i, False, self.cores)
            frames.append(out[:, :3].reshape(H, W, 3).copy())
        return frames

    def load_from(self, nerf):
        """Takes table, parameters and occupancy grids of a device-trained ffnerf_tools.Nerf."""
        nerf.sync_params_from_device()
        st = nerf.state_i32
        for n in self.params:
            if self.params[n].size:
                self.params[n] = st[n].reshape(-1).copy()
        self.table = st["table"].reshape(-1).copy()
        self.occ_in = st["occ_grid_in_u32"].view(np.uint32).reshape(-1).copy()
        self.occ_st = st["occ_grid_st_u32"].view(np.uint32).reshape(-1).copy()


def nibble_max(a, b):
    """Nibble-wise maximum of two occupancy grids (8 nibbles per uint32 word)."""
    out = np.zeros_like(a)
    for sh in range(0, 32, 4):
        out |= np.maximum((a >> sh) & 0xF, (b >> sh) & 0xF) << sh
    return out


class OracleModel:
    """A model trained by the oracle with the deferred table update and the host steps of Nerf.step.
    The rays of a step are split into contiguous chunks run on host threads (the ctypes calls
    release the GIL); each chunk keys its RNG streams by global ray id (ray_offset), so the chunks
    together are the whole-batch step; their table and MLP gradients are summed in chunk order and
    their occupancy proposals merged by nibble-wise maximum (order-independent, like the
    reference's atomic max)."""

    def __init__(self, host, threads=None):
        self.host = host
        self.g = host.geometry(SPR)
        self.cfg = make_orc_config(self.g, table_mode=0)
        self.o = Oracle()
        self.threads = threads or os.cpu_count() or 1
        self.blob = host._blob_from_state()
        self.m, self.v = np.zeros_like(self.blob), np.zeros_like(self.blob)
        self.table = host.state_i32["table"].view(np.float32).copy()
        self.occ_in = host.state_i32["occ_grid_in_u32"].view(np.uint32).copy()
        self.occ_st = host.state_i32["occ_grid_st_u32"].view(np.uint32).copy()

    def _run(self, rays, tg, lr_f, sh, occ_s, seed, train):
        n = rays.shape[0]
        out = np.zeros((n, 4), np.float32)
        bounds = np.linspace(0, n, self.threads + 1).astype(int)

        def work(j):
            a, b = int(bounds[j]), int(bounds[j + 1])
            tgr = np.zeros_like(self.table) if train else None
            mg = np.zeros_like(self.blob) if train else None
            ost = self.occ_st.copy()
            if b > a:
                self.o.forward_backward(self.cfg, OrcStep(lr_f, sh, occ_s, seed, int(train), a), self.blob,
                                        self.table, self.occ_in, ost, np.ascontiguousarray(rays[a:b]),
                                        np.ascontiguousarray(tg[a:b]), out[a:b], tgr, mg)
            return tgr, mg, ost

        with ThreadPoolExecutor(self.threads) as ex:
            res = list(ex.map(work, range(self.threads)))
        return out, res

    def step(self, rays, tg, lr_f, sh, crl, occ_s):
        h = self.host
        seed = int(h._get_rng_u32())
        h.steps_trained += 1
        _, res = self._run(np.ascontiguousarray(rays).view(np.float32).reshape(-1, 8), tg, lr_f, sh, occ_s, seed, True)
        tgr, mg = res[0][0], res[0][1]
        for t_, m_, _ in res[1:]:
            tgr += t_
            mg += m_
        if occ_s > 0.0:                           # proposals are written only while updates are live
            for _, _, ost in res:
                d = np.nonzero(ost != self.occ_st)[0]   # a step proposes into few words: merge those
                if d.size:
                    self.occ_st[d] = nibble_max(self.occ_st[d], ost[d])
        if h.maintenance_due(h.steps_trained, occ_s):
            self.o.decay(self.occ_in, self.occ_st, h.decay_q24(occ_s), seed)
        self.o.mlp_adam(self.cfg, self.blob, mg, self.m, self.v, float(h.lr_t(lr_f)), crl, float(h.ADAM_BETA1),
                        float(h.ADAM_BETA2), float(h.ADAM_EPS))
        self.o.table_apply(self.cfg, self.table, tgr, lr_f)

    def render(self, cams, K, W, H):
        """The views rendered by the oracle's inference path, view i keyed with seed i."""
        uu, vv = np.meshgrid(np.arange(W), np.arange(H))
        frames = []
        for i, c in enumerate(cams):
            rays = np.ascontiguousarray(ft.rays_from_rt_indices(c, uu.ravel(), vv.ravel(), W, H, K))
            out, _ = self._run(rays.view(np.float32).reshape(-1, 8), np.zeros((W * H, 4), np.float32),
                               0.0, 1.0, 0.0, i, False)
            frames.append(out[:, :3].reshape(H, W, 3))
        return frames


def train_device(nerf, data, steps=STEPS, seed=2024):
    images, cams, K, W, H = data
    io = ft.RayBatch.init(nerf.ctx, nerf.queue, RAYS, SPR)
    nerf.setup_buffers(RAYS, SPR)
    for rays, tg, lr_f, sh, crl, occ_s in batches(images, cams, K, W, H, steps, seed):
        io.upload_rays(rays)
        io.upload_targets(tg)
        nerf.step(io, lr_f=lr_f, do_train=True, return_output=False, sh_multiplier=sh, color_MLP_rel_lr=crl,
                  occ_update_strength=occ_s)
    nerf.queue.finish()


def train_cpu(model, data, steps=STEPS, seed=2024):
    images, cams, K, W, H = data
    for b in batches(images, cams, K, W, H, steps, seed):
        model.step(*b)


@pytest.mark.gpu
def test_psnr_matches_reference_after_training(tmp_path):
    """Contracts (PSNR(device) = the median of the device runs): |PSNR(device) - PSNR(reference
    kernels, lockstep)| <= 0.2 dB and
    |PSNR(device) - PSNR(deferred oracle)| <= 0.2 dB; the reference kernels' near-sequential run within
    1 dB of the device (see the module docstring); the device's renderer and the reference's renderer
    agree on the device's model within 0.05 dB."""
    try:
        RefKernels("cfg1")
    except (FileNotFoundError, OSError) as e:
        pytest.skip(f"reference kernels for the CPU not built: {e}")
    data = trainer.synthetic_scene_views("cfg1", 0)
    images, cams, K, W, H = data
    from render_gpu import render_frame
    p_devs = []
    for k in range(DEVICE_RUNS):
        if k:
            dev.native.close()
        dev = trainer.synthetic_nerf("cfg1", "fp32", 0, str(tmp_path / f"dev{k}"))
        train_device(dev, data)
        assert dev.native.status() == 0
        p_devs.append(psnr([render_frame(dev, c, K, W, H, rng_u32=i).cpu().numpy() for i, c in enumerate(cams)],
                           images))
    p_dev = float(np.median(p_devs))
    orc = OracleModel(trainer.synthetic_nerf("cfg1", "fp32", 0, str(tmp_path / "orc"), host_only=True))
    train_cpu(orc, data)
    p_orc = psnr(orc.render(cams, K, W, H), images)
    ref = RefModel(trainer.synthetic_nerf("cfg1", "fp32", 0, str(tmp_path / "ref"), host_only=True))
    train_cpu(ref, data)
    p_ref = psnr(ref.render(cams, K, W, H), images)
    lock = RefModel(trainer.synthetic_nerf("cfg1", "fp32", 0, str(tmp_path / "lock"), host_only=True), lockstep=True)
    train_cpu(lock, data)
    p_lock = psnr(lock.render(cams, K, W, H), images)
    cross = RefModel(trainer.synthetic_nerf("cfg1", "fp32", 0, str(tmp_path / "x"), host_only=True))
    cross.load_from(dev)
    p_dev_refrender = psnr(cross.render(cams, K, W, H), images)
    print(f"PSNR after {STEPS} steps: device {p_dev:.3f} dB (runs {', '.join(f'{p:.3f}' for p in p_devs)}; the last "
          f"one {p_devs[-1]:.3f} dB with the reference renderer {p_dev_refrender:.3f}), "
          f"reference kernels lockstep {p_lock:.3f} dB / near-sequential {p_ref:.3f} dB, deferred oracle {p_orc:.3f} dB")
    assert p_ref > 12.0 and p_orc > 12.0 and p_lock > 12.0, (p_ref, p_orc, p_lock)   # the scene was learned
    assert abs(p_dev - p_lock) <= 0.2, (p_dev, p_lock)
    assert abs(p_dev - p_orc) <= 0.2, (p_dev, p_orc)
    assert abs(p_dev - p_ref) <= 1.0, (p_dev, p_ref)
    assert abs(p_devs[-1] - p_dev_refrender) <= 0.05, (p_devs[-1], p_dev_refrender)
