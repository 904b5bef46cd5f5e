"""Generates the golden fixtures of tests/golden/ from the REFERENCE's own Python host code.

Run where the reference checkout is available:
    python tests/golden/make_golden.py --reference <path to MolSzabi/ffnerf-experimental>

The reference host module imports pyopencl, which has no CPU runtime here; a stub module that
records every kernel launch (name, global/local size, the scalar arguments) stands in for it,
so the reference's own ``Nerf.from_kernels`` / ``Nerf.step`` / ray helpers run unmodified and
their host-side results are captured:
  * golden_host_init.npz   -- Nerf._init_fresh state (seed 777) for two geometries;
  * golden_host_steps.npz  -- per step of Nerf.step: the ffnerf_train_step scalars (lr, seed,
                              sh multiplier, occupancy strength), the decay launch (n_words,
                              decay_q24, seed) when maintenance runs, and the weight-update
                              scalars (B, lr_t, colour lr, Adam betas/eps);
  * golden_rays.npz        -- rays_targets_from_indices / rays_from_rt_indices outputs;
  * golden_schedules.npz   -- run_ffnerf_OG's learning-rate, SH, occupancy and colour-lr
                              schedules over a step range;
  * golden_batch_feedback.npz -- run_ffnerf_OG's pixel-weight feedback (_update_weights_u8 with
                              the make_fg_mask_from_rgb foreground) on small uint8 images;
  * golden_ref_checkpoint.npz -- a checkpoint written by the reference's own Nerf.save (F=2, ND=1,
                              after 70 recorded steps); the stub's device->host copy returns
                              what was uploaded to each buffer, so it holds the initial draws.
The tests compare this repository's host module against these arrays bit for bit.
"""
from __future__ import annotations

import argparse
import importlib
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
LAUNCHES: list[tuple] = []


class _Obj:
    def __init__(self, *a, **k):
        self.args, self.kw = a, k


class _Event:
    class _P:
        start, end = 0, 0

    profile = _P()

    def wait(self):
        return None

    command_execution_status = 0


class _Kernel:
    def __init__(self, prg, name):
        self.name = name
        self.argv = ()

    def set_args(self, *args):
        self.argv = args


class _Program:
    def __init__(self, ctx, src):
        self.src = src

    def build(self, options=None, cache_dir=None):
        self.options = options
        return self


def _enqueue_nd_range_kernel(queue=None, kernel=None, global_work_size=None, local_work_size=None, wait_for=None):
    LAUNCHES.append((kernel.name, tuple(global_work_size), tuple(local_work_size), kernel.argv))
    return _Event()


COPY_FROM_HOSTBUF = [False]


def _enqueue_copy(queue, dst, src, wait_for=None):
    if isinstance(dst, np.ndarray):
        hb = getattr(src, "kw", {}).get("hostbuf") if COPY_FROM_HOSTBUF[0] else None
        if hb is not None and np.asarray(hb).nbytes == dst.nbytes:
            dst.reshape(-1).view(np.uint8)[...] = np.ascontiguousarray(hb).reshape(-1).view(np.uint8)
        else:
            dst[...] = 0
    return _Event()


def install_stubs():
    cl = types.ModuleType("pyopencl")
    cl.Context = cl.CommandQueue = cl.Buffer = cl.Event = _Obj
    cl.Program = _Program
    cl.Kernel = _Kernel
    cl.mem_flags = types.SimpleNamespace(READ_ONLY=1, WRITE_ONLY=2, READ_WRITE=4, COPY_HOST_PTR=8)
    cl.command_queue_properties = types.SimpleNamespace(OUT_OF_ORDER_EXEC_MODE_ENABLE=1, PROFILING_ENABLE=2, COMPLETE=0)
    cl.command_execution_status = types.SimpleNamespace(COMPLETE=0)
    cl.event_info = types.SimpleNamespace(COMMAND_EXECUTION_STATUS=0)
    cl.platform_info = types.SimpleNamespace(NAME=0)
    cl.cltypes = types.SimpleNamespace(make_float3=lambda *v: np.array(list(v) + [0.0], np.float32))
    cl.enqueue_nd_range_kernel = _enqueue_nd_range_kernel
    cl.enqueue_copy = _enqueue_copy
    cl.wait_for_events = lambda evs: None
    sys.modules["pyopencl"] = cl
    sys.modules["pygame"] = types.ModuleType("pygame")


def host_init_and_steps(ft, tmp: Path):
    init = {}
    steps = []
    for tag, F, nd, entries in (("f2nd1", 2, 1, 16 * 2 ** 10), ("f4nd2", 4, 2, 16 * 2 ** 9)):
        ft.F_PER_LEVEL, ft.L_POS, ft.ND, ft.NC = F, 16 * F, nd, 2
        occ = ft.OccParams(G_occ=8, box_min=np.array([-1, -1, -1], np.float32), box_max=np.array([1, 1, 1], np.float32),
                           rho_min=np.float32(1.0), rho_max=np.float32(16.0)).finalize()
        nerf = ft.Nerf.from_kernels(ctx=_Obj(), queue=_Obj(), kernel_file=ft.KERNEL_FILE_DEFAULT,
                                    decay_file=Path(ft.KERNEL_DECAY), weight_update_file=Path(ft.KERNEL_W_B_UPDATES),
                                    background="random", layers={}, edges={}, training_dir=tmp, model_id=f"g_{tag}",
                                    load_id=None, transfer_fmt="fp32", rng_seed=777, occ=occ,
                                    table_size_entries=entries, f_per_level=F)
        for k, v in nerf.state_i32.items():
            init[f"{tag}/{k}"] = np.asarray(v).copy()
        if tag != "f2nd1":
            continue
        io = ft.RayBatch.init(_Obj(), _Obj(), num_rays=4, samples_per_ray=64, with_host_arrays=True)
        for step in range(1, 71):
            LAUNCHES.clear()
            occ_s = 1.0 if step > 30 else 0.0
            lr_f = np.float32(1e-3 * (0.99 ** step))
            nerf.step(io=io, lr_f=float(lr_f), do_train=True, return_output=False, sh_multiplier=0.25,
                      color_MLP_rel_lr=0.4, occ_update_strength=occ_s, rng_u32=None, wait=False)
            rec = {"step": step}
            for name, gws, lws, argv in LAUNCHES:
                if name == "ffnerf_train_step":
                    sc = argv[-18:]   # lr num_rays spr do_train sh occ_in occ_st bmin bmax G rho.. seed strength
                    rec.update(ff_lr=np.float32(sc[0]), ff_nrays=int(sc[1]), ff_spr=int(sc[2]), ff_do_train=int(sc[3]),
                               ff_sh=np.float32(sc[4]), ff_G=int(sc[9]), ff_seed=np.uint32(sc[-2]),
                               ff_occ=np.float32(sc[-1]), ff_gws=gws[0], ff_lws=lws[0])
                elif name == "occ_nibble_decay_write_both_q24":
                    rec.update(dec_n=int(argv[2]), dec_q24=int(argv[3]), dec_seed=np.uint32(argv[4]), dec_gws=gws[0])
                elif name == "update_ffnerf_oneWG":
                    sc = argv[-8:]
                    rec.update(wu_B=int(sc[0]), wu_L=int(sc[1]), wu_M=int(sc[2]), wu_lr_t=np.float32(sc[3]),
                               wu_color=np.float32(sc[4]), wu_b1=np.float32(sc[5]), wu_b2=np.float32(sc[6]),
                               wu_eps=np.float32(sc[7]), wu_gws=gws, wu_lws=lws)
            steps.append(rec)
        # the reference's own checkpoint writer, device buffers read back as uploaded
        COPY_FROM_HOSTBUF[0] = True
        try:
            path = nerf.save(min_new_file_seconds=0)
        finally:
            COPY_FROM_HOSTBUF[0] = False
        (OUT / "golden_ref_checkpoint.npz").write_bytes(Path(path).read_bytes())
    keys = sorted({k for r in steps for k in r})
    cols = {}
    for k in keys:
        vals = [r.get(k) for r in steps]
        if k in ("wu_gws", "wu_lws"):
            cols[k] = np.array([v for v in vals], dtype=np.int64)
        elif k in ("dec_n", "dec_q24", "dec_gws"):
            cols[k] = np.array([-1 if v is None else v for v in vals], dtype=np.int64)
        elif k == "dec_seed":
            cols[k] = np.array([0 if v is None else v for v in vals], dtype=np.uint32)
        else:
            cols[k] = np.array(vals)
    return init, cols


def rays_fixture(ft):
    rng = np.random.default_rng(3)
    N, H, W = 3, 6, 9
    Ims = rng.random((N, H, W, 3), dtype=np.float32)
    c2w = np.tile(np.eye(4, dtype=np.float32), (N, 1, 1))
    for i in range(N):
        a = rng.normal(size=3)
        q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
        c2w[i, :3, :3] = q.astype(np.float32)
        c2w[i, :3, 3] = a.astype(np.float32)
    K = np.array([[7.0, 0, 4.2], [0, 7.5, 3.1], [0, 0, 1]], np.float32)
    im = rng.integers(0, N, 50)
    u = rng.integers(0, W, 50)
    v = rng.integers(0, H, 50)
    r1, t1 = ft.rays_targets_from_indices(im, u, v, Ims, c2w, W, H, K=K)
    r2, t2 = ft.rays_targets_from_indices(im, u, v, Ims, c2w, W, H, K=None)
    Ks = np.stack([K, K * np.float32(1.1)]).astype(np.float32)
    Ks[:, 2, 2] = 1
    r3, _ = ft.rays_targets_from_indices(im % 2, u, v, Ims[:2], c2w[:2], W, H, K=Ks)
    r4 = ft.rays_from_rt_indices(c2w[1], u, v, W, H, K=K)
    r5 = ft.rays_from_rt_indices(c2w[2], u, v, W, H, K=None)
    flat = lambda r: np.ascontiguousarray(r).view(np.float32).reshape(-1, 8)
    return dict(Ims=Ims, c2w=c2w, K=K, Ks=Ks, im=im, u=u, v=v, W=W, H=H, rays_k=flat(r1), tg_k=t1, rays_nok=flat(r2),
                tg_nok=t2, rays_perK=flat(r3), rays_rt=flat(r4), rays_rt_nok=flat(r5))


def schedules_fixture(ref: Path):
    for mod in ("cv2", "tqdm"):
        importlib.import_module(mod)
    run = importlib.import_module("run_ffnerf_OG")
    steps = np.array([0, 1, 100, 1499, 1500, 1501, 2000, 2999, 3000, 3001, 3750, 4500, 6000, 20000])
    return dict(steps=steps, T_MID=np.int64(run.T_MID), LMBDA_BASE=np.float64(run.LMBDA_BASE),
                LR_FLOOR=np.float64(run.LR_FLOOR),
                sh=np.array([float(run.sh_multiplier_function(s)) for s in steps]),
                occ=np.array([float(run.occ_u_multiplier_function(s)) for s in steps]),
                color=np.array([float(run.color_MLP_rel_lr_function(s)) for s in steps]))


def batch_fixture(ref: Path):
    """The trainer's weight-map feedback (_update_weights_u8, run_ffnerf_OG.py:459-490) and its
    RGB-threshold foreground (make_fg_mask_from_rgb, :402-421) on small uint8 images."""
    for mod in ("cv2", "tqdm"):
        importlib.import_module(mod)
    run = importlib.import_module("run_ffnerf_OG")
    rng = np.random.default_rng(11)
    N, H, W = 3, 8, 12
    Ims = rng.integers(0, 256, (N, H, W, 3), dtype=np.uint8)
    Ims[:, :3, :4] = rng.integers(0, 9, (N, 3, 4, 3), dtype=np.uint8)   # dark (background) corner
    weights = [rng.integers(1, 256, (H, W), dtype=np.uint8) for _ in range(N)]
    before = np.stack(weights).copy()
    fg = run.make_fg_mask_from_rgb(Ims, tau=8, dilate=0)
    flat = rng.choice(N * H * W, 120, replace=False)        # distinct pixels: the update is order-free
    im = (flat // (H * W)).astype(np.int32)
    y = ((flat // W) % H).astype(np.int32)
    x = (flat % W).astype(np.int32)
    err = rng.uniform(0.0, 0.6, flat.size).astype(np.float32)
    err[:7] = 0.0
    run._update_weights_u8(weights, fg, im, x, y, err, ema=0.05, bg_cap=16)
    return dict(Ims=Ims, w_before=before, w_after=np.stack(weights), fg=np.stack(fg), im=im, x=x, y=y, err=err,
                median=np.float32(np.median(err)))


def main(argv=None):
    ap = argparse.ArgumentParser(description="golden fixtures from the reference host code")
    ap.add_argument("--reference", type=Path, required=True)
    a = ap.parse_args(argv)
    install_stubs()
    sys.path.insert(0, str(a.reference))
    ft = importlib.import_module("ffnerf_tools")
    with tempfile.TemporaryDirectory() as tmp:
        init, steps = host_init_and_steps(ft, Path(tmp))
    np.savez_compressed(OUT / "golden_host_init.npz", **init)
    np.savez_compressed(OUT / "golden_host_steps.npz", **steps)
    np.savez_compressed(OUT / "golden_rays.npz", **rays_fixture(ft))
    np.savez_compressed(OUT / "golden_schedules.npz", **schedules_fixture(a.reference))
    np.savez_compressed(OUT / "golden_batch_feedback.npz", **batch_fixture(a.reference))
    print("wrote", sorted(p.name for p in OUT.glob("golden_*.npz")))


if __name__ == "__main__":
    main()
