"""Host model and kernel boundary of the fused NeRF step, CUDA edition.

Drop-in replacement for the reference's ``ffnerf_tools`` module (MolSzabi/ffnerf-experimental,
ffnerf_tools.py): the same public surface -- ``Nerf`` (from_kernels, setup_buffers, step, save,
load_latest, sync_params_from_device, steps_trained), ``RayBatch``, ``OccParams``, the ray
helpers, the module constants and the device/queue/event helpers the trainer calls -- with the
OpenCL programs replaced by libffnerf.so (include/ffnerf.h) and OpenCL queues/events by CUDA
streams/events.  Checkpoints use the reference's NPZ layout byte for byte (float tensors stored
as int32 bit patterns), plus a few extra keys the reference loader ignores.

Differences from the reference behaviour (each deliberate):
  * the hash-table SGD update races in-kernel like the reference's (``table_update="immediate"``,
    the default on one GPU) but in one legal order of that race: in the split tensor-core step every
    gather of a step precedes its scatter; ``table_update="deferred"`` (data-parallel runs, the Adam
    table) applies it after the whole batch;
  * ``setup_buffers`` keeps the device state when the batch shape changes (the reference
    re-uploads its last host snapshot then, ffnerf_tools.py:1380-1385);
  * activations never leave the chip; ``transfer_fmt`` ("fp32", "fp16", "fp8") still selects the
    format in which the weight update reads them, quantised as the reference's staging buffers are
    (fp32 MLP; the tensor-core MLP runs with "fp32" only).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from datetime import datetime
from pathlib import Path
from typing import List, Optional

import os

import numpy as np

import ffn_config as fc
import ffn_native

# ---------------------------------------------------------------------------- constants
# (ffnerf_tools.py:18-69; "must match kernel defines")
KERNEL_FILE_DEFAULT = str(ffn_native.LIB_PATH)
KERNEL_NAME = "ffnerf_train_step"
KERNEL_DECAY = str(ffn_native.LIB_PATH)
KERNEL_W_B_UPDATES = str(ffn_native.LIB_PATH)

TABLE_SIZE_ENTRIES = 2_260_992
F_PER_LEVEL = 4
TABLE_ELEMS = TABLE_SIZE_ENTRIES * F_PER_LEVEL
L_POS = 16 * F_PER_LEVEL
D_OUT = fc.D_OUT
L_DIR = fc.L_DIR
C_IN = fc.C_IN
C_OUT = fc.C_OUT
M = fc.M
S_MAX = fc.S_MAX
ND, NC = (2, 2)
NDMAX, NCMAX = (3, 4)
TRANSFER_FMT = "fp32"
transfer_nbytes, transfer_define = 4, 32

ADAM_BETA1 = np.float32(0.9)
ADAM_BETA2 = np.float32(0.999)
ADAM_EPS = np.float32(1e-8)

SIGMA_BIAS = -2.0
OCC_U_STR = 1
DECAY = 0.9
RHO_MIN_DEF = 1.0
RHO_MAX_DEF = 64.0
OCC_INIT_DENSITY = 0xEEEEEEEE
OCC_MAINTENANCE_PERIOD = 32

# Tiling knobs of the reference weight-update kernel, kept for callers that read them.
WU_WG_X_DEFAULT, WU_WG_Y_DEFAULT, WU_REG_X_DEFAULT, WU_REG_Y_DEFAULT, WU_TILEK_DEFAULT = 16, 16, 1, 1, 236


# ---------------------------------------------------------------------------- device / queue / events
class _Profile:
    def __init__(self, start_ns: int, end_ns: int):
        self.start, self.end = start_ns, end_ns


class Event:
    """A completion marker on a stream (the pyopencl.Event subset the trainer uses)."""

    def __init__(self, stream, start=None):
        import torch
        self._start = start
        self._end = torch.cuda.Event(enable_timing=start is not None)
        self._end.record(stream)
        self._on_complete = None      # host work that completes the command (a staged copy's delivery)

    def wait(self):
        self._end.synchronize()
        if self._on_complete is not None:
            done, self._on_complete = self._on_complete, None
            done()

    @property
    def command_execution_status(self):
        return 0 if self._end.query() else 1     # 0 == COMPLETE (CL_COMPLETE)

    @property
    def profile(self):
        self.wait()
        if self._start is None:
            return _Profile(0, 0)
        return _Profile(0, int(self._start.elapsed_time(self._end) * 1e6))


COMPLETE = 0


class Platform:
    def __init__(self):
        import torch
        self.name = "NVIDIA CUDA"
        self.vendor = "NVIDIA"
        self.version = f"CUDA {torch.version.cuda}"


class Device:
    def __init__(self, index: int = 0):
        import torch
        self.index = int(index)
        self.name = torch.cuda.get_device_name(self.index)
        self.vendor = "NVIDIA"
        self.version = "sm_%d%d" % torch.cuda.get_device_capability(self.index)
        self.opencl_c_version = "N/A"


class Context:
    """Stands in for cl.Context: the CUDA device the model lives on."""

    def __init__(self, devices=None):
        self.devices = list(devices) if devices else [Device(0)]

    @property
    def device(self) -> Device:
        return self.devices[0]


class CommandQueue:
    """Stands in for cl.CommandQueue: one CUDA stream (in-order; events give cross-stream order)."""

    def __init__(self, ctx: Context, stream=None):
        import torch
        self.context = ctx
        self.device = ctx.device
        self.stream = stream or torch.cuda.Stream(device=ctx.device.index)
        self._pending = []            # events whose host-side delivery is still due

    def finish(self):
        self.stream.synchronize()
        pending, self._pending = self._pending, []
        for e in pending:
            e.wait()

    def wait_for(self, events):
        for e in events or []:
            if e is not None:
                self.stream.wait_event(e._end)


def event_ms(evt: Event) -> float:
    """Duration of the timed work an event closes, in ms (ffnerf_tools.py:11-13)."""
    p = evt.profile
    return (p.end - p.start) * 1e-6


def pick_first_device():
    """(platform, device) of the first CUDA device (ffnerf_tools.py:109-124)."""
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("No CUDA device found.")
    return Platform(), Device(torch.cuda.current_device())


def make_queue(ctx: Context, dev: Device = None):
    """(queue, is_out_of_order) -- a CUDA stream is in-order (ffnerf_tools.py:127-138)."""
    return CommandQueue(ctx), False


def f32_to_i32_bits(x_f32: np.ndarray) -> np.ndarray:
    return np.asarray(x_f32, dtype=np.float32).view(np.int32)


def i32_bits_to_f32(x_i32: np.ndarray) -> np.ndarray:
    return np.asarray(x_i32, dtype=np.int32).view(np.float32)


def event_is_complete(ev: Event) -> bool:
    return ev.command_execution_status == COMPLETE


def prune_done(events):
    return [e for e in events if not event_is_complete(e)]


# ---------------------------------------------------------------------------- rays & targets
ray_dtype = np.dtype([("o", np.float32, 4), ("d", np.float32, 4)], align=True)
if ray_dtype.itemsize != 32:
    raise RuntimeError(f"Unexpected Ray dtype size: {ray_dtype.itemsize} (expected 32)")


def default_ray_dtype() -> np.dtype:
    return ray_dtype


def _pixel_dirs_cam(u: np.ndarray, v: np.ndarray, W: int, H: int, fx=None, fy=None, cx=None, cy=None) -> np.ndarray:
    """Camera-frame direction (OpenCV: x right, y down, z forward) through each pixel centre, float32:
    ((u + 0.5 - cx) / fx, (v + 0.5 - cy) / fy, 1) with intrinsics, else the reference's fallback
    (u - W/2 + 0.5, v - H/2 + 0.5, sqrt(H W)).  The operation order is the reference's: it decides
    the float32 rounding the golden fixtures pin."""
    uf = np.asarray(u).astype(np.float32)
    vf = np.asarray(v).astype(np.float32)
    if fx is None:
        return np.stack([uf - W / 2.0 + 0.5, vf - H / 2.0 + 0.5, np.full(uf.size, np.sqrt(H * W), dtype=np.float32)], 1)
    return np.stack([(uf + 0.5 - cx) / fx, (vf + 0.5 - cy) / fy, np.ones(uf.size, dtype=np.float32)], 1)


def _pack_rays(origins: np.ndarray, dirs: np.ndarray) -> np.ndarray:
    """Unit directions (d / (|d| + 1e-12) in float32) and origins into the 32-byte Ray records."""
    norm = np.linalg.norm(dirs, axis=1, keepdims=True).astype(np.float32)
    out = np.zeros((dirs.shape[0],), dtype=ray_dtype)
    out["o"][:, :3] = origins
    out["o"][:, 3] = 1.0
    out["d"][:, :3] = dirs / (norm + 1e-12)
    return out


def rays_targets_from_indices(im_idx, u_idx, v_idx, Ims, c2w_all, W, H, K=None):
    """Rays through pixels (u right, v down) of the given images and their colours
    (ffnerf_tools.py:175-234): one camera-to-world pose per ray, K shared ([3,3]), per image
    ([N,3,3]) or None; colours of uint8 images are divided by 255."""
    im_idx = np.asarray(im_idx, dtype=np.int32)
    u_idx = np.asarray(u_idx, dtype=np.int32)
    v_idx = np.asarray(v_idx, dtype=np.int32)
    assert Ims.ndim == 4 and Ims.shape[1] == H and Ims.shape[2] == W, (Ims.shape, H, W)
    assert c2w_all.shape[0] == Ims.shape[0]
    if K is None:
        cam = _pixel_dirs_cam(u_idx, v_idx, W, H)
    elif K.ndim == 2:
        cam = _pixel_dirs_cam(u_idx, v_idx, W, H, float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2]))
    else:
        Kr = K[im_idx].astype(np.float32)
        cam = _pixel_dirs_cam(u_idx, v_idx, W, H, Kr[:, 0, 0], Kr[:, 1, 1], Kr[:, 0, 2], Kr[:, 1, 2])
    pose = c2w_all[im_idx].astype(np.float32)
    # per-ray rotation as the reference computes it (a batched einsum; its summation order matters)
    dirs = np.einsum("nij,nj->ni", pose[:, :3, :3], cam)
    rays = _pack_rays(pose[:, :3, 3], dirs)
    rgb = Ims[im_idx, v_idx, u_idx, :3]
    targets = np.zeros((im_idx.size, 4), dtype=np.float32)
    targets[:, :3] = rgb if rgb.dtype == np.float32 else rgb.astype(np.float32) / 255.0
    return rays, targets


def rays_from_rt_indices(RT, idx, idy, W, H, K=None):
    """Rays through pixels of one camera-to-world pose (ffnerf_tools.py:237-272)."""
    RT = np.asarray(RT, dtype=np.float32)
    if RT.shape != (4, 4):
        raise ValueError(f"RT must be shape (4,4), got {RT.shape}")
    idx = np.asarray(idx, dtype=np.int32).reshape(-1)
    idy = np.asarray(idy, dtype=np.int32).reshape(-1)
    if idx.size != idy.size:
        raise ValueError("idx and idy must have the same length.")
    if K is None:
        cam = _pixel_dirs_cam(idx, idy, W, H)
    else:
        cam = _pixel_dirs_cam(idx, idy, W, H, K[0, 0], K[1, 1], K[0, 2], K[1, 2])
    # one pose for every ray: a matrix product, as the reference computes it
    dirs = cam @ RT[:3, :3].T
    return _pack_rays(np.broadcast_to(RT[:3, 3][None, :], (idx.size, 3)), dirs)


def _write_npz(path: Path, payload: dict, level: int = 1):
    """An .npz archive (a zip of .npy members, deflate) readable by np.load like the reference's
    np.savez_compressed output, written with deflate level 1 (several times faster than savez_compressed's
    default on table data) to a temporary name and renamed into place, so a reader never sees a
    half-written checkpoint."""
    import zipfile
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    with zipfile.ZipFile(tmp, "w", compression=zipfile.ZIP_DEFLATED, compresslevel=level) as zf:
        for key, val in payload.items():
            with zf.open(key + ".npy", "w", force_zip64=True) as f:
                np.lib.format.write_array(f, np.asanyarray(val), allow_pickle=False)
    os.replace(tmp, path)


# ---------------------------------------------------------------------------- IO bundle
@dataclass
class RayBatch:
    """Rays / targets / outputs of one batch on the device plus pinned host staging
    (ffnerf_tools.py:281-395)."""
    ctx: Context
    queue: CommandQueue
    num_rays: int
    samples_per_ray: int
    ray_dtype: np.dtype = None
    ev_last: Optional[Event] = None
    rays_host: Optional[np.ndarray] = None
    targets_host: Optional[np.ndarray] = None
    out_host: Optional[np.ndarray] = None
    rays_buf: object = None
    targets_buf: object = None
    out_buf: object = None
    _stage: dict = field(default_factory=dict, repr=False)

    def __post_init__(self):
        self.num_rays = int(self.num_rays)
        self.samples_per_ray = int(self.samples_per_ray)
        if self.num_rays <= 0 or self.samples_per_ray <= 0:
            raise ValueError("num_rays and samples_per_ray must be > 0")
        if self.ray_dtype is None:
            self.ray_dtype = default_ray_dtype()
        if self.ray_dtype.itemsize != 32:
            raise ValueError("ray_dtype must be 32 bytes (float4 o, float4 d)")

    @property
    def B_total(self) -> int:
        return self.num_rays * self.samples_per_ray

    @classmethod
    def init(cls, ctx: Context, queue: CommandQueue, num_rays: int, samples_per_ray: int,
             ray_dtype: np.dtype = None, with_host_arrays: bool = True, **_flags) -> "RayBatch":
        import torch
        rb = cls(ctx=ctx, queue=queue, num_rays=num_rays, samples_per_ray=samples_per_ray, ray_dtype=ray_dtype)
        dev = f"cuda:{ctx.device.index}"
        rb.rays_buf = torch.zeros((rb.num_rays, 8), dtype=torch.float32, device=dev)
        rb.targets_buf = torch.zeros((rb.num_rays, 4), dtype=torch.float32, device=dev)
        rb.out_buf = torch.zeros((rb.num_rays, 4), dtype=torch.float32, device=dev)
        for k, w in (("rays", 8), ("targets", 4)):
            rb._stage[k] = torch.zeros((rb.num_rays, w), dtype=torch.float32).pin_memory()
            rb._stage[k + "_ev"] = None
        # two pinned slots for read-backs into pageable arrays, so that a non-blocking download can be
        # in flight while the next step runs
        rb._stage["out"] = [torch.zeros((rb.num_rays, 4), dtype=torch.float32).pin_memory() for _ in range(2)]
        rb._stage["out_ev"] = [None, None]
        rb._stage["out_i"] = 0
        if with_host_arrays:
            rb.rays_host = np.empty((rb.num_rays,), dtype=rb.ray_dtype)
            rb.targets_host = np.empty((rb.num_rays, 4), dtype=np.float32)
            # pinned, so that a download into it is one asynchronous copy, as an OpenCL read is
            rb._stage["out_host"] = torch.zeros((rb.num_rays, 4), dtype=torch.float32).pin_memory()
            rb.out_host = rb._stage["out_host"].numpy()
        return rb

    def _h2d(self, key: str, arr: np.ndarray, dst, wait: bool, wait_for=None) -> Event:
        import torch
        prev = self._stage.get(key + "_ev")
        if prev is not None:
            prev.wait()                       # the pinned staging buffer is free again
        stage = self._stage[key]
        stage.numpy()[...] = arr
        self.queue.wait_for(wait_for)
        with torch.cuda.stream(self.queue.stream):
            dst.copy_(stage, non_blocking=True)
            ev = Event(self.queue.stream)
        self._stage[key + "_ev"] = ev
        self.ev_last = ev
        if wait:
            ev.wait()
        return ev

    def upload_rays(self, rays: np.ndarray, wait: bool = False, wait_for=None) -> Event:
        rays = np.asarray(rays)
        if rays.shape != (self.num_rays,):
            raise ValueError(f"rays must be shape ({self.num_rays},), got {rays.shape}")
        if rays.dtype.itemsize != 32:
            raise ValueError(f"rays dtype must be 32B, got {rays.dtype} (itemsize {rays.dtype.itemsize})")
        flat = np.ascontiguousarray(rays).view(np.float32).reshape(self.num_rays, 8)
        return self._h2d("rays", flat, self.rays_buf, wait, wait_for)

    def upload_targets(self, targets: np.ndarray, wait: bool = False, wait_for=None) -> Event:
        targets = np.asarray(targets, dtype=np.float32)
        if targets.shape != (self.num_rays, 4):
            raise ValueError(f"targets must be shape ({self.num_rays},4), got {targets.shape}")
        return self._h2d("targets", targets, self.targets_buf, wait, wait_for)

    def download_out(self, out: Optional[np.ndarray] = None, wait: bool = True,
                     wait_for: List[Event | None] = None) -> tuple[np.ndarray, Event]:
        import torch
        if out is None:
            out = self.out_host
        if out is None:
            out = np.empty((self.num_rays, 4), dtype=np.float32)
        else:
            out = np.asarray(out, dtype=np.float32)
            if out.shape != (self.num_rays, 4):
                raise ValueError(f"out must be shape ({self.num_rays},4), got {out.shape}")
        self.queue.wait_for(wait_for)
        # As with the reference's non-blocking read, `out` holds the colours once the returned event has
        # completed (on return with wait=True).  A pinned `out` (out_host is) receives one asynchronous
        # copy; a pageable one is staged through a pinned slot and filled when the event is waited on
        # or the queue finishes.
        dst = torch.from_numpy(out)
        if dst.is_pinned():
            with torch.cuda.stream(self.queue.stream):
                dst.copy_(self.out_buf, non_blocking=True)
                ev = Event(self.queue.stream)
        else:
            i = self._stage["out_i"]
            self._stage["out_i"] = i ^ 1
            prev = self._stage["out_ev"][i]
            if prev is not None:
                prev.wait()           # that slot's previous download has been delivered
            stage = self._stage["out"][i]
            with torch.cuda.stream(self.queue.stream):
                stage.copy_(self.out_buf, non_blocking=True)
                ev = Event(self.queue.stream)

            def deliver(out=out, stage=stage):
                out[...] = stage.numpy()
            ev._on_complete = deliver
            self._stage["out_ev"][i] = ev
            self.queue._pending.append(ev)
        if wait:
            ev.wait()
        return out, ev

    def ensure_dummy_targets(self) -> np.ndarray:
        if self.targets_host is None:
            self.targets_host = np.zeros((self.num_rays, 4), dtype=np.float32)
        else:
            self.targets_host.fill(0.0)
        return self.targets_host


@dataclass
class OccParams:
    """Occupancy-guided sampling parameters (ffnerf_tools.py:398-424)."""
    G_occ: int = 32
    box_min: np.ndarray = None
    box_max: np.ndarray = None
    rho_min: np.float32 = np.float32(RHO_MIN_DEF)
    rho_max: np.float32 = np.float32(RHO_MAX_DEF)
    dt_min: np.float32 = np.float32(4e-3)
    dt_max: np.float32 = np.float32(0.8)
    t_near_clip: np.float32 = np.float32(0.3)
    t_far_clip: np.float32 = np.float32(1e9)
    occ_update_strength0: np.float32 = np.float32(OCC_U_STR)

    def finalize(self):
        if self.box_min is None:
            self.box_min = np.array([-3.0, -3.0, -3.0], dtype=np.float32)
        if self.box_max is None:
            self.box_max = np.array([+3.0, +3.0, +3.0], dtype=np.float32)
        self.box_min = np.asarray(self.box_min, dtype=np.float32).reshape(3)
        self.box_max = np.asarray(self.box_max, dtype=np.float32).reshape(3)
        self.t_near_clip = np.float32(self.t_near_clip)
        self.t_far_clip = np.float32(self.t_far_clip)
        if not np.isfinite(self.t_near_clip) or self.t_near_clip < 0:
            raise ValueError("t_near_clip must be finite and nonnegative")
        if not np.isfinite(self.t_far_clip) or self.t_far_clip <= self.t_near_clip:
            raise ValueError("t_far_clip must be finite and greater than t_near_clip")
        return self


def _level_log2_for(table_size_entries: int, level_log2=None) -> list[int]:
    if level_log2 is not None:
        return [int(x) for x in level_log2]
    if table_size_entries == TABLE_SIZE_ENTRIES:
        return list(fc.REFERENCE_LEVEL_LOG2)
    per = table_size_entries // fc.N_LEVELS
    if per * fc.N_LEVELS != table_size_entries or per & (per - 1):
        raise ValueError("table_size_entries must be 2,260,992 (the reference's per-level table) or "
                         "16 * 2^k (uniform levels); pass level_log2 for other layouts")
    return [per.bit_length() - 1] * fc.N_LEVELS


class DataParallel:
    """Per-step gradient and occupancy exchange between data-parallel ranks (one process per
    GPU, torch.distributed over NCCL).  Every rank takes a contiguous slice of the ray batch; the
    RNG streams are keyed by the global ray index, so the union of the shards is the batch.

    With ``fused`` (the default when every rank's GPU can map every other's memory), the gradient
    all-reduce and the table SGD step run as one kernel over NVLink peer memory
    (``ffn_dp_reduce_apply``); otherwise the gradient buffer is all-reduced with NCCL and every
    rank applies the update.  The occupancy proposals are merged with an NCCL MAX all-reduce."""

    def __init__(self, group=None, fused: bool | None = None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.want_fused = fused
        self.fused = False
        self.nvls = False
        self._ctx = None

    def ensure_attached(self, nerf: "Nerf"):
        """(Re-)maps the peers after the device context was (re)created; collective."""
        if self._ctx is not nerf.native:
            self.fused = False
            self.nvls = False
            self.attach(nerf)
            self._ctx = nerf.native

    def attach(self, nerf: "Nerf"):
        """Sets up the fused exchange when it can run: SGD table, 2..8 ranks, every GPU pair
        peer-accessible, the same decision on every rank.  When the NVSwitch offers multicast
        (NVLS), the table and the gradient buffer move into symmetric multicast memory and the
        exchange reduces and broadcasts through the switch; otherwise it uses peer loads/stores."""
        import torch
        want = self.want_fused
        if want is None:
            want = os.environ.get("FFNERF_DP_FUSED", "1") != "0"
        ok = bool(want) and nerf.table_optimizer == "sgd" and 2 <= self.world <= 8
        dev = int(nerf.native.device)
        info = [None] * self.world
        self.dist.all_gather_object(info, (dev, ok), group=self.group)
        ok = all(i[1] for i in info) and all(d == dev or torch.cuda.can_device_access_peer(dev, d) for d, _ in info)
        if not self._agree(ok, dev):
            return
        # NVLS moves less data per GPU than peer loads/stores from 4 ranks up (measured on 8 B200:
        # 0.24 vs 0.30 ms per exchange of a 67 MB buffer; on 2: 0.23 vs 0.15 ms)
        mode = os.environ.get("FFNERF_DP_NVLS", "auto")
        use_nvls = mode == "1" or (mode == "auto" and self.world >= 4)
        self.nvls = use_nvls and self._bind_multicast(nerf, dev)
        handles = [None] * self.world
        self.dist.all_gather_object(handles, nerf.native.dp_ipc_handles(), group=self.group)
        nerf.native.dp_attach(self.rank, self.world, handles)
        if self.nvls:
            nerf.native.dp_attach_multicast(*self._mc)
        self.fused = True

    def _agree(self, ok: bool, dev: int) -> bool:
        import torch
        flag = torch.tensor([1 if ok else 0], device=f"cuda:{dev}")
        self.dist.all_reduce(flag, op=self.dist.ReduceOp.MIN, group=self.group)
        return int(flag.item()) == 1

    def _bind_multicast(self, nerf: "Nerf", dev: int) -> bool:
        """Allocates the gradient buffer and the table in symmetric memory with a multicast
        address on every rank (collective); binds them into the context if every rank got one."""
        import torch
        bufs = []
        try:
            import torch.distributed._symmetric_memory as symm_mem
            grp = self.group if self.group is not None else self.dist.group.WORLD
            for bid in (ffn_native.BUF_GRADS, ffn_native.BUF_TABLE):
                t = symm_mem.empty(nerf.native.tensor(bid).numel(), dtype=torch.float32, device=f"cuda:{dev}")
                bufs.append((t, symm_mem.rendezvous(t, grp.group_name)))
            good = all(int(getattr(h, "multicast_ptr", 0) or 0) != 0 for _, h in bufs)
        except Exception:
            good = False
        if not self._agree(good, dev):
            return False
        nerf.native.bind_external(ffn_native.BUF_GRADS, bufs[0][0])
        nerf.native.bind_external(ffn_native.BUF_TABLE, bufs[1][0])
        self._symm = bufs
        self._mc = (int(bufs[0][1].multicast_ptr), int(bufs[1][1].multicast_ptr))
        return True

    def allreduce_grads(self, nerf: "Nerf"):
        self.dist.all_reduce(nerf.native.tensor(ffn_native.BUF_GRADS), op=self.dist.ReduceOp.SUM, group=self.group)

    def merge_occupancy(self, nerf: "Nerf"):
        import torch
        G = int(nerf.occ.G_occ)
        if nerf._occ_bytes is None:
            nerf._occ_bytes = torch.empty(G ** 3 * 8, dtype=torch.uint8, device=f"cuda:{nerf.native.device}")
        nerf.native.occ_st_bytes(nerf._occ_bytes, True)
        self.dist.all_reduce(nerf._occ_bytes, op=self.dist.ReduceOp.MAX, group=self.group)
        nerf.native.occ_st_bytes(nerf._occ_bytes, False)


class Nerf:
    """Fully fused NeRF host-side model container (ffnerf_tools.py:429-1575): numpy state (int32
    bit patterns) for save/load, device state in a libffnerf context, ``step`` runs the step."""

    ADAM_BETA1 = np.float32(0.9)
    ADAM_BETA2 = np.float32(0.999)
    ADAM_EPS = np.float32(1e-6)

    def __init__(self, ctx: Context, queue: CommandQueue, ffnerf_prg=None, ffnerf_suppress_mode_prg=None,
                 decay_prg=None, wu_prg=None, ffnerf_kernel_name: str = KERNEL_NAME,
                 decay_kernel_name: str = "occ_nibble_decay_write_both_q24",
                 wu_kernel_name: str = "update_ffnerf_oneWG", training_dir: str | Path = "training",
                 model_id: str = "ffnerf", layers: dict | None = None, edges: dict | None = None,
                 transfer_fmt: str = "fp16", table_size_entries: int = TABLE_SIZE_ENTRIES,
                 f_per_level: int = F_PER_LEVEL, occ: OccParams | None = None, load_id: str | None = None,
                 rng_seed: int = 777, *, background: str = "black", finest_resolution: float | None = None,
                 level_log2=None, nd: int | None = None, nc: int | None = None, table_optimizer: str = "sgd",
                 mlp_precision: str = "fp32", table_update: str = "immediate", verbose: bool = True):
        self.do_train = True
        self.verbose = verbose
        self.ctx = ctx
        self.queue = queue
        self.library = ffnerf_prg or ffn_native.load_library()
        self.kernel_names = (ffnerf_kernel_name, decay_kernel_name, wu_kernel_name)
        self.training_dir = Path(training_dir)
        self.training_dir.mkdir(parents=True, exist_ok=True)
        self.model_id = model_id
        self.layers = dict(layers or {})
        self.edges = dict(edges or {})
        self.background = background
        self.finest_resolution = float(finest_resolution if finest_resolution is not None else fc.RESOLUTION_LVLMAX)
        self.table_optimizer = table_optimizer
        # "immediate": the SGD step lands in the table inside the fused kernel while other rays read
        # it (the reference's Hogwild update, ffnerf_OG.cl:2155-2168); "deferred": gradients are
        # summed into a buffer and applied after the kernel.  Adam tables and data-parallel runs
        # (whose gradients are all-reduced first) always use "deferred".
        if table_update not in ("immediate", "deferred"):
            raise ValueError("table_update must be 'immediate' or 'deferred'")
        self.table_update = table_update
        if mlp_precision not in ffn_native.MLP_PRECISIONS:
            raise ValueError("mlp_precision must be 'fp32' (CUDA cores) or 'fp16' (tensor cores)")
        self.mlp_precision = mlp_precision
        self.M, self.L_DIR, self.C_OUT, self.D_D_OUT = M, L_DIR, C_OUT, D_OUT
        self.C_IN = D_OUT + L_DIR
        self.NDMAX, self.NCMAX = NDMAX, NCMAX
        self.ND = int(nd if nd is not None else ND)
        self.NC = int(nc if nc is not None else NC)
        self._set_transfer(transfer_fmt)
        if not load_id:
            self._check_transfer()
        self.table_size_entries = int(table_size_entries)
        self.f_per_level = int(f_per_level)
        self.level_log2 = _level_log2_for(self.table_size_entries, level_log2)
        self.table_elems = self.table_size_entries * self.f_per_level
        self.L_POS = fc.N_LEVELS * self.f_per_level
        self._set_arch_from_layer_counts(self.ND, self.NC)
        self.occ = (occ or OccParams()).finalize()
        self.rng = np.random.default_rng(int(rng_seed))
        self.steps_trained = 0
        self.state_i32: dict[str, np.ndarray] = {}
        self.meta: dict = {}
        self._shapes = {}
        self.native: ffn_native.Context | None = None
        self.dp: DataParallel | None = None
        self.ex_events: list = []      # (start, end) CUDA events of the fused exchange, when fb_events is on
        self.ray_offset = 0
        self._occ_bytes = None
        self.fb_events = None      # list -> (start, end) CUDA events around every forward/backward launch
        self.buf, self.io, self.tmp = {}, {}, {}
        if load_id:
            self.load_latest(load_id)
        else:
            self._init_fresh()

    # ---------------------------------------------------------------- construction
    @classmethod
    def from_kernels(cls, ctx, queue, kernel_file=None, decay_file=None, weight_update_file=None,
                     background: str = "black", layers=None, edges=None, training_dir="training",
                     model_id: str = "ffnerf", load_id: str | None = None, transfer_fmt: str = "fp32",
                     ffnerf_kernel_name: str = KERNEL_NAME,
                     decay_kernel_name: str = "occ_nibble_decay_write_both_q24",
                     wu_kernel_name: str = "update_ffnerf_oneWG", build_options_extra: list[str] | None = None,
                     rng_seed: int = 777, occ: OccParams | None = None,
                     table_size_entries: int = TABLE_SIZE_ENTRIES, f_per_level: int = F_PER_LEVEL, **kw):
        """Loads the CUDA library (the reference builds four OpenCL programs here,
        ffnerf_tools.py:583-671).  ``kernel_file`` may name another build of libffnerf.so;
        reference ``.cl`` paths are accepted and ignored.  ``-DND=`` / ``-DNC=`` in
        ``build_options_extra`` select the layer counts as the reference's options do."""
        lib_path = None
        if kernel_file is not None and str(kernel_file).endswith(".so"):
            lib_path = Path(kernel_file)
        lib = ffn_native.load_library(lib_path) if lib_path else ffn_native.load_library()
        for opt in build_options_extra or []:
            if opt.startswith("-DND="):
                kw.setdefault("nd", int(opt[5:]))
            elif opt.startswith("-DNC="):
                kw.setdefault("nc", int(opt[5:]))
        return cls(ctx, queue, lib, lib, lib, lib, ffnerf_kernel_name, decay_kernel_name, wu_kernel_name,
                   training_dir, model_id, layers, edges, transfer_fmt, table_size_entries, f_per_level, occ,
                   load_id, rng_seed, background=background, **kw)

    def _check_transfer(self):
        """The fp16 / fp8 transfer formats quantise the weight-update operands the reference's way
        (ffnerf_OG.cl:85-156) in the fp32 MLP; the tensor-core MLP has its own operand formats."""
        if self.mlp_precision == "fp16" and self.transfer_fmt != "fp32":
            raise ValueError(f"transfer_fmt={self.transfer_fmt!r} needs mlp_precision='fp32' (the tensor-core MLP "
                             "runs with transfer_fmt='fp32' only)")

    def _set_transfer(self, transfer_fmt: str):
        if transfer_fmt not in ("fp32", "fp16", "fp8"):
            raise ValueError("transfer_fmt must be 'fp32', 'fp16', or 'fp8'")
        self.transfer_fmt = transfer_fmt
        self.transfer_nbytes = {"fp32": 4, "fp16": 2, "fp8": 1}[transfer_fmt]
        self.transfer_define = {"fp32": 32, "fp16": 16, "fp8": 8}[transfer_fmt]

    def _set_arch_from_layer_counts(self, ND: int, NC: int):
        """Parameter names, active subsets and placeholder shapes (ffnerf_tools.py:673-802)."""
        ND, NC = int(ND), int(NC)
        if not 1 <= ND <= self.NDMAX:
            raise ValueError(f"ND must be in [1, {self.NDMAX}], got {ND}")
        if not 1 <= NC <= self.NCMAX:
            raise ValueError(f"NC must be in [1, {self.NCMAX}], got {NC}")
        self.ND, self.NC = ND, NC
        self.density_w_all = ["Wd_in", "Wd_01", "Wd_12", "Wd_out"]
        self.density_b_all = ["bd_0", "bd_1", "bd_2", "bd_out"]
        self.color_w_all = ["Wc_in", "Wc_01", "Wc_12", "Wc_23", "Wc_out"]
        self.color_b_all = ["bc_0", "bc_1", "bc_2", "bc_3", "bc_out"]
        self.weight_names = self.density_w_all + self.color_w_all
        self.bias_names = self.density_b_all + self.color_b_all
        aw, ab = ["Wd_in", "Wd_out"], ["bd_0", "bd_out"]
        if ND >= 2: aw.append("Wd_01"); ab.append("bd_1")
        if ND >= 3: aw.append("Wd_12"); ab.append("bd_2")
        cw, cb = ["Wc_in", "Wc_out"], ["bc_0", "bc_out"]
        for k, (w, b) in enumerate((("Wc_01", "bc_1"), ("Wc_12", "bc_2"), ("Wc_23", "bc_3")), start=2):
            if NC >= k:
                cw.append(w); cb.append(b)
        self.active_weight_names = set(aw + cw)
        self.active_bias_names = set(ab + cb)
        L_POS_ = fc.N_LEVELS * self.f_per_level if hasattr(self, "f_per_level") else L_POS
        self.weights_spec = {"Wd_in": (M, L_POS_), "Wd_01": (M, M), "Wd_12": (M, M), "Wd_out": (D_OUT, M),
                             "Wc_in": (M, C_IN), "Wc_01": (M, M), "Wc_12": (M, M), "Wc_23": (M, M),
                             "Wc_out": (C_OUT, M)}
        self.bias_spec = {"bd_0": (M,), "bd_1": (M,), "bd_2": (M,), "bd_out": (D_OUT,), "bc_0": (M,),
                          "bc_1": (M,), "bc_2": (M,), "bc_3": (M,), "bc_out": (C_OUT,)}
        for wn in self.weights_spec:
            if wn not in self.active_weight_names:
                self.weights_spec[wn] = (1, 1)
        for bn in self.bias_spec:
            if bn not in self.active_bias_names:
                self.bias_spec[bn] = (1,)
        self.deltas_spec = {**{f"gl_dd{i}": (M if i <= ND else None) for i in range(1, NDMAX + 1)},
                            "gl_dd_out": D_OUT,
                            **{f"gl_dc{i}": (M if i <= NC else None) for i in range(1, NCMAX + 1)},
                            "gl_dc_out": C_OUT}
        self.activations_spec = {"gl_apos": L_POS_, **{f"gl_ad{i}": (M if i <= ND else None) for i in range(1, NDMAX + 1)},
                                 "gl_ac_in": C_IN, **{f"gl_ac{i}": (M if i <= NC else None) for i in range(1, NCMAX + 1)}}

    def _infer_shapes(self):
        self._shapes.clear()
        for wn, sh in self.weights_spec.items():
            self._shapes[wn] = (int(sh[0]), int(sh[1]))
        for bn, sh in self.bias_spec.items():
            self._shapes[bn] = (int(sh[0]),)
        for n in self.weight_names + self.bias_names:
            self._shapes["m" + n] = self._shapes[n]
            self._shapes["v" + n] = self._shapes[n]
        self._shapes["table"] = (int(self.table_elems),)
        self._shapes["occ_grid_u32"] = (int(self.occ.G_occ) ** 3,)

    def _init_fresh(self):
        """Fresh parameters with the reference's draws, in the reference's order
        (ffnerf_tools.py:836-898): table U(-1e-4, 1e-4); weights N(0, 0.01) for heads with <= 16
        outputs, else He N(0, sqrt(2/fan_in)); biases 0, bd_out[0] = SIGMA_BIAS,
        bc_2 ~ N(-2, 0.05) when active; Adam state 0; occupancy 0xEEEEEEEE."""
        self._infer_shapes()
        self.steps_trained = 0
        table_f = self.rng.uniform(-1e-4, 1e-4, size=self._shapes["table"]).astype(np.float32)
        self.state_i32["table"] = f32_to_i32_bits(table_f).reshape(-1)
        for wn in self.weight_names:
            sh = self._shapes[wn]
            if wn in self.active_weight_names:
                if sh[0] <= 16:
                    w = self.rng.normal(0.0, 0.01, size=sh).astype(np.float32)
                else:
                    w = self.rng.normal(0.0, np.sqrt(2.0 / int(sh[1])), size=sh).astype(np.float32)
            else:
                w = np.zeros(sh, dtype=np.float32)
            self.state_i32[wn] = f32_to_i32_bits(w).reshape(-1)
        for bn in self.bias_names:
            sh = self._shapes[bn]
            b = np.zeros(sh, dtype=np.float32)
            if bn in self.active_bias_names:
                if bn == "bd_out" and b.size > 0:
                    b[0] = SIGMA_BIAS
                if bn == "bc_2":
                    b = self.rng.normal(-2.0, 0.05, size=sh).astype(np.float32)
            self.state_i32[bn] = f32_to_i32_bits(b).reshape(-1)
        for n in self.weight_names + self.bias_names:
            self.state_i32["m" + n] = np.zeros(int(np.prod(self._shapes[n])), dtype=np.int32)
            self.state_i32["v" + n] = np.zeros(int(np.prod(self._shapes[n])), dtype=np.int32)
        occ0 = np.full(self._shapes["occ_grid_u32"], OCC_INIT_DENSITY, dtype=np.uint32).view(np.int32)
        self.state_i32["occ_grid_in_u32"] = occ0.copy()
        self.state_i32["occ_grid_st_u32"] = occ0.copy()
        self.meta = self._build_meta()

    def _build_meta(self) -> dict:
        return dict(timestamp=datetime.now().strftime("%Y%m%d-%H%M%S"), model_id=self.model_id,
                    steps_trained=int(self.steps_trained), transfer_fmt=self.transfer_fmt,
                    table_size_entries=int(self.table_size_entries), f_per_level=int(self.f_per_level),
                    layers=self.layers, G_occ=np.int32(self.occ.G_occ),
                    box_min=np.asarray(self.occ.box_min, np.float32), box_max=np.asarray(self.occ.box_max, np.float32),
                    rho_min=np.float32(self.occ.rho_min), rho_max=np.float32(self.occ.rho_max),
                    dt_min=np.float32(self.occ.dt_min), dt_max=np.float32(self.occ.dt_max),
                    t_near_clip=np.float32(self.occ.t_near_clip), t_far_clip=np.float32(self.occ.t_far_clip),
                    ND=np.int32(self.ND), NC=np.int32(self.NC))

    # ---------------------------------------------------------------- device state
    def geometry(self, samples_per_ray: int = 64) -> dict:
        o = self.occ
        return fc.make_geometry(F=self.f_per_level, ND=self.ND, NC=self.NC, spr=int(samples_per_ray),
                                G=int(o.G_occ), log2_entries=self.level_log2, rmax=self.finest_resolution,
                                box_min=o.box_min, box_max=o.box_max, rho_min=o.rho_min, rho_max=o.rho_max,
                                dt_min=o.dt_min, dt_max=o.dt_max, t_near=o.t_near_clip, t_far=o.t_far_clip,
                                background=self.background)

    def _blob_from_state(self, prefix: str = "") -> np.ndarray:
        lay, total = fc.param_layout(self.f_per_level, self.ND, self.NC)
        blob = np.zeros(total, np.float32)
        for n, (off, sz) in lay.items():
            if sz:
                blob[off:off + sz] = self.state_i32[prefix + n].view(np.float32).reshape(-1)[:sz]
        return blob

    def _state_from_blob(self, blob: np.ndarray, prefix: str = ""):
        lay, _ = fc.param_layout(self.f_per_level, self.ND, self.NC)
        for n, (off, sz) in lay.items():
            if sz:
                self.state_i32[prefix + n] = blob[off:off + sz].copy().view(np.int32)

    def setup_buffers(self, num_rays: int, samples_per_ray: int, do_train=None):
        """Creates the device context on first use and uploads the host state
        (ffnerf_tools.py:926-977).  Later calls keep the device state; there is no per-batch
        scratch to resize (activations stay on chip)."""
        if do_train is not None:
            self.do_train = do_train
        if not 1 <= int(samples_per_ray) <= S_MAX:
            raise ValueError(f"samples_per_ray={samples_per_ray} must be <= S_MAX={S_MAX}")
        self.num_rays = int(num_rays)
        self.samples_per_ray = int(samples_per_ray)
        self.batch_rays = self.num_rays
        self.B = self.num_rays * self.samples_per_ray if self.do_train else None
        if self.native is None:
            self._check_transfer()
            opt = {"sgd": 0, "adam": 1}[self.table_optimizer]
            self.native = ffn_native.Context(self.geometry(self.samples_per_ray), device=self.ctx.device.index,
                                             table_optimizer=opt, adam_beta1=float(self.ADAM_BETA1),
                                             adam_beta2=float(self.ADAM_BETA2), adam_eps=float(self.ADAM_EPS),
                                             mlp_precision=self.mlp_precision, transfer_fmt=self.transfer_fmt)
            self._push_params_to_device()
        self.buf = {"native": self.native}

    def _push_params_to_device(self):
        import torch
        nat = self.native
        dev = f"cuda:{nat.device}"
        with torch.cuda.stream(self.queue.stream):
            nat.tensor(ffn_native.BUF_TABLE).copy_(torch.from_numpy(self.state_i32["table"].view(np.float32)).to(dev))
            nat.tensor(ffn_native.BUF_PARAMS).copy_(torch.from_numpy(self._blob_from_state()).to(dev))
            nat.tensor(ffn_native.BUF_ADAM_M).copy_(torch.from_numpy(self._blob_from_state("m")).to(dev))
            nat.tensor(ffn_native.BUF_ADAM_V).copy_(torch.from_numpy(self._blob_from_state("v")).to(dev))
            nat.tensor(ffn_native.BUF_OCC_IN).copy_(torch.from_numpy(self.state_i32["occ_grid_in_u32"].view(np.int32)).to(dev))
            nat.tensor(ffn_native.BUF_OCC_ST).copy_(torch.from_numpy(self.state_i32["occ_grid_st_u32"].view(np.int32)).to(dev))
        self.queue.finish()

    def sync_params_from_device(self):
        """Pulls table, parameters, Adam state and occupancy grids into state_i32."""
        if self.native is None:
            raise RuntimeError("Buffers not set up. Call setup_buffers(batch_rays, samples_per_ray) first.")
        nat = self.native
        self.queue.finish()
        self.state_i32["table"] = nat.tensor(ffn_native.BUF_TABLE).cpu().numpy().view(np.int32).copy()
        self._state_from_blob(nat.tensor(ffn_native.BUF_PARAMS).cpu().numpy())
        self._state_from_blob(nat.tensor(ffn_native.BUF_ADAM_M).cpu().numpy(), "m")
        self._state_from_blob(nat.tensor(ffn_native.BUF_ADAM_V).cpu().numpy(), "v")
        self.state_i32["occ_grid_in_u32"] = nat.tensor(ffn_native.BUF_OCC_IN).cpu().numpy().copy()
        self.state_i32["occ_grid_st_u32"] = nat.tensor(ffn_native.BUF_OCC_ST).cpu().numpy().copy()

    # ---------------------------------------------------------------- save / load
    def _model_paths(self, save_id: str):
        td = self.training_dir
        td.mkdir(parents=True, exist_ok=True)
        return td / f"{save_id}_weights_latest.npz", sorted(td.glob(f"{save_id}_weights_*.npz"))

    def save(self, min_new_file_seconds: int = 300, async_write: bool = False):
        """Device -> host, then the reference's NPZ layout (ffnerf_tools.py:989-1086): a new
        timestamped file (also copied to ``_latest``) or, within min_new_file_seconds of the last
        one, an overwrite of ``_latest``.  Under data parallelism only rank 0 writes.

        ``async_write``: the device state is copied inside the queue's stream order into a device
        snapshot (a few hundred microseconds for a 67 MB table), read back on a side stream into
        pinned memory and written by a background thread, so training continues meanwhile; returns
        the path the thread will write (``wait_saved()`` joins it)."""
        self.steps_trained = int(self.steps_trained)
        self.meta = self._build_meta()
        if self.dp is not None and self.dp.rank != 0:
            if self.native is not None and not async_write:
                self.sync_params_from_device()
            return None
        latest, _ = self._model_paths(self.model_id)
        make_new = True
        if latest.exists():
            try:
                make_new = (time.time() - latest.stat().st_mtime) >= float(min_new_file_seconds)
            except OSError:
                make_new = True
        ts = datetime.now().strftime("%Y%m%d-%H%M%S")
        fname = (self.training_dir / f"{self.model_id}_weights_{ts}.npz") if make_new else latest
        targets = [fname] + ([latest] if make_new else [])
        if async_write and self.native is not None:
            self.wait_saved()
            grab = self._snapshot_device_async()
            steps = self.steps_trained

            def work():
                grab()
                payload = self._payload(ts, steps)
                for t in targets:
                    _write_npz(t, payload)
            import threading
            self._save_thread = threading.Thread(target=work, name="ffn-save", daemon=False)
            self._save_thread.start()
            return fname
        if self.native is not None:
            self.sync_params_from_device()
        payload = self._payload(ts, self.steps_trained)
        for t in targets:
            _write_npz(t, payload)
        return fname

    def wait_saved(self):
        """Waits for an asynchronous save to finish writing."""
        t = getattr(self, "_save_thread", None)
        if t is not None:
            t.join()
            self._save_thread = None

    def _snapshot_device_async(self):
        """Copies the device state to a device snapshot in stream order and starts its read-back
        into pinned host memory on a side stream; returns a callable that waits for the read-back
        and moves it into state_i32."""
        import torch
        nat = self.native
        ids = (ffn_native.BUF_TABLE, ffn_native.BUF_PARAMS, ffn_native.BUF_ADAM_M, ffn_native.BUF_ADAM_V,
               ffn_native.BUF_OCC_IN, ffn_native.BUF_OCC_ST)
        if getattr(self, "_snap_dev", None) is None:
            self._snap_dev = {i: torch.empty_like(nat.tensor(i)) for i in ids}
            self._snap_host = {i: torch.empty(nat.tensor(i).shape, dtype=nat.tensor(i).dtype).pin_memory() for i in ids}
            self._snap_stream = torch.cuda.Stream(device=f"cuda:{nat.device}")
        with torch.cuda.stream(self.queue.stream):
            for i in ids:
                self._snap_dev[i].copy_(nat.tensor(i), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.queue.stream)
        self._snap_stream.wait_event(ev)
        with torch.cuda.stream(self._snap_stream):
            for i in ids:
                self._snap_host[i].copy_(self._snap_dev[i], non_blocking=True)
            done = torch.cuda.Event()
            done.record(self._snap_stream)

        def grab():
            done.synchronize()
            h = {i: self._snap_host[i].numpy() for i in ids}
            self.state_i32["table"] = h[ffn_native.BUF_TABLE].view(np.int32).copy()
            self._state_from_blob(h[ffn_native.BUF_PARAMS])
            self._state_from_blob(h[ffn_native.BUF_ADAM_M], "m")
            self._state_from_blob(h[ffn_native.BUF_ADAM_V], "v")
            self.state_i32["occ_grid_in_u32"] = h[ffn_native.BUF_OCC_IN].copy()
            self.state_i32["occ_grid_st_u32"] = h[ffn_native.BUF_OCC_ST].copy()
        return grab

    def _payload(self, ts: str, steps_trained: int) -> dict:
        payload = dict(
            timestamp=ts, model_id=self.model_id, steps_trained=np.int32(steps_trained),
            transfer_fmt=np.array(self.transfer_fmt), ND=np.int32(self.ND), NC=np.int32(self.NC),
            table_i=np.asarray(self.state_i32["table"], dtype=np.int32),
            table_size_entries=np.int32(self.table_size_entries), table_f_per_level=np.int32(self.f_per_level),
            occ_grid_in_u32=np.asarray(self.state_i32["occ_grid_in_u32"]).view(np.uint32),
            occ_grid_st_u32=np.asarray(self.state_i32["occ_grid_st_u32"]).view(np.uint32),
            G_occ=np.int32(self.occ.G_occ), box_min=np.asarray(self.occ.box_min, np.float32),
            box_max=np.asarray(self.occ.box_max, np.float32), rho_min=np.float32(self.occ.rho_min),
            rho_max=np.float32(self.occ.rho_max), dt_min=np.float32(self.occ.dt_min),
            dt_max=np.float32(self.occ.dt_max), t_near_clip=np.float32(self.occ.t_near_clip),
            t_far_clip=np.float32(self.occ.t_far_clip),
            # keys of this implementation (ignored by the reference loader)
            ffn_level_log2=np.asarray(self.level_log2, np.int32), ffn_finest_resolution=np.float32(self.finest_resolution),
        )
        active = sorted(list(self.active_weight_names | self.active_bias_names))
        payload["active_params"] = np.array(active, dtype="U32")
        for name in active:
            payload[name + "_i"] = np.asarray(self.state_i32[name], dtype=np.int32)
            payload["m" + name + "_i"] = np.asarray(self.state_i32["m" + name], dtype=np.int32)
            payload["v" + name + "_i"] = np.asarray(self.state_i32["v" + name], dtype=np.int32)
        return payload

    def load_latest(self, load_id: str):
        """Loads the most recently modified checkpoint of ``load_id`` (ffnerf_tools.py:1088-1172)."""
        td = self.training_dir
        pats = sorted(td.glob(f"{load_id}_weights_*.npz"))
        path = max(pats, key=lambda p: p.stat().st_mtime_ns) if pats else None
        if path is None:
            raise FileNotFoundError(f"No saved model found for id='{load_id}' in {td.resolve()}")
        data = np.load(path, allow_pickle=False)
        self.f_per_level = int(data["table_f_per_level"])
        self._set_arch_from_layer_counts(int(data["ND"]), int(data["NC"]))
        self._set_transfer(str(data["transfer_fmt"].item()))
        self.table_size_entries = int(data["table_size_entries"])
        self.table_elems = self.table_size_entries * self.f_per_level
        self.L_POS = fc.N_LEVELS * self.f_per_level
        self.level_log2 = _level_log2_for(self.table_size_entries,
                                          data["ffn_level_log2"].tolist() if "ffn_level_log2" in data else None)
        if "ffn_finest_resolution" in data:
            self.finest_resolution = float(data["ffn_finest_resolution"])
        self.occ = OccParams(G_occ=int(data["G_occ"]), box_min=np.asarray(data["box_min"], np.float32),
                             box_max=np.asarray(data["box_max"], np.float32), rho_min=np.float32(data["rho_min"]),
                             rho_max=np.float32(data["rho_max"]), dt_min=np.float32(data["dt_min"]),
                             dt_max=np.float32(data["dt_max"]), t_near_clip=np.float32(data["t_near_clip"]),
                             t_far_clip=np.float32(data["t_far_clip"])).finalize()
        self._infer_shapes()
        self.steps_trained = int(data["steps_trained"]) if "steps_trained" in data else 0
        self.state_i32["table"] = np.asarray(data["table_i"], dtype=np.int32).reshape(-1)
        for n in self.weight_names + self.bias_names:
            k = int(np.prod(self._shapes[n]))
            self.state_i32[n] = np.zeros(k, np.int32)
            self.state_i32["m" + n] = np.zeros(k, np.int32)
            self.state_i32["v" + n] = np.zeros(k, np.int32)
        for name in [str(x) for x in data["active_params"].tolist()]:
            self.state_i32[name] = np.asarray(data[name + "_i"], dtype=np.int32).reshape(-1)
            self.state_i32["m" + name] = np.asarray(data["m" + name + "_i"], dtype=np.int32).reshape(-1)
            self.state_i32["v" + name] = np.asarray(data["v" + name + "_i"], dtype=np.int32).reshape(-1)
        self.state_i32["occ_grid_in_u32"] = np.asarray(data["occ_grid_in_u32"], np.uint32).reshape(-1).view(np.int32)
        self.state_i32["occ_grid_st_u32"] = np.asarray(data["occ_grid_st_u32"], np.uint32).reshape(-1).view(np.int32)
        self.meta = self._build_meta()
        if self.native is not None:
            self.native.close()
            self.native = None
            self.setup_buffers(self.num_rays, self.samples_per_ray)

    # ---------------------------------------------------------------- stepping
    def _get_rng_u32(self) -> np.uint32:
        return np.uint32(self.rng.integers(0, 2**32, dtype=np.uint32))

    @property
    def table_immediate(self) -> bool:
        return self.table_update == "immediate" and self.table_optimizer == "sgd" and self.dp is None

    def enable_data_parallel(self, group=None, ray_offset: int | None = None, fused: bool | None = None):
        """Shards batches across the ranks of ``group``: this rank's rays start at global index
        ``ray_offset`` (default rank * num_rays of the current batch)."""
        self.dp = DataParallel(group, fused=fused)
        self.ray_offset = ray_offset

    @staticmethod
    def maintenance_due(steps_trained: int, occ_update_strength: float) -> bool:
        """Occupancy maintenance runs every OCC_MAINTENANCE_PERIOD training steps once occupancy
        updates are live (ffnerf_tools.py:1424-1428)."""
        return float(occ_update_strength) > 0.0 and int(steps_trained) % OCC_MAINTENANCE_PERIOD == 0

    @staticmethod
    def decay_q24(occ_update_strength: float) -> int:
        """round((1 - s*(1 - DECAY)) * 2^24) clamped to [0, 2^24] (ffnerf_tools.py:1453-1457)."""
        d = 1 - occ_update_strength * (1 - DECAY)
        return max(0, min(int(round(d * (1 << 24))), 1 << 24))

    def lr_t(self, lr_f: float) -> np.float32:
        """Adam bias correction with t = steps_trained (ffnerf_tools.py:1479-1482)."""
        t = float(self.steps_trained)
        b1t = self.ADAM_BETA1 ** np.float32(t)
        b2t = self.ADAM_BETA2 ** np.float32(t)
        return np.float32(np.float32(lr_f) * np.sqrt(1.0 - b2t) / (1.0 - b1t))

    def step(self, io: RayBatch, lr_f: float, do_train: bool, return_output: bool, sh_multiplier: float = 1.0,
             color_MLP_rel_lr: float = 1.0, occ_update_strength: float | None = None,
             rng_u32: np.uint32 | None = None, wait: bool = False, global_size=None, local_size=None,
             wait_for: list | None = None):
        """One training step (do_train) or one forward render of ``io``'s rays
        (ffnerf_tools.py:1357-1544).  Returns (out or None, event of the last device work)."""
        import torch
        if self.native is None or (do_train and (getattr(self, "num_rays", None) != io.num_rays or
                                                 self.samples_per_ray != io.samples_per_ray)):
            self.setup_buffers(io.num_rays, io.samples_per_ray)
        if occ_update_strength is None:
            occ_update_strength = float(self.occ.occ_update_strength0 if do_train else 0.0)
        if rng_u32 is None:
            rng_u32 = self._get_rng_u32()
        if do_train:
            self.steps_trained = int(self.steps_trained) + 1
        nat = self.native
        q = self.queue
        q.wait_for(wait_for)
        offset = 0
        if self.dp is not None:
            offset = self.ray_offset if self.ray_offset is not None else self.dp.rank * io.num_rays
        do_maint = do_train and self.maintenance_due(self.steps_trained, occ_update_strength)
        timed = do_train and self.steps_trained < 4 and self.verbose
        with torch.cuda.stream(q.stream):
            t_start = torch.cuda.Event(enable_timing=True) if timed else None
            if t_start is not None:
                t_start.record(q.stream)
            if do_train:
                lr_t = self.lr_t(lr_f)
                s = ffn_native.make_step(lr_f=lr_f, lr_t=lr_t, sh_mult=sh_multiplier, color_rel_lr=color_MLP_rel_lr,
                                         occ_strength=occ_update_strength, rng_u32=int(rng_u32), ray_offset=offset,
                                         table_lr_t=lr_t, spr=io.samples_per_ray,
                                         table_immediate=self.table_immediate)
                if self.fb_events is not None:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(q.stream)
                nat.forward_backward(io.rays_buf, io.targets_buf, io.out_buf, io.num_rays, s, q.stream)
                ev_ff = Event(q.stream, t_start)
                if self.fb_events is not None:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(q.stream)
                    self.fb_events.append((e0, e1))
                if self.dp is not None:
                    self.dp.ensure_attached(self)
                    if self.dp.fused:
                        if self.fb_events is not None:
                            x0 = torch.cuda.Event(enable_timing=True)
                            x0.record(q.stream)
                        nat.dp_reduce_apply(s, q.stream)
                        if self.fb_events is not None:
                            x1 = torch.cuda.Event(enable_timing=True)
                            x1.record(q.stream)
                            self.ex_events.append((x0, x1))
                        s = ffn_native.make_step(lr_f=lr_f, lr_t=lr_t, sh_mult=sh_multiplier,
                                                 color_rel_lr=color_MLP_rel_lr, occ_strength=occ_update_strength,
                                                 rng_u32=int(rng_u32), ray_offset=offset, table_lr_t=lr_t,
                                                 spr=io.samples_per_ray, table_applied=True)
                    else:
                        self.dp.allreduce_grads(self)
                if do_maint:
                    if self.dp is not None:
                        self.dp.merge_occupancy(self)
                    nat.occ_maintenance(self.decay_q24(occ_update_strength), int(rng_u32), q.stream)
                nat.apply_updates(s, q.stream)
                ev_last = Event(q.stream)
            else:
                s = ffn_native.make_step(sh_mult=sh_multiplier, rng_u32=int(rng_u32), ray_offset=offset,
                                         spr=io.samples_per_ray)
                nat.render(io.rays_buf, io.out_buf, io.num_rays, s, q.stream)
                ev_ff = ev_last = Event(q.stream, t_start)
        io.ev_last = ev_last
        if timed:
            out, _ = io.download_out(wait=True, wait_for=[ev_last])
            print(f"[I]: ev_ff   do_train  [ms]: {event_ms(ev_ff):.3f}")
            print("          debug vals -", list(out[0:4, 3]))
        if return_output:
            # the reference enqueues the read and returns (ffnerf_tools.py:1533-1540)
            out, ev_dwn = io.download_out(wait=False, wait_for=[ev_last])
            if wait:
                ev_dwn.wait()
            return out, ev_dwn
        if wait:
            ev_last.wait()
        return None, ev_last
