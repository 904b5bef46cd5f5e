"""Headless rendering of a trained model: the B200 counterpart of the reference renderer's snapshot
path (render_nerf.py:646-671), which renders every pixel of one pose with ``Nerf.step(do_train=False)``
and writes a PNG.

Here the view's rays are generated on the device (``ffn_camera_rays``), rendered in chunks by the
inference kernel (``ffn_render``: occupancy-guided sampling with the inference rule, black
background) straight into a device frame, and the frame is read back once.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

import ffn_native


def render_frame(nerf, c2w, K, W: int, H: int, chunk_rays: int = 1 << 16, rng_u32: int = 0, stream=None):
    """Renders the W x H view of camera-to-world ``c2w`` (4x4) with intrinsics ``K`` (3x3 or None:
    the reference's fallback focal) and returns the [H, W, 3] float32 colours as a CUDA tensor.
    Ray i of the view (row-major) keys its sampling RNG with global ray id i.  The work runs on
    ``stream`` (default: the model's queue); torch's current stream is made to wait for it, so the
    returned tensor can be used there directly."""
    import torch
    if nerf.native is None:
        nerf.setup_buffers(min(int(chunk_rays), W * H), nerf.samples_per_ray if getattr(nerf, "samples_per_ray", None)
                           else 64, do_train=False)
    nat = nerf.native
    dev = torch.device("cuda", nat.device)
    c2w = np.ascontiguousarray(np.asarray(c2w, np.float32).reshape(4, 4))
    Kp = None if K is None else np.ascontiguousarray(np.asarray(K, np.float32).reshape(3, 3))
    n_pix = W * H
    chunk = min(int(chunk_rays), n_pix)
    rays = torch.empty((chunk, 8), dtype=torch.float32, device=dev)
    frame = torch.empty((n_pix, 4), dtype=torch.float32, device=dev)
    st = stream if stream is not None else nerf.queue.stream
    sp = ffn_native.Context._stream(st)
    lib = nat.lib
    kp = None if Kp is None else Kp.ctypes.data_as(C.c_void_p)
    for first in range(0, n_pix, chunk):
        n = min(chunk, n_pix - first)
        rc = lib.ffn_camera_rays(c2w.ctypes.data_as(C.c_void_p), kp, int(W), int(H), first, n,
                                 C.c_void_p(rays.data_ptr()), sp)
        if rc != 0:
            raise RuntimeError(f"ffn_camera_rays failed ({rc}): {lib.ffn_last_error(None).decode()}")
        step = ffn_native.make_step(sh_mult=1.0, rng_u32=int(rng_u32), ray_offset=first, spr=nerf.samples_per_ray)
        nat.render(rays, frame[first:first + n], n, step, st)
    if isinstance(st, torch.cuda.Stream):
        torch.cuda.current_stream(dev).wait_stream(st)
    else:
        torch.cuda.synchronize(dev)
    return frame[:, :3].reshape(H, W, 3)


def snapshot(nerf, c2w, K, W: int, H: int, output, chunk_rays: int = 1 << 16, rng_u32: int = 0) -> Path:
    """Renders the view and writes it as an 8-bit PNG the way the reference's snapshot does
    (clip to [0, 1], scale by 255, truncate, RGB -> BGR for cv2.imwrite)."""
    import cv2
    frame = render_frame(nerf, c2w, K, W, H, chunk_rays=chunk_rays, rng_u32=rng_u32)
    nerf.queue.finish()
    img = frame.cpu().numpy()
    if not np.isfinite(img).all():
        raise ValueError("Snapshot contains non-finite pixels")
    output = Path(output)
    output.parent.mkdir(parents=True, exist_ok=True)
    bgr = cv2.cvtColor((np.clip(img, 0, 1) * 255).astype(np.uint8), cv2.COLOR_RGB2BGR)
    if not cv2.imwrite(str(output), bgr):
        raise OSError(f"Could not save snapshot: {output}")
    return output
