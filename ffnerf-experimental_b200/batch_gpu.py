"""Training batches drawn on the device: the B200 counterpart of the reference trainer's batch
producer thread (run_ffnerf_OG.py:585-685) and its pixel-weight feedback (:459-490, :1368-1387).

The images, camera poses and per-image uint8 pixel-weight maps stay in HBM; ``next_batch`` fills a
``RayBatch``'s device buffers (rays, targets) and keeps the drawn (image, x, y) for ``feedback``,
which turns the per-ray colour error of a finished step into the weight-map EMA.  Every kernel is
in libffnerf.so (``ffn_batch_generate``, ``ffn_batch_errors``, ``ffn_batch_feedback``).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

import ffn_native


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def median_like_numpy(x):
    """np.median of a float32 CUDA tensor, on the device: the middle value, or for an even count
    the float32 mean of the two middle values."""
    import torch
    s, _ = torch.sort(x)
    n = s.numel()
    if n % 2:
        return s[n // 2:n // 2 + 1].clone()
    return ((s[n // 2 - 1] + s[n // 2]) / 2).reshape(1)


def batch_metrics(out, targets, n: int, stream=None):
    """The trainer's periodic loss figures (run_ffnerf_OG.py:1389-1391) for one batch, computed on
    the device without a host round trip: a CUDA float64 tensor [mse, rmse, l2]."""
    import torch
    lib = ffn_native.load_library()
    s = torch.zeros(1, dtype=torch.float64, device=out.device)
    rc = lib.ffn_batch_errors(_ptr(out), _ptr(targets), int(n), None, _ptr(s), ffn_native.Context._stream(stream))
    if rc != 0:
        raise RuntimeError(f"ffn_batch_errors failed ({rc}): {lib.ffn_last_error(None).decode()}")
    mse = s / (3.0 * n)
    return torch.cat([mse, mse.sqrt(), (s / n).sqrt()])


class GpuBatchProducer:
    """Draws batches of ``batch_rays`` rays from ``Ims`` ([N, H, W, >=3] uint8 or float32 in [0, 1]),
    ``RTs`` ([N, 4, 4] camera-to-world) and ``K`` ([3, 3], [N, 3, 3] or None), with the reference's
    sampling rule: a uniform image per ray, then a uniform pixel for ``uniform_frac`` of the rays and a
    pixel by rejection against the image's weight map (initialised to 16) for the rest.  ``ema``,
    ``bg_cap`` and ``fg_tau`` are the feedback parameters of the reference's batch producer."""

    def __init__(self, Ims, RTs, K, W: int, H: int, batch_rays: int, rng_seed: int = 0, ema: float = 0.05,
                 bg_cap: int = 16, fg_tau: int = 8, uniform_frac: float = 0.2, max_tries: int = 256,
                 device: int = 0):
        import torch
        Ims = np.asarray(Ims)
        if Ims.ndim != 4 or Ims.shape[1] != H or Ims.shape[2] != W or Ims.shape[3] < 3:
            raise ValueError("Ims must be [N, H, W, >=3]")
        self.dev = torch.device("cuda", device)
        self.f32 = Ims.dtype != np.uint8
        self.images = torch.from_numpy(np.ascontiguousarray(Ims.astype(np.float32) if self.f32 else Ims)).to(self.dev)
        self.n_img, self.H, self.W, self.C = Ims.shape[0], H, W, Ims.shape[3]
        RTs = np.asarray(RTs, np.float32)
        if RTs.shape != (self.n_img, 4, 4):
            raise ValueError("RTs must be [N, 4, 4] camera-to-world")
        self.c2w = torch.from_numpy(np.ascontiguousarray(RTs)).to(self.dev)
        self.K = None if K is None else torch.from_numpy(np.ascontiguousarray(np.asarray(K, np.float32))).to(self.dev)
        self.k_per_image = int(self.K is not None and self.K.ndim == 3)
        self.weights = torch.full((self.n_img, H, W), 16, dtype=torch.uint8, device=self.dev)
        self.batch_rays = int(batch_rays)
        self.seed = int(rng_seed) & 0xFFFFFFFF
        self.ema, self.bg_cap, self.fg_tau = float(ema), int(bg_cap), int(fg_tau)
        self.uniform_frac, self.max_tries = float(uniform_frac), int(max_tries)
        self.draws = 0
        n = self.batch_rays
        self.im = torch.empty(n, dtype=torch.int32, device=self.dev)
        self.x = torch.empty_like(self.im)
        self.y = torch.empty_like(self.im)
        self.err = torch.empty(n, dtype=torch.float32, device=self.dev)
        self.lib = ffn_native.load_library()

    def _check(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed ({rc}): {self.lib.ffn_last_error(None).decode()}")

    def next_batch(self, rays=None, targets=None, stream=None):
        """Draws the next batch into ``rays`` ([n, 8] float32) and ``targets`` ([n, 4] float32) CUDA
        tensors (allocated when None); returns them.  Batch k uses seed hash(rng_seed, k)."""
        import torch
        n = self.batch_rays
        if rays is None:
            rays = torch.empty((n, 8), dtype=torch.float32, device=self.dev)
        if targets is None:
            targets = torch.empty((n, 4), dtype=torch.float32, device=self.dev)
        seed = (self.seed * 0x9E3779B1 + self.draws * 0x85EBCA77 + 1) & 0xFFFFFFFF
        self.draws += 1
        st = ffn_native.Context._stream(stream)
        self._check(self.lib.ffn_batch_generate(_ptr(self.images), int(self.f32), self.C, _ptr(self.weights),
                                                _ptr(self.c2w), _ptr(self.K), self.k_per_image, self.n_img, self.W,
                                                self.H, n, self.uniform_frac, seed, self.max_tries, _ptr(rays),
                                                _ptr(targets), _ptr(self.im), _ptr(self.x), _ptr(self.y), st),
                    "ffn_batch_generate")
        return rays, targets

    def feedback(self, out, targets, stream=None):
        """Weight-map update from the rendered colours ``out`` ([n, 4]) of the last drawn batch and
        its ``targets``: per-ray error, its median (as np.median), then the EMA."""
        n = self.batch_rays
        st = ffn_native.Context._stream(stream)
        self._check(self.lib.ffn_batch_errors(_ptr(out), _ptr(targets), n, _ptr(self.err), None, st), "ffn_batch_errors")
        self.apply_errors(stream)

    def apply_errors(self, stream=None):
        """The weight-map EMA from the per-ray errors held in ``self.err`` (of the last drawn batch)."""
        n = self.batch_rays
        st = ffn_native.Context._stream(stream)
        med = median_like_numpy(self.err)
        self._check(self.lib.ffn_batch_feedback(_ptr(self.weights), _ptr(self.images), int(self.f32), self.C, self.W,
                                                self.H, _ptr(self.im), _ptr(self.x), _ptr(self.y), _ptr(self.err), n,
                                                _ptr(med), self.ema, self.bg_cap, self.fg_tau, st),
                    "ffn_batch_feedback")
