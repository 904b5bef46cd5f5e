"""Seeded synthetic scene: isotropic Gaussian density blobs rendered analytically.

The stand-in for a captured SfM dataset in benchmarks and tests (there is no network for real
data).  Density sigma(x) = sum_k peak * exp(-|x - c_k|^2 / (2 s_k^2)); colour is the
density-weighted mix of the blobs' RGB.  Images are rendered by dense quadrature along each ray
with a black background and quantised to 8 bits, as PNG files are; cameras follow the OpenCV
convention (x right, y down, z forward) used by the reference's ray generation.

Also builds the occupancy grid of the scene (a warmed-up state: the densest ~5% of sub-cells
occupied) and writes the scene as an SfM archive (NPZ with img_paths, K, c2w, posed, X plus
PNG files) that the reference's ``sfm_data.read_scene`` contract accepts.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


class BlobScene:
    def __init__(self, seed: int = 0, n_blobs: int = 6, peak: float = 50.0, sigma_range=(0.05, 0.2),
                 half_extent: float = 0.5, box_min=(-1.0, -1.0, -1.0), box_max=(1.0, 1.0, 1.0)):
        rng = np.random.default_rng(seed)
        self.sigma = rng.uniform(sigma_range[0], sigma_range[1], n_blobs).astype(np.float64)
        lo = -half_extent + self.sigma[:, None]
        hi = half_extent - self.sigma[:, None]
        self.centers = lo + (hi - lo) * rng.random((n_blobs, 3))
        self.rgb = rng.uniform(0.0, 1.0, (n_blobs, 3))
        self.peak = float(peak)
        self.box_min = np.asarray(box_min, np.float64)
        self.box_max = np.asarray(box_max, np.float64)

    def density_color(self, x: np.ndarray):
        """x [..., 3] -> (sigma [...], rgb [..., 3])."""
        d2 = ((x[..., None, :] - self.centers) ** 2).sum(-1)             # [..., K]
        w = self.peak * np.exp(-d2 / (2.0 * self.sigma ** 2))           # [..., K]
        s = w.sum(-1)
        rgb = (w[..., None] * self.rgb).sum(-2) / np.maximum(s, 1e-12)[..., None]
        return s, rgb

    def render(self, rays: np.ndarray, n_quad: int = 192, chunk: int = 8192) -> np.ndarray:
        """rays [n, 8] (o.xyzw, d.xyzw) -> rgb [n, 3] in [0, 1], black background."""
        out = np.zeros((rays.shape[0], 3), np.float32)
        for a in range(0, rays.shape[0], chunk):
            r = rays[a:a + chunk].astype(np.float64)
            o, d = r[:, :3], r[:, 4:7]
            with np.errstate(divide="ignore", invalid="ignore"):
                inv = np.where(d != 0, 1.0 / d, np.inf)
                t0 = np.nanmax(np.minimum((self.box_min - o) * inv, (self.box_max - o) * inv), axis=1)
                t1 = np.nanmin(np.maximum((self.box_min - o) * inv, (self.box_max - o) * inv), axis=1)
            t0 = np.maximum(t0, 0.0)
            hit = t1 > t0
            t0 = np.where(hit, t0, 0.0)
            t1 = np.where(hit, t1, 0.0)
            u = (np.arange(n_quad) + 0.5) / n_quad
            t = t0[:, None] + (t1 - t0)[:, None] * u[None, :]
            dt = ((t1 - t0) / n_quad)[:, None]
            x = o[:, None, :] + t[..., None] * d[:, None, :]
            s, c = self.density_color(x)
            alpha = 1.0 - np.exp(-s * dt)
            T = np.cumprod(np.concatenate([np.ones((x.shape[0], 1)), 1.0 - alpha[:, :-1]], axis=1), axis=1)
            col = ((T * alpha)[..., None] * c).sum(1)
            out[a:a + chunk] = np.where(hit[:, None], col, 0.0)
        return np.clip(out, 0.0, 1.0)

    # -- the same computations on a torch device (data preparation for benchmarks)
    def _t(self, device):
        import torch
        return (torch.as_tensor(self.centers, dtype=torch.float32, device=device),
                torch.as_tensor(self.sigma, dtype=torch.float32, device=device),
                torch.as_tensor(self.rgb, dtype=torch.float32, device=device))

    def density_color_torch(self, x):
        c, s, rgb = self._t(x.device)
        d2 = ((x[..., None, :] - c) ** 2).sum(-1)
        w = self.peak * (-d2 / (2.0 * s ** 2)).exp()
        tot = w.sum(-1)
        col = (w[..., None] * rgb).sum(-2) / tot.clamp_min(1e-12)[..., None]
        return tot, col

    def render_torch(self, rays, n_quad: int = 192, chunk: int = 16384):
        """rays [n, 8] torch tensor -> rgb [n, 3] (black background), on the rays' device."""
        import torch
        out = torch.zeros((rays.shape[0], 3), dtype=torch.float32, device=rays.device)
        bmin = torch.as_tensor(self.box_min, dtype=torch.float32, device=rays.device)
        bmax = torch.as_tensor(self.box_max, dtype=torch.float32, device=rays.device)
        u = (torch.arange(n_quad, device=rays.device, dtype=torch.float32) + 0.5) / n_quad
        for a in range(0, rays.shape[0], chunk):
            o, d = rays[a:a + chunk, :3], rays[a:a + chunk, 4:7]
            inv = torch.where(d != 0, 1.0 / d, torch.full_like(d, float("inf")))
            ta, tb = (bmin - o) * inv, (bmax - o) * inv
            t0 = torch.nan_to_num(torch.minimum(ta, tb), nan=-float("inf")).amax(1).clamp_min(0.0)
            t1 = torch.nan_to_num(torch.maximum(ta, tb), nan=float("inf")).amin(1)
            hit = t1 > t0
            t0 = torch.where(hit, t0, torch.zeros_like(t0))
            t1 = torch.where(hit, t1, torch.zeros_like(t1))
            t = t0[:, None] + (t1 - t0)[:, None] * u[None, :]
            dt = ((t1 - t0) / n_quad)[:, None]
            x = o[:, None, :] + t[..., None] * d[:, None, :]
            sg, c = self.density_color_torch(x)
            alpha = 1.0 - (-sg * dt).exp()
            T = torch.cumprod(torch.cat([torch.ones_like(alpha[:, :1]), 1.0 - alpha[:, :-1]], 1), 1)
            col = ((T * alpha)[..., None] * c).sum(1)
            out[a:a + chunk] = torch.where(hit[:, None], col, torch.zeros_like(col))
        return out.clamp(0.0, 1.0)

    def occupancy_grid_torch(self, G: int, device, occupied_fraction: float = 0.05, q_occupied: int = 15) -> np.ndarray:
        """occupancy_grid computed on a torch device."""
        import torch
        h = torch.as_tensor((self.box_max - self.box_min) / (2 * G), dtype=torch.float32, device=device)
        lo = torch.as_tensor(self.box_min, dtype=torch.float32, device=device)
        idx = torch.arange(2 * G, device=device, dtype=torch.float32) + 0.5
        sub = torch.empty((2 * G, 2 * G, 2 * G), dtype=torch.float32, device=device)
        yy, xx = torch.meshgrid(lo[1] + idx * h[1], lo[0] + idx * h[0], indexing="ij")
        for zi in range(2 * G):
            pts = torch.stack([xx, yy, torch.full_like(xx, float(lo[2] + (zi + 0.5) * h[2]))], -1)
            sub[zi] = self.density_color_torch(pts)[0]
        k = max(1, int(round(occupied_fraction * sub.numel())))
        thr = torch.topk(sub.reshape(-1), k).values[-1]
        occ4 = torch.where(sub >= thr, q_occupied - 1, 0).to(torch.int64).cpu().numpy().astype(np.uint32)
        o = occ4.reshape(G, 2, G, 2, G, 2)
        grid = np.zeros((G, G, G), np.uint32)
        for sz in range(2):
            for sy in range(2):
                for sx in range(2):
                    grid |= o[:, sz, :, sy, :, sx] << np.uint32(4 * (sx + 2 * sy + 4 * sz))
        return grid.reshape(-1)

    def occupancy_grid(self, G: int, occupied_fraction: float = 0.05, q_occupied: int = 15) -> np.ndarray:
        """Packed nibble grid [G^3] uint32 (8 sub-cells per cell, value occ4 = q - 1): the densest
        `occupied_fraction` of sub-cells get occ4 = q_occupied - 1, the rest 0."""
        h = (self.box_max - self.box_min) / (2 * G)          # sub-cell size
        idx = np.arange(2 * G)
        sub = np.zeros((2 * G, 2 * G, 2 * G), np.float32)
        for zi in range(2 * G):                              # slab by slab to bound memory
            z = self.box_min[2] + (zi + 0.5) * h[2]
            yy, xx = np.meshgrid(self.box_min[1] + (idx + 0.5) * h[1], self.box_min[0] + (idx + 0.5) * h[0], indexing="ij")
            pts = np.stack([xx, yy, np.full_like(xx, z)], axis=-1)
            sub[zi] = self.density_color(pts)[0]
        thr = np.quantile(sub, 1.0 - occupied_fraction)
        occ4 = np.where(sub >= thr, q_occupied - 1, 0).astype(np.uint32)   # [z][y][x] at sub-cell res
        # pack: cell (ix,iy,iz), sub = sx + 2 sy + 4 sz (ffnerf_OG.cl:1108-1111)
        o = occ4.reshape(G, 2, G, 2, G, 2)                   # [iz, sz, iy, sy, ix, sx]
        grid = np.zeros((G, G, G), np.uint32)                # [iz][iy][ix] -> cell = ix + G*(iy + G*iz)
        for sz in range(2):
            for sy in range(2):
                for sx in range(2):
                    s = sx + 2 * sy + 4 * sz
                    grid |= o[:, sz, :, sy, :, sx] << np.uint32(4 * s)
        return grid.reshape(-1)


def look_at_c2w(eye, target=(0.0, 0.0, 0.0), world_up=(0.0, 0.0, 1.0)) -> np.ndarray:
    """Camera-to-world 4x4, OpenCV axes (x right, y down, z toward the target)."""
    eye = np.asarray(eye, np.float64)
    z = np.asarray(target, np.float64) - eye
    z /= np.linalg.norm(z)
    x = np.cross(z, world_up)
    if np.linalg.norm(x) < 1e-9:
        x = np.cross(z, (0.0, 1.0, 0.0))
    x /= np.linalg.norm(x)
    y = np.cross(z, x)
    c2w = np.eye(4)
    c2w[:3, 0], c2w[:3, 1], c2w[:3, 2], c2w[:3, 3] = x, y, z, eye
    return c2w.astype(np.float32)


def cameras_sphere(n: int, radius: float, seed: int) -> np.ndarray:
    """n cameras on a sphere (Fibonacci lattice with a seeded rotation) looking at the origin."""
    rng = np.random.default_rng(seed)
    k = np.arange(n) + 0.5
    phi = np.arccos(1 - 2 * k / n)
    theta = np.pi * (1 + 5 ** 0.5) * k + rng.uniform(0, 2 * np.pi)
    eyes = radius * np.stack([np.cos(theta) * np.sin(phi), np.sin(theta) * np.sin(phi), np.cos(phi)], 1)
    return np.stack([look_at_c2w(e) for e in eyes])


def cameras_ring(n: int, radius: float, seed: int, elev_deg=(10.0, 40.0)) -> np.ndarray:
    """n cameras on a seeded ring: azimuth evenly spaced with jitter, elevation in elev_deg."""
    rng = np.random.default_rng(seed)
    az = 2 * np.pi * (np.arange(n) + rng.uniform(-0.3, 0.3, n)) / n
    el = np.deg2rad(rng.uniform(elev_deg[0], elev_deg[1], n))
    eyes = radius * np.stack([np.cos(el) * np.cos(az), np.cos(el) * np.sin(az), np.sin(el)], 1)
    return np.stack([look_at_c2w(e) for e in eyes])


def intrinsics(W: int, H: int, fov_deg: float) -> np.ndarray:
    """Pinhole K with the given horizontal field of view."""
    f = 0.5 * W / np.tan(0.5 * np.deg2rad(fov_deg))
    return np.array([[f, 0, W / 2.0], [0, f, H / 2.0], [0, 0, 1]], np.float32)


def pixel_rays(c2w: np.ndarray, K: np.ndarray, u: np.ndarray, v: np.ndarray) -> np.ndarray:
    """[n, 8] rays through pixel centres (u right, v down) of one camera."""
    x = (u.astype(np.float32) + 0.5 - K[0, 2]) / K[0, 0]
    y = (v.astype(np.float32) + 0.5 - K[1, 2]) / K[1, 1]
    cam = np.stack([x, y, np.ones_like(x)], 1)
    d = cam @ c2w[:3, :3].T
    d /= np.linalg.norm(d, axis=1, keepdims=True) + 1e-12
    rays = np.zeros((u.size, 8), np.float32)
    rays[:, :3] = c2w[:3, 3]
    rays[:, 3] = 1.0
    rays[:, 4:7] = d
    return rays


def random_batch(scene: BlobScene, cams: np.ndarray, K: np.ndarray, W: int, H: int, n: int, seed: int,
                 n_quad: int = 192):
    """n rays through uniformly drawn pixels of random cameras and their 8-bit quantised colours."""
    rng = np.random.default_rng(seed)
    ci = rng.integers(0, cams.shape[0], n)
    u = rng.integers(0, W, n)
    v = rng.integers(0, H, n)
    rays = np.zeros((n, 8), np.float32)
    for c in np.unique(ci):
        sel = ci == c
        rays[sel] = pixel_rays(cams[c], K, u[sel], v[sel])
    rgb = scene.render(rays, n_quad=n_quad)
    tg = np.zeros((n, 4), np.float32)
    tg[:, :3] = np.round(rgb * 255.0) / 255.0
    return rays, tg


def write_sfm_archive(root: Path, scene: BlobScene, cams: np.ndarray, K: np.ndarray, W: int, H: int,
                      n_quad: int = 192) -> Path:
    """Renders every camera and writes PNG images plus the NPZ archive keys that
    sfm_data.read_scene expects (img_paths, K, c2w, posed, X)."""
    import cv2
    root = Path(root)
    (root / "images").mkdir(parents=True, exist_ok=True)
    paths = []
    uu, vv = np.meshgrid(np.arange(W), np.arange(H))
    for i, c2w in enumerate(cams):
        rgb = scene.render(pixel_rays(c2w, K, uu.ravel(), vv.ravel()), n_quad=n_quad).reshape(H, W, 3)
        p = root / "images" / f"{i:03d}.png"
        cv2.imwrite(str(p), cv2.cvtColor((np.round(rgb * 255)).astype(np.uint8), cv2.COLOR_RGB2BGR))
        paths.append(f"images/{i:03d}.png")
    npz = root / "scene.npz"
    np.savez(npz, img_paths=np.array(paths, dtype=object), K=K, c2w=cams, posed=np.ones(len(cams), bool),
             X=scene.centers.astype(np.float32))
    return npz
