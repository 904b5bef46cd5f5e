"""Seeded synthetic inputs shared by the tests (rays, parameters, tables, occupancy grids)."""
from __future__ import annotations

import numpy as np

from ffn_config import param_layout, param_shapes


def rays_toward_box(n: int, seed: int, radius: float = 2.0, spread: float = 0.6, n_miss: int = 0) -> np.ndarray:
    """[n][8] float32 rays: origins on a sphere, directions toward random points near the centre;
    the first n_miss rays point away from the box (no hit)."""
    rng = np.random.default_rng(seed)
    o = rng.normal(size=(n, 3))
    o /= np.linalg.norm(o, axis=1, keepdims=True)
    o *= radius
    tgt = rng.uniform(-spread, spread, size=(n, 3))
    d = tgt - o
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    d[:n_miss] = o[:n_miss] / np.linalg.norm(o[:n_miss], axis=1, keepdims=True)
    rays = np.zeros((n, 8), np.float32)
    rays[:, :3] = o
    rays[:, 3] = 1.0
    rays[:, 4:7] = d
    return rays


def targets(n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed + 1)
    t = np.zeros((n, 4), np.float32)
    t[:, :3] = rng.uniform(0, 1, (n, 3))
    return t


def init_blob(geom: dict, seed: int, sigma_bias: float = 0.5, scale: float = 1.0) -> np.ndarray:
    """Random MLP parameters in the flat blob layout (He-like weights, small heads)."""
    rng = np.random.default_rng(seed)
    F, ND, NC = geom["F"], geom["ND"], geom["NC"]
    lay, total = param_layout(F, ND, NC)
    blob = np.zeros(total, np.float32)
    for n, sh in param_shapes(F, ND, NC).items():
        off, sz = lay[n]
        if n.startswith("W"):
            std = 0.05 if sh[0] <= 16 else np.sqrt(2.0 / sh[1])
            blob[off:off + sz] = (rng.normal(0, std * scale, size=sz)).astype(np.float32)
        else:
            blob[off:off + sz] = rng.normal(0, 0.05, size=sz).astype(np.float32)
    off, _ = lay["bd_out"]
    blob[off] = sigma_bias
    return blob


def init_table(geom: dict, seed: int, amp: float = 1e-1) -> np.ndarray:
    rng = np.random.default_rng(seed + 7)
    return rng.uniform(-amp, amp, geom["table_entries"] * geom["F"]).astype(np.float32)


def init_occ(geom: dict, seed: int, mask: int = 0x77777777) -> np.ndarray:
    rng = np.random.default_rng(seed + 11)
    return (rng.integers(0, 2**32, geom["G"] ** 3, dtype=np.uint64).astype(np.uint32) & np.uint32(mask))


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
