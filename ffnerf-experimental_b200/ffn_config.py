"""Geometry and hyper-parameter tables of the fused NeRF step (host side).

The reference hard-codes most of its geometry as OpenCL ``#define``s; here every knob is a
runtime value carried in one config (``make_geometry``) and passed through the C ABI.  The
derived per-level tables are computed once on the host, in float32, with the same expressions
the reference evaluates per sample inside the kernel:

* level resolution  ``R_l = rint(16 * pow(Rmax/16, l * (1/15)))``, at least 2
  (ffnerf_OG.cl:1308-1311);
* hash learning-rate roll-off ``2^(-0.1 * l)`` (ffnerf_OG.cl:2110-2111);
* per-level table sizes and offsets (ffnerf_OG.cl:187-211).
"""
from __future__ import annotations

import ctypes
import ctypes.util

import numpy as np

N_LEVELS = 16                # ffnerf_OG.cl:166
M = 64                       # hidden width, ffnerf_OG.cl:45
D_OUT = 16                   # ffnerf_OG.cl:42
L_DIR = 16                   # ffnerf_OG.cl:41
C_IN = D_OUT + L_DIR         # ffnerf_OG.cl:43
C_OUT = 3                    # ffnerf_OG.cl:44
S_MAX = 64                   # ffnerf_OG.cl:47
RESOLUTION_LVL0 = 16.0       # ffnerf_OG.cl:163
RESOLUTION_LVLMAX = 1024.0   # ffnerf_OG.cl:164
HASH_W_LVL_SCALE_EXPONENT = 0.1  # ffnerf_OG.cl:66

# The reference's variable per-level table (ffnerf_OG.cl:187-200): 2,260,992 entries in total.
REFERENCE_LEVEL_LOG2 = (13, 13, 13, 13, 15, 15, 15, 15, 17, 17, 17, 17, 18, 18, 19, 19)

BACKGROUNDS = {"black": 0, "white": 1, "random": 2}

PARAM_NAMES = ("Wd_in", "Wd_01", "Wd_12", "Wd_out", "Wc_in", "Wc_01", "Wc_12", "Wc_23", "Wc_out",
               "bd_0", "bd_1", "bd_2", "bd_out", "bc_0", "bc_1", "bc_2", "bc_3", "bc_out")
COLOR_PARAMS = frozenset(n for n in PARAM_NAMES if n.startswith(("Wc_", "bc_")))


def _c_powf():
    """The C library's single-precision pow (numpy's float32 power differs from it by one ulp
    for some arguments; the kernels evaluate powf)."""
    name = ctypes.util.find_library("m")
    if not name:
        return None
    f = ctypes.CDLL(name).powf
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_float, ctypes.c_float]
    return f


_POWF = _c_powf()


def powf(x, y) -> np.float32:
    if _POWF is not None:
        return np.float32(_POWF(float(np.float32(x)), float(np.float32(y))))
    return np.power(np.float32(x), np.float32(y), dtype=np.float32)


def level_resolutions(rmax: float, r0: float = RESOLUTION_LVL0) -> list[int]:
    f32 = np.float32
    inv = f32(1.0) / f32(N_LEVELS - 1)
    ratio = f32(rmax) / f32(r0)
    out = []
    for lvl in range(N_LEVELS):
        t = f32(lvl) * inv
        rf = f32(r0) * powf(ratio, t)
        r = int(np.rint(rf))
        out.append(max(r, 2))
    return out


def hash_lr_scales() -> list[float]:
    f32 = np.float32
    return [float(powf(f32(2.0), f32(-lvl) * f32(HASH_W_LVL_SCALE_EXPONENT))) for lvl in range(N_LEVELS)]


def level_layout(log2_entries) -> tuple[list[int], list[int], int]:
    """Per-level log2 sizes (an int means the same size for every level) -> (log2, offsets, total)."""
    if isinstance(log2_entries, (int, np.integer)):
        log2 = [int(log2_entries)] * N_LEVELS
    else:
        log2 = [int(x) for x in log2_entries]
        if len(log2) != N_LEVELS:
            raise ValueError(f"need {N_LEVELS} per-level table sizes, got {len(log2)}")
    if any(k < 1 or k > 24 for k in log2):
        raise ValueError("per-level table size must be 2^1 .. 2^24 entries")
    offs, o = [], 0
    for k in log2:
        offs.append(o)
        o += 1 << k
    return log2, offs, o


def param_layout(F: int, ND: int, NC: int) -> tuple[dict[str, tuple[int, int]], int]:
    """Offsets/sizes (in floats) of the active parameters in the flat parameter blob.

    Canonical order is the reference kernel argument order (ffnerf_OG.cl:843-861); inactive
    layers have size 0; every segment starts on a 16-byte boundary."""
    lpos = N_LEVELS * F
    sizes = {
        "Wd_in": M * lpos, "Wd_01": M * M if ND >= 2 else 0, "Wd_12": M * M if ND >= 3 else 0,
        "Wd_out": D_OUT * M,
        "Wc_in": M * C_IN, "Wc_01": M * M if NC >= 2 else 0, "Wc_12": M * M if NC >= 3 else 0,
        "Wc_23": M * M if NC >= 4 else 0, "Wc_out": C_OUT * M,
        "bd_0": M, "bd_1": M if ND >= 2 else 0, "bd_2": M if ND >= 3 else 0, "bd_out": D_OUT,
        "bc_0": M, "bc_1": M if NC >= 2 else 0, "bc_2": M if NC >= 3 else 0,
        "bc_3": M if NC >= 4 else 0, "bc_out": C_OUT,
    }
    lay, o = {}, 0
    for n in PARAM_NAMES:
        lay[n] = (o, sizes[n])
        o += (sizes[n] + 3) & ~3
    return lay, o


def param_shapes(F: int, ND: int, NC: int) -> dict[str, tuple[int, ...]]:
    lpos = N_LEVELS * F
    shp = {"Wd_in": (M, lpos), "Wd_01": (M, M), "Wd_12": (M, M), "Wd_out": (D_OUT, M),
           "Wc_in": (M, C_IN), "Wc_01": (M, M), "Wc_12": (M, M), "Wc_23": (M, M), "Wc_out": (C_OUT, M),
           "bd_0": (M,), "bd_1": (M,), "bd_2": (M,), "bd_out": (D_OUT,),
           "bc_0": (M,), "bc_1": (M,), "bc_2": (M,), "bc_3": (M,), "bc_out": (C_OUT,)}
    lay, _ = param_layout(F, ND, NC)
    return {n: s for n, s in shp.items() if lay[n][1] > 0}


def make_geometry(*, F: int = 2, ND: int = 1, NC: int = 2, spr: int = 64, G: int = 64,
                  log2_entries=14, rmax: float = 512.0, box_min=(-1.0, -1.0, -1.0),
                  box_max=(1.0, 1.0, 1.0), rho_min: float = 1.0, rho_max: float = 16.0,
                  dt_min: float | None = None, dt_max: float | None = None, t_near: float = 0.3,
                  t_far: float = 1.0e9, background: str | int = "random") -> dict:
    """One dict with every knob of the step.  dt_min/dt_max default to the trainer's formulas
    (run_ffnerf_OG.py:1050-1051)."""
    if F not in (2, 4):
        raise ValueError("F (features per level) must be 2 or 4")
    if not 1 <= ND <= 3 or not 1 <= NC <= 4:
        raise ValueError("ND must be 1..3 and NC 1..4")
    if spr not in (16, 32, 64):
        raise ValueError(f"samples_per_ray must be 16, 32 or 64 (<= S_MAX={S_MAX}, power of two)")
    if G < 1 or G > 1024:
        raise ValueError("occupancy grid side must be 1..1024")
    bmin = np.asarray(box_min, np.float32).reshape(3)
    bmax = np.asarray(box_max, np.float32).reshape(3)
    if not (np.isfinite(bmin).all() and np.isfinite(bmax).all() and (bmax > bmin).all()):
        raise ValueError("box_max must exceed box_min, finite")
    ext = float(np.max(bmax - bmin))
    if dt_min is None:
        dt_min = np.float32(ext / 8192)
    if dt_max is None:
        dt_max = np.float32(12.8 / spr / 6 * ext)
    log2, offs, total = level_layout(log2_entries)
    bg = BACKGROUNDS[background] if isinstance(background, str) else int(background)
    return dict(F=int(F), ND=int(ND), NC=int(NC), spr=int(spr), G=int(G), background=bg,
                level_log2=log2, level_offset=offs, table_entries=total,
                level_res=level_resolutions(rmax), hash_lr_scale=hash_lr_scales(), rmax=float(rmax),
                box_min=[float(x) for x in bmin], box_max=[float(x) for x in bmax],
                rho_min=float(np.float32(rho_min)), rho_max=float(np.float32(rho_max)),
                dt_min=float(np.float32(dt_min)), dt_max=float(np.float32(dt_max)),
                t_near=float(np.float32(t_near)), t_far=float(np.float32(t_far)))
