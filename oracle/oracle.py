"""ctypes bindings of the CPU oracle and of the reference kernels compiled for the CPU.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline / reference leg.  The product never loads anything from this directory.

* ``Oracle``   -- ``libffn_oracle.so`` built from ``ffn_oracle.cpp`` (restatement of the
                  reference kernels with selectable math and table-update semantics).
* ``RefKernels`` -- ``_ref/libffnref_<variant>.so`` built by ``ref_build.py`` from the
                  reference's own OpenCL sources (run on CPU fibers).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libffn_oracle.so"
N_LEVELS = 16
PARAM_NAMES = ["Wd_in", "Wd_01", "Wd_12", "Wd_out", "Wc_in", "Wc_01", "Wc_12", "Wc_23", "Wc_out",
               "bd_0", "bd_1", "bd_2", "bd_out", "bc_0", "bc_1", "bc_2", "bc_3", "bc_out"]


def build_oracle(cxx: str = "g++") -> Path:
    src = HERE / "ffn_oracle.cpp"
    if ORACLE_SO.exists() and ORACLE_SO.stat().st_mtime >= max(src.stat().st_mtime, (HERE / "ffn_oracle.h").stat().st_mtime):
        return ORACLE_SO
    subprocess.run([cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off",
                    "-fno-fast-math", str(src), "-o", str(ORACLE_SO)], check=True)
    return ORACLE_SO


class OrcConfig(C.Structure):
    _fields_ = [("F", C.c_int32), ("ND", C.c_int32), ("NC", C.c_int32), ("spr", C.c_int32),
                ("G", C.c_int32), ("background", C.c_int32), ("math_mode", C.c_int32),
                ("table_mode", C.c_int32), ("tilek", C.c_int32), ("transfer_fmt", C.c_int32),
                ("level_log2", C.c_uint32 * N_LEVELS), ("level_offset", C.c_uint32 * N_LEVELS),
                ("level_res", C.c_int32 * N_LEVELS), ("hash_lr_scale", C.c_float * N_LEVELS),
                ("box_min", C.c_float * 4), ("box_max", C.c_float * 4),
                ("rho_min", C.c_float), ("rho_max", C.c_float), ("dt_min", C.c_float),
                ("dt_max", C.c_float), ("t_near", C.c_float), ("t_far", C.c_float),
                ("pad1", C.c_float), ("pad2", C.c_float)]


class OrcStep(C.Structure):
    _fields_ = [("lr_f", C.c_float), ("sh_mult", C.c_float), ("occ_strength", C.c_float),
                ("rng_seed", C.c_uint32), ("do_train", C.c_int32), ("ray_offset", C.c_uint32)]


class OrcDebug(C.Structure):
    _fields_ = [("t", C.c_void_p), ("dt", C.c_void_p), ("idx", C.c_void_p), ("flags", C.c_void_p),
                ("sigma", C.c_void_p), ("rgb", C.c_void_p), ("trans", C.c_void_p),
                ("dsigma", C.c_void_p), ("enc", C.c_void_p)]


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def make_orc_config(geom: dict, math_mode: int = 0, table_mode: int = 0, tilek: int = 236,
                    transfer_fmt: int = 32) -> OrcConfig:
    """Builds the C config from a geometry dict (keys as produced by the product's config helper:
    F, ND, NC, spr, G, background, level_log2, level_offset, level_res, hash_lr_scale, box_min,
    box_max, rho_min, rho_max, dt_min, dt_max, t_near, t_far)."""
    c = OrcConfig()
    for k in ("F", "ND", "NC", "spr", "G", "background"):
        setattr(c, k, int(geom[k]))
    c.math_mode, c.table_mode, c.tilek, c.transfer_fmt = math_mode, table_mode, tilek, transfer_fmt
    for i in range(N_LEVELS):
        c.level_log2[i] = int(geom["level_log2"][i])
        c.level_offset[i] = int(geom["level_offset"][i])
        c.level_res[i] = int(geom["level_res"][i])
        c.hash_lr_scale[i] = float(geom["hash_lr_scale"][i])
    for i in range(3):
        c.box_min[i] = float(geom["box_min"][i])
        c.box_max[i] = float(geom["box_max"][i])
    for k in ("rho_min", "rho_max", "dt_min", "dt_max", "t_near", "t_far"):
        setattr(c, k, float(geom[k]))
    return c


class Oracle:
    def __init__(self, so: Path | None = None):
        self.lib = C.CDLL(str(so or build_oracle()))
        L = self.lib
        L.orc_param_layout.restype = C.c_int32
        L.orc_param_layout.argtypes = [C.c_int32] * 3 + [C.c_void_p] * 2
        L.orc_forward_backward.restype = C.c_int32
        L.orc_forward_backward.argtypes = [C.POINTER(OrcConfig), C.POINTER(OrcStep)] + [C.c_void_p] * 7 + [C.c_int32] + [C.c_void_p] * 4
        L.orc_adam.argtypes = [C.c_void_p] * 4 + [C.c_int64] + [C.c_float] * 4
        L.orc_mlp_adam.argtypes = [C.POINTER(OrcConfig)] + [C.c_void_p] * 4 + [C.c_float] * 5
        L.orc_table_apply.argtypes = [C.POINTER(OrcConfig), C.c_void_p, C.c_void_p, C.c_float]
        L.orc_table_adam.argtypes = [C.POINTER(OrcConfig)] + [C.c_void_p] * 4 + [C.c_float] * 4
        L.orc_decay.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_hash_fwd.argtypes = [C.POINTER(OrcConfig), C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
        L.orc_hash_bwd.argtypes = [C.POINTER(OrcConfig), C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
        L.orc_expf.restype = C.c_float
        L.orc_expf.argtypes = [C.c_float]
        L.orc_powr.restype = C.c_float
        L.orc_powr.argtypes = [C.c_float, C.c_float]
        L.orc_hash_u32.restype = C.c_uint32
        L.orc_hash_u32.argtypes = [C.c_uint32]

    def layout(self, F: int, ND: int, NC: int):
        off = np.zeros(18, np.int32)
        sz = np.zeros(18, np.int32)
        total = self.lib.orc_param_layout(F, ND, NC, _p(off), _p(sz))
        return {n: (int(o), int(s)) for n, o, s in zip(PARAM_NAMES, off, sz)}, int(total)

    def forward_backward(self, cfg: OrcConfig, step: OrcStep, params, table, occ_in, occ_st, rays,
                         targets, out, table_grad=None, mlp_grad=None, debug: dict | None = None,
                         bypass=None) -> None:
        dbg = None
        if debug is not None:
            dbg = OrcDebug(*[_p(debug.get(k)) for k, _ in OrcDebug._fields_])
        n = int(rays.shape[0])
        rc = self.lib.orc_forward_backward(C.byref(cfg), C.byref(step), _p(params), _p(table),
                                           _p(occ_in), _p(occ_st), _p(rays), _p(targets), _p(out), n,
                                           _p(table_grad), _p(mlp_grad),
                                           C.byref(dbg) if dbg is not None else None, _p(bypass))
        if rc != 0:
            raise ValueError(f"oracle rejected the configuration (code {rc})")

    def mlp_adam(self, cfg, params, grad, m, v, lr_t, color_rel_lr, b1, b2, eps):
        self.lib.orc_mlp_adam(C.byref(cfg), _p(params), _p(grad), _p(m), _p(v), lr_t, color_rel_lr, b1, b2, eps)

    def adam(self, p, g, m, v, lr_t, b1, b2, eps):
        self.lib.orc_adam(_p(p), _p(g), _p(m), _p(v), p.size, lr_t, b1, b2, eps)

    def table_apply(self, cfg, table, table_grad, lr_f):
        self.lib.orc_table_apply(C.byref(cfg), _p(table), _p(table_grad), lr_f)

    def table_adam(self, cfg, table, table_grad, m, v, lr_t, b1, b2, eps):
        self.lib.orc_table_adam(C.byref(cfg), _p(table), _p(table_grad), _p(m), _p(v), lr_t, b1, b2, eps)

    def decay(self, occ_in, occ_st, decay_q24, seed):
        self.lib.orc_decay(_p(occ_in), _p(occ_st), occ_in.size, decay_q24, seed)

    def hash_fwd(self, cfg, table, pts, enc):
        self.lib.orc_hash_fwd(C.byref(cfg), _p(table), _p(pts), pts.shape[0], _p(enc))

    def hash_bwd(self, cfg, pts, denc, table_grad):
        self.lib.orc_hash_bwd(C.byref(cfg), _p(pts), _p(denc), pts.shape[0], _p(table_grad))


# ----------------------------------------------------------------------------- compiled reference
class RefTrainArgs(C.Structure):
    _fields_ = [("W", C.c_void_p * 9), ("b", C.c_void_p * 9), ("table", C.c_void_p),
                ("rays", C.c_void_p), ("targets", C.c_void_p), ("deltas", C.c_void_p * 9),
                ("acts", C.c_void_p * 9), ("out", C.c_void_p), ("lr", C.c_float),
                ("num_rays", C.c_uint32), ("spr", C.c_uint32), ("do_train", C.c_int32),
                ("sh_mult", C.c_float), ("occ_in", C.c_void_p), ("occ_st", C.c_void_p),
                ("box_min", C.c_float * 3), ("box_max", C.c_float * 3), ("G", C.c_int32),
                ("rho_min", C.c_float), ("rho_max", C.c_float), ("dt_min", C.c_float),
                ("dt_max", C.c_float), ("t_near", C.c_float), ("t_far", C.c_float),
                ("seed", C.c_uint32), ("occ_strength", C.c_float), ("n_threads", C.c_int32),
                ("lockstep", C.c_int32)]


class RefWUArgs(C.Structure):
    _fields_ = [("W", C.c_void_p * 9), ("b", C.c_void_p * 9), ("mW", C.c_void_p * 9),
                ("vW", C.c_void_p * 9), ("mb", C.c_void_p * 9), ("vb", C.c_void_p * 9),
                ("deltas", C.c_void_p * 9), ("acts", C.c_void_p * 9), ("B", C.c_int32),
                ("L", C.c_int32), ("M", C.c_int32), ("lr_t", C.c_float), ("color_rel_lr", C.c_float),
                ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float), ("n_threads", C.c_int32)]


REF_W = ["Wd_in", "Wd_01", "Wd_12", "Wd_out", "Wc_in", "Wc_01", "Wc_12", "Wc_23", "Wc_out"]
REF_B = ["bd_0", "bd_1", "bd_2", "bd_out", "bc_0", "bc_1", "bc_2", "bc_3", "bc_out"]
REF_DELTAS = ["dd1", "dd2", "dd3", "dd_out", "dc1", "dc2", "dc3", "dc4", "dc_out"]
REF_ACTS = ["apos", "ad1", "ad2", "ad3", "ac_in", "ac1", "ac2", "ac3", "ac4"]


def ref_so(variant: str) -> Path:
    return HERE / "_ref" / f"libffnref_{variant}.so"


class RefKernels:
    """The reference kernels, compiled from their own sources for the CPU."""

    def __init__(self, variant: str):
        so = ref_so(variant)
        if not so.exists():
            raise FileNotFoundError(f"{so} not built (oracle/ref_build.py needs the reference checkout)")
        self.lib = C.CDLL(str(so))
        self.lib.ffnref_train.argtypes = [C.POINTER(RefTrainArgs)]
        self.lib.ffnref_weight_update.argtypes = [C.POINTER(RefWUArgs)]
        self.lib.ffnref_decay.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32]
        f, nd, nc, lg, rm = C.c_int32(), C.c_int32(), C.c_int32(), C.c_int32(), C.c_float()
        self.lib.ffnref_info(C.byref(f), C.byref(nd), C.byref(nc), C.byref(lg), C.byref(rm))
        self.F, self.ND, self.NC, self.log2T, self.rmax = f.value, nd.value, nc.value, lg.value, rm.value

    @staticmethod
    def scratch_dims(F: int, ND: int, NC: int) -> dict:
        M, D_OUT, C_IN, C_OUT = 64, 16, 32, 3
        d = {"dd_out": D_OUT, "dc_out": C_OUT, "apos": 16 * F, "ac_in": C_IN}
        for i in range(1, 4):
            d[f"dd{i}"] = M if i <= ND else 0
            d[f"ad{i}"] = M if i <= ND else 0
        for i in range(1, 5):
            d[f"dc{i}"] = M if i <= NC else 0
            d[f"ac{i}"] = M if i <= NC else 0
        return d

    def alloc_scratch(self, n_samples: int) -> dict:
        dims = self.scratch_dims(self.F, self.ND, self.NC)
        return {k: (np.zeros(v * n_samples, np.float32) if v else None) for k, v in dims.items()}

    def train(self, params: dict, table, rays, targets, out, scratch: dict, occ_in, occ_st, geom: dict,
              lr: float, sh_mult: float, occ_strength: float, seed: int, do_train: bool = True,
              n_threads: int = 1, lockstep: bool = False) -> None:
        """One launch of ffnerf_train_step over the rays.  lockstep: every work-group advances barrier
        interval by barrier interval with all the others (each table read of the step precedes each
        in-kernel table update, the schedule of a device running the whole batch at once); else each
        OS thread runs one work-group to completion at a time (n_threads = 1: rays in order)."""
        a = RefTrainArgs()
        keep = []
        for i, n in enumerate(REF_W):
            a.W[i] = params[n].ctypes.data if params[n].size else 0
        for i, n in enumerate(REF_B):
            a.b[i] = params[n].ctypes.data if params[n].size else 0
        for i, n in enumerate(REF_DELTAS):
            a.deltas[i] = scratch[n].ctypes.data if scratch.get(n) is not None else 0
        for i, n in enumerate(REF_ACTS):
            a.acts[i] = scratch[n].ctypes.data if scratch.get(n) is not None else 0
        a.table = table.ctypes.data
        a.rays, a.targets, a.out = rays.ctypes.data, targets.ctypes.data, out.ctypes.data
        a.lr = lr
        a.num_rays, a.spr, a.do_train, a.sh_mult = rays.shape[0], int(geom["spr"]), int(bool(do_train)), sh_mult
        a.occ_in, a.occ_st = occ_in.ctypes.data, occ_st.ctypes.data
        for i in range(3):
            a.box_min[i], a.box_max[i] = float(geom["box_min"][i]), float(geom["box_max"][i])
        a.G = int(geom["G"])
        for k, kk in (("rho_min", "rho_min"), ("rho_max", "rho_max"), ("dt_min", "dt_min"),
                      ("dt_max", "dt_max"), ("t_near", "t_near"), ("t_far", "t_far")):
            setattr(a, k, float(geom[kk]))
        a.seed, a.occ_strength, a.n_threads = int(seed) & 0xFFFFFFFF, occ_strength, n_threads
        a.lockstep = int(bool(lockstep))
        del keep
        self.lib.ffnref_train(C.byref(a))

    def weight_update(self, params: dict, m: dict, v: dict, scratch: dict, B: int, lr_t: float,
                      color_rel_lr: float, beta1: float, beta2: float, eps: float, n_threads: int = 1):
        a = RefWUArgs()
        for i, n in enumerate(REF_W):
            for arr, dst in ((params, a.W), (m, a.mW), (v, a.vW)):
                dst[i] = arr[n].ctypes.data if arr[n].size else 0
        for i, n in enumerate(REF_B):
            for arr, dst in ((params, a.b), (m, a.mb), (v, a.vb)):
                dst[i] = arr[n].ctypes.data if arr[n].size else 0
        for i, n in enumerate(REF_DELTAS):
            a.deltas[i] = scratch[n].ctypes.data if scratch.get(n) is not None else 0
        for i, n in enumerate(REF_ACTS):
            a.acts[i] = scratch[n].ctypes.data if scratch.get(n) is not None else 0
        a.B, a.L, a.M = B, 16 * self.F, 64
        a.lr_t, a.color_rel_lr, a.beta1, a.beta2, a.eps, a.n_threads = lr_t, color_rel_lr, beta1, beta2, eps, n_threads
        self.lib.ffnref_weight_update(C.byref(a))

    def decay(self, occ_in, occ_st, decay_q24, seed):
        self.lib.ffnref_decay(occ_in.ctypes.data, occ_st.ctypes.data, occ_in.size, decay_q24, seed)
