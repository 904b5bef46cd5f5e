"""ctypes binding of libffnerf.so (include/ffnerf.h).

There is no fallback: if the library is missing or a call fails, a RuntimeError / ValueError is
raised.  Device buffers owned by a context are exposed to PyTorch without copies through the
``__cuda_array_interface__`` protocol (``Context.tensor``), so NCCL all-reduce and checkpoint
I/O operate on the very memory the kernels use.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from ffn_config import N_LEVELS, PARAM_NAMES

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libffnerf.so"

FFN_OK, FFN_E_CONFIG, FFN_E_CUDA, FFN_E_CAPACITY, FFN_E_NAME, FFN_E_STATE = 0, -1, -2, -3, -4, -5
BUF_PARAMS, BUF_ADAM_M, BUF_ADAM_V, BUF_TABLE, BUF_OCC_IN, BUF_OCC_ST, BUF_GRADS, BUF_TABLE_M, BUF_TABLE_V = range(9)
BUF_DTYPES = {BUF_PARAMS: np.float32, BUF_ADAM_M: np.float32, BUF_ADAM_V: np.float32, BUF_TABLE: np.float32,
              BUF_OCC_IN: np.uint32, BUF_OCC_ST: np.uint32, BUF_GRADS: np.float32, BUF_TABLE_M: np.float32,
              BUF_TABLE_V: np.float32}


class FfnConfig(C.Structure):
    _fields_ = [("F", C.c_int32), ("ND", C.c_int32), ("NC", C.c_int32), ("spr", C.c_int32),
                ("G", C.c_int32), ("background", C.c_int32), ("table_optimizer", C.c_int32),
                ("max_rays", C.c_int32),
                ("level_log2", C.c_uint32 * N_LEVELS), ("level_offset", C.c_uint32 * N_LEVELS),
                ("level_res", C.c_int32 * N_LEVELS), ("hash_lr_scale", C.c_float * N_LEVELS),
                ("box_min", C.c_float * 4), ("box_max", C.c_float * 4),
                ("rho_min", C.c_float), ("rho_max", C.c_float), ("dt_min", C.c_float),
                ("dt_max", C.c_float), ("t_near", C.c_float), ("t_far", C.c_float),
                ("adam_beta1", C.c_float), ("adam_beta2", C.c_float), ("adam_eps", C.c_float),
                ("table_adam_eps", C.c_float), ("mlp_precision", C.c_int32), ("transfer_fmt", C.c_int32)]


class FfnStep(C.Structure):
    _fields_ = [("lr_f", C.c_float), ("lr_t", C.c_float), ("sh_mult", C.c_float),
                ("color_rel_lr", C.c_float), ("occ_strength", C.c_float), ("rng_u32", C.c_uint32),
                ("ray_offset", C.c_uint32), ("table_lr_t", C.c_float), ("spr", C.c_uint32), ("flags", C.c_uint32)]


STEP_TABLE_IMMEDIATE = 1
STEP_TABLE_APPLIED = 2
STATUS_NONFINITE, STATUS_TC_TIMEOUT, STATUS_DP_TIMEOUT = 1, 4, 8   # ffn_status bits
STAGE_SAMPLES = 1 << 20   # samples per group of the split tensor-core step (ffn_capi.cu)
ABI_VERSION = 6          # include/ffnerf.h FFN_ABI_VERSION


_VP = C.c_void_p
_SIGS = {
    "ffn_abi_version": (C.c_int, []),
    "ffn_last_error": (C.c_char_p, [_VP]),
    "ffn_create": (C.c_int, [C.POINTER(FfnConfig), C.c_int, C.POINTER(_VP)]),
    "ffn_destroy": (C.c_int, [_VP]),
    "ffn_buffer": (C.c_int, [_VP, C.c_int, C.POINTER(_VP), C.POINTER(C.c_size_t)]),
    "ffn_param_layout": (C.c_int, [C.POINTER(FfnConfig), _VP, _VP]),
    "ffn_forward_backward": (C.c_int, [_VP, _VP, _VP, _VP, C.c_uint32, C.POINTER(FfnStep), _VP]),
    "ffn_apply_updates": (C.c_int, [_VP, C.POINTER(FfnStep), _VP]),
    "ffn_train_step": (C.c_int, [_VP, _VP, _VP, _VP, C.c_uint32, C.POINTER(FfnStep), _VP]),
    "ffn_render": (C.c_int, [_VP, _VP, _VP, C.c_uint32, C.POINTER(FfnStep), _VP]),
    "ffn_occ_maintenance": (C.c_int, [_VP, C.c_uint32, C.c_uint32, _VP]),
    "ffn_grad_buffer": (C.c_int, [_VP, C.POINTER(_VP), C.POINTER(C.c_size_t)]),
    "ffn_occ_st_bytes": (C.c_int, [_VP, _VP, C.c_int, _VP]),
    "ffn_probe": (C.c_int, [_VP, _VP, _VP, _VP, C.c_uint32, C.POINTER(FfnStep), _VP] + [_VP] * 7 + [_VP]),
    "ffn_hash_encode": (C.c_int, [_VP, _VP, _VP, C.c_int64, _VP]),
    "ffn_hash_encode_bwd": (C.c_int, [_VP, _VP, _VP, C.c_int64, _VP]),
    "ffn_hash_encode_f16": (C.c_int, [_VP, _VP, _VP, _VP, C.c_int64, _VP]),
    "ffn_pack_x0": (C.c_int, [_VP, _VP, _VP, C.c_int64, _VP]),
    "ffn_mlp_bench": (C.c_int, [_VP, _VP, C.c_int64, _VP]),
    "ffn_mlp_bench_f16": (C.c_int, [_VP, _VP, C.c_int64, _VP]),
    "ffn_hash_encode_bwd_f16": (C.c_int, [_VP, _VP, _VP, _VP, C.c_int64, _VP]),
    "ffn_adam": (C.c_int, [_VP, _VP, _VP, _VP, C.c_int64, C.c_float, C.c_float, C.c_float, C.c_float, _VP]),
    "ffn_status": (C.c_int, [_VP, C.POINTER(C.c_uint32)]),
    "ffn_forward_backward_noalloc": (C.c_int, [C.POINTER(FfnConfig)] + [_VP] * 9 + [C.c_uint32, C.POINTER(FfnStep), _VP]),
    "ffn_dp_ipc_handles": (C.c_int, [_VP, _VP]),
    "ffn_dp_attach": (C.c_int, [_VP, C.c_int, C.c_int, _VP]),
    "ffn_dp_reduce_apply": (C.c_int, [_VP, C.POINTER(FfnStep), _VP]),
    "ffn_dp_set_wait_limit": (C.c_int, [_VP, C.c_uint32]),
    "ffn_bind_external": (C.c_int, [_VP, C.c_int, _VP, C.c_size_t]),
    "ffn_dp_attach_multicast": (C.c_int, [_VP, _VP, _VP]),
    "ffn_kernel_launches": (C.c_uint64, [_VP]),
    "ffn_probe_random_access": (C.c_int, [_VP, C.c_size_t, C.c_int, C.c_uint64, C.c_uint32, _VP]),
    "ffn_batch_generate": (C.c_int, [_VP, C.c_int, C.c_int, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_uint32, C.c_float, C.c_uint32, C.c_uint32, _VP, _VP, _VP, _VP, _VP, _VP]),
    "ffn_batch_errors": (C.c_int, [_VP, _VP, C.c_uint32, _VP, _VP, _VP]),
    "ffn_camera_rays": (C.c_int, [_VP, _VP, C.c_int, C.c_int, C.c_uint32, C.c_uint32, _VP, _VP]),
    "ffn_batch_feedback": (C.c_int, [_VP, _VP, C.c_int, C.c_int, C.c_int, C.c_int, _VP, _VP, _VP, _VP, C.c_uint32,
                                     _VP, C.c_double, C.c_int, C.c_int, _VP]),
}
EXPORTED = tuple(_SIGS)

_lib = None


def load_library(path: Path | None = None):
    """Loads libffnerf.so; raises if it is missing (build it with build_native.py)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: the CUDA library must be built (python build_native.py); "
                           "there is no CPU fallback")
    lib = C.CDLL(str(p))
    lib.ffn_abi_version.restype = C.c_int
    lib.ffn_abi_version.argtypes = []
    if lib.ffn_abi_version() != ABI_VERSION:     # before binding: an older build lacks newer symbols
        raise RuntimeError(f"{p} has ABI version {lib.ffn_abi_version()}, this module expects {ABI_VERSION}: "
                           "rebuild it (python build_native.py)")
    for name, (res, args) in _SIGS.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if path is None:
        _lib = lib
    return lib


MLP_PRECISIONS = {"fp32": 0, "fp16": 1}
TRANSFER_FORMATS = {"fp32": 32, "fp16": 16, "fp8": 8}   # ffn_config.transfer_fmt


def make_ffn_config(geom: dict, table_optimizer: int = 0, max_rays: int = 0, adam_beta1=0.9,
                    adam_beta2=0.999, adam_eps=1e-6, table_adam_eps=1e-15, mlp_precision: str = "fp32",
                    transfer_fmt: str = "fp32") -> FfnConfig:
    c = FfnConfig()
    for k in ("F", "ND", "NC", "spr", "G", "background"):
        setattr(c, k, int(geom[k]))
    c.table_optimizer, c.max_rays = int(table_optimizer), int(max_rays)
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
    c.adam_beta1, c.adam_beta2, c.adam_eps, c.table_adam_eps = adam_beta1, adam_beta2, adam_eps, table_adam_eps
    c.mlp_precision = MLP_PRECISIONS[mlp_precision]
    c.transfer_fmt = TRANSFER_FORMATS[transfer_fmt]
    return c


def make_step(lr_f=0.0, lr_t=0.0, sh_mult=1.0, color_rel_lr=1.0, occ_strength=0.0, rng_u32=0,
              ray_offset=0, table_lr_t=0.0, spr=0, table_immediate: bool = False,
              table_applied: bool = False) -> FfnStep:
    return FfnStep(float(np.float32(lr_f)), float(np.float32(lr_t)), float(np.float32(sh_mult)),
                   float(np.float32(color_rel_lr)), float(np.float32(occ_strength)), int(rng_u32) & 0xFFFFFFFF,
                   int(ray_offset) & 0xFFFFFFFF, float(np.float32(table_lr_t)), int(spr),
                   (STEP_TABLE_IMMEDIATE if table_immediate else 0) | (STEP_TABLE_APPLIED if table_applied else 0))


class _CudaArray:
    """Minimal __cuda_array_interface__ holder (zero-copy view of context memory)."""

    def __init__(self, ptr: int, n: int, dtype, owner):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": np.dtype(dtype).str,
                                         "data": (int(ptr), False), "version": 3, "strides": None}
        self._owner = owner


def _ptr(t) -> int | None:
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr() or None
    return int(t)


class Context:
    """One native context (parameters, optimizer state, table, occupancy grids, gradients)."""

    def __init__(self, geom: dict, device: int = 0, table_optimizer: int = 0, max_rays: int = 0,
                 adam_beta1=0.9, adam_beta2=0.999, adam_eps=1e-6, table_adam_eps=1e-15, mlp_precision: str = "fp32",
                 transfer_fmt: str = "fp32"):
        self.lib = load_library()
        self.geom = dict(geom)
        self.device = int(device)
        self.mlp_precision = mlp_precision
        self.cfg = make_ffn_config(geom, table_optimizer, max_rays, adam_beta1, adam_beta2, adam_eps, table_adam_eps,
                                   mlp_precision, transfer_fmt)
        h = _VP()
        rc = self.lib.ffn_create(C.byref(self.cfg), self.device, C.byref(h))
        if rc != FFN_OK:
            msg = self.lib.ffn_last_error(None).decode()
            raise (ValueError if rc == FFN_E_CONFIG else RuntimeError)(f"ffn_create failed ({rc}): {msg}")
        self.h = h
        off = np.zeros(18, np.int32)
        sz = np.zeros(18, np.int32)
        self.param_total = self.lib.ffn_param_layout(C.byref(self.cfg), off.ctypes.data, sz.ctypes.data)
        self.layout = {n: (int(o), int(s)) for n, o, s in zip(PARAM_NAMES, off, sz)}
        self._views = {}

    # -- lifetime
    def close(self):
        if getattr(self, "h", None):
            self.lib.ffn_destroy(self.h)
            self.h = None
            self._views = {}

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str):
        if rc != FFN_OK:
            msg = self.lib.ffn_last_error(self.h).decode()
            raise (ValueError if rc in (FFN_E_CONFIG, FFN_E_CAPACITY, FFN_E_NAME) else RuntimeError)(
                f"{what} failed ({rc}): {msg}")

    # -- buffers
    def buffer(self, buf_id: int) -> tuple[int, int]:
        p, n = _VP(), C.c_size_t()
        self._check(self.lib.ffn_buffer(self.h, buf_id, C.byref(p), C.byref(n)), "ffn_buffer")
        return int(p.value or 0), int(n.value)

    def tensor(self, buf_id: int):
        """A torch tensor aliasing one context buffer (no copy)."""
        import torch
        if buf_id not in self._views:
            ptr, nbytes = self.buffer(buf_id)
            dt = BUF_DTYPES[buf_id]
            n = nbytes // np.dtype(dt).itemsize
            if dt == np.uint32:
                holder = _CudaArray(ptr, n, np.int32, self)
                t = torch.as_tensor(holder, device=f"cuda:{self.device}")
            else:
                t = torch.as_tensor(_CudaArray(ptr, n, dt, self), device=f"cuda:{self.device}")
            self._views[buf_id] = t
        return self._views[buf_id]

    # -- steps (tensors are torch CUDA tensors on this device; stream = torch stream or None)
    @staticmethod
    def _stream(stream):
        if stream is None:
            import torch
            return torch.cuda.current_stream().cuda_stream
        return getattr(stream, "cuda_stream", stream)

    @property
    def launches(self) -> int:
        """Kernels this context has launched so far, as counted by the library."""
        return int(self.lib.ffn_kernel_launches(self.h)) if getattr(self, "h", None) else 0

    def forward_backward(self, rays, targets, out, n_rays: int, step: FfnStep, stream=None):
        self._check(self.lib.ffn_forward_backward(self.h, _ptr(rays), _ptr(targets), _ptr(out), int(n_rays),
                                                  C.byref(step), self._stream(stream)), "ffn_forward_backward")

    def apply_updates(self, step: FfnStep, stream=None):
        self._check(self.lib.ffn_apply_updates(self.h, C.byref(step), self._stream(stream)), "ffn_apply_updates")

    def train_step(self, rays, targets, out, n_rays: int, step: FfnStep, stream=None):
        self._check(self.lib.ffn_train_step(self.h, _ptr(rays), _ptr(targets), _ptr(out), int(n_rays),
                                            C.byref(step), self._stream(stream)), "ffn_train_step")

    # -- data-parallel exchange over NVLink peer memory
    def dp_ipc_handles(self) -> bytes:
        buf = (C.c_char * 192)()
        self._check(self.lib.ffn_dp_ipc_handles(self.h, buf), "ffn_dp_ipc_handles")
        return bytes(buf)

    def dp_attach(self, rank: int, world: int, handles: list[bytes]):
        blob = b"".join(handles)
        if len(blob) != 192 * world:
            raise ValueError("one 192-byte handle block per rank is required")
        buf = (C.c_char * len(blob)).from_buffer_copy(blob)
        self._check(self.lib.ffn_dp_attach(self.h, int(rank), int(world), buf), "ffn_dp_attach")

    def bind_external(self, buf_id: int, tensor):
        """Moves the table or gradient buffer into ``tensor`` (a CUDA float32 tensor this object keeps
        alive), copying the contents."""
        self._check(self.lib.ffn_bind_external(self.h, int(buf_id), _ptr(tensor), tensor.numel() * tensor.element_size()),
                    "ffn_bind_external")
        self._views.pop(buf_id, None)
        self._external = getattr(self, "_external", []) + [tensor]

    def dp_attach_multicast(self, mc_grads: int, mc_table: int):
        self._check(self.lib.ffn_dp_attach_multicast(self.h, C.c_void_p(int(mc_grads)), C.c_void_p(int(mc_table))),
                    "ffn_dp_attach_multicast")

    def dp_reduce_apply(self, step: FfnStep, stream=None):
        self._check(self.lib.ffn_dp_reduce_apply(self.h, C.byref(step), self._stream(stream)), "ffn_dp_reduce_apply")

    def dp_set_wait_limit(self, polls: int):
        """Polls (~1 us each) per cross-rank wait of the exchange before it sets STATUS_DP_TIMEOUT."""
        self._check(self.lib.ffn_dp_set_wait_limit(self.h, int(polls)), "ffn_dp_set_wait_limit")

    def render(self, rays, out, n_rays: int, step: FfnStep, stream=None):
        self._check(self.lib.ffn_render(self.h, _ptr(rays), _ptr(out), int(n_rays), C.byref(step),
                                        self._stream(stream)), "ffn_render")

    def occ_maintenance(self, decay_q24: int, seed: int, stream=None):
        self._check(self.lib.ffn_occ_maintenance(self.h, int(decay_q24), int(seed) & 0xFFFFFFFF,
                                                 self._stream(stream)), "ffn_occ_maintenance")

    def probe(self, rays, targets, out, n_rays: int, step: FfnStep, bypass=None, t=None, dt=None, idx=None,
              flags=None, sigma=None, rgb=None, trans=None, stream=None):
        self._check(self.lib.ffn_probe(self.h, _ptr(rays), _ptr(targets), _ptr(out), int(n_rays), C.byref(step),
                                       _ptr(bypass), _ptr(t), _ptr(dt), _ptr(idx), _ptr(flags), _ptr(sigma),
                                       _ptr(rgb), _ptr(trans), self._stream(stream)), "ffn_probe")

    def hash_encode(self, pts, enc, n: int, stream=None):
        self._check(self.lib.ffn_hash_encode(self.h, _ptr(pts), _ptr(enc), int(n), self._stream(stream)),
                    "ffn_hash_encode")

    def hash_encode_bwd(self, pts, denc, n: int, stream=None):
        self._check(self.lib.ffn_hash_encode_bwd(self.h, _ptr(pts), _ptr(denc), int(n), self._stream(stream)),
                    "ffn_hash_encode_bwd")

    def hash_encode_f16(self, table16, pts, enc16, n: int, stream=None):
        """Encoding from a caller-owned fp16 table (FFN_BUF_TABLE's layout) into fp16 enc16 [n, 16F]."""
        self._check(self.lib.ffn_hash_encode_f16(self.h, _ptr(table16), _ptr(pts), _ptr(enc16), int(n),
                                                 self._stream(stream)), "ffn_hash_encode_f16")

    def x0_tile_bytes(self, n: int) -> int:
        """Bytes of the packed operand tiles for n rows: an fp16 hi tile and an fp16 lo tile per
        128 rows of 16F features (n * 16F * 4)."""
        return int(n) * 16 * int(self.cfg.F) * 4

    def _check_tiles(self, x16, tiles, n: int):
        need = self.x0_tile_bytes(n)
        have = tiles.numel() * tiles.element_size()
        if have < need:
            raise ValueError(f"tiles holds {have} bytes; {n} rows need {need} (hi and lo fp16 tiles)")
        if x16 is not None and x16.numel() * x16.element_size() < int(n) * 16 * int(self.cfg.F) * 2:
            raise ValueError(f"x16 holds fewer than {n} rows of 16F fp16 features")

    def pack_x0(self, x16, tiles, n: int, stream=None):
        """Packs fp16 rows x16 [n, 16F] (n a multiple of 128) into the MLP kernels' operand tiles
        (x0_tile_bytes(n) bytes)."""
        self._check_tiles(x16, tiles, n)
        self._check(self.lib.ffn_pack_x0(self.h, _ptr(x16), _ptr(tiles), int(n), self._stream(stream)), "ffn_pack_x0")

    def mlp_bench(self, tiles, n: int, stream=None):
        """The MLP microbenchmark over packed inputs: gradients of sum 0.5 (rgb - 0.5)^2 added to the
        MLP part of BUF_GRADS (view direction (0.36, 0.48, 0.8), sh multiplier 1)."""
        self._check_tiles(None, tiles, n)
        self._check(self.lib.ffn_mlp_bench(self.h, _ptr(tiles), int(n), self._stream(stream)), "ffn_mlp_bench")

    def mlp_bench_f16(self, tiles, n: int, stream=None):
        """mlp_bench with plain fp16 operands (one MMA per product, no compensation)."""
        self._check_tiles(None, tiles, n)
        self._check(self.lib.ffn_mlp_bench_f16(self.h, _ptr(tiles), int(n), self._stream(stream)),
                    "ffn_mlp_bench_f16")

    def hash_encode_bwd_f16(self, grad16, pts, denc, n: int, stream=None):
        """Scatter-adds fp32 upstream gradients denc [n, 16F] into the caller-owned fp16 table grad16."""
        self._check(self.lib.ffn_hash_encode_bwd_f16(self.h, _ptr(grad16), _ptr(pts), _ptr(denc), int(n),
                                                     self._stream(stream)), "ffn_hash_encode_bwd_f16")

    def occ_st_bytes(self, buf, to_bytes: bool, stream=None):
        self._check(self.lib.ffn_occ_st_bytes(self.h, _ptr(buf), 1 if to_bytes else 0, self._stream(stream)),
                    "ffn_occ_st_bytes")

    def status(self) -> int:
        """Device status word since the last call (0 = every kernel completed normally)."""
        v = C.c_uint32()
        self._check(self.lib.ffn_status(self.h, C.byref(v)), "ffn_status")
        return int(v.value)

    def grad_buffer(self):
        p, n = _VP(), C.c_size_t()
        self._check(self.lib.ffn_grad_buffer(self.h, C.byref(p), C.byref(n)), "ffn_grad_buffer")
        return int(p.value), int(n.value)


def adam(p, g, m, v, n: int, lr_t: float, beta1: float, beta2: float, eps: float, stream=None):
    lib = load_library()
    rc = lib.ffn_adam(_ptr(p), _ptr(g), _ptr(m), _ptr(v), int(n), lr_t, beta1, beta2, eps, Context._stream(stream))
    if rc != FFN_OK:
        raise RuntimeError(f"ffn_adam failed ({rc})")


PROBE_GATHER, PROBE_RED = 0, 1


def probe_random_access(buf, mode: int, n_ops: int, seed: int = 1, stream=None):
    """n_ops fully random 8-byte loads (PROBE_GATHER) or vector reductions (PROBE_RED) over the
    device tensor ``buf`` (the ceiling probe of ffn_probe_random_access)."""
    lib = load_library()
    rc = lib.ffn_probe_random_access(_ptr(buf), buf.numel() * buf.element_size(), int(mode), int(n_ops),
                                     int(seed) & 0xFFFFFFFF, Context._stream(stream))
    if rc != FFN_OK:
        raise RuntimeError(f"ffn_probe_random_access failed ({rc}): {lib.ffn_last_error(None).decode()}")
