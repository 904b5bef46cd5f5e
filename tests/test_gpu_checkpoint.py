"""Asynchronous checkpointing of a model training on the device (Nerf.save(async_write=True)).

Contracts: the file holds the state at the point of the save in the queue's order, even though
training steps run while it is read back and written; it loads into a fresh Nerf (and with np.load,
as the reference's loader does) with table, parameters, Adam moments and occupancy grids bit-exact.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ffn_native as fn
import ffnerf_tools as ft
from _helpers import rays_toward_box, targets


def _nerf(tmp_path, model_id):
    ctx = ft.Context([ft.Device(0)])
    queue = ft.CommandQueue(ctx)
    occ = ft.OccParams(G_occ=32, box_min=np.array([-1, -1, -1], np.float32), box_max=np.array([1, 1, 1], np.float32),
                       rho_min=np.float32(1.0), rho_max=np.float32(16.0)).finalize()
    return ft.Nerf(ctx, queue, training_dir=tmp_path, model_id=model_id, transfer_fmt="fp32",
                   table_size_entries=16 << 12, f_per_level=2, occ=occ, rng_seed=5, background="random",
                   finest_resolution=512.0, nd=1, nc=2, mlp_precision="fp16", verbose=False)


def test_async_save_captures_state_at_save_point(tmp_path):
    nerf = _nerf(tmp_path, "ck")
    n = 256
    io = ft.RayBatch.init(nerf.ctx, nerf.queue, n, 64)
    nerf.setup_buffers(n, 64)

    def step(k):
        io.upload_rays(rays_toward_box(n, 40 + k, radius=2.0).view(ft.ray_dtype).reshape(-1))
        io.upload_targets(targets(n, 40 + k))
        nerf.step(io, lr_f=5e-2, do_train=True, return_output=False, occ_update_strength=1.0)

    for k in range(3):
        step(k)
    path = nerf.save(min_new_file_seconds=0, async_write=True)
    nat = nerf.native
    nerf.queue.finish()
    at_save = {i: nat.tensor(i).cpu().numpy().copy() for i in (fn.BUF_TABLE, fn.BUF_PARAMS, fn.BUF_ADAM_M,
                                                                fn.BUF_OCC_IN, fn.BUF_OCC_ST)}
    for k in range(3, 6):                       # training continues while the file is written
        step(k)
    nerf.wait_saved()
    nerf.queue.finish()
    assert not np.array_equal(nat.tensor(fn.BUF_TABLE).cpu().numpy(), at_save[fn.BUF_TABLE])
    data = np.load(path, allow_pickle=False)
    assert np.array_equal(data["table_i"].view(np.float32), at_save[fn.BUF_TABLE])
    other = _nerf(tmp_path, "ck2")
    other.load_latest("ck")
    other.setup_buffers(n, 64)
    assert np.array_equal(other.native.tensor(fn.BUF_TABLE).cpu().numpy(), at_save[fn.BUF_TABLE])
    assert np.array_equal(other.native.tensor(fn.BUF_PARAMS).cpu().numpy(), at_save[fn.BUF_PARAMS])
    assert np.array_equal(other.native.tensor(fn.BUF_ADAM_M).cpu().numpy(), at_save[fn.BUF_ADAM_M])
    assert np.array_equal(other.native.tensor(fn.BUF_OCC_IN).cpu().numpy(), at_save[fn.BUF_OCC_IN])
    assert np.array_equal(other.native.tensor(fn.BUF_OCC_ST).cpu().numpy(), at_save[fn.BUF_OCC_ST])
    assert int(data["steps_trained"]) == 3
