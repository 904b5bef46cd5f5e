"""The colour read-back of Nerf.step(return_output=True) and RayBatch.download_out, with the
reference's semantics (ffnerf_tools.py:372-385, 1533-1540): the read is enqueued and (out, event)
returned at once; `out` holds the step's colours once the event has completed (on return with
wait=True).

Contracts, on the same rays and seeds: the pipelined form (step i+1 enqueued before step i's colours
are taken; two pinned host arrays) returns the colours of the blocking form, step for step (within
1e-3 absolute: the Hogwild table update adds its float atomics in a different order from run to
run, and after five training steps at lr 5e-2 the two runs' colours drift apart by up to ~2e-4,
while the rays of consecutive steps differ completely, so their colours differ by more than
1e-2); a pageable array passed as `out` is filled when its event is
waited on, or when the queue finishes.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ffnerf_tools as ft
from _helpers import rays_toward_box, targets

N = 256


def _nerf(tmp_path, model_id):
    ctx = ft.Context([ft.Device(0)])
    queue = ft.CommandQueue(ctx)
    occ = ft.OccParams(G_occ=32, box_min=np.array([-1, -1, -1], np.float32), box_max=np.array([1, 1, 1], np.float32),
                       rho_min=np.float32(1.0), rho_max=np.float32(16.0)).finalize()
    nerf = ft.Nerf(ctx, queue, training_dir=tmp_path, model_id=model_id, transfer_fmt="fp32",
                   table_size_entries=16 << 12, f_per_level=2, occ=occ, rng_seed=5, background="random",
                   finest_resolution=512.0, nd=1, nc=2, mlp_precision="fp16", verbose=False)
    nerf.setup_buffers(N, 64)
    return nerf, ft.RayBatch.init(ctx, queue, N, 64)


def _upload(io, k):
    io.upload_rays(rays_toward_box(N, 70 + k, radius=2.0).view(ft.ray_dtype).reshape(-1))
    io.upload_targets(targets(N, 70 + k))


def test_pipelined_readback_matches_blocking(tmp_path):
    steps = 6
    a, io_a = _nerf(tmp_path / "a", "a")
    blocking = []
    for k in range(steps):
        _upload(io_a, k)
        out, ev = a.step(io_a, lr_f=5e-2, do_train=True, return_output=True, wait=True)
        blocking.append(out.copy())
    b, io_b = _nerf(tmp_path / "b", "b")
    slots = [torch.zeros((N, 4), dtype=torch.float32).pin_memory().numpy() for _ in range(2)]
    pipelined, pending = [], None
    for k in range(steps):
        io_b.out_host = slots[k % 2]
        _upload(io_b, k)
        out, ev = b.step(io_b, lr_f=5e-2, do_train=True, return_output=True)
        if pending is not None:
            pending[1].wait()
            pipelined.append(pending[0].copy())
        pending = (out, ev)
    pending[1].wait()
    pipelined.append(pending[0].copy())
    for k in range(steps):
        np.testing.assert_allclose(pipelined[k], blocking[k], rtol=0, atol=1e-3, err_msg=f"step {k}")
        if k:
            assert np.abs(blocking[k] - blocking[k - 1]).max() > 1e-2   # consecutive steps are told apart
    assert np.isfinite(blocking[-1]).all() and np.abs(blocking[-1][:, :3]).sum() > 0


def test_pageable_out_delivered_on_wait_or_finish(tmp_path):
    nerf, io = _nerf(tmp_path, "p")
    _upload(io, 0)
    nerf.step(io, lr_f=5e-2, do_train=True, return_output=False)
    ref, _ = io.download_out(np.empty((N, 4), np.float32), wait=True)
    page = np.full((N, 4), -1.0, np.float32)
    out, ev = io.download_out(page, wait=False)
    assert out is page
    ev.wait()
    assert np.array_equal(page, ref)
    page2 = np.full((N, 4), -1.0, np.float32)
    io.download_out(page2, wait=False)
    nerf.queue.finish()
    assert np.array_equal(page2, ref)
