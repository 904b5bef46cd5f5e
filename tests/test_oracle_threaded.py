"""The threaded deferred-update oracle of the end-of-training PSNR test (OracleModel: a step's rays
split into chunks on host threads, gradients summed, occupancy proposals merged by nibble maximum)
against the same oracle on one thread: parameters and table equal up to float summation order
(rel-L2 1e-5), occupancy grids identical, including steps with live occupancy updates."""
import tempfile

import numpy as np
import pytest

pytest.importorskip("torch")

import trainer
from _helpers import rays_toward_box, rel_l2, targets
from ffn_config import param_layout
from test_gpu_psnr_reference import OracleModel, nibble_max


def test_nibble_max():
    a = np.array([0x0123ABCD, 0xFFFFFFFF, 0], np.uint32)
    b = np.array([0x3210DCBA, 0x00000000, 0x11111111], np.uint32)
    assert nibble_max(a, b).tolist() == [0x3223DCCD, 0xFFFFFFFF, 0x11111111]


def test_threaded_oracle_matches_single_thread():
    models = [OracleModel(trainer.synthetic_nerf("cfg1", "fp32", 0, tempfile.mkdtemp(), host_only=True), threads=t)
              for t in (1, 4)]
    off = param_layout(2, 1, 2)[0]["bd_out"][0]
    for m in models:                              # a sparse grid and a dense field, so that proposals raise nibbles
        m.occ_in[:] = 0x11111111
        m.occ_st[:] = 0x11111111
        m.blob[off] = 5.0
    n = 96
    for k in range(4):
        rays, tg = rays_toward_box(n, 70 + k, radius=2.0, n_miss=3), targets(n, 70 + k)
        occ_s = 1.0 if k >= 2 else 0.0          # proposals live in the last two steps
        for m in models:
            m.step(rays, tg, 5e-3, 1.0, 1.0, occ_s)
    a, b = models
    assert rel_l2(b.table, a.table) < 1e-5
    assert rel_l2(b.blob, a.blob) < 1e-5
    assert np.array_equal(a.occ_st, b.occ_st) and np.array_equal(a.occ_in, b.occ_in)
    init = np.full_like(a.occ_st, 0x11111111)
    assert not np.array_equal(a.occ_st, init), "the occupancy merge was not exercised"
