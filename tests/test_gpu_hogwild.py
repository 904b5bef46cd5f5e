"""Immediate (Hogwild) hash-table updates -- the reference's own semantics, where every sample's
table gradient is added into the table as -lr * 2^(-0.1 l) * 0.5 * g * w while other rays of the
same step read it (ffnerf_OG.cl:2155-2168) -- against the CPU oracle in sequential table mode
(rays in order, each update applied at once: one legal schedule of the same race).

Contracts:
  * one step: the table change matches the oracle's within rel-L2 1e-3 (both MLP precisions), the
    gradient buffer's table part stays zero;
  * an Adam table refuses immediate updates.
The table starts at amplitude 1e-3 (the reference initialises at 1e-4).  At the helpers' usual 0.1
the comparison measures float rounding, not the update: every one of a step's many small adds into
an entry of size ~0.1 rounds to that entry's ulp, so the reference's per-sample adds (the oracle's
sequential mode) and one exact sum of the same contributions (its deferred mode) end 1.2e-2 apart
(rel-L2 of the change), and the device, which sums the contributions of a cell's samples before one
add, sits between the two.  At 1e-3 that rounding is 1e-4 of the change and the remaining
difference is the schedule's: which adds a gather sees (the oracle's sequential mode in forward and
in reverse ray order: 4.8e-4 apart).
(100-step training runs in this mode are in test_gpu_train100.py.)
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from _helpers import init_blob, init_occ, init_table, rays_toward_box, rel_l2, targets
from ffn_config import make_geometry
from oracle import OrcStep, make_orc_config
import ffn_native as fn

GEOM = dict(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0)
TOL = {"fp32": (1e-3,), "fp16": (1e-3,)}
MLP_GRAD_TOL = {"fp32": 1e-3, "fp16": 1e-2}


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _make(prec, seed, n_rays, table_amp=1e-1):
    g = make_geometry(**GEOM)
    ctx = fn.Context(g, mlp_precision=prec)
    blob, table, occ = init_blob(g, seed), init_table(g, seed, table_amp), init_occ(g, seed)
    ctx.tensor(fn.BUF_PARAMS).copy_(_cuda(blob))
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    ctx.tensor(fn.BUF_OCC_IN).copy_(_cuda(occ.view(np.int32)))
    ctx.tensor(fn.BUF_OCC_ST).copy_(_cuda(occ.view(np.int32)))
    rays = rays_toward_box(n_rays, seed, radius=2.0, n_miss=0)
    return g, ctx, blob, table, occ, rays, targets(n_rays, seed)


@pytest.mark.parametrize("prec", ["fp32", "fp16"])
def test_immediate_one_step(oracle, prec):
    g, ctx, blob, table, occ, rays, tg = _make(prec, 21, 128, table_amp=1e-3)
    n, lr_f, seed = rays.shape[0], np.float32(1e-2), 4242
    cfg = make_orc_config(g, table_mode=1)
    tab_o = table.copy()
    out_o = np.zeros((n, 4), np.float32)
    mgo = np.zeros(blob.size, np.float32)
    oracle.forward_backward(cfg, OrcStep(lr_f, 1.0, 0.0, seed, 1, 0), blob, tab_o, occ.copy(), occ.copy(), rays, tg,
                            out_o, None, mgo)
    assert not np.array_equal(tab_o, table)
    dout = torch.zeros((n, 4), device="cuda")
    ctx.forward_backward(_cuda(rays), _cuda(tg), dout, n, fn.make_step(lr_f=lr_f, rng_u32=seed, table_immediate=True))
    torch.cuda.synchronize()
    tab_g = ctx.tensor(fn.BUF_TABLE).cpu().numpy()
    assert rel_l2(tab_g - table, tab_o - table) < TOL[prec][0], rel_l2(tab_g - table, tab_o - table)
    grads = ctx.tensor(fn.BUF_GRADS).cpu().numpy()
    assert not grads[:table.size].any()
    assert rel_l2(grads[table.size:], mgo) < MLP_GRAD_TOL[prec]
    assert np.abs(dout.cpu().numpy()[:, :3] - out_o[:, :3]).max() < 1e-3
    assert ctx.status() == 0


def test_immediate_needs_sgd_table():
    g = make_geometry(**GEOM)
    ctx = fn.Context(g, table_optimizer=1)   # Adam
    rays = _cuda(rays_toward_box(8, 0))
    with pytest.raises(ValueError):
        ctx.forward_backward(rays, _cuda(targets(8, 0)), torch.zeros((8, 4), device="cuda"), 8,
                             fn.make_step(lr_f=1e-3, table_immediate=True))
