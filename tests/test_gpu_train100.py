"""100 training steps on the device against the deferred CPU oracle (every ray of a step reads the
step-start table; table gradients summed, then applied), for both table-update modes of the
device (deferred; immediate = the reference's Hogwild update inside the fused kernel) and both
MLP precisions.

Contracts (fp32 MLP / fp16 tensor-core MLP; the north-star tolerances for both):
  * per-step loss within 1e-3 relative of the oracle's, every step;
  * parameters and table within rel-L2 1e-2 of the oracle's after 100 steps;
  * gradients after 100 steps, evaluated on the device's own state (so that the comparison
    measures the kernels, not the divergence of two trajectories): MLP gradients within rel-L2
    1e-4 (fp32) / 1e-2 (fp16, measured ~1e-4: the backward's fp16 operand rounding); table
    gradients (deferred) within the same, or the step's table change
    (immediate) within 5e-2 of the deferred change: in immediate mode a ray's gather sees the
    updates of rays that scattered before it, which on this trained state moves the step's table
    change by about 2e-2 (rel-L2) from the deferred schedule's.
Two trajectories that differ only in float summation order drift apart chaotically under Adam:
the oracle against itself with another weight-gradient chunking (TILEK 64 instead of 236) ends
100 steps with parameters 4e-3 and MLP gradients 4e-2 apart (rel-L2) on this geometry.  That is
why the per-trajectory gradient is not compared, and the parameter bound is the oracle's own
spread, not bit-level.
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
TOL = {  # loss rel, params, table, gradients on the device state, immediate table change
    "fp32": (1e-3, 1e-2, 1e-2, 1e-4, 5e-2),
    "fp16": (1e-3, 1e-2, 1e-2, 1e-2, 5e-2),
}


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("prec", ["fp32", "fp16"])
@pytest.mark.parametrize("mode", ["deferred", "immediate"])
def test_training_100_steps(oracle, prec, mode):
    tol_loss, tol_p, tol_t, tol_g, tol_dt = TOL[prec]
    imm = mode == "immediate"
    n, steps = 128, 100
    g = make_geometry(**GEOM)
    ctx = fn.Context(g, mlp_precision=prec)
    blob, table, occ = init_blob(g, 11), init_table(g, 11), init_occ(g, 11)
    ctx.tensor(fn.BUF_PARAMS).copy_(_cuda(blob))
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    ctx.tensor(fn.BUF_OCC_IN).copy_(_cuda(occ.view(np.int32)))
    ctx.tensor(fn.BUF_OCC_ST).copy_(_cuda(occ.view(np.int32)))
    rays_all, tg_all = rays_toward_box(n * steps, 11, radius=2.0, n_miss=0), targets(n * steps, 11)
    cfg = make_orc_config(g)
    b1, b2 = np.float32(0.9), np.float32(0.999)
    p, m, v, tab, oi, os_ = blob.copy(), np.zeros_like(blob), np.zeros_like(blob), table.copy(), occ.copy(), occ.copy()
    lo, lg = [], []
    for step in range(1, steps + 1):
        rays, tg = rays_all[(step - 1) * n: step * n], tg_all[(step - 1) * n: step * n]
        lr_f = np.float32(5e-3)
        lr_t = np.float32(lr_f * np.sqrt(1.0 - b2 ** np.float32(step)) / (1.0 - b1 ** np.float32(step)))
        seed = (step * 2654435761) & 0xFFFFFFFF
        ost = OrcStep(lr_f, 1.0, 0.0, seed, 1, 0)
        tgo, mgo = np.zeros(table.size, np.float32), np.zeros(blob.size, np.float32)
        out_o = np.zeros((n, 4), np.float32)
        oracle.forward_backward(cfg, ost, p, tab, oi, os_, rays, tg, out_o, tgo, mgo)
        oracle.mlp_adam(cfg, p, mgo, m, v, lr_t, 0.5, b1, b2, np.float32(1e-6))
        oracle.table_apply(cfg, tab, tgo, lr_f)
        st = fn.make_step(lr_f=lr_f, lr_t=lr_t, color_rel_lr=0.5, rng_u32=seed, table_immediate=imm)
        dout = torch.zeros((n, 4), device="cuda")
        if step < steps:
            ctx.train_step(_cuda(rays), _cuda(tg), dout, n, st)
        else:
            # the last step's gradients against the oracle on the device's own state
            p_dev, t_dev = ctx.tensor(fn.BUF_PARAMS).cpu().numpy(), ctx.tensor(fn.BUF_TABLE).cpu().numpy()
            tgs, mgs = np.zeros(table.size, np.float32), np.zeros(blob.size, np.float32)
            oracle.forward_backward(cfg, ost, p_dev, t_dev.copy(), occ.copy(), occ.copy(), rays, tg,
                                    np.zeros((n, 4), np.float32), tgs, mgs)
            ctx.forward_backward(_cuda(rays), _cuda(tg), dout, n, st)
            grads = ctx.tensor(fn.BUF_GRADS).cpu().numpy()
            assert rel_l2(grads[table.size:], mgs) < tol_g, rel_l2(grads[table.size:], mgs)
            if imm:
                t_after = ctx.tensor(fn.BUF_TABLE).cpu().numpy()
                t_exp = t_dev.copy()
                oracle.table_apply(cfg, t_exp, tgs, lr_f)
                assert rel_l2(t_after - t_dev, t_exp - t_dev) < tol_dt, rel_l2(t_after - t_dev, t_exp - t_dev)
            else:
                assert rel_l2(grads[:table.size], tgs) < tol_g, rel_l2(grads[:table.size], tgs)
            ctx.apply_updates(st)
        lo.append(float(np.mean((out_o[:, :3] - tg[:, :3]) ** 2)))
        lg.append(float(np.mean((dout.cpu().numpy()[:, :3] - tg[:, :3]) ** 2)))
    lo, lg = np.array(lo), np.array(lg)
    assert np.all(np.abs(lg - lo) <= tol_loss * lo), (np.abs(lg - lo) / lo).max()
    p_g, tab_g = ctx.tensor(fn.BUF_PARAMS).cpu().numpy(), ctx.tensor(fn.BUF_TABLE).cpu().numpy()
    assert rel_l2(p_g, p) < tol_p, rel_l2(p_g, p)
    assert rel_l2(tab_g, tab) < tol_t, rel_l2(tab_g, tab)
    assert ctx.status() == 0
