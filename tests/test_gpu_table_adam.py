"""The opt-in Adam optimizer for the hash table (table_optimizer = 1; no reference counterpart:
the reference trains the table with its in-kernel SGD step) against the oracle's restatement
(orc_table_adam: the reference's Adam update, weight_update.cl:177-201, per level with step
lr_t * 2^(-0.1 l)).

Contracts:
  * given the same gradients and moments, the table, both moments and the cleared gradient are
    bit-exact (the Adam arithmetic is the MLP Adam's, which test_adam_bit_exact pins);
  * 10 training steps (fp32 MLP, deferred table gradients, Adam on table and MLP): per-step loss
    within 1e-3 relative of the oracle, parameters and table within rel-L2 1e-2.
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
B1, B2, EPS_T = np.float32(0.9), np.float32(0.999), np.float32(1e-15)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_table_adam_bit_exact(oracle):
    g = make_geometry(**GEOM)
    ctx = fn.Context(g, table_optimizer=1)
    n = ctx.tensor(fn.BUF_TABLE).numel()
    rng = np.random.default_rng(17)
    table = rng.uniform(-1e-1, 1e-1, n).astype(np.float32)
    grad = rng.normal(0.0, 1e-3, n).astype(np.float32)
    grad[rng.random(n) < 0.3] = 0.0                     # untouched entries: zero gradient
    m = rng.normal(0.0, 1e-4, n).astype(np.float32)
    v = np.abs(rng.normal(0.0, 1e-7, n)).astype(np.float32)
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    ctx.tensor(fn.BUF_GRADS)[:n].copy_(_cuda(grad))
    ctx.tensor(fn.BUF_TABLE_M).copy_(_cuda(m))
    ctx.tensor(fn.BUF_TABLE_V).copy_(_cuda(v))
    lr_t = np.float32(3e-3)
    ctx.apply_updates(fn.make_step(table_lr_t=lr_t))
    torch.cuda.synchronize()
    oracle.table_adam(make_orc_config(g), table, grad, m, v, lr_t, B1, B2, EPS_T)
    assert np.array_equal(ctx.tensor(fn.BUF_TABLE).cpu().numpy(), table)
    assert np.array_equal(ctx.tensor(fn.BUF_TABLE_M).cpu().numpy(), m)
    assert np.array_equal(ctx.tensor(fn.BUF_TABLE_V).cpu().numpy(), v)
    assert not ctx.tensor(fn.BUF_GRADS)[:n].any().item()
    assert ctx.status() == 0


def test_table_adam_training_run(oracle):
    g = make_geometry(**GEOM)
    ctx = fn.Context(g, table_optimizer=1)
    blob, table, occ = init_blob(g, 23), init_table(g, 23), init_occ(g, 23)
    ctx.tensor(fn.BUF_PARAMS).copy_(_cuda(blob))
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    ctx.tensor(fn.BUF_OCC_IN).copy_(_cuda(occ.view(np.int32)))
    ctx.tensor(fn.BUF_OCC_ST).copy_(_cuda(occ.view(np.int32)))
    cfg = make_orc_config(g)
    n, steps = 128, 10
    rays_all, tg_all = rays_toward_box(n * steps, 23, radius=2.0, n_miss=0), targets(n * steps, 23)
    p, pm, pv = blob.copy(), np.zeros_like(blob), np.zeros_like(blob)
    tab, tm, tv = table.copy(), np.zeros_like(table), np.zeros_like(table)
    oi, os_ = occ.copy(), occ.copy()
    lo, lg = [], []
    for step in range(1, steps + 1):
        rays, tg = rays_all[(step - 1) * n: step * n], tg_all[(step - 1) * n: step * n]
        lr_f = np.float32(5e-3)
        lr_t = np.float32(lr_f * np.sqrt(1.0 - B2 ** np.float32(step)) / (1.0 - B1 ** np.float32(step)))
        seed = (step * 2654435761) & 0xFFFFFFFF
        tgo, mgo = np.zeros(table.size, np.float32), np.zeros(blob.size, np.float32)
        out_o = np.zeros((n, 4), np.float32)
        oracle.forward_backward(cfg, OrcStep(lr_f, 1.0, 0.0, seed, 1, 0), p, tab, oi, os_, rays, tg, out_o, tgo, mgo)
        oracle.mlp_adam(cfg, p, mgo, pm, pv, lr_t, 0.5, B1, B2, np.float32(1e-6))
        oracle.table_adam(cfg, tab, tgo, tm, tv, lr_t, B1, B2, EPS_T)
        dout = torch.zeros((n, 4), device="cuda")
        ctx.train_step(_cuda(rays), _cuda(tg), dout, n,
                       fn.make_step(lr_f=lr_f, lr_t=lr_t, color_rel_lr=0.5, rng_u32=seed, table_lr_t=lr_t))
        lo.append(float(np.mean((out_o[:, :3] - tg[:, :3]) ** 2)))
        lg.append(float(np.mean((dout.cpu().numpy()[:, :3] - tg[:, :3]) ** 2)))
    lo, lg = np.array(lo), np.array(lg)
    assert np.all(np.abs(lg - lo) <= 1e-3 * lo), (np.abs(lg - lo) / lo).max()
    assert rel_l2(ctx.tensor(fn.BUF_PARAMS).cpu().numpy(), p) < 1e-2
    t_dev = ctx.tensor(fn.BUF_TABLE).cpu().numpy()
    assert rel_l2(t_dev, tab) < 1e-2, rel_l2(t_dev, tab)
    assert (t_dev != table).sum() > 1000                  # Adam moved the table
    assert ctx.status() == 0
