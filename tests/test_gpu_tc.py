"""The tensor-core fused step (mlp_precision = fp16: compensated fp16 operand pairs in the
forward, fp16 backward operands, fp32 accumulation, tcgen05) against the CPU oracle, through the C
ABI, with the same tolerances as the fp32 path where the contract sets them.

Contracts:
  * bit-exact (same ray-phase code as the fp32 path): sample times / indices / run-start bits,
    occupancy proposals and transmittance when sigma/rgb are given;
  * forward: sigma and rgb within rel 1e-4 (the hi/lo forward is as close to fp32 as the fp32 path),
    ray colours within 1e-4 absolute of the fp32 oracle;
  * one step's gradients within rel-L2 1e-2 (the contract; measured 2e-5..6e-4 -- the backward's
    fp16 operand rounding);
  * 20 training steps: per-step loss within 1e-3 relative of the oracle, parameter and table
    updates within rel-L2 1e-2;
  * the device status word stays 0 (no tensor-core wait ran out).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from _helpers import init_blob, init_occ, init_table, rays_toward_box, rel_l2, targets
from ffn_config import REFERENCE_LEVEL_LOG2, make_geometry
from oracle import OrcStep, make_orc_config
import ffn_native as fn

GEOMS = {
    "cfg1": dict(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0),
    "f4nd2": dict(F=4, ND=2, NC=2, spr=64, G=32, log2_entries=list(REFERENCE_LEVEL_LOG2), rmax=1024.0,
                  box_min=(-3, -3, -3), box_max=(3, 3, 3)),
    "f2nd2_spr32": dict(F=2, ND=2, NC=2, spr=32, G=64, log2_entries=12, rmax=512.0),
    "f4nd1_spr16": dict(F=4, ND=1, NC=2, spr=16, G=64, log2_entries=13, rmax=2048.0),
    # the benchmarked geometry (BASELINE cfg2/cfg3): T = 2^19 per level, finest level 2048, 128^3 grid
    "cfg3": dict(F=2, ND=1, NC=2, spr=64, G=128, log2_entries=19, rmax=2048.0),
}
N_RAYS = {"cfg3": 2048}   # rays per call of the single-step tests (default 192)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _make(name, seed=0, n_rays=None, n_miss=4):
    if n_rays is None:
        n_rays = N_RAYS.get(name, 192)
    g = make_geometry(**GEOMS[name])
    ctx = fn.Context(g, mlp_precision="fp16")
    blob, table, occ = init_blob(g, seed), init_table(g, seed), init_occ(g, seed)
    ctx.tensor(fn.BUF_PARAMS).copy_(_cuda(blob))
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    ctx.tensor(fn.BUF_OCC_IN).copy_(_cuda(occ.view(np.int32)))
    ctx.tensor(fn.BUF_OCC_ST).copy_(_cuda(occ.view(np.int32)))
    rays = rays_toward_box(n_rays, seed, radius=6.0 if name == "f4nd2" else 2.0, n_miss=n_miss)
    return g, ctx, blob, table, occ, rays, targets(n_rays, seed)


@pytest.mark.parametrize("name", list(GEOMS))
def test_tc_sampler_exact_and_forward_close(oracle, name):
    g, ctx, blob, table, occ, rays, tg = _make(name)
    n, spr = rays.shape[0], g["spr"]
    seed = 31337
    dbg = {k: np.zeros(n * spr, np.float32) for k in ("t", "dt", "sigma")}
    dbg["idx"] = np.zeros(n * spr, np.int32)
    dbg["flags"] = np.zeros(n * 2, np.uint32)
    dbg["rgb"] = np.zeros(n * spr * 3, np.float32)
    out_o = np.zeros((n, 4), np.float32)
    oracle.forward_backward(make_orc_config(g), OrcStep(1e-3, 0.7, 0.0, seed, 1, 0), blob, table.copy(), occ.copy(),
                            occ.copy(), rays, tg, out_o, None, None, dbg)
    t = torch.zeros(n * spr, device="cuda"); dt = torch.zeros_like(t); sg = torch.zeros_like(t)
    idx = torch.zeros(n * spr, dtype=torch.int32, device="cuda")
    fl = torch.zeros(n * 2, dtype=torch.int32, device="cuda")
    rgb = torch.zeros(n * spr * 3, device="cuda")
    dout = torch.zeros((n, 4), device="cuda")
    ctx.probe(_cuda(rays), _cuda(tg), dout, n, fn.make_step(sh_mult=0.7, rng_u32=seed), t=t, dt=dt, idx=idx, flags=fl,
              sigma=sg, rgb=rgb)
    torch.cuda.synchronize()
    assert np.array_equal(t.cpu().numpy(), dbg["t"]) and np.array_equal(dt.cpu().numpy(), dbg["dt"])
    assert np.array_equal(idx.cpu().numpy(), dbg["idx"])
    assert np.array_equal(fl.cpu().numpy().view(np.uint32), dbg["flags"])
    hit = np.repeat((dbg["dt"].reshape(n, spr) > 0).any(1), spr)
    np.testing.assert_allclose(sg.cpu().numpy()[hit], dbg["sigma"][hit], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(rgb.cpu().numpy().reshape(-1, 3)[hit], dbg["rgb"].reshape(-1, 3)[hit], rtol=1e-4, atol=1e-6)
    assert np.abs(dout.cpu().numpy()[:, :3] - out_o[:, :3]).max() < 1e-4
    assert ctx.status() == 0


@pytest.mark.parametrize("name", ["cfg1", "f4nd2", "cfg3"])
def test_tc_occupancy_bypass_bit_exact(oracle, name):
    g, ctx, blob, table, occ, rays, tg = _make(name, seed=3)
    n, spr = rays.shape[0], g["spr"]
    rng = np.random.default_rng(5)
    bypass = np.zeros((n * spr, 4), np.float32)
    bypass[:, 0] = rng.exponential(20.0, n * spr).astype(np.float32)
    bypass[:, 1:] = rng.uniform(0, 1, (n * spr, 3)).astype(np.float32)
    occ_st_o = occ.copy()
    out_o = np.zeros((n, 4), np.float32)
    oracle.forward_backward(make_orc_config(g), OrcStep(0.0, 1.0, 1.0, 99, 1, 0), blob, table.copy(), occ.copy(),
                            occ_st_o, rays, tg, out_o, None, None, None, bypass)
    dout = torch.zeros((n, 4), device="cuda")
    ctx.probe(_cuda(rays), _cuda(tg), dout, n, fn.make_step(occ_strength=1.0, rng_u32=99), bypass=_cuda(bypass))
    torch.cuda.synchronize()
    assert (occ_st_o != occ).sum() > 0
    assert np.array_equal(ctx.tensor(fn.BUF_OCC_ST).cpu().numpy().view(np.uint32), occ_st_o)
    assert np.array_equal(dout.cpu().numpy(), out_o)


@pytest.mark.parametrize("name", list(GEOMS))
def test_tc_gradients_close(oracle, name):
    g, ctx, blob, table, occ, rays, tg = _make(name, seed=7)
    n = rays.shape[0]
    tgo = np.zeros(table.size, np.float32)
    mgo = np.zeros(blob.size, np.float32)
    out_o = np.zeros((n, 4), np.float32)
    oracle.forward_backward(make_orc_config(g), OrcStep(1e-2, 0.8, 0.0, 42, 1, 0), blob, table.copy(), occ.copy(),
                            occ.copy(), rays, tg, out_o, tgo, mgo)
    dout = torch.zeros((n, 4), device="cuda")
    ctx.forward_backward(_cuda(rays), _cuda(tg), dout, n, fn.make_step(lr_f=1e-2, sh_mult=0.8, rng_u32=42))
    torch.cuda.synchronize()
    grads = ctx.tensor(fn.BUF_GRADS).cpu().numpy()
    assert np.abs(dout.cpu().numpy()[:, :3] - out_o[:, :3]).max() < 1e-4
    assert rel_l2(grads[:table.size], tgo) < 1e-2, rel_l2(grads[:table.size], tgo)
    for pname, (off, sz) in ctx.layout.items():
        if sz:
            e = rel_l2(grads[table.size + off: table.size + off + sz], mgo[off:off + sz])
            assert e < 1e-2, (pname, e)
    assert ctx.status() == 0


def test_tc_training_run(oracle):
    g, ctx, blob, table, occ, rays_all, tg_all = _make("cfg1", seed=11, n_rays=128 * 20, n_miss=0)
    cfg = make_orc_config(g)
    b1, b2 = np.float32(0.9), np.float32(0.999)
    p, m, v, tab, oi, os_ = blob.copy(), np.zeros_like(blob), np.zeros_like(blob), table.copy(), occ.copy(), occ.copy()
    lo, lg = [], []
    n = 128
    for step in range(1, 21):
        rays, tg = rays_all[(step - 1) * n: step * n], tg_all[(step - 1) * n: step * n]
        lr_f = np.float32(5e-3)
        lr_t = np.float32(lr_f * np.sqrt(1.0 - b2 ** np.float32(step)) / (1.0 - b1 ** np.float32(step)))
        seed = (step * 2654435761) & 0xFFFFFFFF
        tgo = np.zeros(table.size, np.float32)
        mgo = np.zeros(blob.size, np.float32)
        out_o = np.zeros((n, 4), np.float32)
        oracle.forward_backward(cfg, OrcStep(lr_f, 1.0, 0.0, seed, 1, 0), p, tab, oi, os_, rays, tg, out_o, tgo, mgo)
        oracle.mlp_adam(cfg, p, mgo, m, v, lr_t, 0.5, b1, b2, np.float32(1e-6))
        oracle.table_apply(cfg, tab, tgo, lr_f)
        dout = torch.zeros((n, 4), device="cuda")
        ctx.train_step(_cuda(rays), _cuda(tg), dout, n, fn.make_step(lr_f=lr_f, lr_t=lr_t, color_rel_lr=0.5, rng_u32=seed))
        lo.append(float(np.mean((out_o[:, :3] - tg[:, :3]) ** 2)))
        lg.append(float(np.mean((dout.cpu().numpy()[:, :3] - tg[:, :3]) ** 2)))
    lo, lg = np.array(lo), np.array(lg)
    assert np.all(np.abs(lg - lo) <= 1e-3 * lo), np.abs(lg - lo) / lo
    assert rel_l2(ctx.tensor(fn.BUF_PARAMS).cpu().numpy() - blob, p - blob) < 1e-2
    assert rel_l2(ctx.tensor(fn.BUF_TABLE).cpu().numpy() - table, tab - table) < 1e-2
    assert ctx.status() == 0


def test_tc_render_close(oracle):
    g, ctx, blob, table, occ, rays, tg = _make("cfg1", seed=9)
    n = rays.shape[0]
    out_o = np.zeros((n, 4), np.float32)
    oracle.forward_backward(make_orc_config(g), OrcStep(0.0, 1.0, 0.0, 5, 0, 0), blob, table.copy(), occ.copy(),
                            occ.copy(), rays, np.zeros((n, 4), np.float32), out_o)
    dout = torch.zeros((n, 4), device="cuda")
    ctx.render(_cuda(rays), dout, n, fn.make_step(rng_u32=5))
    torch.cuda.synchronize()
    assert np.abs(dout.cpu().numpy() - out_o).max() < 1e-4
    assert not ctx.tensor(fn.BUF_GRADS).cpu().numpy().any()
