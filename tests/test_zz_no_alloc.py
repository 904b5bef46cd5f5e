"""ffn_forward_backward_noalloc (the entry point for callers that cannot allocate device memory)
against ffn_forward_backward on the same inputs, through the C ABI, on calls in a row.

The caller owns every buffer; the library's static scratch array is shared by all calls, so the
second call (other rays, fewer CTAs, occupancy proposals on) also checks that nothing of the first
call's scratch leaks into it.  Tolerances are the fp32 parity tests' own: ray colours within
1e-4 absolute, gradients within rel-L2 1e-4 (both paths run the same arithmetic; only the order of
the table's atomic adds differs), occupancy proposals and the status word exact.

Further contracts:
  * the device's free memory is the same before and after a call (the entry point allocates
    nothing; checked from the second call on, after the CUDA driver has loaded the kernel);
  * with FFN_STEP_TABLE_IMMEDIATE the table changes by the SGD step of the deferred gradient
    (rel-L2 1e-3): the call is one 128-sample tile, whose table reads all precede its updates, so
    the immediate and the deferred schedule see the same table;
  * a non-finite target makes both entry points report the same status bits.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from _helpers import init_blob, init_occ, init_table, rays_toward_box, rel_l2, targets
from ffn_config import make_geometry
import ffn_native as fn

GEOM = dict(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _setup(prec, seed=3):
    g = make_geometry(**GEOM)
    ctx = fn.Context(g, mlp_precision=prec)
    blob, table, occ = init_blob(g, seed), init_table(g, seed), init_occ(g, seed)
    ctx.tensor(fn.BUF_PARAMS).copy_(_cuda(blob))
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    ctx.tensor(fn.BUF_OCC_IN).copy_(_cuda(occ.view(np.int32)))
    ctx.tensor(fn.BUF_OCC_ST).copy_(_cuda(occ.view(np.int32)))
    return g, ctx, blob, table, occ


def _noalloc(lib, ctx, params, tab, occ_in, occ_st, rays, tg, out, grads, status, n, step):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.ffn_forward_backward_noalloc(C.byref(ctx.cfg), _ptr(params), _ptr(tab), _ptr(occ_in), _ptr(occ_st),
                                            _ptr(rays), _ptr(tg), _ptr(out), _ptr(grads), _ptr(status), n,
                                            C.byref(step), C.c_void_p(stream))


@pytest.mark.parametrize("prec", ["fp32", "fp16"])
def test_noalloc_matches_context_entry_point(prec):
    g, ctx, blob, table, occ = _setup(prec)
    lib = fn.load_library()
    # the caller's own buffers for the no-allocation entry point
    params, tab = _cuda(blob), _cuda(table)
    occ_in, occ_st = _cuda(occ.view(np.int32)), _cuda(occ.view(np.int32))
    grads = torch.full((table.size + blob.size,), 7.0, device="cuda")   # overwritten, not accumulated
    status = torch.full((1,), 5, dtype=torch.int32, device="cuda")
    low = _cuda(np.full(occ.size, 0x11111111, np.uint32).view(np.int32))   # proposals raise these nibbles
    calls = ((512, 101, 0.0), (96, 202, 1.0), (300, 303, 0.0))
    for call, (n, seed, occs) in enumerate(calls):
        rays, tg = _cuda(rays_toward_box(n, seed, radius=2.0, n_miss=4)), _cuda(targets(n, seed))
        step = fn.make_step(lr_f=1e-2, sh_mult=0.8, occ_strength=occs, rng_u32=seed)
        ctx.tensor(fn.BUF_GRADS).zero_()
        ctx.tensor(fn.BUF_OCC_ST).copy_(low)
        occ_st.copy_(low)
        out_ref = torch.zeros((n, 4), device="cuda")
        ctx.forward_backward(rays, tg, out_ref, n, step)
        out = torch.zeros((n, 4), device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = _noalloc(lib, ctx, params, tab, occ_in, occ_st, rays, tg, out, grads, status, n, step)
        assert rc == 0, lib.ffn_last_error(None)
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        if call > 0:
            assert free_after == free_before, (call, free_before - free_after)
        assert (out - out_ref)[:, :3].abs().max().item() < 1e-4, call
        g_ref = ctx.tensor(fn.BUF_GRADS).cpu().numpy()
        g_new = grads.cpu().numpy()
        assert rel_l2(g_new[:table.size], g_ref[:table.size]) < 1e-4, call
        assert rel_l2(g_new[table.size:], g_ref[table.size:]) < 1e-4, call
        assert torch.equal(occ_st, ctx.tensor(fn.BUF_OCC_ST)), call
        if occs:
            assert not torch.equal(occ_st, low)
        assert int(status.item()) == 0
        assert torch.equal(tab, _cuda(table))          # deferred mode: the table is only read
    assert ctx.status() == 0
    ctx.close()


@pytest.mark.parametrize("prec", ["fp32", "fp16"])
def test_noalloc_immediate_table_update(prec):
    """FFN_STEP_TABLE_IMMEDIATE: the scatter adds -(lr 2^(-0.1 l)) 0.5 g w straight into the
    caller's table, which must equal the deferred gradient's SGD step.  Two rays (one tile): every
    table read of the call precedes its updates.  Table values of the reference's initial scale
    (1e-4), so that the change is far above the rounding of the table values."""
    g, ctx, blob, table, occ = _setup(prec, seed=5)
    table = init_table(g, 5, amp=1e-4)
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    lib = fn.load_library()
    n, seed, lr = 2, 77, 1e-2
    rays, tg = _cuda(rays_toward_box(n, seed, radius=2.0, n_miss=0)), _cuda(targets(n, seed))
    # deferred gradient from the context entry point, applied on the host side
    ctx.forward_backward(rays, tg, torch.zeros((n, 4), device="cuda"), n, fn.make_step(lr_f=lr, rng_u32=seed))
    gt = ctx.tensor(fn.BUF_GRADS).cpu().numpy()[:table.size].reshape(-1, g["F"])
    coef = np.zeros(gt.shape[0], np.float32)
    for lvl in range(16):
        lo, sz = g["level_offset"][lvl], 1 << g["level_log2"][lvl]
        coef[lo:lo + sz] = -(np.float32(lr) * np.float32(g["hash_lr_scale"][lvl])) * np.float32(0.5)
    expect = (coef[:, None] * gt).ravel()
    params, tab = _cuda(blob), _cuda(table)
    occ_in, occ_st = _cuda(occ.view(np.int32)), _cuda(occ.view(np.int32))
    grads = torch.zeros(table.size + blob.size, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros((n, 4), device="cuda")
    step = fn.make_step(lr_f=lr, rng_u32=seed, table_immediate=True)
    for call in range(2):
        tab.copy_(_cuda(table))
        rc = _noalloc(lib, ctx, params, tab, occ_in, occ_st, rays, tg, out, grads, status, n, step)
        assert rc == 0, lib.ffn_last_error(None)
        torch.cuda.synchronize()
        change = tab.cpu().numpy() - table
        assert np.abs(expect).max() > 0
        assert rel_l2(change, expect) < 1e-3, (call, rel_l2(change, expect))
        assert not grads[:table.size].any().item()     # immediate: the table gradient is not kept
        assert int(status.item()) == 0
    ctx.close()


@pytest.mark.parametrize("prec", ["fp32", "fp16"])
def test_noalloc_reports_nonfinite_like_context(prec):
    """A NaN target makes the MLP gradient non-finite: both entry points set the same status bit."""
    g, ctx, blob, table, occ = _setup(prec, seed=9)
    lib = fn.load_library()
    n, seed = 128, 55
    tg_np = targets(n, seed)
    tg_np[7, 1] = np.nan
    rays, tg = _cuda(rays_toward_box(n, seed, radius=2.0, n_miss=0)), _cuda(tg_np)
    step = fn.make_step(lr_f=1e-2, rng_u32=seed)
    assert ctx.status() == 0
    ctx.forward_backward(rays, tg, torch.zeros((n, 4), device="cuda"), n, step)
    torch.cuda.synchronize()
    st_ctx = ctx.status()
    params, tab = _cuda(blob), _cuda(table)
    occ_in, occ_st = _cuda(occ.view(np.int32)), _cuda(occ.view(np.int32))
    grads = torch.zeros(table.size + blob.size, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _noalloc(lib, ctx, params, tab, occ_in, occ_st, rays, tg, torch.zeros((n, 4), device="cuda"), grads, status,
                  n, step)
    assert rc == 0, lib.ffn_last_error(None)
    torch.cuda.synchronize()
    assert st_ctx & fn.STATUS_NONFINITE, st_ctx
    assert int(status.item()) == st_ctx
    ctx.close()
