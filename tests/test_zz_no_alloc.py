"""ffn_forward_backward_noalloc (the entry point for callers that cannot allocate device memory)
against ffn_forward_backward on the same inputs, through the C ABI, on two calls in a row.

The caller owns every buffer; the library's static scratch array is shared by all calls, so the
second call (other rays, fewer CTAs, occupancy proposals on) also checks that nothing of the first
call's scratch leaks into it.  Tolerances are the fp32 parity tests' own: ray colours within
1e-4 absolute, gradients within rel-L2 1e-4 (both paths run the same kernel; only the order of
the table's atomic adds differs), occupancy proposals and the status word exact.
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


@pytest.mark.parametrize("prec", ["fp32", "fp16"])
def test_noalloc_matches_context_entry_point(prec):
    g = make_geometry(**GEOM)
    ctx = fn.Context(g, mlp_precision=prec)
    lib = fn.load_library()
    blob, table, occ = init_blob(g, 3), init_table(g, 3), init_occ(g, 3)
    ctx.tensor(fn.BUF_PARAMS).copy_(_cuda(blob))
    ctx.tensor(fn.BUF_TABLE).copy_(_cuda(table))
    ctx.tensor(fn.BUF_OCC_IN).copy_(_cuda(occ.view(np.int32)))
    # the caller's own buffers for the no-allocation entry point
    params, tab = _cuda(blob), _cuda(table)
    occ_in, occ_st = _cuda(occ.view(np.int32)), _cuda(occ.view(np.int32))
    grads = torch.full((table.size + blob.size,), 7.0, device="cuda")   # overwritten, not accumulated
    status = torch.full((1,), 5, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for call, (n, seed, occs) in enumerate(((512, 101, 0.0), (96, 202, 1.0))):
        rays, tg = _cuda(rays_toward_box(n, seed, radius=2.0, n_miss=4)), _cuda(targets(n, seed))
        step = fn.make_step(lr_f=1e-2, sh_mult=0.8, occ_strength=occs, rng_u32=seed)
        ctx.tensor(fn.BUF_GRADS).zero_()
        low = np.full(occ.size, 0x11111111, np.uint32).view(np.int32)   # proposals raise these nibbles
        ctx.tensor(fn.BUF_OCC_ST).copy_(_cuda(low))
        occ_st.copy_(_cuda(low))
        out_ref = torch.zeros((n, 4), device="cuda")
        ctx.forward_backward(rays, tg, out_ref, n, step)
        out = torch.zeros((n, 4), device="cuda")
        rc = lib.ffn_forward_backward_noalloc(C.byref(ctx.cfg), _ptr(params), _ptr(tab), _ptr(occ_in), _ptr(occ_st),
                                              _ptr(rays), _ptr(tg), _ptr(out), _ptr(grads), _ptr(status), n,
                                              C.byref(step), C.c_void_p(stream))
        assert rc == 0, lib.ffn_last_error(None)
        torch.cuda.synchronize()
        assert (out - out_ref)[:, :3].abs().max().item() < 1e-4, call
        g_ref = ctx.tensor(fn.BUF_GRADS).cpu().numpy()
        g_new = grads.cpu().numpy()
        assert rel_l2(g_new[:table.size], g_ref[:table.size]) < 1e-4, call
        assert rel_l2(g_new[table.size:], g_ref[table.size:]) < 1e-4, call
        assert torch.equal(occ_st, ctx.tensor(fn.BUF_OCC_ST)), call
        if occs:
            assert not torch.equal(occ_st, _cuda(low))
        assert int(status.item()) == 0
        assert torch.equal(tab, _cuda(table))          # deferred mode: the table is only read
    assert ctx.status() == 0
    ctx.close()
