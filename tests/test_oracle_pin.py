"""The oracle against the reference kernels compiled from their own OpenCL sources.

oracle/_ref/libffnref_<variant>.so runs ffnerf_train_step, update_ffnerf_oneWG and
occ_nibble_decay_write_both_q24 unmodified on CPU fibers (oracle/ref_build.py).  With the C
library's exp/pow (math mode 1), one OS thread (work-groups in ray order) and the oracle's
sequential table mode (the Hogwild schedule that order produces), every output is bit-identical:
ray colours, the table after the in-kernel SGD adds, occupancy proposals, and all MLP parameters
and Adam moments after the weight update -- also with the reference's fp16 and fp8 transfer
formats, where the weight update reads the staged activations and deltas quantised.  Skipped where
the reference library was not built."""
import numpy as np
import pytest

from _helpers import init_blob, init_occ, init_table, rays_toward_box, targets
from ffn_config import REFERENCE_LEVEL_LOG2, make_geometry, param_layout, param_shapes
from oracle import OrcStep, RefKernels, make_orc_config, ref_so

VARIANTS = {
    "cfg1": dict(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0),
    "default": dict(F=4, ND=2, NC=2, spr=64, G=32, log2_entries=list(REFERENCE_LEVEL_LOG2), rmax=1024.0,
                    box_min=(-3, -3, -3), box_max=(3, 3, 3)),
    "cfg3": dict(F=2, ND=1, NC=2, spr=64, G=128, log2_entries=19, rmax=2048.0),
    # the reference's fp16 / fp8 transfer formats of the activations and deltas the weight update reads
    "cfg1_t16": dict(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0),
    "cfg1_t8": dict(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0),
}
TRANSFER = {"cfg1_t16": 16, "cfg1_t8": 8}


def _split(blob, geom):
    lay, _ = param_layout(geom["F"], geom["ND"], geom["NC"])
    shapes = param_shapes(geom["F"], geom["ND"], geom["NC"])
    out = {}
    for n, (off, sz) in lay.items():
        out[n] = blob[off:off + sz].copy() if n in shapes else np.zeros(0, np.float32)
    return out


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("occ_strength,sh_mult", [(0.0, 0.0), (1.0, 1.0)])
def test_oracle_matches_compiled_reference(oracle, variant, occ_strength, sh_mult):
    if not ref_so(variant).exists():
        pytest.skip("reference kernels not compiled here (needs the reference checkout)")
    ref = RefKernels(variant)
    g = make_geometry(**VARIANTS[variant])
    assert (ref.F, ref.ND, ref.NC) == (g["F"], g["ND"], g["NC"])
    n = 40
    rays = rays_toward_box(n, 21, radius=6.0 if variant == "default" else 2.0, n_miss=3)
    tg = targets(n, 21)
    blob = init_blob(g, 21, sigma_bias=2.0)
    table0 = init_table(g, 21)
    occ0 = init_occ(g, 21, mask=0x33333333)
    lr, seed = np.float32(5e-2), 2024
    # compiled reference, one thread
    params = {k: v.view(np.int32).copy() for k, v in _split(blob, g).items()}
    tab_r = table0.copy()
    out_r = np.zeros((n, 4), np.float32)
    occ_st_r = occ0.copy()
    scr = ref.alloc_scratch(n * g["spr"])
    ref.train(params, tab_r.view(np.int32), rays, tg, out_r, scr, occ0.copy(), occ_st_r, g, float(lr), sh_mult,
              occ_strength, seed, True, 1)
    m = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
    v_ = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
    ref.weight_update(params, m, v_, scr, n * g["spr"], 1e-3, 0.15, 0.9, 0.999, 1e-6)
    # oracle: libm math, sequential table updates
    cfg = make_orc_config(g, math_mode=1, table_mode=1, transfer_fmt=TRANSFER.get(variant, 32))
    tab_o = table0.copy()
    out_o = np.zeros((n, 4), np.float32)
    occ_st_o = occ0.copy()
    mg = np.zeros(blob.size, np.float32)
    oracle.forward_backward(cfg, OrcStep(lr, sh_mult, occ_strength, seed, 1, 0), blob, tab_o, occ0.copy(), occ_st_o,
                            rays, tg, out_o, None, mg)
    p_o, m_o, v_o = blob.copy(), np.zeros_like(blob), np.zeros_like(blob)
    oracle.mlp_adam(cfg, p_o, mg, m_o, v_o, np.float32(1e-3), np.float32(0.15), np.float32(0.9), np.float32(0.999),
                    np.float32(1e-6))
    assert np.array_equal(out_r, out_o)
    assert np.array_equal(tab_r, tab_o) and (tab_r != table0).sum() > 1000
    assert np.array_equal(occ_st_r, occ_st_o)
    if occ_strength > 0:
        assert (occ_st_r != occ0).sum() > 0
    lay, _ = param_layout(g["F"], g["ND"], g["NC"])
    for name, (off, sz) in lay.items():
        if sz:
            assert np.array_equal(params[name].view(np.float32), p_o[off:off + sz]), name
            assert np.array_equal(m[name], m_o[off:off + sz]), name
            assert np.array_equal(v_[name], v_o[off:off + sz]), name


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_decay_matches_compiled_reference(oracle, variant):
    if not ref_so(variant).exists():
        pytest.skip("reference kernels not compiled here")
    ref = RefKernels(variant)
    rng = np.random.default_rng(8)
    a = rng.integers(0, 2**32, 40000, dtype=np.uint64).astype(np.uint32)
    b = a.copy()
    sel = rng.random(a.size) < 0.4
    b[sel] = rng.integers(0, 2**32, sel.sum(), dtype=np.uint64).astype(np.uint32)
    for dq, seed in ((15099494, 3), (1 << 24, 4), (0, 5)):
        a1, b1, a2, b2 = a.copy(), b.copy(), a.copy(), b.copy()
        ref.decay(a1, b1, dq, seed)
        oracle.decay(a2, b2, dq, seed)
        assert np.array_equal(a1, a2) and np.array_equal(b1, b2)


@pytest.mark.parametrize("variant", ["cfg1", "default"])
def test_reference_lockstep_matches_deferred_oracle(oracle, variant):
    """The reference kernels with every work-group of the step in lockstep (barrier interval by
    barrier interval, on 4 OS threads: the schedule of a device that holds the whole batch, where
    each ray's table reads precede every ray's in-kernel table update) against the oracle's deferred
    table mode: ray colours, occupancy proposals and the weight update + Adam are bit-identical; the
    tables after the step (the reference adds each -lr 2^(-0.1 l) 0.5 g w with a CAS loop, the oracle
    sums g w per entry first) agree within float rounding of the table values.  The near-sequential schedule (one work-group at a
    time, rays in order) gives other colours."""
    if not ref_so(variant).exists():
        pytest.skip("reference kernels not compiled here")
    ref = RefKernels(variant)
    g = make_geometry(**VARIANTS[variant])
    n = 48
    rays = rays_toward_box(n, 31, radius=6.0 if variant == "default" else 2.0, n_miss=3)
    tg = targets(n, 31)
    blob = init_blob(g, 31, sigma_bias=2.0)
    table0 = init_table(g, 31)
    occ0 = init_occ(g, 31, mask=0x33333333)
    lr, seed = np.float32(5e-2), 77
    runs = {}
    for mode in ("lockstep", "sequential"):
        params = {k: v.view(np.int32).copy() for k, v in _split(blob, g).items()}
        tab, out, occ_st = table0.copy(), np.zeros((n, 4), np.float32), occ0.copy()
        scr = ref.alloc_scratch(n * g["spr"])
        ref.train(params, tab.view(np.int32), rays, tg, out, scr, occ0.copy(), occ_st, g, float(lr), 1.0, 1.0, seed,
                  True, 4 if mode == "lockstep" else 1, lockstep=mode == "lockstep")
        m = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
        v_ = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
        ref.weight_update(params, m, v_, scr, n * g["spr"], 1e-3, 0.15, 0.9, 0.999, 1e-6)
        runs[mode] = (params, m, v_, tab, out, occ_st)
    cfg = make_orc_config(g, math_mode=1, table_mode=0)
    tab_o, out_o, occ_st_o = table0.copy(), np.zeros((n, 4), np.float32), occ0.copy()
    tgr, mg = np.zeros_like(table0), np.zeros(blob.size, np.float32)
    oracle.forward_backward(cfg, OrcStep(lr, 1.0, 1.0, seed, 1, 0), blob, tab_o, occ0.copy(), occ_st_o, rays, tg, out_o,
                            tgr, mg)
    oracle.table_apply(cfg, tab_o, tgr, lr)
    p_o, m_o, v_o = blob.copy(), np.zeros_like(blob), np.zeros_like(blob)
    oracle.mlp_adam(cfg, p_o, mg, m_o, v_o, np.float32(1e-3), np.float32(0.15), np.float32(0.9), np.float32(0.999),
                    np.float32(1e-6))
    params, m, v_, tab, out, occ_st = runs["lockstep"]
    assert np.array_equal(out, out_o)
    assert np.array_equal(occ_st, occ_st_o) and (occ_st != occ0).sum() > 0
    lay, _ = param_layout(g["F"], g["ND"], g["NC"])
    for name, (off, sz) in lay.items():
        if sz:
            assert np.array_equal(params[name].view(np.float32), p_o[off:off + sz]), name
            assert np.array_equal(m[name], m_o[off:off + sz]) and np.array_equal(v_[name], v_o[off:off + sz]), name
    # each of the reference's in-kernel adds rounds to the table value's ulp (~1e-8 here, about the size of
    # one add), so the two tables agree to float rounding of the table, not of the change
    assert (tab_o != table0).sum() > 1000
    assert np.linalg.norm((tab - tab_o).astype(np.float64)) <= 1e-6 * np.linalg.norm(table0.astype(np.float64))
    assert not np.array_equal(runs["sequential"][4], out)
