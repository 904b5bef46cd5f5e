"""This repository's host module against fixtures produced by the reference's own host code
(tests/golden/make_golden.py): parameter initialisation, per-step seeds, Adam bias correction,
occupancy-maintenance schedule, ray generation and trainer schedules -- all bit-exact."""
from pathlib import Path

import numpy as np
import pytest

import ffnerf_tools as ft
import schedules

G = Path(__file__).resolve().parent / "golden"


def _nerf(tmp_path, F, nd, entries):
    occ = ft.OccParams(G_occ=8, box_min=np.array([-1, -1, -1], np.float32), box_max=np.array([1, 1, 1], np.float32),
                       rho_min=np.float32(1.0), rho_max=np.float32(16.0)).finalize()
    return ft.Nerf(None, None, training_dir=tmp_path, model_id="t", transfer_fmt="fp32", table_size_entries=entries,
                   f_per_level=F, occ=occ, rng_seed=777, nd=nd, nc=2)


@pytest.mark.parametrize("tag,F,nd,entries", [("f2nd1", 2, 1, 16 * 2 ** 10), ("f4nd2", 4, 2, 16 * 2 ** 9)])
def test_init_matches_reference(tmp_path, tag, F, nd, entries):
    gold = np.load(G / "golden_host_init.npz")
    nerf = _nerf(tmp_path, F, nd, entries)
    keys = {k.split("/", 1)[1] for k in gold.files if k.startswith(tag + "/")}
    assert keys == set(nerf.state_i32)
    for k in keys:
        assert np.array_equal(np.asarray(nerf.state_i32[k]), gold[f"{tag}/{k}"]), k


def test_step_scalars_match_reference(tmp_path):
    gold = np.load(G / "golden_host_steps.npz")
    nerf = _nerf(tmp_path, 2, 1, 16 * 2 ** 10)
    for i, step in enumerate(gold["step"]):
        nerf.steps_trained = int(step)
        assert np.uint32(nerf._get_rng_u32()) == gold["ff_seed"][i]
        assert nerf.lr_t(gold["ff_lr"][i]) == gold["wu_lr_t"][i]
        occ_s = float(gold["ff_occ"][i])
        due = nerf.maintenance_due(step, occ_s)
        assert due == (gold["dec_q24"][i] >= 0), step
        if due:
            assert nerf.decay_q24(occ_s) == gold["dec_q24"][i]
            assert gold["dec_seed"][i] == gold["ff_seed"][i]      # decay reuses the step seed
            assert gold["dec_n"][i] == 8 ** 3
    assert np.all(gold["wu_b1"] == ft.Nerf.ADAM_BETA1) and np.all(gold["wu_b2"] == ft.Nerf.ADAM_BETA2)
    assert np.all(gold["wu_eps"] == ft.Nerf.ADAM_EPS)
    assert np.all(gold["ff_do_train"] == 1) and np.all(gold["ff_spr"] == 64)


def test_rays_match_reference():
    g = np.load(G / "golden_rays.npz")
    flat = lambda r: np.ascontiguousarray(r).view(np.float32).reshape(-1, 8)
    W, H = int(g["W"]), int(g["H"])
    r, t = ft.rays_targets_from_indices(g["im"], g["u"], g["v"], g["Ims"], g["c2w"], W, H, K=g["K"])
    assert np.array_equal(flat(r), g["rays_k"]) and np.array_equal(t, g["tg_k"])
    r, t = ft.rays_targets_from_indices(g["im"], g["u"], g["v"], g["Ims"], g["c2w"], W, H, K=None)
    assert np.array_equal(flat(r), g["rays_nok"]) and np.array_equal(t, g["tg_nok"])
    r, _ = ft.rays_targets_from_indices(g["im"] % 2, g["u"], g["v"], g["Ims"][:2], g["c2w"][:2], W, H, K=g["Ks"])
    assert np.array_equal(flat(r), g["rays_perK"])
    assert np.array_equal(flat(ft.rays_from_rt_indices(g["c2w"][1], g["u"], g["v"], W, H, K=g["K"])), g["rays_rt"])
    assert np.array_equal(flat(ft.rays_from_rt_indices(g["c2w"][2], g["u"], g["v"], W, H, K=None)), g["rays_rt_nok"])


def test_review_rays_match_training_intrinsics():
    """The reference's own consistency check (tests/test_scene_workflow.py:64-72) on this module."""
    K = np.array([[40, 0, 10], [0, 40, 20], [0, 0, 1]], np.float32)
    poses = np.tile(np.eye(4), (2, 1, 1))
    poses[1, :3, 3] = [1, 2, 3]
    images = np.zeros((2, 80, 40, 3), np.float32)
    u, v = np.array([0, 19, 39]), np.array([0, 29, 79])
    training, _ = ft.rays_targets_from_indices(np.ones(3, np.int32), u, v, images, poses, 40, 80, K=K)
    review = ft.rays_from_rt_indices(poses[1], u, v, 40, 80, K=K)
    np.testing.assert_allclose(training["o"], review["o"])
    np.testing.assert_allclose(training["d"], review["d"], atol=1e-7)


def test_schedules_match_reference():
    g = np.load(G / "golden_schedules.npz")
    assert schedules.T_MID == int(g["T_MID"]) and schedules.LMBDA_BASE == float(g["LMBDA_BASE"])
    assert schedules.LR_FLOOR == float(g["LR_FLOOR"])
    for i, s in enumerate(g["steps"]):
        assert float(schedules.sh_multiplier_function(s)) == g["sh"][i]
        assert float(schedules.occ_u_multiplier_function(s)) == g["occ"][i]
        assert float(schedules.color_MLP_rel_lr_function(s)) == g["color"][i]


def test_checkpoint_roundtrip_reference_layout(tmp_path):
    """save() writes the reference's NPZ keys; load_latest() restores the state bit for bit."""
    nerf = _nerf(tmp_path, 2, 1, 16 * 2 ** 10)
    nerf.steps_trained = 17
    path = nerf.save(min_new_file_seconds=0)
    d = np.load(path)
    for k in ("timestamp", "model_id", "steps_trained", "transfer_fmt", "ND", "NC", "table_i", "table_size_entries",
              "table_f_per_level", "occ_grid_in_u32", "occ_grid_st_u32", "G_occ", "box_min", "box_max", "rho_min",
              "rho_max", "dt_min", "dt_max", "t_near_clip", "t_far_clip", "active_params"):
        assert k in d.files, k
    assert d["table_i"].dtype == np.int32 and d["occ_grid_in_u32"].dtype == np.uint32
    assert sorted(d["active_params"].tolist()) == sorted(["Wd_in", "Wd_out", "Wc_in", "Wc_01", "Wc_out",
                                                          "bd_0", "bd_out", "bc_0", "bc_1", "bc_out"])
    other = ft.Nerf(None, None, training_dir=tmp_path, model_id="t2", load_id="t", rng_seed=1)
    assert other.steps_trained == 17 and (other.ND, other.NC, other.f_per_level) == (1, 2, 2)
    for k, v in nerf.state_i32.items():
        assert np.array_equal(np.asarray(other.state_i32[k]).ravel(), np.asarray(v).ravel()), k


def test_checkpoint_written_by_reference_loads(tmp_path):
    """A checkpoint written by the reference's own Nerf.save (golden_ref_checkpoint.npz, from
    make_golden.py) loads through load_latest with every array, the geometry, the occupancy
    parameters and the step count; saving it again writes the same values under the same keys."""
    import shutil
    ref = np.load(G / "golden_ref_checkpoint.npz")
    mid = str(ref["model_id"])
    shutil.copy(G / "golden_ref_checkpoint.npz", tmp_path / f"{mid}_weights_20260101-000000.npz")
    nerf = ft.Nerf(None, None, training_dir=tmp_path, model_id="again", load_id=mid, rng_seed=1)
    assert nerf.steps_trained == int(ref["steps_trained"])
    assert (nerf.ND, nerf.NC, nerf.f_per_level) == (int(ref["ND"]), int(ref["NC"]), int(ref["table_f_per_level"]))
    assert nerf.transfer_fmt == str(ref["transfer_fmt"])
    assert np.array_equal(nerf.state_i32["table"], ref["table_i"])
    for name in ref["active_params"].tolist():
        for pre in ("", "m", "v"):
            assert np.array_equal(np.asarray(nerf.state_i32[pre + name]).ravel(), ref[pre + name + "_i"]), pre + name
    assert np.array_equal(nerf.state_i32["occ_grid_in_u32"].view(np.uint32), ref["occ_grid_in_u32"])
    assert np.array_equal(nerf.state_i32["occ_grid_st_u32"].view(np.uint32), ref["occ_grid_st_u32"])
    for k in ("box_min", "box_max"):
        assert np.array_equal(getattr(nerf.occ, k), ref[k])
    for k in ("rho_min", "rho_max", "dt_min", "dt_max", "t_near_clip", "t_far_clip"):
        assert np.float32(getattr(nerf.occ, k)) == ref[k], k
    out = np.load(nerf.save(min_new_file_seconds=0))
    for k in ref.files:
        if k in ("timestamp", "model_id"):
            continue
        assert k in out.files, k
        assert out[k].dtype == ref[k].dtype and np.array_equal(out[k], ref[k]), k
