"""The reference's CLI on this build, host side (no GPU): ``run_reference.py`` runs the
reference's unmodified ``ffnerf_cli.py inspect`` on a synthetic scene in the reference's SfM
archive format, and inside that process ``ffnerf_tools``, ``pyopencl`` and ``render_nerf`` resolve
to this package's modules, not the reference's.  Skipped where the reference's modules are not
installed in baseline/_ref (oracle/ref_install.py)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
PKG = ROOT / "ffnerf-experimental_b200"


def _scene(tmp_path):
    from synthetic_scene import BlobScene, cameras_sphere, intrinsics, write_sfm_archive
    npz = write_sfm_archive(tmp_path / "scene", BlobScene(0), cameras_sphere(8, 2.0, 0), intrinsics(64, 64, 50.0), 64, 64)
    cfg = {"data": {"reconstruction": str(npz)}, "scene": {"box_min": [-1.0, -1.0, -1.0], "box_max": [1.0, 1.0, 1.0]},
           "training": {"directory": str(tmp_path / "training"), "model_id": "refcli"}}
    p = tmp_path / "scene.json"
    p.write_text(json.dumps(cfg))
    return p


def test_reference_inspect_through_launcher(tmp_path):
    if not (REF / "ffnerf_cli.py").exists():
        pytest.skip("the reference's modules are not installed in baseline/_ref")
    cfg = _scene(tmp_path)
    r = subprocess.run([sys.executable, str(PKG / "run_reference.py"), "--reference", str(REF), "inspect",
                        "--config", str(cfg)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "Registered cameras: 8" in r.stdout
    assert '"box_min": [-1.0, -1.0, -1.0]' in r.stdout


def test_launcher_binds_this_package(tmp_path):
    if not (REF / "ffnerf_cli.py").exists():
        pytest.skip("the reference's modules are not installed in baseline/_ref")
    probe = tmp_path / "probe"
    probe.mkdir()
    (probe / "ffnerf_cli.py").write_text(
        "import ffnerf_tools, pyopencl, render_nerf, scene_config\n"
        "print(ffnerf_tools.__file__); print(pyopencl.__file__); print(render_nerf.__file__); "
        "print(scene_config.__file__)\n")
    (probe / "scene_config.py").write_text("ROOT = None\n")
    r = subprocess.run([sys.executable, str(PKG / "run_reference.py"), "--reference", str(probe)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    tools, cl, render, scfg = [Path(x) for x in r.stdout.split()]
    assert tools == PKG / "ffnerf_tools.py"
    assert cl == PKG / "dropin" / "pyopencl" / "__init__.py"
    assert render == PKG / "dropin" / "render_nerf.py"
    assert scfg == probe / "scene_config.py"


def test_build_c2w_yaw_pitch_axes():
    sys.path.insert(0, str(PKG / "dropin"))
    import numpy as np
    import render_nerf
    rt = render_nerf.build_c2w_rt_yaw_pitch([1.0, 2.0, 3.0], 0.3, -0.2)
    R = rt[:3, :3]
    assert np.allclose(R.T @ R, np.eye(3), atol=1e-5)          # orthonormal
    assert np.allclose(rt[:3, 3], [1, 2, 3]) and np.allclose(rt[3], [0, 0, 0, 1])
    fwd = np.array([np.cos(0.3) * np.cos(-0.2), np.sin(0.3) * np.cos(-0.2), np.sin(-0.2)])
    assert np.allclose(R[:, 2], fwd, atol=1e-6)                # camera +z looks forward
    assert R[2, 1] < 0                                         # camera +y (image down) points down in world z
    assert abs(R[2, 0]) < 1e-6                                 # no roll: the right axis is horizontal
