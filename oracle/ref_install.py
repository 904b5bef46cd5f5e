"""Installs the reference's Python modules into the git-ignored ``baseline/_ref/`` (TEST
INFRASTRUCTURE ONLY): the reference trainer and CLI are then run unmodified on this build by
``tests/test_gpu_reference_cli.py`` (through ``ffnerf-experimental_b200/run_reference.py``).

The reference checkout is not an installable package (no setup.py / pyproject.toml:
``pip install --target baseline/_ref <checkout>`` refuses it).  This recipe copies the checkout to
a temporary directory, adds packaging metadata that lists its top-level modules, and installs that
copy with pip (offline, no build isolation) into ``baseline/_ref/``.  Nothing is written into the
checkout or into the repository's tracked files.

    python oracle/ref_install.py --reference <checkout>
"""
from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
TARGET = ROOT / "baseline" / "_ref"
MODULES = ["ffnerf_cli", "run_ffnerf_OG", "scene_config", "sfm_data", "ffnerf_tools", "render_nerf",
           "nerf_web_remote", "inspect_npz"]


def install(reference: Path, target: Path = TARGET) -> Path:
    reference = Path(reference).resolve()
    missing = [m for m in MODULES if not (reference / f"{m}.py").exists()]
    if missing:
        raise FileNotFoundError(f"not a reference checkout ({reference}): missing {missing}")
    with tempfile.TemporaryDirectory(prefix="ffnerf_ref_") as tmp:
        src = Path(tmp) / "src"
        shutil.copytree(reference, src, ignore=shutil.ignore_patterns(".git", "training", "__pycache__"))
        (src / "pyproject.toml").write_text(
            "[build-system]\nrequires = [\"setuptools\"]\nbuild-backend = \"setuptools.build_meta\"\n\n"
            "[project]\nname = \"ffnerf-reference\"\nversion = \"0\"\n\n"
            "[tool.setuptools]\npy-modules = [" + ", ".join(f'"{m}"' for m in MODULES) + "]\n")
        if target.exists():
            shutil.rmtree(target)
        target.parent.mkdir(parents=True, exist_ok=True)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", str(target), str(src)]
        subprocess.run(cmd, check=True, capture_output=True, text=True)
    return target


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", type=Path, required=True)
    print(install(ap.parse_args().reference))
