"""Runs the reference's own command-line entry (MolSzabi/ffnerf-experimental ``ffnerf_cli.py``:
inspect / train / snapshot, with its ``run_ffnerf_OG.train`` loop, scene_config JSON and sfm_data
loaders) unmodified on this build:

    python run_reference.py --reference <checkout of the reference> train --config scene.json --no-web

The reference's Python modules are imported from its checkout; ``ffnerf_tools`` (this package's
CUDA edition), ``pyopencl`` (the transport subset over CUDA streams) and a headless ``render_nerf``
come first on the import path, so the trainer's ``import ffnerf_tools as ft`` and ``import
pyopencl as cl`` bind to libffnerf.so instead of OpenCL.  Everything after ``--reference DIR`` is
passed to ffnerf_cli.py as its own arguments.
"""
from __future__ import annotations

import runpy
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if len(argv) < 2 or argv[0] != "--reference":
        sys.exit("usage: run_reference.py --reference <reference checkout> <ffnerf_cli.py arguments>")
    ref = Path(argv[1]).resolve()
    cli = ref / "ffnerf_cli.py"
    if not cli.exists():
        sys.exit(f"{cli} not found")
    for p in (str(ref), str(HERE), str(HERE / "dropin")):     # dropin first, the reference last
        while p in sys.path:
            sys.path.remove(p)
    sys.path[:0] = [str(HERE / "dropin"), str(HERE), str(ref)]
    sys.argv = [str(cli)] + argv[2:]
    runpy.run_path(str(cli), run_name="__main__")


if __name__ == "__main__":
    main()
