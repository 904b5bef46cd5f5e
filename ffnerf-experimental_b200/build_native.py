"""Build recipe of libffnerf.so (the C-ABI library in include/ffnerf.h) for B200 / sm_100a.

Compiles csrc/ffn_capi.cu (which includes the kernels) with nvcc into
``libffnerf.so`` next to this file.  Rebuilds only when a source is newer than the library.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SO = HERE / "libffnerf.so"
SOURCES = [HERE / "csrc" / n for n in ("ffn_capi.cu", "ffn_step.cu", "ffn_common.cuh", "ffn_raymarch.cuh", "ffn_hashgrid.cuh", "ffn_tcgen05.cuh", "ffn_step_tc.cu", "ffn_noalloc.cu", "ffn_dp.cu", "ffn_batch.cu", "ffn_probe.cu")] + [ROOT / "include" / "ffnerf.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def build(force: bool = False, verbose: bool = False) -> Path:
    newest = max(p.stat().st_mtime for p in SOURCES)
    if SO.exists() and SO.stat().st_mtime >= newest and not force:
        return SO
    tmp = SO.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{ROOT / 'include'}", str(HERE / "csrc" / "ffn_capi.cu"), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stderr)
    tmp.replace(SO)
    return SO


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
