"""The C-ABI library loads without a GPU and exports every entry point include/ffnerf.h declares;
host-side configuration logic matches the oracle's restatement."""
import re
from pathlib import Path

import numpy as np
import pytest

import ffn_native as fn
from ffn_config import (REFERENCE_LEVEL_LOG2, hash_lr_scales, level_layout, level_resolutions, make_geometry,
                        param_layout)

ROOT = Path(__file__).resolve().parents[1]


def test_header_symbols_exported():
    header = (ROOT / "include" / "ffnerf.h").read_text()
    declared = set(re.findall(r"^\s*(?:int|uint64_t|const char\*)\s+(ffn_\w+)\s*\(", header, flags=re.M))
    assert declared, "no declarations parsed"
    lib = fn.load_library()
    for name in declared:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert declared == set(fn.EXPORTED), declared ^ set(fn.EXPORTED)
    assert lib.ffn_abi_version() == fn.ABI_VERSION


def test_param_layout_matches_oracle(oracle):
    for F, ND, NC in [(2, 1, 2), (4, 2, 2), (2, 3, 4), (4, 1, 1)]:
        lay, total = param_layout(F, ND, NC)
        lay_o, total_o = oracle.layout(F, ND, NC)
        assert total == total_o and lay == lay_o
        g = make_geometry(F=F, ND=ND, NC=NC)
        c = fn.make_ffn_config(g)
        off = np.zeros(18, np.int32)
        sz = np.zeros(18, np.int32)
        assert fn.load_library().ffn_param_layout(c, off.ctypes.data, sz.ctypes.data) == total
        assert [lay[n] for n in lay] == list(zip(off.tolist(), sz.tolist()))


def test_level_tables():
    # finest resolution reached exactly, coarsest is 16 (ffnerf_OG.cl:1308-1311)
    for rmax in (512.0, 1024.0, 2048.0):
        r = level_resolutions(rmax)
        assert r[0] == 16 and r[-1] == int(rmax) and all(a <= b for a, b in zip(r, r[1:]))
    assert level_resolutions(512.0) == [16, 20, 25, 32, 40, 51, 64, 81, 102, 128, 161, 203, 256, 323, 406, 512]
    s = hash_lr_scales()
    assert s[0] == 1.0 and s[10] == 0.5 and abs(s[5] - 2 ** -0.5) < 1e-7
    log2, offs, total = level_layout(list(REFERENCE_LEVEL_LOG2))
    assert total == 2_260_992   # ffnerf_tools.py:26
    assert offs[15] == 1736704  # ffnerf_OG.cl:199


def test_geometry_validation():
    with pytest.raises(ValueError):
        make_geometry(spr=128)      # > S_MAX (scene_config.py:48-50)
    with pytest.raises(ValueError):
        make_geometry(F=3)
    with pytest.raises(ValueError):
        make_geometry(box_min=(0, 0, 0), box_max=(1, 0, 1))
    g = make_geometry(spr=64, box_min=(-1, -1, -1), box_max=(1, 1, 1))
    # trainer defaults (run_ffnerf_OG.py:1050-1051)
    assert g["dt_min"] == float(np.float32(2.0 / 8192))
    assert g["dt_max"] == float(np.float32(12.8 / 64 / 6 * 2.0))


def test_library_missing_or_of_another_abi_is_refused(tmp_path):
    """No silent fallback: a missing library, or one built for another ABI version (which may lack
    newer entry points), makes load_library raise before anything is bound."""
    import shutil
    import subprocess
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        fn.load_library(tmp_path / "absent.so")
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "old.c"
    src.write_text(f"int ffn_abi_version(void) {{ return {fn.ABI_VERSION - 1}; }}\n")
    so = tmp_path / "libold.so"
    subprocess.run([cc, "-shared", "-fPIC", str(src), "-o", str(so)], check=True)
    with pytest.raises(RuntimeError, match="ABI version"):
        fn.load_library(so)
