"""Build recipe for the reference kernels compiled for the CPU (TEST INFRASTRUCTURE ONLY).

Reads the reference's three OpenCL C sources where they lie (``ffnerf_OG.cl``,
``weight_update.cl``, ``decay_occ_grid_in-st.cl`` in the reference checkout), applies a
mechanical OpenCL-C -> C++ rewrite, and compiles them with ``clemu.cpp`` (fiber work-groups)
into ``oracle/_ref/libffnref_<variant>.so``.  Nothing from the reference is written outside
``oracle/_ref/`` (git-ignored).

Rewrites (syntax only):
  * ``(float3)(a,b,c)`` / ``(float4)(a,b,c,d)`` vector literals -> braced initialisers (which keep
    OpenCL's left-to-right evaluation of the components), ``(float3)(s)`` -> broadcast;
  * ``.xyz`` swizzle -> ``.xyz()``;
  * ``__local`` variable declarations inside kernels -> references into the local memory of the
    running work-group (``clemu::local_ref``, shared by its fibers, separate per work-group, so that
    several work-groups can be in flight on one OS thread); every other ``__local`` / ``__global``
    qualifier is dropped;
  * ``__constant`` -> ``static const``; OpenCL extension pragmas are removed.

Patches (semantics), each asserted to apply exactly once:
  * geometry of the variant: per-level table sizes/offsets and the finest resolution
    (``RESOLUTION_LVLMAX`` is not ``#ifndef``-guarded in the reference);
  * ``scan_excl_seg`` stores the scan total through a pointer for lane 0 only, and lanes != 0
    later read their own, never-written copy (``T_final`` in the occupancy proposal).  That read
    has no defined value; the patch makes every lane read the total, which is what lane 0 holds.
"""
from __future__ import annotations

import argparse
import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_ROOT = HERE / "_ref"

# name -> (F, ND, NC, log2 entries per level or None for the reference's own table, finest res)
VARIANTS = {
    "default": dict(F=4, ND=2, NC=2, log2T=None, rmax=None),
    "cfg1": dict(F=2, ND=1, NC=2, log2T=14, rmax=512.0),
    "cfg3": dict(F=2, ND=1, NC=2, log2T=19, rmax=2048.0),
    # the reference's fp16 and fp8 transfer formats of the staged activations / deltas
    "cfg1_t16": dict(F=2, ND=1, NC=2, log2T=14, rmax=512.0, transfer=16),
    "cfg1_t8": dict(F=2, ND=1, NC=2, log2T=14, rmax=512.0, transfer=8),
}


def _match_paren(s: str, i: int) -> int:
    """Index of the ')' matching the '(' at s[i]."""
    depth = 0
    for j in range(i, len(s)):
        if s[j] == "(":
            depth += 1
        elif s[j] == ")":
            depth -= 1
            if depth == 0:
                return j
    raise ValueError("unbalanced parentheses")


def _split_top(s: str) -> list[str]:
    parts, depth, cur = [], 0, []
    for ch in s:
        if ch == "(":
            depth += 1
        elif ch == ")":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    parts.append("".join(cur))
    return parts


def _rewrite_vector_literals(src: str) -> str:
    pat = re.compile(r"\((float3|float4)\)\s*\(")
    while True:
        m = pat.search(src)
        if not m:
            return src
        typ = m.group(1)
        open_i = m.end() - 1
        close_i = _match_paren(src, open_i)
        args = _split_top(src[open_i + 1:close_i])
        if len(args) == 1:
            rep = f"{'f3_bcast' if typ == 'float3' else 'f4_bcast'}({args[0].strip()})"
        elif typ == "float3" and len(args) == 3:
            rep = "float3{" + ", ".join(a.strip() for a in args) + ", 0.0f}"
        elif typ == "float4" and len(args) == 4:
            rep = "float4{" + ", ".join(a.strip() for a in args) + "}"
        else:
            raise ValueError(f"unsupported vector literal: {src[m.start():close_i + 1]}")
        src = src[:m.start()] + rep + src[close_i + 1:]


def _sub_once(pattern: str, repl: str, src: str, flags=0) -> str:
    out, n = re.subn(pattern, repl, src, flags=flags)
    if n != 1:
        raise RuntimeError(f"patch {pattern!r} applied {n} times (expected 1)")
    return out


_LOCAL_ID = [0]


def _local_decl(m: re.Match) -> str:
    """``__local T a[N], b;`` -> one reference per name into the running work-group's local memory
    (clemu::local_ref: allocated zeroed on first use by the group, shared by its work-items)."""
    indent, typ, names = m.group(1), m.group(2), m.group(3)
    out = []
    for part in names.split(","):
        part = part.strip()
        nm = re.match(r"(\w+)\s*(\[[^\]]*\])?", part)
        name, dim = nm.group(1), nm.group(2) or ""
        if _LOCAL_ID[0] >= 64:
            raise ValueError("more __local declarations than clemu::kMaxLocals")
        out.append(f"auto& {name} = ::clemu::local_ref<{typ}{dim}>({_LOCAL_ID[0]});")
        _LOCAL_ID[0] += 1
    return indent + " ".join(out)


def translate(src: str) -> str:
    _LOCAL_ID[0] = 0        # __local ids are per translation unit (clemu::kMaxLocals of them)
    src = re.sub(r"^\s*#pragma\s+OPENCL.*$", "", src, flags=re.M)
    src = _rewrite_vector_literals(src)
    src = re.sub(r"\.xyz\b", ".xyz()", src)
    src = re.sub(
        r"^(\s*)__local\s+(\w+)\s+(\w+\s*(?:\[[^\]]*\])?(?:\s*,\s*\w+\s*(?:\[[^\]]*\])?)*)\s*;",
        _local_decl, src, flags=re.M)
    src = src.replace("__local", "")
    src = re.sub(r"\b__kernel\b", "", src)
    src = re.sub(r"\b__global\b", "", src)
    src = re.sub(r"\b__constant\b", "static const", src)
    return src


def patch_train(src: str, v: dict) -> str:
    src = _sub_once(r"if \(lid == 0\) \*total_out = segs\[WG - 1\];", "*total_out = segs[WG - 1];", src)
    if v["rmax"] is not None:
        src = _sub_once(r"#define RESOLUTION_LVLMAX\s+[0-9.]+f", f"#define RESOLUTION_LVLMAX {v['rmax']:.1f}f", src)
    if v["log2T"] is not None:
        k = v["log2T"]
        log2 = ", ".join(f"{k}u" for _ in range(16))
        offs = ", ".join(f"{l << k}u" for l in range(16))
        src = _sub_once(r"__constant uint LEVEL_LOG2\[N_LEVELS\] = \{[^}]*\};",
                        f"__constant uint LEVEL_LOG2[N_LEVELS] = {{{log2}}};", src)
        src = _sub_once(r"__constant uint LEVEL_OFFSET_ENTRIES\[N_LEVELS\] = \{[^}]*\};",
                        f"__constant uint LEVEL_OFFSET_ENTRIES[N_LEVELS] = {{{offs}}};", src)
        src = _sub_once(r"#define TABLE_TOTAL_ENTRIES\s+\d+u", f"#define TABLE_TOTAL_ENTRIES {16 << k}u", src)
    return src


TRAIN_LAUNCHER = r"""
extern "C" void ffnref_train(const ffnref_train_args* a) {
    using namespace clemu;
    using namespace clemu::k_train;
    auto T = [](float* p) { return reinterpret_cast<TRANSFER_T*>(p); };   // scratch in the transfer format
    const float3 bmin = f3_make(a->box_min[0], a->box_min[1], a->box_min[2]);
    const float3 bmax = f3_make(a->box_max[0], a->box_max[1], a->box_max[2]);
    const Ray* rays = (const Ray*)a->rays;
    const float4* tg = (const float4*)a->targets;
    float4* out = (float4*)a->out;
    const long n = (long)a->num_rays;
    const int nt = a->n_threads > 0 ? a->n_threads : 1;
    auto body = [&]() {
            ffnerf_train_step(a->W[0], a->W[1], a->W[2], a->W[3], a->b[0], a->b[1], a->b[2], a->b[3],
                              a->W[4], a->W[5], a->W[6], a->W[7], a->W[8],
                              a->b[4], a->b[5], a->b[6], a->b[7], a->b[8],
                              a->table, rays, tg,
                              T(a->deltas[0]), T(a->deltas[1]), T(a->deltas[2]), T(a->deltas[3]), T(a->deltas[4]),
                              T(a->deltas[5]), T(a->deltas[6]), T(a->deltas[7]), T(a->deltas[8]),
                              T(a->acts[0]), T(a->acts[1]), T(a->acts[2]), T(a->acts[3]), T(a->acts[4]),
                              T(a->acts[5]), T(a->acts[6]), T(a->acts[7]), T(a->acts[8]),
                              out, a->lr, a->num_rays, a->spr, a->do_train, a->sh_mult,
                              a->occ_in, a->occ_st, bmin, bmax, a->G, a->rho_min, a->rho_max,
                              a->dt_min, a->dt_max, a->t_near, a->t_far, a->seed, a->occ_strength);
    };
    if (a->lockstep) {
        run_work_groups_lockstep((size_t)n, a->spr, body, nt);
        return;
    }
    #pragma omp parallel for schedule(dynamic, 4) num_threads(nt)
    for (long g = 0; g < n; ++g) run_work_group((size_t)g, 0, a->spr, 1, body);
}

extern "C" void ffnref_info(int32_t* f_, int32_t* nd_, int32_t* nc_, int32_t* log2T, float* rmax) {
    using namespace clemu::k_train;
    *f_ = F_PER_LEVEL; *nd_ = ND; *nc_ = NC; *log2T = (int32_t)LEVEL_LOG2[0]; *rmax = RESOLUTION_LVLMAX;
}
"""

WU_LAUNCHER = r"""
extern "C" void ffnref_weight_update(const ffnref_wu_args* a) {
    using namespace clemu;
    using namespace clemu::k_wu;
    auto T = [](float* p) { return reinterpret_cast<TRANSFER_T*>(p); };   // scratch in the transfer format
    const int max_in = a->M > 32 ? (a->M > a->L ? a->M : a->L) : (32 > a->L ? 32 : a->L);
    const int ngx = (max_in + INT - 1) / INT;
    const int ngy = (a->M + OUTT - 1) / OUTT;
    const int nt = a->n_threads > 0 ? a->n_threads : 1;
    #pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(nt)
    for (int gy = 0; gy < ngy; ++gy)
        for (int gx = 0; gx < ngx; ++gx)
            run_work_group((size_t)gx, (size_t)gy, WG_X, WG_Y, [&]() {
                update_ffnerf_oneWG(a->W[0], a->W[1], a->W[2], a->W[3], a->W[4], a->W[5], a->W[6], a->W[7], a->W[8],
                                    a->b[0], a->b[1], a->b[2], a->b[3], a->b[4], a->b[5], a->b[6], a->b[7], a->b[8],
                                    a->mW[0], a->mW[1], a->mW[2], a->mW[3], a->mW[4], a->mW[5], a->mW[6], a->mW[7], a->mW[8],
                                    a->vW[0], a->vW[1], a->vW[2], a->vW[3], a->vW[4], a->vW[5], a->vW[6], a->vW[7], a->vW[8],
                                    a->mb[0], a->mb[1], a->mb[2], a->mb[3], a->mb[4], a->mb[5], a->mb[6], a->mb[7], a->mb[8],
                                    a->vb[0], a->vb[1], a->vb[2], a->vb[3], a->vb[4], a->vb[5], a->vb[6], a->vb[7], a->vb[8],
                                    T(a->deltas[0]), T(a->deltas[1]), T(a->deltas[2]), T(a->deltas[3]), T(a->deltas[4]),
                                    T(a->deltas[5]), T(a->deltas[6]), T(a->deltas[7]), T(a->deltas[8]),
                                    T(a->acts[0]), T(a->acts[1]), T(a->acts[2]), T(a->acts[3]), T(a->acts[4]),
                                    T(a->acts[5]), T(a->acts[6]), T(a->acts[7]), T(a->acts[8]),
                                    a->B, a->L, a->M, a->lr_t, a->color_rel_lr, a->beta1, a->beta2, a->eps);
            });
}
"""

DECAY_LAUNCHER = r"""
extern "C" void ffnref_decay(uint32_t* occ_in, uint32_t* occ_st, uint32_t n_words, uint32_t dq, uint32_t seed) {
    using namespace clemu;
    using namespace clemu::k_decay;
    const size_t groups = (n_words + 63u) / 64u;
    for (size_t g = 0; g < groups; ++g)
        run_work_group(g, 0, 64, 1, [&]() { occ_nibble_decay_write_both_q24(occ_in, occ_st, n_words, dq, seed); });
}
"""


def _unit(ns: str, body: str, launcher: str, fname: str) -> str:
    return ("#include \"clemu.h\"\n#include \"ref_abi.h\"\n#include <cstdint>\n"
            f"namespace clemu {{ namespace {ns} {{\n#line 1 \"{fname}\"\n{body}\n}} }}\n{launcher}")


def build_variant(ref_dir: Path, name: str, cxx: str = "g++", quiet: bool = True) -> Path:
    v = VARIANTS[name]
    out_dir = OUT_ROOT / name
    out_dir.mkdir(parents=True, exist_ok=True)
    train = translate(patch_train((ref_dir / "ffnerf_OG.cl").read_text(encoding="utf-8"), v))
    wu = translate((ref_dir / "weight_update.cl").read_text(encoding="utf-8"))
    dec = translate((ref_dir / "decay_occ_grid_in-st.cl").read_text(encoding="utf-8"))
    units = {
        "k_train.cpp": _unit("k_train", train, TRAIN_LAUNCHER, "ffnerf_OG.cl"),
        "k_wu.cpp": _unit("k_wu", wu, WU_LAUNCHER, "weight_update.cl"),
        "k_decay.cpp": _unit("k_decay", dec, DECAY_LAUNCHER, "decay_occ_grid_in-st.cl"),
    }
    for fn, text in units.items():
        (out_dir / fn).write_text(text, encoding="utf-8")
    # Same -D options the reference host passes (ffnerf_tools.py:618-637), BACKGROUND_COLOR=2 as
    # selected by the trainer for SfM scenes (run_ffnerf_OG.py:1082), fp32 transfer unless the
    # variant names another.
    defs = [f"-DND={v['ND']}", f"-DNC={v['NC']}", "-DNDMAX=3", "-DNCMAX=4", f"-DTRANSFER_FMT={v.get('transfer', 32)}",
            "-DWG_X=16", "-DWG_Y=16", "-DREG_X=1", "-DREG_Y=1", "-DTILEK=236",
            "-DBACKGROUND_COLOR=2", f"-DF_PER_LEVEL={v['F']}"]
    so = OUT_ROOT / f"libffnref_{name}.so"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-w", f"-I{HERE}", *defs,
           str(out_dir / "k_train.cpp"), str(out_dir / "k_wu.cpp"), str(out_dir / "k_decay.cpp"),
           str(HERE / "clemu.cpp"), "-o", str(so)]
    subprocess.run(cmd, check=True, capture_output=quiet)
    return so


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", type=Path, required=True, help="reference checkout")
    ap.add_argument("--variant", action="append", choices=sorted(VARIANTS))
    a = ap.parse_args(argv)
    for name in a.variant or sorted(VARIANTS):
        print(build_variant(a.reference, name, quiet=False))
    return 0


if __name__ == "__main__":
    sys.exit(main())
