"""Builds the package's native libraries in-tree.

* ``libshield_b200.so`` — the CUDA library (sm_100a kernels + the C ABI of
  include/shield_b200.h), compiled by nvcc for ``compute_100a``/``sm_100a``.
* ``libshield_synth.so`` — the host-side synthetic checkpoint generator.

Both land beside this file so they travel with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
REPO = PKG.parent
INCLUDE = REPO / "include"

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def main_lib_path() -> Path:
    return PKG / "libshield_b200.so"


def synth_lib_path() -> Path:
    return PKG / "libshield_synth.so"


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def build_synth(force: bool = False) -> Path:
    out = synth_lib_path()
    src = CSRC / "synth.c"
    if force or _stale(out, [src]):
        cc = os.environ.get("CC", "gcc")
        subprocess.run([cc, "-O2", "-std=c11", "-fPIC", "-mf16c", "-ffp-contract=off", "-shared",
                        "-o", str(out), str(src), "-lm", "-lpthread"], check=True)
    return out


def build_main(force: bool = False, verbose: bool = False) -> Path:
    out = main_lib_path()
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    deps = srcs + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    if not (force or _stale(out, deps)):
        return out
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    # -fmad=false / -ffp-contract=off: no multiply-add is fused unless the
    # source spells it (__fmaf_rn, fmaf), so every rounding matches the
    # reference's separate operations.
    common = ["-std=c++17", "-O3", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC,-ffp-contract=off",
              "-I", str(INCLUDE), "-I", str(CSRC), "--expt-relaxed-constexpr"]
    objs = []
    procs = []
    for s in srcs:
        o = objdir / (s.stem + ".o")
        objs.append(o)
        cmd = [nvcc, *NVCC_ARCH, *common, "-c", str(s), "-o", str(o)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for s, p in procs:
        outp = p.communicate()[0].decode()
        if p.returncode != 0 or verbose:
            print(outp)
        if p.returncode != 0:
            failed.append(s.name)
    if failed:
        raise RuntimeError("nvcc failed on " + ", ".join(failed))
    subprocess.run([nvcc, *NVCC_ARCH, "-shared", "-o", str(out), *map(str, objs), "-lcudart", "-lpthread"],
                   check=True)
    return out


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_main(force)


if __name__ == "__main__":
    import sys
    build_synth(force=True)
    build_main(force=True, verbose="-v" in sys.argv)
