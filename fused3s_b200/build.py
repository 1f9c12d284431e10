"""Build libfused3s.so in-tree with nvcc for sm_100a.

    python -m fused3s_b200.build [--verbose-ptxas]

The shared library lands next to this file (fused3s_b200/libfused3s.so) so
it travels with the source tree.  cudart is linked statically: the library
needs only the NVIDIA driver at run time and coexists with the runtime that
PyTorch loads.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libfused3s.so"
SOURCES = ["f3s_api.cu", "f3s_format.cu", "f3s_forward.cu", "f3s_peer.cu", "f3s_probe.cu", "f3s_text.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def build(verbose_ptxas: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    if not force and LIB.exists() and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    common = [nvcc_path(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              f"-I{INCLUDE}", f"-I{CSRC}"]
    if verbose_ptxas:
        common += ["-Xptxas", "-v"]
    objs = []
    for s in srcs:
        o = objdir / (s.stem + ".o")
        cmd = common + ["-c", str(s), "-o", str(o)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose_ptxas:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s.name}")
        objs.append(str(o))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB)
    shutil.rmtree(objdir, ignore_errors=True)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    p = build(verbose_ptxas=a.verbose_ptxas, force=a.force)
    print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
