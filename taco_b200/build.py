"""Builds the B200 HardShell backend into taco_b200/libhardshell_b200.so (in the source tree, so
the built library travels with the repository to the GPU box).

    python -m taco_b200.build            # build if a source is newer than the library
    python -m taco_b200.build --force

nvcc compiles every CUDA source for sm_100a only (the kernels use tcgen05 and TMA) and the host
C++ sources with the same toolchain. No GPU is needed to build.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libhardshell_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list(CSRC.glob("*.inc")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    out_dir = PKG / "_build"
    out_dir.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = out_dir / (src.name + ".o")
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
               "-c", str(src), "-o", str(obj)]
        if src.suffix == ".cu":
            cmd[1:1] = ["-Xptxas", "-v"] if verbose else []
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0 or verbose:
            sys.stderr.write(out.decode())
        if p.returncode != 0:
            failed = True
            sys.stderr.write(f"error: compiling {src.name} failed\n")
    if failed:
        raise RuntimeError("the CUDA build failed")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
