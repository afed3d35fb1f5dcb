"""Build the sm_100a shared library ``libheartmula_b200.so`` in-tree with nvcc.

    python -m estudiocanciones_b200.build [--verbose]

Every ``csrc/*.cu`` is compiled for ``sm_100a`` only and linked into one
shared library exporting the C ABI declared in ``include/heartmula_b200.h``.
The CUDA runtime is linked statically, so the library needs only the driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libheartmula_b200.so"
BUILD = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2",
         "-Xptxas", "-O3", f"-I{INCLUDE}"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]
    return obj.stat().st_mtime < max(d.stat().st_mtime for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_info or _stale(obj, src):
            cmd = [cc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed on {src.name}")
            if verbose or ptxas_info:
                sys.stderr.write(r.stderr)
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, ptxas_info="--ptxas" in sys.argv, force="--force" in sys.argv)
    print(LIB)
