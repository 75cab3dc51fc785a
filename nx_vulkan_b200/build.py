"""Build libnxv_b200.so (the nxv_* C ABI on sm_100a) in-tree.

Each csrc/*.cu file is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``), in parallel, and linked into
``nx_vulkan_b200/lib/libnxv_b200.so`` with a static CUDA runtime so the
library carries no dependency on a particular libcudart on the host.

Usage: ``python -m nx_vulkan_b200.build [--force] [--ptxas-v]``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = PKG / "lib" / "obj"
LIB = PKG / "lib" / "libnxv_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
    f"-I{CSRC}",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (looked at $NVCC, /usr/local/cuda/bin/nvcc, PATH)")


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "nx_vulkan_shim.h"]


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, ptxas_v: bool) -> tuple[Path, str]:
    obj = OBJ / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{p.stdout}\n{p.stderr}")
    return obj, p.stderr


def build(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library."""
    OBJ.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    todo = [s for s in sources if force or ptxas_v or _stale(OBJ / (s.stem + ".o"), _deps(s))]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, log in ex.map(lambda s: _compile(s, ptxas_v), todo):
                logs.append((obj.name, log))
    objs = [OBJ / (s.stem + ".o") for s in sources]
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stdout}\n{p.stderr}")
    if verbose or ptxas_v:
        for name, log in logs:
            if log.strip():
                print(f"== {name}\n{log}", file=sys.stderr)
    return LIB


if __name__ == "__main__":
    lib = build(force="--force" in sys.argv, ptxas_v="--ptxas-v" in sys.argv, verbose=True)
    print(lib)
