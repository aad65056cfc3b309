"""Builds libkd_b200.so (every CUDA source under csrc/) in-tree for sm_100a with nvcc.

``python -m karpo_decision_b200.build`` or ``build()``. The library is rebuilt when any source or header is newer than
it. It cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIBRARY = PACKAGE / "libkd_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-Xptxas",
         "-warn-spills"]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: libkd_b200 needs the CUDA toolkit to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = [*sources(), *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h"), Path(__file__)]
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every ``csrc/*.cu`` to an object (in parallel) and links ``libkd_b200.so``; returns its path."""
    if not force and not _stale():
        return LIBRARY
    nvcc = _nvcc()
    objdir = PACKAGE / "_build"
    objdir.mkdir(exist_ok=True)
    procs = []
    objects = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        objects.append(obj)
        cmd = [nvcc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if verbose and out:
            print(out, file=sys.stderr)
        if proc.returncode != 0:
            failed.append(f"{src.name}:\n{out}")
    if failed:
        raise RuntimeError("libkd_b200 build failed:\n" + "\n".join(failed))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objects)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError("libkd_b200 link failed:\n" + result.stdout + result.stderr)
    tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
