"""Builds the sm_100a shared library ``forma_b200/libforma_b200.so`` in-tree.

Every CUDA translation unit is compiled by nvcc for ``compute_100a/sm_100a``
with precise f32 arithmetic (no fast-math, no flush-to-zero, IEEE divide and
square root), the host C++ by nvcc's host compiler, and the CUDA runtime is
linked statically so the library only needs the driver at run time.
Objects are rebuilt only when a source or header is newer.

Usage: ``python -m forma_b200.build [--force] [-j N]``
"""

from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libforma_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include")]
CUDA_FLAGS = ARCH + [
    "-lineinfo",
    "-ftz=false",
    "-prec-div=true",
    "-prec-sqrt=true",
    "-fmad=true",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
]


def sources() -> list[Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def headers() -> list[Path]:
    hs = [p for p in CSRC.iterdir() if p.suffix in (".h", ".cuh")]
    return hs + [ROOT / "include" / "forma_b200.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path) -> None:
    cmd = [NVCC, "-c", str(src), "-o", str(obj)] + COMMON
    if src.suffix == ".cu":
        cmd += CUDA_FLAGS
    else:
        cmd += ["-x", "c++", "-Wno-deprecated-gpu-targets"]
    subprocess.run(cmd, check=True)


def build(force: bool = False, jobs: int | None = None) -> Path:
    OBJ.mkdir(exist_ok=True)
    hdrs = headers()
    todo = []
    objs = []
    for src in sources():
        obj = OBJ / (src.name + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            todo.append((src, obj))
    with futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        for f in [pool.submit(_compile, s, o) for s, o in todo]:
            f.result()
    if force or todo or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run(
            [NVCC, "-shared", "-o", str(tmp)] + ARCH + [str(o) for o in objs] + ["-cudart", "static", "-lpthread", "-ldl"],
            check=True,
        )
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args(argv)
    print(build(a.force, a.j))
    return 0


if __name__ == "__main__":
    sys.exit(main())
