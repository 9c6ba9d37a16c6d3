"""Build libnpu_b200.so (sm_100a) in-tree with nvcc.

Objects go to ``_build/`` at the repository root and the shared library to
``llm_compiler_3_b200/lib/libnpu_b200.so``; both are git-ignored but travel with
the source tree, so a machine with a GPU and no compiler can load the prebuilt
library.  Only sources newer than their object are recompiled.

    python -m llm_compiler_3_b200.build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBDIR = PACKAGE / "lib"
LIBRARY = LIBDIR / "libnpu_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-rdc=true", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden", "-I", str(INCLUDE), "-I", str(CSRC),
    "-DNPU_B200_BUILD",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libnpu_b200")
    return found


def _headers_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: Path, force: bool, hdr_mtime: float, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
            and obj.stat().st_mtime >= hdr_mtime):
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{done.stdout}\n{done.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libnpu_b200.so; return its path."""
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    hdr = _headers_mtime()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as pool:
        objects = list(pool.map(lambda s: _compile(s, force, hdr, extra), sources))
    newest = max(o.stat().st_mtime for o in objects)
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-rdc=true", *[str(o) for o in objects],
               "-o", str(tmp), "-ldl", "-lpthread"]
        done = subprocess.run(cmd, capture_output=True, text=True)
        if done.returncode:
            raise RuntimeError(f"link of libnpu_b200.so failed:\n{done.stdout}\n{done.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true",
                    help="print registers/spills/shared memory per kernel")
    a = ap.parse_args(argv)
    path = build(force=a.force or a.ptxas_verbose, jobs=a.jobs, verbose_ptxas=a.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
