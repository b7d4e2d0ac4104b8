"""Builds the native library libint8linear_b200.so from int8_linear/csrc with nvcc.

    python -m int8_linear.build [--force] [--verbose]

The library is compiled for sm_100a only (tcgen05, TMA) and links the CUDA runtime
statically, so it loads without a GPU and depends on nothing but the driver at run
time.  Objects are rebuilt when a source or header is newer than the library.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libint8linear_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-Xptxas", "-O3"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is needed to build int8_linear")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile every csrc/*.cu for sm_100a and link the shared library; returns its path."""
    OUT_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    srcs = sources()
    if not force and not _stale(LIB, srcs + headers + [Path(__file__)]):
        return LIB
    cc = nvcc()
    objs = []
    jobs = []
    for src in srcs:
        obj = OUT_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers + [Path(__file__)]):
            cmd = [cc, *ARCH, *FLAGS, *(extra or []), f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(run, jobs))
    tmp = LIB.with_suffix(".so.tmp")
    run([cc, *ARCH, "-shared", "-cudart", "static", *map(str, objs), "-o", str(tmp)])
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_info else None
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose or a.ptxas_info, extra=extra))


if __name__ == "__main__":
    sys.exit(main())
