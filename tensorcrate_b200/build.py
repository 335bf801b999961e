"""Build the CUDA library in-tree: tensorcrate_b200/_lib/libtccuda.so.

Every kernel is compiled for sm_100a only (B200).  Objects go to
tensorcrate_b200/_build/; the shared object is linked against the static
CUDA runtime, so it needs nothing from the environment but the driver.

    python -m tensorcrate_b200.build [--force] [-v]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libtccuda.so"
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2,-Wall", "-I", str(ROOT / "include"),
]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src] + _headers()
    if _stale(obj, deps):
        # the object is dated from its sources as they were when the compile
        # began, so a source edited while it runs is rebuilt next time
        seen = max(d.stat().st_mtime for d in deps)
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, flush=True)
        os.utime(obj, (seen, seen))
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose or ptxas_verbose, extra), srcs))
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-ldl", "-lpthread", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))


if __name__ == "__main__":
    sys.exit(main())
