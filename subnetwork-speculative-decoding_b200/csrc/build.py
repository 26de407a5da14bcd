"""Build libssd_b200.so (sm_100a) in-tree with nvcc.

    python subnetwork-speculative-decoding_b200/csrc/build.py [--force] [-j N]

Each .cu file is compiled to an object under csrc/_build/ (skipped when the
object is newer than every source and header), then linked into
ssd/libssd_b200.so next to the Python package that loads it.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent / "ssd"
OUT = PKG / "libssd_b200.so"
INCLUDE = HERE.parent.parent / "include"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", str(INCLUDE)]


def sources() -> list[Path]:
    return sorted(HERE.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(HERE.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int = 8, verbose: bool = False, extra: list[str] | None = None) -> Path:
    extra = list(extra or [])
    bdir = HERE / "_build"
    bdir.mkdir(exist_ok=True)
    newest_hdr = max((h.stat().st_mtime for h in headers()), default=0.0)
    todo, objs = [], []
    for src in sources():
        obj = bdir / (src.stem + ".o")
        objs.append(obj)
        stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_hdr)
        if stale:
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for obj, err in ex.map(lambda a: _compile(*a, extra), todo):
                if verbose and err.strip():
                    print(f"[{obj.name}]\n{err}", file=sys.stderr)
    link_needed = force or todo or not OUT.exists() or OUT.stat().st_mtime < max(o.stat().st_mtime for o in objs)
    if link_needed:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--force", action="store_true")
    p.add_argument("-j", "--jobs", type=int, default=os.cpu_count() or 4)
    p.add_argument("-v", "--verbose", action="store_true", help="print ptxas / compiler warnings")
    p.add_argument("--ptxas-info", action="store_true", help="add -Xptxas -v (registers, spills, smem)")
    a = p.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    out = build(force=a.force or a.ptxas_info, jobs=a.jobs, verbose=a.verbose or a.ptxas_info, extra=extra)
    print(out)


if __name__ == "__main__":
    main()
