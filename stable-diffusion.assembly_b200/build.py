"""Builds libsdb.so, the sm_100a kernel library, in place.

    python stable-diffusion.assembly_b200/build.py [--verbose] [--checks]

Each csrc/*.cu is compiled by nvcc for sm_100a only (-gencode
arch=compute_100a,code=sm_100a) into _build/, then linked into
stable-diffusion.assembly_b200/libsdb.so next to this file.  Objects are
rebuilt when their source or any header under csrc/ or include/ is newer.
--checks adds -DSDB_CHECKS (device-side index checks that record an error
bit instead of faulting).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "libsdb.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _newest_header() -> float:
    newest = 0.0
    for d in (CSRC, INCLUDE):
        for p in list(d.glob("*.h")) + list(d.glob("*.cuh")):
            newest = max(newest, p.stat().st_mtime)
    return newest


def _compile(src: Path, obj: Path, extra: list[str], verbose: bool) -> tuple[Path, str]:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
    return obj, res.stderr if verbose else ""


def build(verbose: bool = False, checks: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    extra = ["-DSDB_CHECKS"] if checks else []
    headers = _newest_header()
    sources = sorted(CSRC.glob("*.cu"))
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + (".checks" if checks else "") + ".o")
        objs.append(obj)
        if not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, headers):
            jobs.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for obj, log in ex.map(lambda j: _compile(j[0], j[1], extra, verbose), jobs):
            if log:
                print(f"== {obj.name}\n{log}")
    lib = LIB if not checks else HERE / "libsdb_checks.so"
    if not lib.exists() or any(o.stat().st_mtime > lib.stat().st_mtime for o in objs):
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs),
               "-o", str(lib), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--checks", action="store_true")
    ns = ap.parse_args()
    print(build(verbose=ns.verbose, checks=ns.checks))
    sys.exit(0)
