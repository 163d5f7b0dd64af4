"""Builds libcacheflow_b200.so in-tree with nvcc for sm_100a.

    python -m cacheflow_b200.build [--force] [--verbose]

Objects go to cacheflow_b200/_build/, the shared library next to this file,
so it travels with the source tree.  cudart is linked statically (nvcc's
default), so the library does not depend on the CUDA runtime that PyTorch
bundles.
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
LIB = PKG / "libcacheflow_b200.so"

SOURCES = ["paged_attention.cu", "prefill_attention.cu", "cache_ops.cu", "capi.cu", "static_scratch.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build cacheflow_b200")
    return cand


def _flags(extra: list[str]) -> list[str]:
    return [
        *ARCH,
        "-std=c++17",
        "-O3",
        "-lineinfo",
        "-Xcompiler",
        "-fPIC,-O3,-fvisibility=hidden",
        "-Xptxas",
        "-v" if os.environ.get("CF_PTXAS_VERBOSE") else "-O3",
        f"-I{ROOT / 'include'}",
        *extra,
    ]


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compiles every .cu under csrc/ and links the shared library; returns its path."""
    extra = extra or []
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    cc = nvcc()
    jobs = []
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (Path(src).stem + ".o")
        objs.append(o)
        if force or _stale(o, [s, *headers]):
            cmd = [cc, *_flags(extra), "-c", str(s), "-o", str(o)]
            jobs.append(cmd)

    def run(cmd: list[str]) -> None:
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stdout.write(r.stdout)
            sys.stderr.write(r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({r.returncode}): {' '.join(cmd)}")

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        link = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp)]
        run(link)
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
