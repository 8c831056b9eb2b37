"""Build libla_attention.so (sm_100a) in-tree with nvcc.

    python -m trainium_linear_attention_b200.build [--force] [--verbose]

Every ``csrc/*.cu`` is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into ``_build/`` and
linked into ``trainium_linear_attention_b200/lib/libla_attention.so``.  The
CUDA runtime is linked statically; the CUDA driver is reached at run time
through ``cudaGetDriverEntryPoint`` (TMA descriptors), so the library has no
link-time dependency on ``libcuda``.  Objects are rebuilt only when a source
or header is newer than they are.
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
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "lib" / "libla_attention.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
          "--expt-relaxed-constexpr", "-I" + str(INCLUDE), "-I" + str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set $NVCC)")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH_FLAGS, *CFLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return res.stderr if verbose else ""


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel source and link the shared library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    srcs = sorted(CSRC.glob("*.cu"))
    jobs = []
    for src in srcs:
        obj = BUILD / (src.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for out in ex.map(lambda j: _compile(j[0], j[1], verbose), jobs):
                if out:
                    print(out, file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    newest = max(o.stat().st_mtime for o in objs)
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
