"""Build liborin_b200.so (the sm_100a kernels and the C ABI) in-tree.

    python -m orininfer_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` and linked into
``orininfer_b200/liborin_b200.so`` next to this file, so the library travels
with the source tree.  Objects are rebuilt when their source or any header
changed.  The CUDA runtime is linked statically; NCCL dynamically.
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
BUILD = ROOT / "_build" / "orininfer_b200"
LIB = PKG / "liborin_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3",
    "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build liborin_b200.so")


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, flush=True)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library if anything changed; return its path."""
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = [ex.submit(_compile, s, o, verbose) for s, o in jobs]
            for f in futs:
                f.result()
    if force or jobs or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs),
               "-cudart", "static", "-lnccl", "-ldl", "-lpthread", "-lrt"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    path = build(force=a.force, verbose=a.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
