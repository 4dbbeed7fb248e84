"""Build the sm_100a shared library ``csahca_b200/_lib/libcsahca_b200.so``.

    python -m csahca_b200.build            # incremental
    python -m csahca_b200.build --force    # rebuild everything
    python -m csahca_b200.build --ptxas-verbose   # registers / spills / shared memory

Every ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` only (no PTX for other
targets, no JIT cache) and linked into one shared library with the CUDA runtime
linked statically.  The library is built in-tree so it travels with the
repository; ``csahca_b200._native`` loads it and raises if it is missing.
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
BUILD = ROOT / "_build"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libcsahca_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
    f"-I{ROOT / 'include'}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout, res.stderr, sep="\n")


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    hdr_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    jobs, objs = [], []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_verbose or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_mtime):
            jobs.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(lambda j: _compile(j[0], j[1], extra, verbose or ptxas_verbose), jobs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills / shared memory")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
