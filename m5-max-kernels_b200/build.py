"""Build libm5b200.so (the C-ABI CUDA library) in-tree for sm_100a.

    python m5-max-kernels_b200/build.py [--force] [--verbose]

Each csrc/*.cu is compiled to an object with nvcc (in parallel), then linked
into m5kernels_b200/lib/libm5b200.so.  Objects are rebuilt only when a source
or header is newer than them.  `-Xptxas -v` output (registers, spills, shared
memory) is written to _build/ptxas_<name>.txt when --verbose is given.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG_DIR / "_build"
LIB_DIR = PKG_DIR / "m5kernels_b200" / "lib"
LIB = LIB_DIR / "libm5b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libm5b200.so")
    return found


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src),
           "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        (BUILD / f"ptxas_{src.stem}.txt").write_text(proc.stdout + proc.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    workers = min(len(sources), os.cpu_count() or 1)
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose), sources))
    if LIB.exists() and not force and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static",
           "-Xcompiler", "-fPIC"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
