"""Build the CUDA backend in-tree: mlir-cim22_b200/cim22_b200/libcim22_cuda.so.

    python mlir-cim22_b200/build.py          # incremental
    python mlir-cim22_b200/build.py --force  # rebuild everything

Every translation unit is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) and linked into one shared
library with the static CUDA runtime. nvcc cross-compiles, so no GPU is
needed to build.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "cim22_b200" / "libcim22_cuda.so"
OBJ = HERE / "_build"
INCLUDE = HERE.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", *ARCH]
EXPORTS = HERE / "csrc" / "exports.map"


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return path


def sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def headers() -> list[Path]:
    return [*CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]


def compile_one(src: Path, force: bool, verbose: bool) -> Path:
    obj = OBJ / (src.name + ".o")
    newest = max(p.stat().st_mtime for p in [src, *headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(lambda s: compile_one(s, force, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < max(newest, EXPORTS.stat().st_mtime):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(OUT), *map(str, objs),
               "-Xlinker", f"--version-script={EXPORTS}", "-lpthread", "-ldl"]
        subprocess.run(cmd, check=True)
    return OUT


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = parser.parse_args()
    print(build(args.force, args.verbose))


if __name__ == "__main__":
    sys.exit(main())
