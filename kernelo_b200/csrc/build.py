"""Build libkernelo_b200.so for sm_100a with nvcc.

Each ``.cu`` file in this directory is compiled to an object in parallel and
the objects are linked into ``kernelo_b200/_native/libkernelo_b200.so``. The
library is built in-tree so that it travels with the source tree to the GPU
host; nothing is installed. A rebuild happens only when the content hash of
the sources and headers differs from the one recorded at the last build (or
when ``force=True``).

Run directly: ``python -m kernelo_b200.csrc.build [--force]``.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PACKAGE = CSRC.parent
REPO = PACKAGE.parent
INCLUDE = REPO / "include"
OUT_DIR = PACKAGE / "_native"
LIB_NAME = "libkernelo_b200.so"
LIB_PATH = OUT_DIR / LIB_NAME
BUILD_DIR = OUT_DIR / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc_path() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME to a CUDA 12.8+ toolkit")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")])


HASH_PATH = OUT_DIR / (LIB_NAME + ".sha256")


def source_digest() -> str:
    """Content hash of every input of the build (sources, headers, this script).

    Content rather than mtimes: a copied tree keeps its library valid even when
    the copy reorders timestamps.
    """
    h = hashlib.sha256()
    for path in [*sources(), *headers(), Path(__file__)]:
        h.update(path.name.encode())
        h.update(path.read_bytes())
    return h.hexdigest()


def is_stale() -> bool:
    if not LIB_PATH.exists() or not HASH_PATH.exists():
        return True
    return HASH_PATH.read_text().strip() != source_digest()


def _compile(nvcc: str, src: Path, extra: list[str], verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-I", str(CSRC), "-c",
           str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, flush=True)
    return obj


def build(*, force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile and link the library if it is missing or out of date."""
    if not force and not ptxas_info and not is_stale():
        return LIB_PATH
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    with ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as pool:
        objs = list(pool.map(lambda s: _compile(nvcc, s, extra, verbose or ptxas_info), sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    HASH_PATH.write_text(source_digest() + "\n")
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v usage lines")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
