"""Build the sm_100a library libcg_b200.so in-tree (create_graph_b200/_lib/).

    python -m create_graph_b200.build [--verbose]

Each ``csrc/*.cu`` compiles to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and they link into
one shared library with a plain C ABI (``include/cg_b200.h``). Objects are
rebuilt only when a source or header is newer than them.
"""

from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
OBJ_DIR = OUT_DIR / "obj"
LIB = OUT_DIR / "libcg_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found: the sm_100a library needs the CUDA toolkit")
    return found


def _flags(verbose: bool) -> list[str]:
    flags = [
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "--expt-relaxed-constexpr",
        f"-I{ROOT / 'include'}",
        f"-I{CSRC}",
    ]
    if verbose:
        flags += ["-Xptxas", "-v"]
    return flags


def _stale(obj: pathlib.Path, src: pathlib.Path, headers: list[pathlib.Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def build(verbose: bool = False, jobs: int | None = None) -> pathlib.Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    headers = [*CSRC.glob("*.cuh"), *(ROOT / "include").glob("*.h")]
    sources = sorted(CSRC.glob("*.cu"))
    compiler = nvcc()
    flags = _flags(verbose)

    def compile_one(src: pathlib.Path):
        obj = OBJ_DIR / (src.stem + ".o")
        if not verbose and not _stale(obj, src, headers):
            return obj, ""
        cmd = [compiler, *flags, "-c", str(src), "-o", str(obj)]
        run = subprocess.run(cmd, capture_output=True, text=True)
        if run.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{run.stderr}")
        return obj, run.stderr

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_one, sources))
    if verbose:
        for _, log in results:
            if log:
                print(log)
    objs = [obj for obj, _ in results]
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [compiler, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        run = subprocess.run(cmd, capture_output=True, text=True)
        if run.returncode != 0:
            raise RuntimeError(f"linking libcg_b200.so failed:\n{run.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = parser.parse_args()
    print(build(verbose=args.verbose))


if __name__ == "__main__":
    main()
