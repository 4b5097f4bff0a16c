"""Build libcuda_operator_lab.so for sm_100a from csrc/*.cu.

Each translation unit is compiled in parallel with nvcc
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) and linked into
``build/lib/libcuda_operator_lab.so`` next to this file, the path the Python
bindings load by default.  Objects are rebuilt only when a source or header is
newer than the object.  Usage: ``python build.py [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
OBJ_DIR = ROOT / "build" / "obj"
LIB_DIR = ROOT / "build" / "lib"
LIB_PATH = LIB_DIR / "libcuda_operator_lab.so"
INCLUDE = ROOT.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    fallback = Path("/usr/local/cuda/bin/nvcc")
    if fallback.is_file():
        return str(fallback)
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build the library")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.is_file():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def _compile(src: Path, obj: Path) -> tuple[Path, int, str]:
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    return src, proc.returncode, proc.stdout + proc.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    headers = _headers()
    todo = []
    for src in sources:
        obj = OBJ_DIR / (src.stem + ".o")
        if force or _stale(obj, src, headers):
            todo.append((src, obj))
    workers = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    failures = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        for src, rc, log in pool.map(lambda so: _compile(*so), todo):
            if verbose or rc != 0:
                sys.stderr.write(f"[build] {src.name}: rc={rc}\n{log}")
            if rc != 0:
                failures.append(src.name)
    if failures:
        raise RuntimeError(f"nvcc failed for: {', '.join(failures)}")
    objs = [OBJ_DIR / (s.stem + ".o") for s in sources]
    if force or todo or not LIB_PATH.is_file():
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))


if __name__ == "__main__":
    main()
