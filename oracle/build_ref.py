"""Build the reference's own CUDA library for sm_100a into oracle/_ref/.

TEST INFRASTRUCTURE ONLY: the result is a second checker (the reference's own
kernels run on the same B200 and the same inputs as ours) and a timing
yardstick; the product never loads it.

Compiles every ``csrc/*/*.cu`` of the reference checkout where it lies (no
copy, no CMake: plain nvcc, the same flags for every file) and links them into
``oracle/_ref/libcuda_operator_lab_ref.so``, which exports the reference's 54
``cuda_operator_*`` symbols.  Its cuBLAS/cuBLASLt versions dlopen the CUDA
libraries at run time, as the reference does.

Usage: python oracle/build_ref.py [/path/to/reference]; without an argument the
checkout is taken from ``$COL_REFERENCE_DIR``, else from ``reference/`` beside
this repository.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "libcuda_operator_lab_ref.so"
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC"]


def default_reference_root() -> Path:
    """The reference checkout: ``$COL_REFERENCE_DIR`` or ``../reference``
    relative to the repository root."""
    override = os.environ.get("COL_REFERENCE_DIR")
    return Path(override) if override else HERE.parent.parent / "reference"


def build(reference_root: Path | None = None) -> Path | None:
    if reference_root is None:
        reference_root = default_reference_root()
    sources = sorted((reference_root / "csrc").glob("*/*.cu"))
    if not sources:
        return None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)

    def compile_one(src: Path) -> tuple[Path, int, str]:
        obj = obj_dir / (src.stem + ".o")
        if obj.is_file() and obj.stat().st_mtime >= src.stat().st_mtime:
            return obj, 0, ""
        proc = subprocess.run([nvcc, *FLAGS, f"-I{src.parent}", "-c", str(src), "-o", str(obj)],
                              capture_output=True, text=True)
        return obj, proc.returncode, proc.stdout + proc.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=len(sources)) as pool:
        results = list(pool.map(compile_one, sources))
    for obj, rc, log in results:
        if rc != 0:
            raise RuntimeError(f"nvcc failed for {obj.name}:\n{log}")
    objs = [str(r[0]) for r in results]
    proc = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o",
                           str(LIB), *objs, "-ldl"], capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}{proc.stderr}")
    return LIB


if __name__ == "__main__":
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else default_reference_root()
    print(build(root))
