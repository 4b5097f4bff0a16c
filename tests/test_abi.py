"""The C-ABI library builds, loads and exports every declared symbol (CPU).

No compute call is made: these run without a GPU.
"""

from __future__ import annotations

import ctypes
import re
import subprocess

from conftest import PACKAGE_DIR, ROOT

HEADER = ROOT / "include" / "cuda_operator_lab.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cuda_operator_\w+)\s*\(", text)))


def library():
    from cuda_operator_lab import bindings

    path = bindings.library_path()
    if not path.is_file():
        import importlib.util

        spec = importlib.util.spec_from_file_location("col_build", PACKAGE_DIR / "build.py")
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
        module.build()
    return path


def test_header_declares_reference_abi_and_extensions():
    names = declared_symbols()
    from cuda_operator_lab import bindings

    assert len(bindings.REFERENCE_SYMBOLS) == 54
    assert set(bindings.REFERENCE_SYMBOLS) <= set(names)
    assert set(names) == set(bindings._SIGNATURES)


def test_library_exports_every_declared_symbol():
    path = library()
    handle = ctypes.CDLL(str(path))
    for name in declared_symbols():
        assert hasattr(handle, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (cuda_operator_\w+)", out.stdout))
    assert exported == set(declared_symbols())


def test_bindings_load_library_and_report_build_tag():
    library()
    from cuda_operator_lab import bindings

    assert "sm_100a" in bindings.build_tag()


def test_error_strings_cover_library_codes():
    library()
    from cuda_operator_lab import bindings

    lib = bindings._library()
    assert b"invalid argument" in lib.handle.cuda_operator_error_string(1)
    assert b"cuTensorMapEncodeTiled" in lib.handle.cuda_operator_error_string(10001)
    try:
        lib.check(1)
    except RuntimeError as exc:
        assert str(exc).startswith("CUDA error 1:")
    else:
        raise AssertionError("check(1) did not raise")


def test_plain_c_program_links_against_the_library(tmp_path):
    """A C99 caller (no PyTorch, no CUDA headers beyond the library's) includes
    the header, links the shared library and calls its host-only entry points."""
    import shutil

    import pytest

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    libdir = library().parent
    src = tmp_path / "caller.c"
    src.write_text(
        '#include "cuda_operator_lab.h"\n'
        "#include <stdio.h>\n"
        "#include <string.h>\n"
        "int main(void) {\n"
        "  const char* tag = cuda_operator_lab_build_tag();\n"
        "  const char* msg = cuda_operator_error_string(10005);\n"
        "  if (!tag || !strstr(tag, \"sm_100a\") || !msg || !strstr(msg, \"gathering\")) return 1;\n"
        "  if (cuda_operator_lab_peer_handle_bytes() != 64) return 2;\n"
        "  printf(\"%s\\n\", tag);\n"
        "  return 0;\n"
        "}\n")
    exe = tmp_path / "caller"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(src),
                    f"-L{libdir}", "-lcuda_operator_lab", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out
    assert "sm_100a" in out.stdout
    # the header is also valid C++
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-x", "c++", f"-I{ROOT / 'include'}",
                    str(HEADER)], check=True)
