"""The reference's own Python bindings drive this library (CPU, no compute).

The drop-in claim, checked with the reference's module itself rather than a
restatement: ``python/cuda_operator_lab/bindings.py`` of the reference checkout
is imported from where it lies, ``CUDA_OPERATOR_LIB`` points it at this
library, and its ``_Library`` resolves every symbol it declares (eagerly, as
it does on its first call) with its own argtypes and restypes.  Those
declarations must equal this library's (``include/cuda_operator_lab.h`` via
``bindings._SIGNATURES``), its error path must decode this library's codes,
and its host-side validation must behave like ours on the inputs its tests
reject.  No kernel is launched (there is no GPU here); the reference's GPU
tests cannot run on the GPU box, which has no reference checkout, so the
contract tests in ``test_gpu_contract.py`` restate them there.

Skipped when the checkout is absent (``$COL_REFERENCE_DIR``, else
``reference/`` beside this repository).
"""

from __future__ import annotations

import ctypes
import importlib.util
import os
from pathlib import Path

import pytest
import torch

from conftest import ROOT
from cuda_operator_lab import bindings as ours


def _reference_root() -> Path:
    override = os.environ.get("COL_REFERENCE_DIR")
    return Path(override) if override else ROOT.parent / "reference"


@pytest.fixture()
def reference_bindings(monkeypatch):
    path = _reference_root() / "python" / "cuda_operator_lab" / "bindings.py"
    if not path.is_file():
        pytest.skip("reference checkout not present")
    if not ours.library_path().is_file():
        pytest.skip("library not built")
    monkeypatch.setenv("CUDA_OPERATOR_LIB", str(ours.library_path()))
    spec = importlib.util.spec_from_file_location("reference_bindings_under_test", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_reference_module_resolves_every_symbol_with_our_signatures(reference_bindings):
    lib = reference_bindings._library()
    assert lib.handle._name == str(ours.library_path())
    checked = 0
    for name in ours.REFERENCE_SYMBOLS:
        fn = getattr(lib.handle, name)
        assert fn.argtypes is not None, f"the reference declares no argtypes for {name}"
        assert list(fn.argtypes) == list(ours._SIGNATURES[name]), name
        expected_res = ctypes.c_char_p if name == "cuda_operator_error_string" else ctypes.c_int
        assert fn.restype is expected_res, name
        checked += 1
    assert checked == 54


def test_reference_module_decodes_our_error_codes(reference_bindings):
    lib = reference_bindings._library()
    with pytest.raises(RuntimeError, match=r"CUDA error 1: invalid argument"):
        lib.check(1)
    with pytest.raises(RuntimeError, match=r"CUDA error 10004: "):
        lib.check(10004)  # a library code: the message comes from this library


@pytest.mark.parametrize("name", ["reduction_v5", "softmax_v5", "rmsnorm_v4", "layernorm_v5",
                                  "fused_residual_layernorm_v4", "fused_bias_gelu_v2",
                                  "swiglu_v2", "gemm_bias_gelu_v6", "gemm_swiglu_v11"])
def test_reference_and_our_wrappers_reject_cpu_tensors_alike(reference_bindings, name):
    shapes = {
        "reduction_v5": [(8,)], "softmax_v5": [(2, 8)], "rmsnorm_v4": [(2, 8), (8,)],
        "layernorm_v5": [(2, 8), (8,), (8,)], "fused_residual_layernorm_v4": [(2, 8)] * 2 + [(8,)] * 2,
        "fused_bias_gelu_v2": [(2, 8), (8,)], "swiglu_v2": [(2, 8), (2, 8)],
        "gemm_bias_gelu_v6": [(2, 8), (4, 8), (4,)], "gemm_swiglu_v11": [(2, 8), (8, 8)],
    }[name]
    args = [torch.zeros(s, dtype=torch.bfloat16 if name == "gemm_swiglu_v11" else torch.float32)
            for s in shapes]
    errors = []
    for module in (reference_bindings, ours):
        with pytest.raises((ValueError, TypeError)) as info:
            getattr(module, name)(*args)
        errors.append(type(info.value))
        assert "CUDA" in str(info.value)
    assert errors[0] is errors[1]
