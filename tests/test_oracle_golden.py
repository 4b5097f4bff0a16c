"""Pins the CPU oracle to the reference's own outputs (CPU).

tests/golden/reference_cases.pt was produced by importing the reference's
python/cuda_operator_lab/references.py (tests/golden/make_golden.py).  The
oracle must reproduce every case; most are bit-identical because the oracle
runs the same PyTorch CPU ops.
"""

from __future__ import annotations

import pytest
import torch

from oracle import reference_math as oracle

TOL = {
    # (rtol, atol); fp32 element-wise and row ops are expected to be exact
    "default": (1e-6, 1e-7),
    "reduction_sum": (1e-6, 1e-6),
}


def test_golden_file_covers_every_reference_function(golden):
    names = {c["fn"] for c in golden}
    expected = {
        "reduction_sum", "row_softmax", "rmsnorm", "layernorm", "fused_residual_layernorm",
        "fused_bias_gelu", "swiglu", "gemm_bias_gelu", "gemm_bias_gelu_tanh", "gemm_swiglu",
        "gemm_swiglu_packed", "gemm_swiglu_bf16_fp32_reference",
        "gemm_swiglu_bf16_workspace_reference", "gemm_swiglu_bf16_dual_fp32_reference",
    }
    assert expected <= names


def test_oracle_matches_reference_outputs(golden):
    failures = []
    for case in golden:
        fn = getattr(oracle, case["fn"])
        actual = fn(*case["args"], **case["kwargs"])
        rtol, atol = TOL.get(case["fn"], TOL["default"])
        try:
            torch.testing.assert_close(actual, case["expected"], rtol=rtol, atol=atol)
        except AssertionError as exc:  # collect all mismatches
            failures.append(f"{case['fn']}[{case['tag']}]: {exc}")
    assert not failures, "\n".join(failures)


def test_reduction_known_answer(golden):
    case = next(c for c in golden if c["tag"] == "arange_1_1025")
    assert float(case["expected"]) == 1025 * 1026 / 2
    assert oracle.reduction_sum_f64(case["args"][0]) == 525825.0


def test_softmax_large_logits_rows_sum_to_one(golden):
    case = next(c for c in golden if c["fn"] == "row_softmax" and c["tag"] == "large_logits")
    torch.testing.assert_close(case["expected"].sum(dim=-1), torch.ones(2), rtol=2e-6, atol=2e-6)


def test_oracle_rejects_what_the_reference_rejects():
    with pytest.raises(ValueError):
        oracle.rmsnorm(torch.ones(2, 4), torch.ones(3))
    with pytest.raises(ValueError):
        oracle.rmsnorm(torch.ones(2, 4), torch.ones(4), eps=0.0)
    with pytest.raises(ValueError):
        oracle.gemm_swiglu_packed(torch.ones(2, 4), torch.ones(3, 4))
