"""Parity of bias+GELU, SwiGLU and the global sum with the CPU oracle (GPU).

Reduction sizes follow the reference (tests/test_reduction_v5.py:16-44): 0,
1, around warp/block/vector boundaries, the 524287/524288/524289 dispatch
thresholds and an odd 1,000,003, plus the benchmark's 16,777,216 and a
~2^28-element case checked against a float64 sum (relative error <= 1e-6).
"""

from __future__ import annotations

import pytest
import torch

from conftest import seeded
from cuda_operator_lab import bindings as b
from oracle import reference_math as oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
RTOL, ATOL = 1e-5, 1e-6


def close(actual, expected, rtol=RTOL, atol=ATOL):
    torch.cuda.synchronize()
    torch.testing.assert_close(actual.cpu(), expected, rtol=rtol, atol=atol)


SIZES_2D = [(0, 16), (1, 1), (1, 3), (17, 31), (64, 256), (3, 4097), (1024, 4096), (7, 1000)]


@pytest.mark.parametrize("version", range(3))
@pytest.mark.parametrize(("rows", "cols"), SIZES_2D)
def test_bias_gelu_matches_oracle(version, rows, cols):
    g = seeded(20261007 + rows * 10000 + cols)
    x = torch.randn(rows, cols, generator=g) * 2.0
    bias = torch.randn(cols, generator=g) * 0.1
    fn = getattr(b, f"fused_bias_gelu_v{version}")
    actual = fn(x.to(DEV), bias.to(DEV))
    # the fp32 bar (rtol 1e-5 / atol 1e-6) against the exact function of the fp32 inputs.  PyTorch's
    # own fp32 CPU GELU is off by up to 1.2e-6 near |z| = 3.5, so against the
    # reference's CPU path the reference tests' bar (5e-6) applies.
    exact = torch.nn.functional.gelu((x + bias).double()).float()
    close(actual, exact)
    close(actual, oracle.fused_bias_gelu(x, bias), rtol=5e-6, atol=5e-6)


@pytest.mark.parametrize("version", range(3))
@pytest.mark.parametrize(("rows", "cols"), SIZES_2D)
def test_swiglu_matches_oracle(version, rows, cols):
    g = seeded(20261008 + rows * 10000 + cols)
    gate = torch.randn(rows, cols, generator=g) * 3.0
    up = torch.randn(rows, cols, generator=g)
    fn = getattr(b, f"swiglu_v{version}")
    close(fn(gate.to(DEV), up.to(DEV)), oracle.swiglu(gate, up))


def test_swiglu_extremes_and_1d():
    gate = torch.tensor([-100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 100.0])
    up = torch.linspace(-2, 2, 7)
    close(b.swiglu_v0(gate.to(DEV), up.to(DEV)), oracle.swiglu(gate, up))


def test_pointwise_unaligned_views():
    g = seeded(20261212)
    storage = torch.randn(2 * 4096 + 1, generator=g).to(DEV)
    gate = storage[1:].view(2, 4096)
    up = torch.randn(2, 4096, generator=g).to(DEV)
    close(b.swiglu_v1(gate, up), oracle.swiglu(gate.cpu(), up.cpu()))
    bias = torch.randn(4096, generator=g).to(DEV)
    actual = b.fused_bias_gelu_v1(gate, bias)
    # as in test_bias_gelu_matches_oracle: the fp32 bar against the exact
    # function, the reference tests' bar against PyTorch's fp32 CPU GELU
    exact = torch.nn.functional.gelu((gate.cpu() + bias.cpu()).double()).float()
    close(actual, exact)
    close(actual, oracle.fused_bias_gelu(gate.cpu(), bias.cpu()), rtol=5e-6, atol=5e-6)


def test_pointwise_golden_cases(golden):
    seen = 0
    for case in golden:
        args = [a.to(DEV) for a in case["args"]]
        if case["fn"] == "fused_bias_gelu":
            actual = b.fused_bias_gelu_v2(*args)
            close(actual, case["expected"], rtol=5e-6, atol=5e-6)
        elif case["fn"] == "swiglu":
            actual = b.swiglu_v0(*args)
            close(actual, case["expected"])
        else:
            continue
        seen += 1
    assert seen >= 8


REDUCTION_SIZES = [0, 1, 2, 3, 4, 5, 31, 32, 33, 255, 256, 257, 1023, 1024, 1025, 16384, 16385,
                   32767, 32768, 32769, 262144, 524287, 524288, 524289, 1_000_003]


@pytest.mark.parametrize("version", range(6))
@pytest.mark.parametrize("n", REDUCTION_SIZES)
def test_reduction_matches_oracle(version, n):
    x = torch.rand(n, generator=seeded(20261004 + n))
    fn = getattr(b, f"reduction_v{version}")
    actual = fn(x.to(DEV))[0].cpu()
    expected64 = oracle.reduction_sum_f64(x)
    # fp64 accumulation: within one fp32 rounding of the exact sum
    assert abs(float(actual) - expected64) <= 1e-6 * max(1.0, abs(expected64))
    torch.testing.assert_close(actual, oracle.reduction_sum(x), rtol=5e-5, atol=5e-4)


def test_reduction_known_answer_resets_dirty_output(golden):
    x = torch.arange(1, 1026, dtype=torch.float32, device=DEV)
    out = torch.full((1,), 12345.0, device=DEV)
    b.reduction_v5_into(x, out)
    torch.cuda.synchronize()
    assert float(out[0]) == 525825.0
    for case in golden:
        if case["fn"] == "reduction_sum":
            actual = b.reduction_v3(case["args"][0].to(DEV))[0].cpu()
            torch.testing.assert_close(actual, case["expected"], rtol=1e-6, atol=1e-6)


def test_reduction_unaligned_and_deterministic():
    storage = torch.randn(1_000_004, generator=seeded(20261004)).to(DEV)
    x = storage[1:]
    assert x.data_ptr() % 16 == 4
    first = b.reduction_v4(x)[0].item()
    for _ in range(3):
        assert b.reduction_v4(x)[0].item() == first
    expected64 = oracle.reduction_sum_f64(x.cpu())
    assert abs(first - expected64) <= 1e-6 * max(1.0, abs(expected64))


@pytest.mark.parametrize("n", [16_777_216, (1 << 28) + 3])
def test_reduction_large_relative_error(n):
    g = torch.Generator(device=DEV)
    g.manual_seed(20261201)
    x = torch.rand(n, device=DEV, generator=g) * 2 - 1
    actual = b.reduction_v5(x)[0].item()
    expected64 = float(x.double().sum().item())
    assert abs(actual - expected64) <= 1e-6 * abs(expected64)
    partial = b.reduction_partial_f64(x)[0].item()
    assert abs(partial - expected64) <= 1e-9 * abs(expected64)
