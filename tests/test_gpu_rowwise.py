"""Parity of the row-wise kernels (RMSNorm, LayerNorm, residual+LayerNorm,
residual+RMSNorm, softmax) with the CPU oracle and the reference's golden
outputs (GPU).

Shapes follow the reference's tests (tests/test_rmsnorm_v0.py:16-32,
tests/test_softmax_v2.py:16-41): empty, single element, widths around the
warp (31/32/33) and vector boundaries, odd widths (4097, 8193), the
benchmark-workload shapes and rows wider than the register path (the streaming
kernel).  Tolerance: the fp32 bar, rtol 1e-5 / atol 1e-6.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import seeded
from cuda_operator_lab import bindings as b
from oracle import reference_math as oracle

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6
SHAPES = [(0, 128), (1, 1), (1, 3), (2, 31), (2, 32), (2, 33), (7, 127), (64, 128), (33, 512),
          (17, 1024), (8, 4097), (11, 257), (32, 4096), (128, 4096), (128, 8192), (5, 12289),
          (3, 33000), (2, 40000),
          # few wide rows, 8 vectors per thread, and more rows than SMs
          (3, 2052), (7, 6144), (100, 16384), (296, 4096)]
DEV = "cuda"


def close(actual: torch.Tensor, expected: torch.Tensor, rtol=RTOL, atol=ATOL) -> None:
    torch.cuda.synchronize()
    torch.testing.assert_close(actual.cpu(), expected, rtol=rtol, atol=atol)


@pytest.mark.parametrize("version", range(5))
@pytest.mark.parametrize(("rows", "cols"), SHAPES)
def test_rmsnorm_matches_oracle(version, rows, cols):
    g = seeded(20261005 + rows * 10000 + cols)
    x = torch.randn(rows, cols, generator=g)
    w = torch.rand(cols, generator=g) + 0.5
    fn = getattr(b, f"rmsnorm_v{version}")
    close(fn(x.to(DEV), w.to(DEV), 1e-6), oracle.rmsnorm(x, w, 1e-6))


def test_rmsnorm_large_magnitude_signed_weight():
    x = torch.tensor([[1000.0, -1000.0, 500.0, -500.0]])
    w = torch.tensor([1.0, 0.5, -2.0, 3.0])
    close(b.rmsnorm_v4(x.to(DEV), w.to(DEV)), oracle.rmsnorm(x, w))


@pytest.mark.parametrize(("rows", "cols"), [(1, 1), (3, 100), (16384 // 64, 4096), (7, 4104),
                                            (5, 2000), (2, 70000)])
def test_rmsnorm_bf16_matches_oracle(rows, cols):
    g = seeded(20261201 + rows + cols)
    x = torch.randn(rows, cols, generator=g).to(torch.bfloat16)
    w = (torch.rand(cols, generator=g) + 0.5).to(torch.bfloat16)
    actual = b.rmsnorm_bf16(x.to(DEV), w.to(DEV), 1e-6).cpu().float()
    expected = oracle.rmsnorm_bf16(x, w, 1e-6).float()
    # one bf16 rounding step of difference at most (2^-8 relative)
    torch.testing.assert_close(actual, expected, rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("version", range(6))
@pytest.mark.parametrize(("rows", "cols"), SHAPES)
def test_layernorm_matches_oracle(version, rows, cols):
    g = seeded(20261005 + rows * 10000 + cols)
    x = torch.randn(rows, cols, generator=g)
    w = torch.rand(cols, generator=g) + 0.5
    bias = torch.randn(cols, generator=g) * 0.1
    fn = getattr(b, f"layernorm_v{version}")
    close(fn(x.to(DEV), w.to(DEV), bias.to(DEV), 1e-5), oracle.layernorm(x, w, bias, 1e-5))


def test_layernorm_large_offset_against_float64():
    # reference tests/test_layernorm_v3.py:56-84
    g = seeded(20261005)
    x = torch.randn(64, 4096, generator=g) * 0.1 + 1000.0
    w = torch.randn(4096, generator=g)
    bias = torch.randn(4096, generator=g)
    actual = b.layernorm_v3(x.to(DEV), w.to(DEV), bias.to(DEV)).cpu()
    x64 = x.double()
    mean = x64.mean(dim=-1, keepdim=True)
    var = (x64 - mean).square().mean(dim=-1, keepdim=True)
    expected = ((x64 - mean) * torch.rsqrt(var + 1e-5) * w.double() + bias.double()).float()
    err = (actual - expected).abs()
    assert float(err.max()) < 2.5e-3
    assert float(err.mean()) < 2.5e-4


@pytest.mark.parametrize("version", range(5))
@pytest.mark.parametrize(("rows", "cols"), SHAPES)
def test_residual_layernorm_matches_oracle(version, rows, cols):
    g = seeded(20261006 + rows * 10000 + cols)
    x = torch.randn(rows, cols, generator=g)
    r = torch.randn(rows, cols, generator=g)
    w = torch.rand(cols, generator=g) + 0.5
    bias = torch.randn(cols, generator=g) * 0.1
    fn = getattr(b, f"fused_residual_layernorm_v{version}")
    close(fn(x.to(DEV), r.to(DEV), w.to(DEV), bias.to(DEV)),
          oracle.fused_residual_layernorm(x, r, w, bias))


@pytest.mark.parametrize(("rows", "cols"), SHAPES)
def test_residual_layernorm_h_stores_sum_and_norm(rows, cols):
    g = seeded(20261007 + rows * 10000 + cols)
    x = torch.randn(rows, cols, generator=g)
    r = torch.randn(rows, cols, generator=g)
    w = torch.rand(cols, generator=g) + 0.5
    bias = torch.randn(cols, generator=g) * 0.1
    h, y = b.fused_residual_layernorm_h(x.to(DEV), r.to(DEV), w.to(DEV), bias.to(DEV))
    h_ref, y_ref = oracle.fused_residual_layernorm_h(x, r, w, bias)
    close(h, h_ref, rtol=0, atol=0)
    close(y, y_ref)


@pytest.mark.parametrize(("rows", "cols"), SHAPES)
def test_residual_rmsnorm_fp32_stores_sum_and_norm(rows, cols):
    g = seeded(20261208 + rows * 10000 + cols)
    x = torch.randn(rows, cols, generator=g)
    r = torch.randn(rows, cols, generator=g)
    w = torch.rand(cols, generator=g) + 0.5
    h, y = b.fused_residual_rmsnorm(x.to(DEV), r.to(DEV), w.to(DEV), 1e-6)
    h_ref, y_ref = oracle.fused_residual_rmsnorm(x, r, w, 1e-6)
    close(h, h_ref, rtol=0, atol=0)
    close(y, y_ref)


@pytest.mark.parametrize(("rows", "cols"), [(0, 64), (1, 1), (3, 100), (16384 // 64, 4096),
                                            (7, 4104), (5, 2000), (2, 70000)])
def test_residual_rmsnorm_bf16_stores_sum_and_norm(rows, cols):
    g = seeded(20261209 + rows + cols)
    x = torch.randn(rows, cols, generator=g).to(torch.bfloat16)
    r = torch.randn(rows, cols, generator=g).to(torch.bfloat16)
    w = (torch.rand(cols, generator=g) + 0.5).to(torch.bfloat16)
    h, y = b.fused_residual_rmsnorm(x.to(DEV), r.to(DEV), w.to(DEV), 1e-6)
    h_ref, y_ref = oracle.fused_residual_rmsnorm(x, r, w, 1e-6)
    torch.cuda.synchronize()
    # h: one bf16 add, bit for bit; y: within one bf16 rounding step
    assert torch.equal(h.cpu(), h_ref)
    torch.testing.assert_close(y.cpu().float(), y_ref.float(), rtol=2 ** -7, atol=1e-6)


def test_residual_rmsnorm_argument_checks():
    x = torch.randn(4, 64, device=DEV)
    w = torch.ones(64, device=DEV)
    with pytest.raises(ValueError):
        b.fused_residual_rmsnorm(x, x[:, :32].contiguous(), w)
    with pytest.raises(ValueError):
        b.fused_residual_rmsnorm(x, x, w, eps=0.0)
    out = torch.empty_like(x)
    P, U, F = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_float
    lib = b._library()
    # rows == 0 succeeds before pointer checks; a NULL pointer is invalid (1)
    assert lib.handle.cuda_operator_fused_residual_rmsnorm_h(
        None, None, None, None, None, U(0), U(64), F(1e-5), None) == 0
    assert lib.handle.cuda_operator_fused_residual_rmsnorm_h(
        P(x.data_ptr()), None, P(w.data_ptr()), P(out.data_ptr()), P(out.data_ptr()), U(4), U(64),
        F(1e-5), None) == 1


@pytest.mark.parametrize("version", range(6))
@pytest.mark.parametrize(("rows", "cols"), SHAPES + [(1024, 128), (33, 8193)])
def test_softmax_matches_oracle(version, rows, cols):
    g = seeded(20261005 + rows * 10000 + cols)
    x = torch.randn(rows, cols, generator=g) * 2.0  # logits ~ N(0, 4)
    fn = getattr(b, f"softmax_v{version}")
    close(fn(x.to(DEV)), oracle.row_softmax(x))


def test_softmax_large_logits_and_normalisation():
    x = torch.tensor([[1000.0, 1001.0, 999.0, 998.0], [-1000.0, -999.0, -1001.0, -1002.0]])
    y = b.softmax_v5(x.to(DEV))
    close(y, oracle.row_softmax(x))
    close(y.sum(dim=-1), torch.ones(2), rtol=2e-6, atol=2e-6)
    z = b.softmax_v2(torch.randn(128, 4097, device=DEV))
    close(z.sum(dim=-1), torch.ones(128), rtol=4e-6, atol=4e-6)


def test_rowwise_golden_cases(golden):
    ops = {
        "row_softmax": lambda x: b.softmax_v5(x),
        "rmsnorm": lambda x, w, eps=1e-5: b.rmsnorm_v4(x, w, eps),
        "layernorm": lambda x, w, bias: b.layernorm_v5(x, w, bias),
        "fused_residual_layernorm": lambda x, r, w, bias: b.fused_residual_layernorm_v4(x, r, w, bias),
    }
    seen = 0
    for case in golden:
        if case["fn"] not in ops:
            continue
        args = [a.to(DEV) for a in case["args"]]
        actual = ops[case["fn"]](*args, **case["kwargs"])
        if case["tag"] == "offset_1000":
            # rows of 1000 + 0.1 N(0,1): fp32 LayerNorm is only accurate to
            # ~1e-3 here (PyTorch's CPU result is off by up to 4e-3 from the
            # float64 value), so check against float64 as the reference's own
            # test does (tests/test_layernorm_v3.py:56-84) and loosely against
            # the recorded CPU result.
            x64, w64, b64 = (a.double() for a in case["args"])
            mean = x64.mean(dim=-1, keepdim=True)
            var = (x64 - mean).square().mean(dim=-1, keepdim=True)
            exact = ((x64 - mean) * torch.rsqrt(var + 1e-5) * w64 + b64).float()
            assert float((actual.cpu() - exact).abs().max()) < 2.5e-3
            close(actual, case["expected"], rtol=RTOL, atol=1e-2)
        else:
            close(actual, case["expected"], rtol=RTOL, atol=ATOL)
        seen += 1
    assert seen >= 20


def test_unaligned_rows_use_scalar_path():
    storage = torch.randn(4 * 256 + 1, device=DEV)
    x = storage[1:].view(4, 256)
    assert x.data_ptr() % 16 != 0
    w = torch.rand(256, device=DEV) + 0.5
    close(b.rmsnorm_v3(x, w), oracle.rmsnorm(x.cpu(), w.cpu()))
    close(b.softmax_v4(x), oracle.row_softmax(x.cpu()))
