"""Parity of the GEMM epilogue kernels with the CPU oracle (GPU).

bf16 operands run on the tcgen05 tensor-core kernel (TMA-addressable shapes)
or the CUDA-core kernel (K not a multiple of 8); fp32 operands run on the same
tensor-core kernel through a three-part bf16 split (m*n*k >= 4e6) or on the
CUDA-core kernel (smaller problems).  Tolerances: bf16 epilogues rtol 2e-2 / atol 2e-2 against
the fp32-accumulated reference (the project's bf16 bar), fp32 epilogues rtol/atol 3e-4
(reference tests/test_gemm_bias_gelu_v0.py).  Shapes follow the reference's
tests (tests/test_gemm_swiglu_v4.py:16-28, test_gemm_swiglu_v11.py:19-31)
plus tile-boundary and benchmark-workload shapes.
"""

from __future__ import annotations

import pytest
import torch

from conftest import seeded
from cuda_operator_lab import bindings as b
from oracle import reference_math as oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF_RTOL, BF_ATOL = 2e-2, 2e-2
F32_TOL = 3e-4


@pytest.fixture(autouse=True)
def no_wait_timeouts():
    b.gemm_status(clear=True)
    yield
    assert b.gemm_status(clear=True) == 0, "a bounded mbarrier wait timed out"


def bf16_inputs(m, k, n, seed, scale=None):
    g = seeded(seed)
    s = scale if scale is not None else k ** -0.5
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wg = (torch.randn(n, k, generator=g) * s).to(torch.bfloat16)
    wu = (torch.randn(n, k, generator=g) * s).to(torch.bfloat16)
    return x, wg, wu


def close(actual, expected, rtol, atol):
    torch.cuda.synchronize()
    torch.testing.assert_close(actual.cpu().float(), expected.float(), rtol=rtol, atol=atol)


BF16_SHAPES = [
    (1, 8, 1), (4, 16, 32), (16, 64, 64), (17, 40, 24), (32, 128, 256), (64, 256, 512),
    (128, 64, 2048), (128, 512, 1024), (129, 72, 130), (200, 136, 300), (128, 1024, 4096),
    (512, 1024, 4096), (384, 4096, 256), (1000, 520, 700),
]


@pytest.mark.parametrize("version", [4, 10, 11])
@pytest.mark.parametrize(("m", "k", "n"), BF16_SHAPES)
def test_packed_bf16_swiglu_fp32_out(version, m, k, n):
    x, wg, wu = bf16_inputs(m, k, n, 20261025 + m * 1000000 + k * 1000 + n)
    packed = torch.cat((wg, wu), dim=0).contiguous()
    fn = getattr(b, f"gemm_swiglu_v{version}")
    actual = fn(x.to(DEV), packed.to(DEV))
    close(actual, oracle.gemm_swiglu_bf16_fp32_reference(x, packed), BF_RTOL, BF_ATOL)


@pytest.mark.parametrize(("m", "k", "n"), [(1, 1, 1), (4, 16, 32), (17, 31, 63), (33, 100, 70)])
def test_packed_bf16_swiglu_unaddressable_k_uses_cuda_cores(m, k, n):
    x, wg, wu = bf16_inputs(m, k, n, 20261026 + m + k + n)
    packed = torch.cat((wg, wu), dim=0).contiguous()
    close(b.gemm_swiglu_v4(x.to(DEV), packed.to(DEV)),
          oracle.gemm_swiglu_bf16_fp32_reference(x, packed), BF_RTOL, BF_ATOL)


@pytest.mark.parametrize(("m", "k", "n"), [(16, 64, 64), (32, 128, 256), (256, 512, 384),
                                           (128, 1024, 4096)])
def test_packed_bf16_swiglu_bf16_workspace_semantics(m, k, n):
    x, wg, wu = bf16_inputs(m, k, n, 20261027 + m + k + n)
    packed = torch.cat((wg, wu), dim=0).contiguous()
    close(b.gemm_swiglu_v5(x.to(DEV), packed.to(DEV)),
          oracle.gemm_swiglu_bf16_workspace_reference(x, packed), 1e-2, 1e-1)


@pytest.mark.parametrize(("version", "m", "k", "n"), [
    (6, 16, 16, 64), (6, 32, 128, 256), (6, 48, 80, 16), (7, 16, 16, 64), (7, 128, 512, 1024),
    (8, 32, 64, 128), (8, 64, 256, 512), (9, 16, 16, 128), (9, 128, 1024, 4096)])
def test_dual_bf16_swiglu(version, m, k, n):
    x, wg, wu = bf16_inputs(m, k, n, 20261019 + m * 1000000 + k * 1000 + n, scale=1.0)
    fn = getattr(b, f"gemm_swiglu_v{version}")
    actual = fn(x.to(DEV), wg.to(DEV), wu.to(DEV))
    # unit-variance weights as in the reference tests: values grow with sqrt(k)
    close(actual, oracle.gemm_swiglu_bf16_dual_fp32_reference(x, wg, wu), 5e-3, 5e-2 * (k ** 0.5))


@pytest.mark.parametrize(("version", "m", "k", "n"), [(6, 17, 32, 64), (7, 32, 33, 64),
                                                      (8, 16, 16, 64), (9, 16, 16, 64)])
def test_dual_bf16_swiglu_shape_guards(version, m, k, n):
    x, wg, wu = bf16_inputs(m, k, n, 1)
    with pytest.raises(ValueError):
        getattr(b, f"gemm_swiglu_v{version}")(x.to(DEV), wg.to(DEV), wu.to(DEV))


# (16384, 512, 1792) and (8192, 1024, 1792): many tiles per CTA pair, ending in a
# nearly empty last wave (the 8-GPU shard shape of the benchmark, shorter K)
@pytest.mark.parametrize(("m", "k", "n"), [(1, 8, 1), (16, 64, 64), (100, 256, 300),
                                           (128, 64, 2048), (512, 4096, 4096), (1000, 1024, 1500),
                                           (16384, 512, 1792), (8192, 1024, 1792)])
def test_gemm_swiglu_bf16_output(m, k, n):
    x, wg, wu = bf16_inputs(m, k, n, 20261201 + m + k + n)
    packed = torch.cat((wg, wu), dim=0).contiguous()
    actual = b.gemm_swiglu_bf16(x.to(DEV), packed.to(DEV))
    assert actual.dtype == torch.bfloat16
    close(actual, oracle.gemm_swiglu_bf16_fp32_reference(x, packed), BF_RTOL, BF_ATOL)


# (512, 4096, 4096), (300, 2048, 1000), (512, 1024, 4096), (256, 8192, 512) and
# (768, 4096, 2048) run the split-K cluster kernel (two CTA pairs per tile,
# each half of K, partial accumulator exchanged through distributed shared
# memory), the others one CTA (pair) per tile
@pytest.mark.parametrize(("m", "k", "n"), [(1, 8, 1), (16, 64, 64), (100, 256, 300),
                                           (512, 4096, 4096), (257, 520, 1000), (3, 30, 5),
                                           (300, 2048, 1000), (512, 1024, 4096),
                                           (256, 8192, 512), (768, 4096, 2048)])
def test_gemm_bias_gelu_bf16(m, k, n):
    g = seeded(20261202 + m + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    bias = torch.randn(n, generator=g) * 0.1
    actual = b.gemm_bias_gelu_bf16(x.to(DEV), w.to(DEV), bias.to(DEV))
    close(actual, oracle.gemm_bias_gelu(x.float(), w.float(), bias), BF_RTOL, BF_ATOL)


# below 4e6 multiply-adds: CUDA cores; from (64, 256, 512) on: tensor cores,
# including ragged K (77, 520: split parts padded to 64) and ragged M/N
FP32_SHAPES = [(1, 1, 1), (1, 7, 13), (4, 16, 32), (17, 31, 63), (32, 128, 256), (64, 256, 512),
               (300, 77, 515), (1, 1024, 4096), (257, 520, 1000), (128, 512, 1024)]


@pytest.mark.parametrize("version", range(7))
@pytest.mark.parametrize(("m", "k", "n"), FP32_SHAPES)
def test_fp32_gemm_bias_gelu(version, m, k, n):
    g = seeded(20261005 + m * 1000000 + k * 1000 + n)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g)
    bias = torch.randn(n, generator=g)
    fn = getattr(b, f"gemm_bias_gelu_v{version}")
    ref = oracle.gemm_bias_gelu if version <= 1 else oracle.gemm_bias_gelu_tanh
    close(fn(x.to(DEV), w.to(DEV), bias.to(DEV)), ref(x, w, bias), F32_TOL, F32_TOL)


@pytest.mark.parametrize("version", range(4))
@pytest.mark.parametrize(("m", "k", "n"), FP32_SHAPES[:-1])
def test_fp32_gemm_swiglu(version, m, k, n):
    g = seeded(20261010 + m * 1000000 + k * 1000 + n)
    x = torch.randn(m, k, generator=g)
    wg = torch.randn(n, k, generator=g)
    wu = torch.randn(n, k, generator=g)
    fn = getattr(b, f"gemm_swiglu_v{version}")
    if version <= 1:
        actual = fn(x.to(DEV), wg.to(DEV), wu.to(DEV))
    else:
        actual = fn(x.to(DEV), torch.cat((wg, wu), 0).to(DEV))
    expected = oracle.gemm_swiglu(x, wg, wu)
    close(actual, expected, F32_TOL, F32_TOL * max(1.0, float(expected.abs().max()) / 100))


@pytest.mark.parametrize(("m", "k", "n"), [(256, 2048, 512), (130, 4000, 260)])
def test_fp32_tensor_core_split_matches_float64(m, k, n):
    # The three-part split keeps ~24 significand bits per operand and the
    # chunked accumulation keeps the tensor core's truncating adds short:
    # against a float64 GEMM the error stays below 3e-7 of sum_k |x||w| (one
    # unchunked accumulation reaches ~4e-6 at k = 2048, a bf16-only GEMM ~1e-4).
    g = seeded(20261130 + m + k + n)
    x = torch.randn(m, k, generator=g) * torch.exp(torch.randn(m, 1, generator=g))
    w = torch.randn(n, k, generator=g)
    bias = torch.zeros(n)
    actual = b.gemm_bias_gelu_v0(x.to(DEV), w.to(DEV), bias.to(DEV)).cpu().double()
    pre = x.double() @ w.double().T
    expected = torch.nn.functional.gelu(pre)
    scale = x.double().abs() @ w.double().abs().T
    err = (actual - expected).abs() / (scale + 1e-30)
    assert float(err.max()) < 3e-7, float(err.max())


# Few tiles and long K, including ragged K and N: SwiGLU (fp32 out) and
# bias+GELU (bf16 out) against the oracle, and reproducible bit for bit.
@pytest.mark.parametrize(("m", "k", "n"), [(128, 2048, 4096), (256, 1024, 1536), (100, 3000, 300),
                                           (512, 4096, 4096), (384, 8192, 1000)])
def test_long_k_few_tiles(m, k, n):
    x, wg, wu = bf16_inputs(m, k, n, 20261203 + m + k + n)
    packed = torch.cat((wg, wu), dim=0).contiguous()
    xd, pd = x.to(DEV), packed.to(DEV)
    expected = oracle.gemm_swiglu_bf16_fp32_reference(x, packed)
    first = b.gemm_swiglu_v11(xd, pd)
    close(first, expected, BF_RTOL, BF_ATOL)
    assert torch.equal(first, b.gemm_swiglu_v11(xd, pd)), "results must be reproducible"
    bias = torch.randn(n, generator=seeded(m + n)) * 0.1
    out = b.gemm_bias_gelu_bf16(xd, wg.to(DEV), bias.to(DEV))
    close(out, oracle.gemm_bias_gelu(x.float(), wg.float(), bias), BF_RTOL, BF_ATOL)


@pytest.mark.parametrize(("m", "k", "n"), [(1, 8, 1), (16, 64, 64), (100, 256, 300),
                                           (512, 14336, 4096), (257, 520, 1000), (3, 30, 5),
                                           (1024, 4096, 4096), (300, 2048, 1000)])
def test_gemm_residual_bf16(m, k, n):
    g = seeded(20261210 + m + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16)
    actual = b.gemm_residual_bf16(x.to(DEV), w.to(DEV), res.to(DEV))
    close(actual, oracle.gemm_residual_bf16(x, w, res), BF_RTOL, BF_ATOL)


def test_gemm_residual_bf16_in_place():
    g = seeded(20261211)
    m, k, n = 384, 1024, 768
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(torch.bfloat16).to(DEV)
    h = torch.randn(m, n, generator=g).to(torch.bfloat16).to(DEV)
    expected = oracle.gemm_residual_bf16(x.cpu(), w.cpu(), h.cpu())
    b.gemm_residual_bf16_into(x, w, h, h)  # h += x @ w.T
    close(h, expected, BF_RTOL, BF_ATOL)


@pytest.mark.parametrize(("m", "k", "n"), [(1, 8, 1), (100, 256, 300), (512, 4096, 4096),
                                           (257, 520, 1000), (2048, 4096, 14336 // 8)])
def test_rmsnorm_folded_into_gemm_swiglu(m, k, n):
    g = seeded(20261213 + m + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w_norm = (torch.rand(k, generator=g) + 0.5).to(torch.bfloat16)
    _, wg, wu = bf16_inputs(m, k, n, 20261214 + m + k + n)
    packed = torch.cat((wg, wu), 0).contiguous()
    folded = b.fold_rmsnorm_weight(packed, w_norm)
    xd = x.to(DEV)
    rstd = b.rmsnorm_rstd_bf16(xd, 1e-6)
    torch.cuda.synchronize()
    torch.testing.assert_close(rstd.cpu(), oracle.rmsnorm_rstd(x, 1e-6), rtol=1e-5, atol=1e-7)
    actual = b.gemm_swiglu_rowscale_bf16(xd, rstd, folded.to(DEV))
    close(actual, oracle.gemm_swiglu_rowscale_bf16(x, rstd.cpu(), folded), BF_RTOL, BF_ATOL)
    # Against the unfused block (RMSNorm to bf16, then the packed GEMM+SwiGLU)
    # the folded form agrees within 3e-2, not the 2e-2 bar: its one bf16
    # rounding falls on W * w instead of on the normalised X, and at the 2e-2
    # bar a few elements in a million differ by more (a CPU emulation of both
    # on 4M outputs: max 1.34x the bound).  The benchmark's headline step is
    # therefore the unfused block, pinned at 2e-2 in test_gpu_headline.py.
    unfused = oracle.gemm_swiglu_bf16_fp32_reference(oracle.rmsnorm_bf16(x, w_norm, 1e-6), packed)
    close(actual, unfused, 3e-2, 3e-2)


def test_gemm_golden_cases(golden):
    seen = 0
    for case in golden:
        args = [a.to(DEV) for a in case["args"]]
        fn = case["fn"]
        if fn == "gemm_swiglu_bf16_fp32_reference":
            actual, tol = b.gemm_swiglu_v11(*args), (BF_RTOL, BF_ATOL)
        elif fn == "gemm_swiglu_bf16_dual_fp32_reference":
            x, wg, wu = args
            actual, tol = b.gemm_swiglu_v10(x, torch.cat((wg, wu), 0)), (BF_RTOL, BF_ATOL)
        elif fn == "gemm_swiglu_bf16_workspace_reference":
            actual, tol = b.gemm_swiglu_v5(*args), (1e-2, 1e-1)
        elif fn == "gemm_bias_gelu":
            actual, tol = b.gemm_bias_gelu_v0(*args), (F32_TOL, F32_TOL)
        elif fn == "gemm_bias_gelu_tanh":
            actual, tol = b.gemm_bias_gelu_v6(*args), (F32_TOL, F32_TOL)
        elif fn == "gemm_swiglu":
            actual, tol = b.gemm_swiglu_v1(*args), (F32_TOL, F32_TOL)
        elif fn == "gemm_swiglu_packed":
            actual, tol = b.gemm_swiglu_v3(*args), (F32_TOL, F32_TOL)
        else:
            continue
        close(actual, case["expected"], *tol)
        seen += 1
    assert seen >= 20


def test_tensor_core_path_is_exact_on_integer_inputs():
    # Small integers are exact in bf16 and their products/sums exact in fp32:
    # the tensor-core result must equal the CPU result bit for bit.
    g = seeded(5)
    m, k, n = 256, 512, 384
    x = torch.randint(-3, 4, (m, k), generator=g).to(torch.bfloat16)
    wg = torch.randint(-2, 3, (n, k), generator=g).to(torch.bfloat16)
    wu = torch.randint(-2, 3, (n, k), generator=g).to(torch.bfloat16)
    packed = torch.cat((wg, wu), 0).contiguous()
    gate = x.float() @ wg.float().T
    up = x.float() @ wu.float().T
    actual = b.gemm_swiglu_v4(x.to(DEV), packed.to(DEV)).cpu()
    expected = torch.nn.functional.silu(gate) * up
    torch.testing.assert_close(actual, expected, rtol=1e-6, atol=1e-5)


def test_packed_versions_agree_bit_for_bit():
    # reference tests/test_gemm_swiglu_v11.py:51 (v11 equals v10 exactly); here
    # every packed bf16 version with fp32 output runs the same kernel
    x, wg, wu = bf16_inputs(384, 1024, 768, 91)
    packed = torch.cat((wg, wu), 0).contiguous().to(DEV)
    xd = x.to(DEV)
    v4, v10, v11 = (getattr(b, f"gemm_swiglu_v{v}")(xd, packed) for v in (4, 10, 11))
    torch.cuda.synchronize()
    assert torch.equal(v10, v11) and torch.equal(v4, v11)


def test_split_k_gemm_is_bitwise_stable():
    # the split-K cluster kernel adds the two halves of K in a fixed order
    g = seeded(78)
    x = torch.randn(512, 4096, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(4096, 4096, generator=g) * 4096 ** -0.5).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(4096, generator=g) * 0.1).to(DEV)
    first = b.gemm_bias_gelu_bf16(x, w, bias)
    for _ in range(3):
        assert torch.equal(b.gemm_bias_gelu_bf16(x, w, bias), first)


def test_many_tiles_per_pair_is_bitwise_stable():
    # several tiles per CTA pair, both TMEM accumulators in turn
    x, wg, wu = bf16_inputs(8192, 1024, 1792, 79)
    packed = torch.cat((wg, wu), 0).contiguous().to(DEV)
    xd = x.to(DEV)
    first = b.gemm_swiglu_bf16(xd, packed)
    for _ in range(3):
        assert torch.equal(b.gemm_swiglu_bf16(xd, packed), first)


def test_gemm_repeated_calls_are_bitwise_stable():
    x, wg, wu = bf16_inputs(512, 1024, 1024, 77)
    packed = torch.cat((wg, wu), 0).contiguous().to(DEV)
    xd = x.to(DEV)
    first = b.gemm_swiglu_bf16(xd, packed)
    for _ in range(3):
        assert torch.equal(b.gemm_swiglu_bf16(xd, packed), first)
