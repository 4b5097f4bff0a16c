"""Guard regions around every output (GPU): no kernel writes outside its output.

The stand-in for a memory checker on this pool: each output is a view into a
larger buffer whose head and tail are filled with a sentinel bit pattern (a
quiet-NaN payload no kernel produces).  After the call the head and tail must
hold the sentinel bit for bit, and the output itself must hold no sentinel
(every element was written).  Shapes are the ragged ones: GEMM M/N/K tails
(129x72x130, 1000x520x700, 257x520x1000, 1x8x1), row widths that are not a
multiple of the vector width, single rows and columns, and pointwise sizes
that leave a partial vector.  Outputs start both 16-byte aligned (vector
stores) and one element off (scalar stores).  Inputs are checked unchanged.
"""

from __future__ import annotations

import pytest
import torch

from conftest import seeded
from cuda_operator_lab import bindings as b

pytestmark = pytest.mark.gpu
DEV = "cuda"
GUARD = 256  # elements of sentinel before and after the output
SENTINEL = {torch.float32: (0x7FC0DEAD, torch.int32), torch.bfloat16: (0x7FDE, torch.int16),
            torch.float64: (0x7FF8DEADBEEF0001, torch.int64)}


class Guarded:
    """A `shape` output of `dtype` inside a sentinel-filled buffer; `offset`
    shifts its start by that many elements (1 = not 16-byte aligned)."""

    def __init__(self, shape, dtype, offset=0):
        count = 1
        for s in shape:
            count *= s
        self.count, self.offset = count, offset
        bits, self.itype = SENTINEL[dtype]
        self.buf = torch.full((GUARD + offset + count + GUARD,), bits, dtype=self.itype, device=DEV)
        self.out = self.buf[GUARD + offset:GUARD + offset + count].view(dtype).view(*shape)
        self.bits = bits

    def check(self):
        torch.cuda.synchronize()
        head = self.buf[:GUARD + self.offset]
        tail = self.buf[GUARD + self.offset + self.count:]
        body = self.buf[GUARD + self.offset:GUARD + self.offset + self.count]
        assert bool((head == self.bits).all()), "a kernel wrote before its output"
        assert bool((tail == self.bits).all()), "a kernel wrote past its output"
        assert not bool((body == self.bits).any()), "an output element was not written"


def unchanged(*tensors):
    copies = [t.clone() for t in tensors]

    def verify():
        torch.cuda.synchronize()
        for t, c in zip(tensors, copies):
            assert torch.equal(t, c), "an input was modified"
    return verify


def randn(*shape, seed, dtype=torch.float32, scale=1.0):
    return (torch.randn(*shape, generator=seeded(seed)) * scale).to(dtype).to(DEV)


@pytest.fixture(autouse=True)
def no_wait_timeouts():
    b.gemm_status(clear=True)
    yield
    assert b.gemm_status(clear=True) == 0


# (300, 2048, 1000) and (384, 1024, 264) take the split-K cluster kernel for
# bias+GELU and the residual GEMM
GEMM_SHAPES = [(129, 72, 130), (1000, 520, 700), (257, 520, 1000), (1, 8, 1), (128, 64, 2048),
               (384, 1024, 264), (300, 2048, 1000)]


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize(("m", "k", "n"), GEMM_SHAPES)
def test_gemm_outputs_stay_inside(m, k, n, offset):
    x = randn(m, k, seed=m + k, dtype=torch.bfloat16)
    wp = randn(2 * n, k, seed=n + k, dtype=torch.bfloat16, scale=k ** -0.5)
    w = wp[:n].contiguous()
    bias = randn(n, seed=n, scale=0.1)
    res = randn(m, n, seed=m + n, dtype=torch.bfloat16)
    rs = torch.rand(m, generator=seeded(m)).to(DEV) + 0.5
    verify = unchanged(x, wp, w, bias, res, rs)

    g = Guarded((m, n), torch.bfloat16, offset)
    b.gemm_swiglu_bf16_into(x, wp, g.out)
    g.check()
    g = Guarded((m, n), torch.bfloat16, offset)
    b.gemm_bias_gelu_bf16_into(x, w, bias, g.out)
    g.check()
    g = Guarded((m, n), torch.bfloat16, offset)
    b.gemm_residual_bf16_into(x, w, res, g.out)
    g.check()
    g = Guarded((m, n), torch.bfloat16, offset)
    b.gemm_swiglu_rowscale_bf16_into(x, rs, wp, g.out)
    g.check()
    g = Guarded((m, n), torch.float32, offset)
    ws = torch.empty(m, 2 * n, device=DEV)
    b.gemm_swiglu_v11_into(x, wp, ws, g.out)
    g.check()
    verify()


@pytest.mark.parametrize(("m", "k", "n"), [(129, 72, 130), (257, 520, 1000), (300, 1000, 200)])
def test_fp32_gemm_outputs_stay_inside(m, k, n):
    # m*n*k >= 4e6 takes the tensor-core split path, smaller the CUDA-core one
    x = randn(m, k, seed=m)
    wp = randn(2 * n, k, seed=n, scale=k ** -0.5)
    w = wp[:n].contiguous()
    bias = randn(n, seed=k, scale=0.1)
    verify = unchanged(x, wp, w, bias)
    for offset in (0, 1):
        g = Guarded((m, n), torch.float32, offset)
        b.gemm_bias_gelu_v0_into(x, w, bias, g.out)
        g.check()
        g = Guarded((m, n), torch.float32, offset)
        b.gemm_swiglu_v3_into(x, wp, torch.empty(m, 2 * n, device=DEV), g.out)
        g.check()
    verify()


ROW_SHAPES = [(1, 1), (3, 33), (17, 4097), (128, 4096), (2, 40000), (5, 1023)]


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize(("rows", "cols"), ROW_SHAPES)
def test_row_outputs_stay_inside(rows, cols, offset):
    x = randn(rows, cols, seed=rows * 7 + cols)
    r = randn(rows, cols, seed=rows + cols * 3)
    w = torch.rand(cols, generator=seeded(cols)).to(DEV) + 0.5
    beta = randn(cols, seed=cols + 1, scale=0.1)
    verify = unchanged(x, r, w, beta)
    calls = {
        "rmsnorm": lambda o: b.rmsnorm_v4_into(x, w, o, 1e-6),
        "softmax": lambda o: b.softmax_v5_into(x, o),
        "layernorm": lambda o: b.layernorm_v5_into(x, w, beta, o),
        "residual_layernorm": lambda o: b.fused_residual_layernorm_v4_into(x, r, w, beta, o),
    }
    for name, call in calls.items():
        g = Guarded((rows, cols), torch.float32, offset)
        call(g.out)
        g.check()
    gh, gy = Guarded((rows, cols), torch.float32, offset), Guarded((rows, cols), torch.float32, offset)
    b.fused_residual_layernorm_h_into(x, r, w, beta, gh.out, gy.out)
    gh.check()
    gy.check()
    gh, gy = Guarded((rows, cols), torch.float32, offset), Guarded((rows, cols), torch.float32, offset)
    b.fused_residual_rmsnorm_into(x, r, w, gh.out, gy.out, 1e-6)
    gh.check()
    gy.check()
    xb, rb, wb = x.to(torch.bfloat16), r.to(torch.bfloat16), w.to(torch.bfloat16)
    g = Guarded((rows, cols), torch.bfloat16, offset)
    b.rmsnorm_bf16_into(xb, wb, g.out, 1e-6)
    g.check()
    gh, gy = Guarded((rows, cols), torch.bfloat16, offset), Guarded((rows, cols), torch.bfloat16, offset)
    b.fused_residual_rmsnorm_into(xb, rb, wb, gh.out, gy.out, 1e-6)
    gh.check()
    gy.check()
    g = Guarded((rows,), torch.float32, offset)
    b.rmsnorm_rstd_bf16_into(xb, g.out, 1e-6)
    g.check()
    verify()


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize(("rows", "cols"), [(1, 3), (17, 4097), (1024, 4096), (7, 5)])
def test_pointwise_outputs_stay_inside(rows, cols, offset):
    x = randn(rows, cols, seed=rows + cols)
    u = randn(rows, cols, seed=rows * cols)
    bias = randn(cols, seed=cols, scale=0.1)
    verify = unchanged(x, u, bias)
    g = Guarded((rows, cols), torch.float32, offset)
    b.fused_bias_gelu_v2_into(x, bias, g.out)
    g.check()
    g = Guarded((rows, cols), torch.float32, offset)
    b.swiglu_v2_into(x, u, g.out)
    g.check()
    g = Guarded((rows, cols), torch.float32, offset)
    b.swiglu_v0_into(x, u, g.out)
    g.check()
    verify()


@pytest.mark.parametrize("n", [1, 1025, 16_777_216 + 3])
def test_reduction_outputs_stay_inside(n):
    x = torch.rand(n, generator=seeded(n)).to(DEV) * 2 - 1
    verify = unchanged(x)
    for offset in (0, 1):
        g = Guarded((1,), torch.float32, offset)
        b.reduction_v5_into(x, g.out)
        g.check()
        g = Guarded((1,), torch.float64, offset)
        b.reduction_partial_f64_into(x, g.out)
        g.check()
    verify()
