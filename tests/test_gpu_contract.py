"""Drop-in API contract of the bindings on a GPU.

The behaviours the reference's tests pin for every op: ``_into`` returns the
caller's storage (tests/test_softmax_v2.py:102-110), work is enqueued on the
current stream (tests/test_reduction_v5.py:88-96), bad arguments raise
ValueError/TypeError with the reference's keywords
(tests/test_rmsnorm_v0.py:101-114), empty inputs succeed without a launch,
and C-level argument errors surface as RuntimeError("CUDA error ...").
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from cuda_operator_lab import bindings as b
from oracle import reference_math as oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_into_variants_return_caller_storage():
    x = torch.randn(11, 257, device=DEV)
    w = torch.randn(257, device=DEV)
    bias = torch.randn(257, device=DEV)
    for fn, args in [
        (b.softmax_v2_into, (x,)),
        (b.rmsnorm_v0_into, (x, w)),
        (b.layernorm_v3_into, (x, w, bias)),
        (b.fused_residual_layernorm_v1_into, (x, x, w, bias)),
        (b.fused_bias_gelu_v1_into, (x, bias)),
        (b.swiglu_v2_into, (x, x)),
    ]:
        out = torch.full_like(x, float("nan"))
        returned = fn(*args, out) if fn is not b.rmsnorm_v0_into else fn(x, w, out)
        torch.cuda.synchronize()
        assert returned.data_ptr() == out.data_ptr()
        assert not torch.isnan(out).any()
    s = torch.full((1,), 7.0, device=DEV)
    assert b.reduction_v1_into(x.flatten(), s).data_ptr() == s.data_ptr()


def test_ops_use_the_current_stream():
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        x = torch.randn(32, 513, device=DEV)
        w = torch.randn(513, device=DEV)
        y = b.rmsnorm_v2(x, w)
        s = b.reduction_v5(torch.arange(4099, device=DEV, dtype=torch.float32))
        xb = torch.randn(128, 256, device=DEV).to(torch.bfloat16)
        wb = torch.randn(512, 256, device=DEV).to(torch.bfloat16)
        z = b.gemm_swiglu_v11(xb, wb)
    stream.synchronize()
    torch.testing.assert_close(y.cpu(), oracle.rmsnorm(x.cpu(), w.cpu()), rtol=1e-5, atol=1e-6)
    assert float(s[0]) == 4098 * 4099 / 2
    torch.testing.assert_close(z.cpu(), oracle.gemm_swiglu_bf16_fp32_reference(xb.cpu(), wb.cpu()),
                               rtol=2e-2, atol=2e-2)


def test_validation_errors_match_reference_keywords():
    x = torch.randn(8, 64, device=DEV)
    with pytest.raises(ValueError, match="weight"):
        b.rmsnorm_v0(x, torch.randn(63, device=DEV))
    with pytest.raises(ValueError, match="positive"):
        b.rmsnorm_v4(x, torch.randn(64, device=DEV), eps=0.0)
    with pytest.raises(ValueError, match="positive"):
        b.layernorm_v1(x, torch.randn(64, device=DEV), torch.randn(64, device=DEV), eps=-1.0)
    with pytest.raises(TypeError):
        b.softmax_v0(x.double())
    with pytest.raises(ValueError, match="cols > 0"):
        b.softmax_v0(torch.empty(4, 0, device=DEV))
    with pytest.raises(ValueError, match="contiguous"):
        b.reduction_v0(torch.randn(8, 2, device=DEV)[:, 0])
    with pytest.raises(ValueError, match="alias"):
        ws = torch.empty(4, 8, device=DEV)
        b.gemm_swiglu_v0_into(torch.randn(4, 16, device=DEV), torch.randn(8, 16, device=DEV),
                              torch.randn(8, 16, device=DEV), ws, ws)
    with pytest.raises(ValueError, match="even"):
        b.gemm_swiglu_v4(torch.randn(4, 16, device=DEV).bfloat16(),
                         torch.randn(7, 16, device=DEV).bfloat16())


def test_empty_work_succeeds():
    assert b.softmax_v1(torch.empty(0, 128, device=DEV)).shape == (0, 128)
    assert b.rmsnorm_v3(torch.empty(0, 8, device=DEV), torch.ones(8, device=DEV)).shape == (0, 8)
    assert b.swiglu_v0(torch.empty(0, device=DEV), torch.empty(0, device=DEV)).numel() == 0
    assert float(b.reduction_v2(torch.empty(0, device=DEV))[0]) == 0.0
    out = b.gemm_bias_gelu_v2(torch.empty(0, 32, device=DEV), torch.randn(64, 32, device=DEV),
                              torch.randn(64, device=DEV))
    assert out.shape == (0, 64)


def test_c_abi_argument_errors():
    lib = b._library().handle
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    x = torch.randn(4, 8, device=DEV)
    null = ctypes.c_void_p()
    # rows == 0 succeeds before any pointer check (softmax.cu:342-344)
    assert lib.cuda_operator_softmax_v0(null, null, 0, 8, stream) == 0
    # NULL input, cols == 0, eps <= 0 are cudaErrorInvalidValue (1)
    assert lib.cuda_operator_softmax_v0(null, ctypes.c_void_p(x.data_ptr()), 4, 8, stream) == 1
    assert lib.cuda_operator_rmsnorm_v0(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                        ctypes.c_void_p(x.data_ptr()), 4, 0, ctypes.c_float(1e-5),
                                        stream) == 1
    assert lib.cuda_operator_rmsnorm_v0(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                        ctypes.c_void_p(x.data_ptr()), 4, 8, ctypes.c_float(0.0),
                                        stream) == 1
    assert lib.cuda_operator_reduction_v0(ctypes.c_void_p(x.data_ptr()), null, 8, stream) == 1
    assert lib.cuda_operator_gemm_swiglu_v4(ctypes.c_void_p(x.data_ptr()), null, null, null, 4, 0,
                                            8, stream) == 1
    # m == 0 succeeds first
    assert lib.cuda_operator_gemm_swiglu_v4(null, null, null, null, 0, 0, 8, stream) == 0
    with pytest.raises(RuntimeError, match="CUDA error 1"):
        b._library().check(1)


def test_device_info_reports_b200():
    info = b.device_info()
    assert info["cc_major"] == 10
    assert info["sm_count"] >= 100
