"""Our kernels against the reference's own CUDA kernels on the same B200 (GPU).

oracle/_ref/libcuda_operator_lab_ref.so is the reference's csrc/ compiled for
sm_100a by oracle/build_ref.py (built where the reference checkout exists; the
tests skip without it).  Both libraries export the same 54 symbols, so each
case calls one symbol of each library on the same device buffers and
compares the outputs: the reference's kernels are a second checker beside
the CPU oracle.  Its GEMM versions that call cuBLAS (v4, v10/v11 off the WMMA
region, bias+GELU v2..v6 through cuBLASLt) run NVIDIA's library kernels.

With COL_REF_TIMING=path set, the device time of both libraries per case is
written there as JSON (timing is recorded, not asserted): `reps` calls are
captured into a CUDA graph and replayed, so the figure is device time per call
without the host's ctypes/launch cost (eager back-to-back timing if a library
call cannot be captured).
"""

from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

import pytest
import torch

from conftest import ROOT, seeded
from cuda_operator_lab import bindings as b

pytestmark = pytest.mark.gpu
REF_LIB = ROOT / "oracle" / "_ref" / "libcuda_operator_lab_ref.so"
DEV = "cuda"
TIMINGS: dict[str, dict] = {}


@pytest.fixture(scope="module")
def libs():
    if not REF_LIB.is_file():
        pytest.skip("reference library not built (oracle/build_ref.py)")
    ref = b._Library(REF_LIB, symbols=b.REFERENCE_SYMBOLS)
    ours = b._library()
    yield ours, ref
    out = os.environ.get("COL_REF_TIMING")
    if out and TIMINGS:
        Path(out).write_text(json.dumps(TIMINGS, indent=1, sort_keys=True))


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _s() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _time_us(fn, reps=20) -> float:
    """fn() takes no arguments and enqueues on torch's current stream.  The
    warm-up calls run on the stream that is then captured, as a caller that
    graphs its steady state would (the library keeps per-stream scratch for
    the reduction; a stream it has not served yet gets graph memory nodes)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        start.record()
        for _ in range(5):
            graph.replay()
        end.record()
        end.synchronize()
        del graph
        return start.elapsed_time(end) * 1000.0 / (5 * reps)
    except RuntimeError:
        torch.cuda.synchronize()
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) * 1000.0 / reps


def run_both(libs, symbol, make_args, out_ours, out_ref, name, time_it=True):
    ours, ref = libs
    ours.check(getattr(ours.handle, symbol)(*make_args(out_ours)))
    ref.check(getattr(ref.handle, symbol)(*make_args(out_ref)))
    torch.cuda.synchronize()
    if time_it:
        TIMINGS[name] = {
            "ours_us": round(_time_us(lambda: getattr(ours.handle, symbol)(*make_args(out_ours))), 3),
            "reference_us": round(_time_us(lambda: getattr(ref.handle, symbol)(*make_args(out_ref))), 3),
        }


@pytest.mark.parametrize(("rows", "cols"), [(1, 1), (7, 127), (128, 4096), (8, 4097), (128, 8192)])
def test_rowwise_vs_reference_kernels(libs, rows, cols):
    g = seeded(rows * 7 + cols)
    x = torch.randn(rows, cols, generator=g).to(DEV)
    r = torch.randn(rows, cols, generator=g).to(DEV)
    w = (torch.rand(cols, generator=g) + 0.5).to(DEV)
    bias = (torch.randn(cols, generator=g) * 0.1).to(DEV)
    n, c = ctypes.c_uint64(rows), ctypes.c_uint64(cols)
    eps = ctypes.c_float(1e-5)
    cases = {
        "cuda_operator_softmax_v5": lambda o: (_p(x), _p(o), n, c, _s()),
        "cuda_operator_rmsnorm_v4": lambda o: (_p(x), _p(w), _p(o), n, c, eps, _s()),
        "cuda_operator_layernorm_v5": lambda o: (_p(x), _p(w), _p(bias), _p(o), n, c, eps, _s()),
        "cuda_operator_fused_residual_layernorm_v4":
            lambda o: (_p(x), _p(r), _p(w), _p(bias), _p(o), n, c, eps, _s()),
        "cuda_operator_fused_bias_gelu_v2": lambda o: (_p(x), _p(bias), _p(o), n, c, _s()),
        "cuda_operator_swiglu_v2": lambda o: (_p(x), _p(r), _p(o), n, c, _s()),
    }
    for symbol, make in cases.items():
        o1, o2 = torch.empty_like(x), torch.empty_like(x)
        run_both(libs, symbol, make, o1, o2, f"{symbol}[{rows}x{cols}]", time_it=rows >= 128)
        torch.testing.assert_close(o1, o2, rtol=3e-5, atol=5e-6, msg=symbol)


@pytest.mark.parametrize("n", [1, 1025, 524289, 16_777_216])
def test_reduction_vs_reference_kernel(libs, n):
    x = (torch.rand(n, generator=seeded(n)) * 2 - 1).to(DEV)
    o1, o2 = torch.zeros(1, device=DEV), torch.zeros(1, device=DEV)
    run_both(libs, "cuda_operator_reduction_v5",
             lambda o: (_p(x), _p(o), ctypes.c_uint64(n), _s()), o1, o2,
             f"reduction_v5[{n}]", time_it=n >= 1 << 20)
    exact = float(x.double().sum())
    # ours is within one fp32 rounding of the exact sum; the reference's fp32
    # atomics are within its tests' 5e-4 absolute bar
    assert abs(float(o1) - exact) <= 1e-6 * max(1.0, abs(exact))
    assert abs(float(o2) - exact) <= 5e-3 + 5e-5 * abs(exact)


@pytest.mark.parametrize(("m", "k", "n"), [(128, 64, 2048), (512, 4096, 4096), (256, 1024, 1536)])
def test_gemm_swiglu_vs_reference_kernels(libs, m, k, n):
    g = seeded(m + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(2 * n, k, generator=g) * k ** -0.5).to(torch.bfloat16).to(DEV)
    ws1 = torch.empty(m, 2 * n, device=DEV)
    ws2 = torch.empty(m, 2 * n, device=DEV)
    args = lambda ws: (lambda o: (_p(x), _p(w), _p(ws), _p(o), ctypes.c_uint64(m),  # noqa: E731
                                  ctypes.c_uint64(k), ctypes.c_uint64(n), _s()))
    o1, o2 = torch.empty(m, n, device=DEV), torch.empty(m, n, device=DEV)
    ours, ref = libs
    ours.check(ours.handle.cuda_operator_gemm_swiglu_v11(*args(ws1)(o1)))
    ref.check(ref.handle.cuda_operator_gemm_swiglu_v11(*args(ws2)(o2)))
    torch.cuda.synchronize()
    TIMINGS[f"gemm_swiglu_v11[{m}x{k}x{n}]"] = {
        "ours_us": round(_time_us(lambda: ours.handle.cuda_operator_gemm_swiglu_v11(*args(ws1)(o1))), 3),
        "reference_us": round(_time_us(lambda: ref.handle.cuda_operator_gemm_swiglu_v11(*args(ws2)(o2))), 3),
    }
    torch.testing.assert_close(o1, o2, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize(("m", "k", "n"), [(17, 31, 63), (128, 512, 1024), (512, 4096, 4096)])
def test_fp32_gemm_bias_gelu_vs_reference_kernels(libs, m, k, n):
    g = seeded(m * 3 + k + n)
    x = torch.randn(m, k, generator=g).to(DEV)
    w = torch.randn(n, k, generator=g).to(DEV)
    bias = torch.randn(n, generator=g).to(DEV)
    for version in (0, 2):
        symbol = f"cuda_operator_gemm_bias_gelu_v{version}"
        o1, o2 = torch.empty(m, n, device=DEV), torch.empty(m, n, device=DEV)
        run_both(libs, symbol, lambda o: (_p(x), _p(w), _p(bias), _p(o), ctypes.c_uint64(m),
                                          ctypes.c_uint64(k), ctypes.c_uint64(n), _s()),
                 o1, o2, f"{symbol}[{m}x{k}x{n}]", time_it=m >= 512)
        # unit-variance operands: |x.w| ~ sqrt(k); fp32 sums in a different
        # order differ by ~1e-7 * k relative to that scale
        torch.testing.assert_close(o1, o2, rtol=3e-4, atol=3e-4 * k ** 0.5, msg=symbol)


@pytest.mark.parametrize(("m", "k", "n"), [(512, 4096, 4096)])
def test_fp32_gemm_swiglu_vs_reference_kernels(libs, m, k, n):
    g = seeded(m * 5 + k + n)
    x = torch.randn(m, k, generator=g).to(DEV)
    w = (torch.randn(2 * n, k, generator=g) * k ** -0.5).to(DEV)
    ws1, ws2 = torch.empty(m, 2 * n, device=DEV), torch.empty(m, 2 * n, device=DEV)
    o1, o2 = torch.empty(m, n, device=DEV), torch.empty(m, n, device=DEV)
    ours, ref = libs
    make = lambda ws: (lambda o: (_p(x), _p(w), _p(ws), _p(o), ctypes.c_uint64(m),  # noqa: E731
                                  ctypes.c_uint64(k), ctypes.c_uint64(n), _s()))
    ours.check(ours.handle.cuda_operator_gemm_swiglu_v3(*make(ws1)(o1)))
    ref.check(ref.handle.cuda_operator_gemm_swiglu_v3(*make(ws2)(o2)))
    torch.cuda.synchronize()
    TIMINGS[f"gemm_swiglu_v3_fp32[{m}x{k}x{n}]"] = {
        "ours_us": round(_time_us(lambda: ours.handle.cuda_operator_gemm_swiglu_v3(*make(ws1)(o1)), 5), 3),
        "reference_us": round(_time_us(lambda: ref.handle.cuda_operator_gemm_swiglu_v3(*make(ws2)(o2)), 5), 3),
    }
    torch.testing.assert_close(o1, o2, rtol=3e-4, atol=3e-4)
