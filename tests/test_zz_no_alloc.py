"""The allocation-free global sum, called through the C ABI (GPU).

cuda_operator_lab_reduction_noalloc exists for callers that cannot let a
library allocate device memory (a server that handed the whole device to its
own allocator at start-up, a host whose plugins must not allocate, a loop
where an allocator call could synchronise).  It keeps its scratch in a fixed
array inside the library image, so these tests check that, called twice in a
row on different inputs, it returns what the regular entry point returns
(within the reduction tolerance of the other tests: 1e-6 relative to the
float64 sum), and that it refuses inputs larger than that array serves.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from cuda_operator_lab import bindings as b

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_ELEMENTS = 1 << 28
CAPACITY_ERROR = 10004


def _noalloc(x: torch.Tensor, out: torch.Tensor) -> int:
    lib = b._library().handle
    return lib.cuda_operator_lab_reduction_noalloc(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_uint64(x.numel()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _regular(x: torch.Tensor, out: torch.Tensor) -> int:
    lib = b._library().handle
    return lib.cuda_operator_reduction_v5(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_uint64(x.numel()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_sum_matches_regular_entry_point_on_two_calls_in_a_row():
    g = torch.Generator(device=DEV)
    g.manual_seed(20261201)
    inputs = [torch.rand(16_777_216, device=DEV, generator=g) * 2 - 1,
              torch.rand(1_000_003, device=DEV, generator=g) * 2 - 1]
    outs = [torch.full((1,), float("nan"), device=DEV) for _ in inputs]
    for x, out in zip(inputs, outs):  # two calls in a row on one stream
        assert _noalloc(x, out) == 0
    for x, out in zip(inputs, outs):
        expected = torch.empty(1, device=DEV)
        assert _regular(x, expected) == 0
        torch.cuda.synchronize()
        exact = float(x.double().sum())
        assert abs(float(out) - exact) <= 1e-6 * abs(exact)
        assert abs(float(out) - float(expected)) <= 1e-6 * abs(exact)


def test_noalloc_sum_unaligned_and_empty_inputs():
    storage = torch.rand(65_537, device=DEV)
    x = storage[1:]
    out = torch.empty(1, device=DEV)
    assert _noalloc(x, out) == 0
    torch.cuda.synchronize()
    exact = float(x.double().sum())
    assert abs(float(out) - exact) <= 1e-6 * abs(exact)
    empty = torch.empty(0, device=DEV)
    out.fill_(7.0)
    assert _noalloc(empty, out) == 0
    torch.cuda.synchronize()
    assert float(out) == 0.0


def test_noalloc_sum_rejects_inputs_beyond_its_scratch():
    # The size check runs on the host before anything is launched, so a small
    # buffer with an oversized count is rejected without being read.
    x = torch.zeros(16, device=DEV)
    out = torch.zeros(1, device=DEV)
    lib = b._library().handle
    code = lib.cuda_operator_lab_reduction_noalloc(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_uint64(MAX_ELEMENTS + 1), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code == CAPACITY_ERROR
    assert b"2^28" in lib.cuda_operator_error_string(code)
