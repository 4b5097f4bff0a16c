"""The entry points inside CUDA graph capture (GPU).

Captured on a stream the library has never seen, so the reduction's
per-stream scratch does not exist yet and the stream-ordered fallbacks run
while capturing: the graph's replay must equal the eager result bit for bit.
"""

from __future__ import annotations

import pytest
import torch

from conftest import seeded
from cuda_operator_lab import bindings as b

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_capture_reduction_norm_and_fp32_gemm():
    g = seeded(424242)
    x = (torch.rand(3_000_001, generator=g) * 2 - 1).to(DEV)
    rows = torch.randn(64, 4096, generator=g).to(DEV)
    w = (torch.rand(4096, generator=g) + 0.5).to(DEV)
    a = torch.randn(256, 512, generator=g).to(DEV)
    wg = torch.randn(1024, 512, generator=g).to(DEV)
    bias = torch.randn(1024, generator=g).to(DEV)

    eager_sum = b.reduction_v5(x)
    eager_norm = b.rmsnorm_v4(rows, w, 1e-6)
    eager_gemm = b.gemm_bias_gelu_v0(a, wg, bias)
    torch.cuda.synchronize()

    out_sum = torch.empty(1, device=DEV)
    out_norm = torch.empty_like(rows)
    out_gemm = torch.empty(256, 1024, device=DEV)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):  # a fresh capture stream
        b.reduction_v5_into(x, out_sum)
        b.rmsnorm_v4_into(rows, w, out_norm, 1e-6)
        b.gemm_bias_gelu_v0_into(a, wg, bias, out_gemm)
    for _ in range(2):
        out_sum.zero_()
        out_norm.zero_()
        out_gemm.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_sum, eager_sum)
        assert torch.equal(out_norm, eager_norm)
        assert torch.equal(out_gemm, eager_gemm)
    del graph
