"""The entry points inside CUDA graph capture (GPU).

A captured reduction takes graph-owned scratch (never a stream's persistent
block, which a graph replayed elsewhere would share): the graph's replay must
equal the eager result bit for bit, also while eager calls run beside it.
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


def test_captured_reduction_does_not_share_the_capture_streams_scratch():
    """A graph captured on a stream the library already served, replayed on
    another stream while eager reductions run on the first: each must keep its
    own scratch (partials and the finishing-CTA counter), so both results stay
    exact in every round."""
    g = seeded(515151)
    x_graph = (torch.rand(4_000_000, generator=g) * 2 - 1).to(DEV)
    x_eager = (torch.rand(4_000_000, generator=g) * 2 - 1).to(DEV)
    want_graph = b.reduction_v5(x_graph)
    want_eager = b.reduction_v5(x_eager)
    torch.cuda.synchronize()

    served, other = torch.cuda.Stream(), torch.cuda.Stream()
    out_graph = torch.zeros(1, device=DEV)
    out_eager = [torch.zeros(1, device=DEV) for _ in range(16)]
    with torch.cuda.stream(served):
        b.reduction_v5_into(x_eager, out_eager[0])  # the stream's own scratch exists now
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=served):
        b.reduction_v5_into(x_graph, out_graph)
    outs_graph = []
    for i in range(16):
        with torch.cuda.stream(other):
            graph.replay()
            outs_graph.append(out_graph.clone())
        with torch.cuda.stream(served):
            b.reduction_v5_into(x_eager, out_eager[i])
    torch.cuda.synchronize()
    for o in outs_graph:
        assert torch.equal(o, want_graph)
    for o in out_eager:
        assert torch.equal(o, want_eager)
    del graph
