"""Sharded workloads reproduce the unsharded results on one GPU (GPU).

Each rank of the multi-GPU plan is emulated in turn on the same device: the
N-sharded GEMM+SwiGLU column blocks concatenate to the full output bit for
bit (every output element is the same dot product, accumulated in the same
k order, whichever tile computes it), row-sharded RMSNorm concatenates to the
full RMSNorm, and the chunked sum with fp64 partials matches the float64 sum.
"""

from __future__ import annotations

import pytest
import torch

from conftest import seeded
from cuda_operator_lab import bindings as b
from cuda_operator_lab import sharding

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize(("m", "k", "n"), [(512, 1024, 1792), (300, 512, 1000)])
def test_n_sharded_gemm_swiglu_matches_full(world, m, k, n):
    g = seeded(world * 1000 + m + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w_norm = (torch.rand(k, generator=g) + 0.5).to(torch.bfloat16).to(DEV)
    packed = (torch.randn(2 * n, k, generator=g) * k ** -0.5).to(torch.bfloat16).to(DEV)
    full = sharding.mlp_block_sharded(x, w_norm, packed)
    parts = [sharding.mlp_block_sharded(x, w_norm, sharding.pack_gate_up_shard(packed, r, world))
             for r in range(world)]
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts, dim=1), full)


@pytest.mark.parametrize("world", [2, 8])
def test_row_sharded_rmsnorm_matches_full(world):
    g = seeded(world)
    x = torch.randn(1000, 4096, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.rand(4096, generator=g) + 0.5).to(torch.bfloat16).to(DEV)
    full = b.rmsnorm_bf16(x, w, 1e-6)
    parts = [b.rmsnorm_bf16(sharding.shard_rows(x, r, world), w, 1e-6) for r in range(world)]
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts), full)


@pytest.mark.parametrize("world", [2, 8])
def test_chunked_sum_with_fp64_partials(world):
    g = torch.Generator(device=DEV)
    g.manual_seed(world)
    x = torch.rand(1 << 24, device=DEV, generator=g) * 2 - 1
    total = 0.0
    for r in range(world):
        lo, hi = sharding.shard_range(x.numel(), r, world)
        total += float(b.reduction_partial_f64(x[lo:hi]))
    exact = float(x.double().sum())
    assert abs(total - exact) <= 1e-9 * abs(exact)
    single = float(sharding.distributed_sum(x))  # no process group: one "rank"
    assert abs(single - exact) <= 1e-6 * abs(exact)
