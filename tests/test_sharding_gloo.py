"""Multi-rank host logic of the sharded workloads on CPU ranks (gloo, world 2).

The per-rank compute is the CPU oracle here; on GPUs it is the library.  The
tests check that the partition and the combine reproduce the unsharded
result: column blocks of the N-sharded GEMM+SwiGLU gather to the full
output, row shards of RMSNorm concatenate to the full output, and the fp64
partial all-reduce gives the global sum.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cuda_operator_lab import sharding
from oracle import reference_math as oracle


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator()
        g.manual_seed(1234)
        m, k, n = 24, 32, 20
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        w_norm = (torch.rand(k, generator=g) + 0.5).to(torch.bfloat16)
        packed = (torch.randn(2 * n, k, generator=g) * k ** -0.5).to(torch.bfloat16)

        # N-sharded GEMM+SwiGLU: local column block, then gather
        shard = sharding.pack_gate_up_shard(packed, rank, world)
        local = oracle.mlp_block_bf16(x, w_norm, shard)
        full = sharding.gather_columns(local.float())
        ref = oracle.mlp_block_bf16(x, w_norm, packed).float()
        gemm_ok = torch.equal(full, ref)

        # row-sharded RMSNorm: concatenating the shards gives the full output
        rows = sharding.shard_rows(x, rank, world)
        local_norm = oracle.rmsnorm_bf16(rows, w_norm).float()
        parts = [torch.empty_like(local_norm) for _ in range(world)]
        dist.all_gather(parts, local_norm)
        norm_ok = torch.equal(torch.cat(parts), oracle.rmsnorm_bf16(x, w_norm).float())

        # chunked sum with an fp64 partial all-reduce
        v = torch.rand(1001, generator=g) * 2 - 1
        lo, hi = sharding.shard_range(v.numel(), rank, world)
        total = sharding.distributed_sum(
            v[lo:hi], partial_fn=lambda t: torch.tensor([oracle.reduction_sum_f64(t)],
                                                        dtype=torch.float64))
        sum_ok = abs(float(total) - oracle.reduction_sum_f64(v)) <= 1e-6 * max(
            1.0, abs(oracle.reduction_sum_f64(v)))
        results[rank] = (gemm_ok, norm_ok, sum_ok)
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions_exactly():
    for total in (0, 1, 7, 14336, 16385):
        for world in (1, 2, 3, 4, 8):
            ranges = [sharding.shard_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    with pytest.raises(ValueError):
        sharding.shard_range(10, 2, 2)


def test_pack_gate_up_shard_layout():
    n, k = 8, 3
    packed = torch.arange(2 * n * k, dtype=torch.float32).view(2 * n, k)
    s1 = sharding.pack_gate_up_shard(packed, 1, 2)
    assert torch.equal(s1[:4], packed[4:8])
    assert torch.equal(s1[4:], packed[12:16])
    assert s1.is_contiguous()


def test_two_gloo_ranks_reproduce_unsharded_results():
    world = 2
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True,
                       start_method="spawn")
    assert dict(results) == {0: (True, True, True), 1: (True, True, True)}
