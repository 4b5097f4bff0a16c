"""GEMM+SwiGLU with the column all-gather fused into its epilogue (GPU).

On one GPU every rank of a g-way N split is run in turn, each storing its
column block into g [M, N] buffers of the same device (the epilogue cannot
tell a peer mapping from a local address): every buffer must equal the
unsharded GEMM bit for bit.  The device flag barrier is checked for one rank
and for a wait that runs out (a flag that nothing sets: the kernel must give
up after its limit, report it in the peer status word and leave the context
usable).  With two or more GPUs, ranks in separate processes exchange CUDA
IPC handles and gather over NVLink through ``sharding.PeerColumnGather``.
The row-sharded RMSNorm with its all-gather (``rmsnorm_allgather_bf16`` and
``sharding.RowNormGather``, peer stores or copy engines) runs as one rank here
and across every GPU the box has, bit for bit against the unsharded RMSNorm.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import seeded
from cuda_operator_lab import bindings as b
from cuda_operator_lab import sharding

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _operands(m, k, n, seed):
    g = seeded(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    packed = (torch.randn(2 * n, k, generator=g) * k ** -0.5).to(torch.bfloat16).to(DEV)
    rs = (torch.rand(m, generator=g) + 0.5).to(DEV)
    return x, packed, rs


@pytest.mark.parametrize("scaled", [False, True])
@pytest.mark.parametrize(("world", "m", "k", "n"), [
    (2, 512, 1024, 1792), (4, 300, 512, 1024), (8, 256, 2048, 14336 // 8), (8, 130, 256, 1000),
    (3, 1, 64, 96), (2, 2048, 512, 2 * 112), (2, 640, 512, 2 * 96), (2, 384, 256, 2 * 64),
    (1, 2048, 1024, 1792)])
def test_gather_epilogue_fills_every_destination(world, m, k, n, scaled):
    # (1, 2048, 1024, 1792): 112 CTA-pair tiles, more than one per pair
    x, packed, rs = _operands(m, k, n, world * 7 + m)
    rs = rs if scaled else None
    if scaled:
        full = b.gemm_swiglu_rowscale_bf16(x, rs, packed)
    else:
        full = b.gemm_swiglu_bf16(x, packed)
    bufs = [torch.full((m, n), float("nan"), device=DEV, dtype=torch.bfloat16)
            for _ in range(world)]
    b.gemm_status(clear=True)
    for r in range(world):
        lo, _ = sharding.shard_range(n, r, world)
        shard = sharding.pack_gate_up_shard(packed, r, world)
        dests = [bufs[(r + j) % world].data_ptr() + lo * 2 for j in range(world)]
        b.gemm_swiglu_allgather_bf16(x, rs, shard, dests, n)
    torch.cuda.synchronize()
    assert b.gemm_status() == 0
    for buf in bufs:
        assert torch.equal(buf, full)


def test_gather_at_the_headline_shard_shape_matches_the_oracle():
    """The 8-rank N split of the benchmark workload (K=4096, N=14336, each rank
    1792 columns; M=2048 of its 16384 rows), ranks emulated in turn: every
    destination holds the same blocks, and 256 rows of them match the CPU
    oracle of the row-scaled GEMM+SwiGLU at the bf16 bar."""
    from oracle import reference_math as oracle

    world, m, k, n = 8, 2048, 4096, 14336
    x, packed, rs = _operands(m, k, n, 20261230)
    bufs = [torch.full((m, n), float("nan"), device=DEV, dtype=torch.bfloat16)
            for _ in range(world)]
    b.gemm_status(clear=True)
    for r in range(world):
        lo, _ = sharding.shard_range(n, r, world)
        shard = sharding.pack_gate_up_shard(packed, r, world)
        dests = [bufs[(r + j) % world].data_ptr() + lo * 2 for j in range(world)]
        b.gemm_swiglu_allgather_bf16(x, rs, shard, dests, n)
    torch.cuda.synchronize()
    assert b.gemm_status() == 0
    for buf in bufs[1:]:
        assert torch.equal(buf, bufs[0])
    rows = torch.arange(0, m, 8) + torch.arange(0, m, 8) % 7
    expected = oracle.gemm_swiglu_rowscale_bf16(x[rows.to(DEV)].cpu(), rs[rows.to(DEV)].cpu(),
                                                packed.cpu())
    torch.testing.assert_close(bufs[0][rows.to(DEV)].cpu().float(), expected.float(),
                               rtol=2e-2, atol=2e-2)


def test_gather_argument_checks():
    x, packed, _ = _operands(64, 64, 64, 1)
    out = torch.empty(64, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        b.gemm_swiglu_allgather_bf16(x, None, packed, [], 64)
    with pytest.raises(ValueError):
        b.gemm_swiglu_allgather_bf16(x, None, packed, [out.data_ptr()] * 9, 64)
    with pytest.raises(ValueError):
        b.gemm_swiglu_allgather_bf16(x, None, packed, [out.data_ptr()], 32)
    # k not a multiple of 8: the tensor path cannot take it (library code 10005)
    x7 = torch.zeros(64, 60, device=DEV, dtype=torch.bfloat16)
    w7 = torch.zeros(128, 60, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="10005"):
        b.gemm_swiglu_allgather_bf16(x7, None, w7, [out.data_ptr()], 64)


def test_peer_barrier_single_rank_passes():
    flags = torch.zeros(8, device=DEV, dtype=torch.int32)
    b.peer_status(clear=True)
    for epoch in (1, 2, 3):
        b.peer_barrier([flags.data_ptr()], 0, epoch)
    assert b.peer_status() == 0
    assert flags[0].item() == 3


def test_peer_barrier_wait_runs_out_and_reports():
    """Rank 0 of 2 with nobody playing rank 1: the wait gives up after its
    limit (20 ms), sets bit 1 of the peer status, and the device stays usable."""
    flags = torch.zeros(2, 8, device=DEV, dtype=torch.int32)
    b.peer_status(clear=True)
    b.peer_barrier([flags[0].data_ptr(), flags[1].data_ptr()], 0, 1, timeout_ns=20_000_000)
    assert b.peer_status() == 1
    assert flags[0, 0].item() == 1 and flags[1, 0].item() == 1 and flags[0, 1].item() == 0
    assert b.peer_status() == 0
    x, packed, _ = _operands(128, 128, 128, 3)
    assert torch.equal(b.gemm_swiglu_bf16(x, packed), b.gemm_swiglu_bf16(x, packed))


def test_peer_alloc_is_zeroed_and_freed():
    addr, handle = b.peer_alloc(1 << 20)
    assert len(handle) == 64 and addr % 256 == 0
    view = sharding.LibraryPeers().view(addr, 512, 1024)
    assert int(view.view(torch.int16).abs().sum().item()) == 0
    del view
    b.peer_free(addr)


def _as_layout(full: torch.Tensor, world: int, layout: str) -> torch.Tensor:
    if layout == "columns":
        return full
    nl = full.shape[1] // world
    return torch.stack([full[:, r * nl:(r + 1) * nl] for r in range(world)])


@pytest.mark.parametrize("layout", ["blocks", "columns"])
def test_peer_column_gather_one_rank(layout):
    x, packed, rs = _operands(256, 512, 768, 11)
    gather = sharding.PeerColumnGather(256, 768, layout=layout)
    try:
        a = gather(x, packed, rs)
        first = a.data_ptr()
        assert torch.equal(a, _as_layout(b.gemm_swiglu_rowscale_bf16(x, rs, packed), 1, layout))
        c = gather(x, packed)
        assert c.data_ptr() != first
        assert torch.equal(c, _as_layout(b.gemm_swiglu_bf16(x, packed), 1, layout))
        assert gather(x, packed, rs).data_ptr() == first
        assert b.peer_status() == 0 and b.gemm_status() == 0
        del a, c
    finally:
        gather.close()


# ---------------------------------------------------------------- several GPUs


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ranks_worker(rank: int, world: int, port: int, results, layout: str) -> None:
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    gather = None
    try:
        m, k, n = 1000, 1024, 256 * world
        x, packed, rs = _operands(m, k, n, 99)  # the same operands on every rank
        full = b.gemm_swiglu_rowscale_bf16(x, rs, packed)
        shard = sharding.pack_gate_up_shard(packed, rank, world)
        gather = sharding.PeerColumnGather(m, n, layout=layout)
        ok = True
        for call in range(6):
            scale = rs * (1 + 0.25 * call)
            out = gather(x, shard, scale)
            expected = _as_layout(b.gemm_swiglu_rowscale_bf16(x, scale, packed), world, layout)
            ok = ok and torch.equal(out, expected)
        last = gather(x, shard, rs)
        ok = ok and torch.equal(last, _as_layout(full, world, layout))
        # and against the CPU oracle on a row sample, at the bf16 bar
        from oracle import reference_math as oracle

        rows = torch.arange(0, m, 37)
        expected = _as_layout(oracle.gemm_swiglu_rowscale_bf16(
            x[rows.to(x.device)].cpu(), rs[rows.to(x.device)].cpu(), packed.cpu()), world, layout)
        got = last[:, rows.to(x.device)] if layout == "blocks" else last[rows.to(x.device)]
        ok = ok and torch.allclose(got.cpu().float(), expected.float(), rtol=2e-2, atol=2e-2)
        gather.check()
        del out, last
        results[rank] = (ok, b.peer_status(), b.gemm_status())
    finally:
        if gather is not None:
            gather.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
@pytest.mark.parametrize("layout", ["blocks", "columns"])
def test_peer_column_gather_across_gpus(layout):
    world = min(torch.cuda.device_count(), 8)
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_ranks_worker, args=(world, _free_port(), results, layout),
                       nprocs=world, join=True, start_method="spawn")
    assert dict(results) == {r: (True, 0, 0) for r in range(world)}


# ---------------------------------------------------------------- row-sharded RMSNorm + all-gather


def _row_norm_case(rng, rank, world, m, k, pipelined):
    """Six calls of the row-sharded RMSNorm (whole X and own rows alternating),
    each output against the unsharded bf16 RMSNorm bit for bit and fed to a
    GEMM; in the pipelined form the calls run on a side stream while the
    previous call's GEMM runs, ordered by events as in the benchmark."""
    g = seeded(555)
    w = (torch.rand(k, generator=g) + 0.5).to(torch.bfloat16).to(DEV)
    packed = (torch.randn(2 * 128, k, generator=g) * k ** -0.5).to(torch.bfloat16).to(DEV)
    xs = [torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV) for _ in range(6)]
    rows = m // world
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream() if pipelined else main
    consumed = [torch.cuda.Event() for _ in range(2)]
    outs = []
    for call, x in enumerate(xs):
        j = call % 2
        side.wait_event(consumed[j])
        with torch.cuda.stream(side):
            arg = x if call % 2 == 0 else x[rank * rows:(rank + 1) * rows]
            xn = rng(arg, w, 1e-6, slot=j)
            normed = torch.cuda.Event()
            normed.record(side)
        main.wait_event(normed)
        outs.append((xn.clone(), b.gemm_swiglu_bf16(xn, packed)))
        consumed[j].record(main)
    ok = True
    for x, (xn, y) in zip(xs, outs):
        expected = b.rmsnorm_bf16(x, w, 1e-6)
        ok = ok and torch.equal(xn, expected)
        ok = ok and torch.equal(y, b.gemm_swiglu_bf16(expected, packed))
    rng.check()
    return ok


@pytest.mark.parametrize(("rows", "cols"), [(1, 8), (4, 256), (5, 512), (33, 1024), (9, 2048),
                                         (300, 2056), (136, 4096), (7, 8192)])
def test_rmsnorm_allgather_matches_rmsnorm_bit_for_bit(rows, cols):
    """Every width class of the row engine (8 to 8192 columns): each of three
    destinations receives exactly what rmsnorm_bf16 writes, and nothing
    outside its rows (sentinel guard before and after each)."""
    g = seeded(rows * 31 + cols)
    x = (torch.randn(rows, cols, generator=g) * 3).to(torch.bfloat16).to(DEV)
    w = (torch.rand(cols, generator=g) * 2 - 0.5).to(torch.bfloat16).to(DEV)
    guard = 64
    bufs = [torch.full((guard + rows * cols + guard,), 0x7FDE, dtype=torch.int16, device=DEV)
            for _ in range(3)]
    dests = [buf[guard:].data_ptr() for buf in bufs]
    b.rmsnorm_allgather_bf16(x, w, dests, 1e-6)
    expected = b.rmsnorm_bf16(x, w, 1e-6)
    torch.cuda.synchronize()
    for buf in bufs:
        assert torch.equal(buf[guard:guard + rows * cols].view(torch.bfloat16).view(rows, cols),
                           expected)
        assert bool((buf[:guard] == 0x7FDE).all()) and bool((buf[guard + rows * cols:] == 0x7FDE).all())


def test_rmsnorm_allgather_rejects_what_it_cannot_take():
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(64, dtype=torch.bfloat16, device=DEV)
    out = torch.empty(4 * 64 + 8, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        b.rmsnorm_allgather_bf16(x[:, :60].contiguous(), w[:60], [out.data_ptr()], 1e-6)
    with pytest.raises(ValueError):
        b.rmsnorm_allgather_bf16(x, w, [out.data_ptr()] * 9, 1e-6)
    with pytest.raises(RuntimeError, match="CUDA error 1"):  # a destination off 16 bytes
        b.rmsnorm_allgather_bf16(x, w, [out[1:].data_ptr()], 1e-6)
    b.rmsnorm_allgather_bf16(x[:0], w, [out.data_ptr()], 1e-6)  # no rows: nothing to do


@pytest.mark.parametrize("exchange", ["stores", "copies"])
def test_row_norm_gather_one_rank(exchange):
    rng = sharding.RowNormGather(384, 4096, exchange=exchange)
    try:
        assert _row_norm_case(rng, 0, 1, 384, 4096, pipelined=True)
    finally:
        rng.close()
    assert b.peer_status(clear=True) == 0


def _row_norm_worker(rank: int, world: int, port: int, results) -> None:
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    rng = None
    try:
        m, k = 136 * world, 4096  # 136 rows per rank: not a multiple of a CTA's rows
        ok = True
        for exchange in ("stores", "copies"):
            rng = sharding.RowNormGather(m, k, exchange=exchange)
            ok = _row_norm_case(rng, rank, world, m, k, pipelined=False) and ok
            ok = _row_norm_case(rng, rank, world, m, k, pipelined=True) and ok
            rng.close()
            rng = None
        results[rank] = (ok, b.peer_status(), b.gemm_status())
    finally:
        if rng is not None:
            rng.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_row_norm_gather_across_gpus():
    """Each rank normalises its rows of X and places them in every rank's
    buffer over NVLink (peer stores from the norm kernel, and copy engines):
    every rank's buffer must equal the unsharded RMSNorm bit for bit after
    every call."""
    world = min(torch.cuda.device_count(), 8)
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_row_norm_worker, args=(world, _free_port(), results),
                       nprocs=world, join=True, start_method="spawn")
    assert dict(results) == {r: (True, 0, 0) for r in range(world)}
