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
from multiprocessing import shared_memory

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


class HostPeers:
    """Host stand-ins for the peer operations of :class:`sharding.PeerColumnGather`.

    "Device memory" is POSIX shared memory that every rank process can map;
    an address is (segment number << 40) + byte offset.  The GEMM is the CPU
    oracle writing its block to every destination with row stride ld; the
    barrier writes this rank's epoch into slot `rank` of every flag array,
    meets the other ranks at a gloo barrier and checks that every slot of its
    own array has reached the epoch -- the protocol of the device barrier, with
    the waiting done by gloo.
    """

    def __init__(self) -> None:
        self.segments: dict[int, shared_memory.SharedMemory] = {}
        self.next = 1
        self.epochs_seen: list[bool] = []
        self.normed_rows: list[int] = []

    def _map(self, shm: shared_memory.SharedMemory) -> int:
        base = self.next << 40
        self.next += 1
        self.segments[base] = shm
        return base

    def _resolve(self, addr: int) -> tuple[shared_memory.SharedMemory, int]:
        base = (addr >> 40) << 40
        return self.segments[base], addr - base

    def alloc(self, nbytes: int) -> tuple[int, bytes]:
        shm = shared_memory.SharedMemory(create=True, size=nbytes)
        shm.buf[:nbytes] = bytes(nbytes)
        return self._map(shm), shm.name.encode()

    def open(self, handle: bytes) -> int:
        return self._map(shared_memory.SharedMemory(name=handle.decode()))

    def close(self, addr: int) -> None:
        self.segments.pop(addr).close()

    def free(self, addr: int) -> None:
        shm = self.segments.pop(addr)
        shm.close()
        shm.unlink()

    def view(self, addr: int, m: int, n: int) -> torch.Tensor:
        shm, off = self._resolve(addr)
        return torch.frombuffer(shm.buf, dtype=torch.bfloat16, count=m * n, offset=off).view(m, n)

    def gemm(self, x, row_scale, packed_shard, dests, ld) -> None:
        block = oracle.gemm_swiglu_rowscale_bf16(x, row_scale, packed_shard)
        m, n = block.shape
        for d in dests:
            shm, off = self._resolve(d)
            rows = torch.frombuffer(shm.buf, dtype=torch.bfloat16, count=(m - 1) * ld + n,
                                    offset=off)
            rows.as_strided((m, n), (ld, 1)).copy_(block)
            del rows

    def rmsnorm_gather(self, x, weight, dests, eps) -> None:
        """The fused RMSNorm: the oracle's rows written to every destination."""
        self.normed_rows.append(x.shape[0])
        rows = oracle.rmsnorm_bf16(x, weight, eps)
        for d in dests:
            shm, off = self._resolve(d)
            torch.frombuffer(shm.buf, dtype=torch.bfloat16, count=rows.numel(),
                             offset=off).copy_(rows.reshape(-1))

    def barrier(self, flag_addrs, rank, epoch) -> None:
        world = len(flag_addrs)
        for a in flag_addrs:
            shm, off = self._resolve(a)
            flags = torch.frombuffer(shm.buf, dtype=torch.int32, count=world, offset=off)
            flags[rank] = epoch
            del flags
        dist.barrier()
        shm, off = self._resolve(flag_addrs[rank])
        own = torch.frombuffer(shm.buf, dtype=torch.int32, count=world, offset=off).tolist()
        # another rank may already have arrived at the next epoch: at least this one
        self.epochs_seen.append(all(v >= epoch for v in own))

    def status(self) -> int:
        return 0


def _gather_worker(rank: int, world: int, port: int, results, layout: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator()
        g.manual_seed(4321)
        m, k, n = 24, 32, 20
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        packed = (torch.randn(2 * n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
        rs = torch.rand(m, generator=g) + 0.5
        peers = HostPeers()
        gather = sharding.PeerColumnGather(m, n, peers=peers, layout=layout)
        shard = sharding.pack_gate_up_shard(packed, rank, world)
        nl = n // world
        ok = []
        outs = []
        for call in range(3):
            out = gather(x, shard, rs * (1 + call))
            full = oracle.gemm_swiglu_rowscale_bf16(x, rs * (1 + call), packed)
            if layout == "blocks":
                full = torch.stack([full[:, r * nl:(r + 1) * nl] for r in range(world)])
            ok.append(torch.equal(out, full))
            outs.append(out.data_ptr())
        alternate = outs[0] == outs[2] != outs[1]
        first = gather.destinations(0)[0] - gather.addrs[0][rank]
        first_ok = first == (rank * m * nl * 2 if layout == "blocks" else rank * nl * 2)
        epochs = peers.epochs_seen == [True] * 3
        del out
        gather.close()
        results[rank] = (all(ok), alternate, first_ok, epochs, not peers.segments)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", ["blocks", "columns"])
def test_peer_column_gather_two_gloo_ranks(layout):
    """Host logic of the fused GEMM + all-gather: handle exchange, the
    destination addresses (this rank's column block in every rank's buffer,
    in either layout), alternating buffers, epochs of the flag barrier and
    the collective close."""
    world = 2
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_gather_worker, args=(world, _free_port(), results, layout),
                       nprocs=world, join=True, start_method="spawn")
    assert dict(results) == {r: (True, True, True, True, True) for r in range(world)}


def _row_norm_worker(rank: int, world: int, port: int, results, exchange: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator()
        g.manual_seed(8765)
        m, k = 16, 40
        xs = [torch.randn(m, k, generator=g).to(torch.bfloat16) for _ in range(3)]
        w = (torch.rand(k, generator=g) + 0.5).to(torch.bfloat16)
        normed_rows = []

        def norm(x, weight, out, eps):
            normed_rows.append(x.shape[0])
            out.copy_(oracle.rmsnorm_bf16(x, weight, eps))

        peers = HostPeers()
        rng = sharding.RowNormGather(m, k, peers=peers, norm=norm, exchange=exchange)
        rows = m // world
        ok, ptrs = [], []
        for call, x in enumerate(xs):
            # whole X on even calls, only this rank's rows on odd ones
            arg = x if call % 2 == 0 else x[rank * rows:(rank + 1) * rows]
            out = rng(arg, w, 1e-6)
            dist.barrier()  # the host stand-in copies synchronously: every rank done
            ok.append(torch.equal(out, oracle.rmsnorm_bf16(x, w, 1e-6)))
            ptrs.append(out.data_ptr())
            dist.barrier()  # every rank checked before the buffer is reused
        alternate = ptrs[0] == ptrs[2] != ptrs[1]
        own_rows_only = (normed_rows if exchange == "copies" else peers.normed_rows) == [rows] * 3
        first = rng.dest_addrs[0][0] - rng.addrs[0][rank] == rank * rows * k * 2
        own_rows_only = own_rows_only and first
        epochs = peers.epochs_seen == [True] * 6 and rng.epoch == 6
        del out
        rng.close()
        results[rank] = (all(ok), alternate, own_rows_only, epochs, not peers.segments)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["stores", "copies"])
@pytest.mark.parametrize("world", [2, 4])
def test_row_norm_gather_gloo_ranks(world, exchange):
    """Host logic of the row-sharded RMSNorm with its all-gather: each rank
    normalises only its M/g rows, its rows land in every rank's buffer, two
    barrier epochs per call, alternating buffers, collective close."""
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_row_norm_worker, args=(world, _free_port(), results, exchange),
                       nprocs=world, join=True, start_method="spawn")
    assert dict(results) == {r: (True, True, True, True, True) for r in range(world)}


def test_row_norm_gather_rejects_bad_shapes():
    peers = HostPeers()
    rng = sharding.RowNormGather(8, 16, peers=peers, norm=lambda *a: None)
    with pytest.raises(ValueError):
        rng(torch.zeros(4, 8, dtype=torch.bfloat16), torch.zeros(16), 1e-6)
    with pytest.raises(ValueError):
        rng(torch.zeros(8, 16, dtype=torch.bfloat16), torch.zeros(16), 1e-6, slot=2)
    with pytest.raises(ValueError):
        sharding.RowNormGather(8, 16, peers=peers, exchange="nccl")
    rng.close()
    assert not peers.segments


def test_peer_column_gather_rejects_bad_shapes():
    peers = HostPeers()
    gather = sharding.PeerColumnGather(8, 20, peers=peers)
    with pytest.raises(ValueError):
        gather(torch.zeros(4, 8), torch.zeros(40, 8))
    with pytest.raises(ValueError):
        sharding.PeerColumnGather(8, 20, peers=peers, layout="rows")
    gather.close()
    assert not peers.segments


def test_peer_column_gather_check_raises_after_a_barrier_timeout():
    """A barrier that gave up leaves a non-zero status word: check() turns it
    into an error (and passes when every barrier completed)."""

    class TimedOutPeers(HostPeers):
        def __init__(self) -> None:
            super().__init__()
            self.code = 0

        def barrier(self, flag_addrs, rank, epoch) -> None:
            pass  # one rank: nothing to wait for

        def status(self) -> int:
            code, self.code = self.code, 0
            return code

    peers = TimedOutPeers()
    gather = sharding.PeerColumnGather(8, 20, peers=peers)
    g = torch.Generator()
    g.manual_seed(7)
    x = torch.randn(8, 16, generator=g).to(torch.bfloat16)
    packed = torch.randn(40, 16, generator=g).to(torch.bfloat16)
    gather(x, packed, torch.ones(8))
    gather.check()
    peers.code = 2  # bit 1: the wait for a peer's flag ran out
    with pytest.raises(RuntimeError, match="timed out"):
        gather.check()
    gather.check()  # the status word was cleared by the failing check
    gather.close()
    assert not peers.segments


def test_peer_column_gather_releases_memory_when_setup_fails():
    class FailingPeers(HostPeers):
        def __init__(self) -> None:
            super().__init__()
            self.allocs = 0

        def alloc(self, nbytes):
            self.allocs += 1
            if self.allocs == 2:
                raise RuntimeError("CUDA error 2: out of memory")
            return super().alloc(nbytes)

    peers = FailingPeers()
    with pytest.raises(RuntimeError, match="out of memory"):
        sharding.PeerColumnGather(8, 20, peers=peers)
    assert not peers.segments  # the first buffer was freed again


@pytest.mark.parametrize("layout", ["blocks", "columns"])
def test_peer_column_gather_destinations_at_eight_ranks(monkeypatch, layout):
    """Destination arithmetic of rank 3 of 8 (one process; the collective calls
    replaced): its block goes to its own buffer first, then to ranks 4, 5, ...,
    2, at the block's origin in each rank's buffer of the current call."""
    world, rank, m, n = 8, 3, 6, 64
    peers = HostPeers()
    handles_seen = []
    others = []  # the other ranks' buffers, made here

    def all_gather_object(out, obj, group=None):
        handles_seen.append(obj)
        for j in range(world):
            if j == rank:
                out[j] = obj
                continue
            made = [peers.alloc(4096) for _ in range(2)]
            others.extend(addr for addr, _ in made)
            out[j] = [handle for _, handle in made]

    monkeypatch.setattr(sharding.dist, "is_initialized", lambda: True)
    monkeypatch.setattr(sharding.dist, "get_world_size", lambda group=None: world)
    monkeypatch.setattr(sharding.dist, "get_rank", lambda group=None: rank)
    monkeypatch.setattr(sharding.dist, "all_gather_object", all_gather_object)
    monkeypatch.setattr(sharding.dist, "barrier", lambda group=None: None)
    gather = sharding.PeerColumnGather(m, n, peers=peers, layout=layout)
    nl = n // world
    for call in range(3):
        dests = gather.destinations(call)
        order = [(rank + j) % world for j in range(world)]
        offset = rank * m * nl * 2 if layout == "blocks" else rank * nl * 2
        assert dests == [gather.addrs[call % 2][r] + offset for r in order]
        assert dests[0] - gather.addrs[call % 2][rank] == offset
    assert gather.ld == (nl if layout == "blocks" else n)
    assert len(handles_seen) == 1 and len(handles_seen[0]) == 2
    gather.outputs = []
    gather.close()
    for addr in others:
        peers.free(addr)
    assert not peers.segments


def test_shard_plans_partition_and_repack_exactly():
    """Property check over many sizes: row ranges tile [0, total) in rank order
    with sizes differing by at most one, and the per-rank packed gate/up shards
    hold exactly the packed weight's rows (gate block, then up block)."""
    hypothesis = pytest.importorskip("hypothesis")
    given, settings, st = hypothesis.given, hypothesis.settings, hypothesis.strategies

    @settings(max_examples=200, deadline=None)
    @given(total=st.integers(0, 5000), world=st.integers(1, 8))
    def ranges(total, world):
        spans = [sharding.shard_range(total, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [hi - lo for lo, hi in spans]
        assert max(sizes) - min(sizes) <= 1

    @settings(max_examples=100, deadline=None)
    @given(n=st.integers(1, 40), k=st.integers(1, 5), world=st.integers(1, 8))
    def repack(n, k, world):
        packed = torch.arange(2 * n * k, dtype=torch.float32).view(2 * n, k)
        gates, ups = [], []
        for r in range(world):
            shard = sharding.pack_gate_up_shard(packed, r, world)
            lo, hi = sharding.shard_range(n, r, world)
            assert shard.shape == (2 * (hi - lo), k)
            gates.append(shard[: hi - lo])
            ups.append(shard[hi - lo:])
        assert torch.equal(torch.cat(gates), packed[:n])
        assert torch.equal(torch.cat(ups), packed[n:])

    ranges()
    repack()
