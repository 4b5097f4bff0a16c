"""Multi-GPU partitioning of the large workloads (one process per GPU).

The reference is single-GPU; these helpers add a sharding plan for one box:

* row-wise ops (norms, softmax, pointwise) split rows into contiguous ranges,
  one per rank, with no exchange;
* GEMM+SwiGLU splits the N output columns: rank r keeps rows
  [r*N/g, (r+1)*N/g) of the gate half and the same rows of the up half of
  the packed W[2N, K], re-packed as its own contiguous [2N/g, K] (gate block
  first), and X is replicated; the optional output gather is a column-block
  all-gather;
* the global sum reduces each rank's chunk to an fp64 partial and
  all-reduces the partials (the only collective on the data path);
* :class:`PeerColumnGather` fuses the optional output gather into the GEMM:
  each rank's epilogue stores its column block straight into every rank's
  [M, N] output over NVLink (CUDA IPC peer mappings), then a device-side flag
  barrier tells each rank that the other blocks have landed.

Collectives go through ``torch.distributed`` (NCCL on GPUs, gloo on CPU for
tests of this host logic).  Per-rank compute is injectable so the partition
and combine logic is testable on CPU ranks.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of `total` items owned by `rank`; the first
    total % world ranks own one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def shard_rows(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows of a 2-D tensor owned by `rank` (a contiguous view)."""
    lo, hi = shard_range(x.shape[0], rank, world)
    return x[lo:hi]


def pack_gate_up_shard(packed_weight: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """[2N/g, K] packed weight of one rank: its gate rows, then its up rows."""
    if packed_weight.ndim != 2 or packed_weight.shape[0] % 2:
        raise ValueError("packed_weight must be [2N, K]")
    n = packed_weight.shape[0] // 2
    lo, hi = shard_range(n, rank, world)
    return torch.cat((packed_weight[lo:hi], packed_weight[n + lo:n + hi]), dim=0).contiguous()


def gather_columns(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather column blocks [M, N/g] of every rank into [M, N] (equal
    blocks).  The optional output gather of the N-sharded GEMM."""
    world = dist.get_world_size(group)
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def _library_partial(x: torch.Tensor) -> torch.Tensor:
    from . import bindings

    return bindings.reduction_partial_f64(x)


def distributed_sum(x_local: torch.Tensor, group=None,
                    partial_fn: Callable[[torch.Tensor], torch.Tensor] = _library_partial
                    ) -> torch.Tensor:
    """Global fp32 sum of the chunks held by all ranks.

    Each rank reduces its chunk to a one-element float64 partial
    (``reduction_partial_f64`` on a GPU), the partials are summed with one
    all-reduce, and the result is rounded once to fp32.
    """
    partial = partial_fn(x_local).reshape(1).to(torch.float64)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(partial, group=group)
    return partial.to(torch.float32)


def mlp_block_sharded(x: torch.Tensor, norm_weight: torch.Tensor, packed_shard: torch.Tensor,
                      eps: float = 1e-6, xn_out: torch.Tensor | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """One rank's part of RMSNorm -> N-sharded GEMM+SwiGLU (bf16).

    Every rank normalises all rows of the replicated X (the GEMM of each N
    slice needs all of them) and multiplies by its packed weight shard;
    the result is the rank's [M, N/g] output column block.
    """
    from . import bindings

    xn = xn_out if xn_out is not None else torch.empty_like(x)
    bindings.rmsnorm_bf16_into(x, norm_weight, xn, eps)
    if out is None:
        out = torch.empty((x.shape[0], packed_shard.shape[0] // 2), device=x.device,
                          dtype=torch.bfloat16)
    return bindings.gemm_swiglu_bf16_into(xn, packed_shard, out)


# ---------------------------------------------------------------- fused output gather

_FLAG_BYTES = 256  # one uint32 per rank (up to 8), padded


class _CudaWords:
    """__cuda_array_interface__ view of raw device memory as int16 words."""

    def __init__(self, addr: int, shape: tuple[int, ...]) -> None:
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<i2", "data": (addr, False),
                                         "version": 3, "strides": None}


class LibraryPeers:
    """Peer memory, fused gather GEMM and RMSNorm, and barrier of the CUDA
    library.

    The operations :class:`PeerColumnGather` and :class:`RowNormGather` need,
    as one object so that a test can substitute host-side stand-ins for them."""

    def __init__(self, timeout_ns: int = 5_000_000_000) -> None:
        from . import bindings

        self._b = bindings
        self.timeout_ns = timeout_ns

    def alloc(self, nbytes: int) -> tuple[int, bytes]:
        return self._b.peer_alloc(nbytes)

    def open(self, handle: bytes) -> int:
        return self._b.peer_open(handle)

    def close(self, addr: int) -> None:
        self._b.peer_close(addr)

    def free(self, addr: int) -> None:
        self._b.peer_free(addr)

    def view(self, addr: int, m: int, n: int) -> torch.Tensor:
        return torch.as_tensor(_CudaWords(addr, (m, n)), device="cuda").view(torch.bfloat16)

    def gemm(self, x: torch.Tensor, row_scale: torch.Tensor | None, packed_shard: torch.Tensor,
             dests: Sequence[int], ld: int) -> None:
        self._b.gemm_swiglu_allgather_bf16(x, row_scale, packed_shard, dests, ld)

    def rmsnorm_gather(self, x: torch.Tensor, weight: torch.Tensor, dests: Sequence[int],
                       eps: float) -> None:
        self._b.rmsnorm_allgather_bf16(x, weight, dests, eps)

    def barrier(self, flag_addrs: Sequence[int], rank: int, epoch: int) -> None:
        self._b.peer_barrier(flag_addrs, rank, epoch, self.timeout_ns)

    def status(self) -> int:
        return self._b.peer_status(clear=True)


class PeerColumnGather:
    """N-sharded GEMM+SwiGLU with its column all-gather fused into the GEMM.

    Every rank holds two bf16 output buffers of M * N elements in memory the
    other ranks have mapped (CUDA IPC), plus a flag array.  A call runs the
    rank's GEMM with the gathering epilogue -- each finished tile of its
    [M, N/g] column block is stored into the same place of every rank's
    current buffer, the NVLink transfers overlapping the remaining tiles --
    and then the device barrier, after which the returned buffer holds all g
    blocks.  Everything is stream-ordered on the current stream; the host
    never waits.

    ``layout`` places the blocks: ``"blocks"`` (default) returns
    [g, M, N/g] with rank r's block contiguous at [r] -- the layout of
    ``torch.distributed.all_gather_into_tensor``; ``"columns"`` returns the
    [M, N] matrix itself.  The block layout is the fast one: a tile's rows
    then lie within one 2 MiB page of each peer's buffer, while in [M, N] a
    page holds only 2 MiB / (2N) rows and the peer stores of all tiles in
    flight touch g - 1 times as many pages (measured at 8 GPUs, M = 16384,
    N = 14336: 0.73 ms per step against 2.6 ms).

    The two buffers alternate.  A returned output stays valid until the call
    after the next one, provided each rank reads it on the current stream
    before its own next call: rank r's GEMM of call c + 2 runs after r passed
    barrier c + 1, which every other rank p entered only after its GEMM
    c + 1, and so after p's reads of the output of call c.

    Construction and :meth:`close` are collective (``torch.distributed``
    object all-gather and barriers on ``group``).  ``peers`` supplies the
    memory, GEMM and barrier operations (default: the CUDA library).
    """

    def __init__(self, m: int, n: int, group=None, peers=None, layout: str = "blocks") -> None:
        if layout not in ("blocks", "columns"):
            raise ValueError("layout must be 'blocks' or 'columns'")
        self.layout = layout
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if not 1 <= self.world <= 8:
            raise ValueError("the fused gather supports 1 to 8 ranks")
        if n % self.world:
            raise ValueError("N must divide evenly between the ranks")
        self.m, self.n, self.n_local = m, n, n // self.world
        self.group = group
        self.peers = peers if peers is not None else LibraryPeers()
        out_bytes = m * n * 2
        self._flag_offset = -(-out_bytes // 256) * 256
        nbytes = self._flag_offset + _FLAG_BYTES
        self._local: list[int] | None = []
        self._opened: list[int] = []
        handles: list[bytes] = []
        try:
            for _ in range(2):
                addr, handle = self.peers.alloc(nbytes)
                self._local.append(addr)
                handles.append(handle)
            every = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(every, handles, group=group)
            else:
                every = [handles]
            # addrs[i][j]: rank j's buffer i as mapped here
            self.addrs = [[0] * self.world for _ in range(2)]
            for j in range(self.world):
                for i in range(2):
                    if j == self.rank:
                        self.addrs[i][j] = self._local[i]
                    else:
                        self.addrs[i][j] = self.peers.open(every[j][i])
                        self._opened.append(self.addrs[i][j])
        except Exception:
            # release what this rank holds; the other ranks' next collective on
            # `group` then fails with the process group's timeout
            for addr in self._opened:
                self.peers.close(addr)
            for addr in self._local:
                self.peers.free(addr)
            self._local = None
            raise
        self.outputs = [self.peers.view(self._local[i], m, n) for i in range(2)]
        if layout == "blocks":
            self.outputs = [o.view(self.world, m, self.n_local) for o in self.outputs]
        self.flag_addrs = [self.addrs[0][j] + self._flag_offset for j in range(self.world)]
        self.calls = 0
        if self.world > 1:
            dist.barrier(group=group)  # every mapping exists before any peer store

    @property
    def ld(self) -> int:
        """Row stride (elements) of a block in the output buffers."""
        return self.n_local if self.layout == "blocks" else self.n

    def destinations(self, call: int) -> list[int]:
        """Addresses the gathering epilogue of `call` stores to: this rank's
        block in its own buffer first, then in rank+1, rank+2, ... (mod g)."""
        i = call % 2
        if self.layout == "blocks":
            offset = self.rank * self.m * self.n_local * 2
        else:
            offset = self.rank * self.n_local * 2
        order = [(self.rank + j) % self.world for j in range(self.world)]
        return [self.addrs[i][r] + offset for r in order]

    def __call__(self, x: torch.Tensor, packed_shard: torch.Tensor,
                 row_scale: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's GEMM (packed_shard [2N/g, K], optional row scale) and the
        gather; returns the output holding every rank's block ([g, M, N/g] or
        [M, N], see ``layout``).

        The barrier that completes the gather waits a bounded time
        (``peers.timeout_ns``); when it gives up, the returned buffer may miss
        other ranks' blocks and nothing is raised here, because the host never
        waits for the device.  Call :meth:`check` (it synchronises) before
        trusting an output: it raises if any barrier since the last check
        timed out."""
        if x.shape[0] != self.m or packed_shard.shape[0] != 2 * self.n_local:
            raise ValueError(f"expected x[{self.m}, K] and a packed shard of "
                             f"{2 * self.n_local} rows")
        call = self.calls
        self.calls += 1
        self.peers.gemm(x, row_scale, packed_shard, self.destinations(call), self.ld)
        self.peers.barrier(self.flag_addrs, self.rank, self.calls)
        return self.outputs[call % 2]

    def check(self) -> None:
        """Raise RuntimeError if a peer barrier of an earlier call gave up
        waiting (its output may lack other ranks' blocks).  Synchronises the
        device and clears the status word."""
        code = self.peers.status()
        if code != 0:
            raise RuntimeError(f"fused all-gather: a peer barrier timed out (status {code}); "
                               "outputs since the last check may miss other ranks' blocks")

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective).  Output
        tensors returned by earlier calls must not be used afterwards."""
        if self._local is None:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank still stores into a buffer
        for addr in self._opened:
            self.peers.close(addr)
        if self.world > 1:
            dist.barrier(group=self.group)  # every mapping closed before the frees
        self.outputs = []
        for addr in self._local:
            self.peers.free(addr)
        self._local = None


# ---------------------------------------------------------------- row-sharded norm, all-gathered


def _library_rmsnorm(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, eps: float) -> None:
    from . import bindings

    bindings.rmsnorm_bf16_into(x, weight, out, eps)


class RowNormGather:
    """bf16 RMSNorm of X[M, K] sharded by rows, the normalised rows
    all-gathered to every rank over NVLink.

    The large MLP workload needs the whole normalised X on every rank (each
    rank's GEMM owns an N slice, all M rows).  Instead of every rank
    normalising all M rows, rank r normalises its M/g rows and places them in
    the same rows of every rank's [M, K] buffer (memory shared with CUDA IPC).
    Two exchanges:

    * ``"stores"`` (default): one kernel, ``rmsnorm_allgather_bf16``, whose
      threads store each normalised vector into all g buffers, the NVLink
      traffic spread over the kernel;
    * ``"copies"``: the RMSNorm into this rank's own buffer, then one
      ``cudaMemcpyAsync`` per peer on its own stream (copy engines, no SMs).

    Two device flag barriers bracket a call: the first makes sure no rank
    still reads the buffer (its previous use), the second that every rank's
    rows have landed.  Run on a second stream, a call overlaps the previous
    step's GEMM.

    It is for X that arrives sharded by rows (each rank uploads or produces
    only its rows).  When every rank already holds all of X, normalising all
    rows locally is faster: at 8 GPUs that reads and writes 268 MB of the
    rank's own HBM in ~40 us, where this exchange writes 117 MB over NVLink
    into every rank (~200 us alone) and slows a GEMM running beside it.

    Two buffers alternate (``slot``).  Before a call the caller must have
    ordered, on the current stream, every read of that slot's previous
    contents on this rank; the first barrier extends that to all ranks.
    Construction and :meth:`close` are collective; ``peers`` supplies memory,
    views, the fused RMSNorm and the barrier (default: the CUDA library),
    ``norm`` the per-shard RMSNorm of the copy exchange (default:
    ``bindings.rmsnorm_bf16_into``).  The barriers wait a bounded time;
    :meth:`check` raises if one gave up.
    """

    def __init__(self, m: int, k: int, group=None, peers=None,
                 norm: Callable[[torch.Tensor, torch.Tensor, torch.Tensor, float], None] | None = None,
                 exchange: str = "stores") -> None:
        if exchange not in ("stores", "copies"):
            raise ValueError("exchange must be 'stores' or 'copies'")
        self.exchange = exchange
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if not 1 <= self.world <= 8:
            raise ValueError("the row-sharded norm gather supports 1 to 8 ranks")
        if m % self.world:
            raise ValueError("M must divide evenly between the ranks")
        self.m, self.k, self.rows = m, k, m // self.world
        self.group = group
        self.peers = peers if peers is not None else LibraryPeers()
        self.norm = norm if norm is not None else _library_rmsnorm
        buf_bytes = m * k * 2
        self._flag_offset = -(-buf_bytes // 256) * 256
        nbytes = self._flag_offset + _FLAG_BYTES
        self._local: list[int] | None = []
        self._opened: list[int] = []
        handles: list[bytes] = []
        try:
            for _ in range(2):
                addr, handle = self.peers.alloc(nbytes)
                self._local.append(addr)
                handles.append(handle)
            every = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(every, handles, group=group)
            else:
                every = [handles]
            self.addrs = [[0] * self.world for _ in range(2)]
            for j in range(self.world):
                for i in range(2):
                    if j == self.rank:
                        self.addrs[i][j] = self._local[i]
                    else:
                        self.addrs[i][j] = self.peers.open(every[j][i])
                        self._opened.append(self.addrs[i][j])
        except Exception:
            for addr in self._opened:
                self.peers.close(addr)
            for addr in self._local:
                self.peers.free(addr)
            self._local = None
            raise
        self.outputs = [self.peers.view(self._local[i], m, k) for i in range(2)]
        row_bytes = self.rank * self.rows * k * 2
        # dests[i][j]: this rank's rows inside rank j's buffer i, as mapped here
        self.dests = [[self.peers.view(self.addrs[i][j] + row_bytes, self.rows, k)
                       for j in range(self.world)] for i in range(2)]
        self.flag_addrs = [self.addrs[0][j] + self._flag_offset for j in range(self.world)]
        # where this rank's rows go in buffer i of every rank: its own first,
        # then rank+1, rank+2, ... (mod g), so that the ranks' first peer
        # stores go to different GPUs
        order = [(self.rank + j) % self.world for j in range(self.world)]
        self.dest_addrs = [[self.addrs[i][r] + row_bytes for r in order] for i in range(2)]
        self.epoch = 0
        self.calls = 0
        self._streams = None
        if exchange == "copies" and torch.cuda.is_available() and self.outputs[0].is_cuda:
            self._streams = [torch.cuda.Stream() for _ in range(self.world)]
        if self.world > 1:
            dist.barrier(group=group)  # every mapping exists before any copy

    def _barrier(self) -> None:
        self.epoch += 1
        self.peers.barrier(self.flag_addrs, self.rank, self.epoch)

    def __call__(self, x: torch.Tensor, weight: torch.Tensor, eps: float,
                 slot: int | None = None) -> torch.Tensor:
        """RMSNorm of every row of X (bf16), this rank computing its M/g rows.
        `x` is either the whole X [M, K] or only this rank's rows [M/g, K]
        (rows r*M/g to (r+1)*M/g - 1).  Returns buffer `slot` (default:
        alternating) holding all M normalised rows once the current stream
        reaches it."""
        lo = self.rank * self.rows
        if tuple(x.shape) == (self.m, self.k):
            x = x[lo:lo + self.rows]
        elif tuple(x.shape) != (self.rows, self.k):
            raise ValueError(f"expected x[{self.m}, {self.k}] or this rank's rows "
                             f"x[{self.rows}, {self.k}]")
        i = self.calls % 2 if slot is None else slot
        if i not in (0, 1):
            raise ValueError("slot must be 0 or 1")
        self.calls += 1
        self._barrier()  # nobody still reads buffer i
        if self.exchange == "stores":
            self.peers.rmsnorm_gather(x, weight, self.dest_addrs[i], eps)
            self._barrier()  # every rank's rows have landed
            return self.outputs[i]
        own = self.outputs[i][lo:lo + self.rows]
        self.norm(x, weight, own, eps)
        if self.world > 1:
            if self._streams is not None:
                current = torch.cuda.current_stream()
                for j in range(self.world):
                    if j == self.rank:
                        continue
                    s = self._streams[j]
                    s.wait_stream(current)
                    with torch.cuda.stream(s):
                        self.dests[i][j].copy_(own, non_blocking=True)
                for j in range(self.world):
                    if j != self.rank:
                        current.wait_stream(self._streams[j])
            else:
                for j in range(self.world):
                    if j != self.rank:
                        self.dests[i][j].copy_(own)
        self._barrier()  # every rank's rows have landed
        return self.outputs[i]

    def check(self) -> None:
        """Raise RuntimeError if a barrier of an earlier call gave up waiting
        (a buffer may then miss other ranks' rows).  Synchronises the device."""
        code = self.peers.status()
        if code != 0:
            raise RuntimeError(f"row-sharded norm gather: a peer barrier timed out (status {code})")

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective)."""
        if self._local is None:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        self.dests = []
        for addr in self._opened:
            self.peers.close(addr)
        if self.world > 1:
            dist.barrier(group=self.group)
        self.outputs = []
        for addr in self._local:
            self.peers.free(addr)
        self._local = None
