"""Multi-GPU partitioning of the large workloads (one process per GPU).

The reference is single-GPU; these helpers add the BASELINE sharding plan:

* row-wise ops (norms, softmax, pointwise) split rows into contiguous ranges,
  one per rank, with no exchange;
* GEMM+SwiGLU splits the N output columns: rank r keeps rows
  [r*N/g, (r+1)*N/g) of the gate half and the same rows of the up half of
  the packed W[2N, K], re-packed as its own contiguous [2N/g, K] (gate block
  first), and X is replicated; the optional output gather is a column-block
  all-gather;
* the global sum reduces each rank's chunk to an fp64 partial and
  all-reduces the partials (the only collective on the data path).

Collectives go through ``torch.distributed`` (NCCL on GPUs, gloo on CPU for
tests of this host logic).  Per-rank compute is injectable so the partition
and combine logic is testable on CPU ranks.
"""

from __future__ import annotations

from typing import Callable

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
