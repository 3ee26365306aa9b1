"""Column (N) sharding of one block-scaled GEMM over the ranks of a node.

C[:, n0:n1] = A . B[n0:n1, :]^T depends only on B's rows n0..n1 and their
scales, so every rank keeps its slice of the weights (pre-sharded) and of
their scales, receives the replicated activation A once, and computes its
column block of C with the single-GPU kernels -- no collective on the data
path.  The optional gather of the bf16 column blocks uses one all-gather into
a rank-major [P][M][N/P] buffer, then a device transpose to [M, N].

Shard boundaries are multiples of `granularity` columns:
  128 for the fp32 and E8M0 block-scale families (one weight scale per
      128 x 128 block),
  16 for weights in shuffle_weight(16,16) layout (16-row tiles),
  8 otherwise (16-byte bf16 output rows).
"""
from __future__ import annotations

import torch


def shard_bounds(n: int, world: int, rank: int, granularity: int = 128) -> tuple[int, int]:
    """Columns [n0, n1) of rank `rank` when n columns are split over `world`
    ranks in blocks of `granularity` (the last shard may be short or empty)."""
    if world <= 0 or not 0 <= rank < world or granularity <= 0 or n < 0:
        raise ValueError("bad shard request")
    units = -(-n // granularity)
    per = -(-units // world)
    n0 = min(n, rank * per * granularity)
    n1 = min(n, n0 + per * granularity)
    return n0, n1


def shard_rows(t: torch.Tensor, n0: int, n1: int, rows_per_entry: int = 1) -> torch.Tensor:
    """Rows of a weight-side tensor that belong to columns [n0, n1) of C:
    B [N, K] (rows_per_entry 1), per-32-K scales [N, K/32] (1), block scales
    [N/128, K/128] (rows_per_entry 128, n0 and n1 multiples of 128)."""
    if n0 % rows_per_entry or (n1 % rows_per_entry and n1 != n0):
        raise ValueError("shard bounds must be multiples of rows_per_entry")
    return t[n0 // rows_per_entry: -(-n1 // rows_per_entry)].contiguous()


def assemble_columns(gathered: torch.Tensor) -> torch.Tensor:
    """[P, M, Ns] rank-major column blocks -> [M, P * Ns]."""
    p, m, ns = gathered.shape
    return gathered.permute(1, 0, 2).reshape(m, p * ns)


def allgather_columns(c_shard: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather equal-width column blocks [M, Ns] of every rank into C [M, P*Ns]."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    gathered = torch.empty((world,) + tuple(c_shard.shape), dtype=c_shard.dtype, device=c_shard.device)
    dist.all_gather(list(gathered.unbind(0)), c_shard.contiguous(), group=group)
    return assemble_columns(gathered)
