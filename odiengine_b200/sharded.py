"""Row-sharded quantized matrix product over the ranks of a process group.

A weight of N output rows is split by rows: rank r of g holds rows
[r * S, min(N, (r + 1) * S)) with S = ceil(N / g).  Rows are independent dot
products and GGUF blocks run along K, so a shard is a contiguous run of
whole block-rows of the GGUF tensor (no block is split, nothing to repack
across ranks).  Every rank computes y_r = x . W_r^T for the same x, the
slices (padded to S rows) are all-gathered (NCCL over NVLink on GPUs), and
the rank-major result [g][M][S] is permuted to [M][N].

One process per GPU; torch.distributed is the plumbing.  The product itself
is the library's CUDA path (odi_cuda_matmul); ``local_fn`` exists so the
host-side sharding and gathering can be exercised on CPU ranks with a
stand-in product.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np


def shard_rows(N: int, world: int, rank: int) -> tuple[int, int, int]:
    """(first row, end row, padded shard size S) of `rank`'s shard."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    S = math.ceil(N / world)
    lo = min(N, rank * S)
    hi = min(N, lo + S)
    return lo, hi, S


def shard_blocks(blocks: np.ndarray, dtype: int, N: int, K: int, world: int, rank: int) -> np.ndarray:
    """This rank's GGUF block-rows (a contiguous slice of the packed tensor)."""
    from . import BLOCK_BYTES, BLOCK_ELEMS

    row_bytes = (K + BLOCK_ELEMS[dtype] - 1) // BLOCK_ELEMS[dtype] * BLOCK_BYTES[dtype]
    flat = np.ascontiguousarray(blocks).reshape(-1)
    if flat.size != N * row_bytes:
        raise ValueError(f"expected {N * row_bytes} bytes of blocks, got {flat.size}")
    lo, hi, _ = shard_rows(N, world, rank)
    return flat[lo * row_bytes: hi * row_bytes]


def gather_rows(local_y, N: int, S: int, group=None):
    """All-gather the ranks' [M, S] slices and return the [M, N] product."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    M = local_y.shape[0]
    # rank-major concatenation along dim 0 ([world * M, S]), viewed [world, M, S]
    flat = torch.empty((world * M, S), dtype=local_y.dtype, device=local_y.device)
    dist.all_gather_into_tensor(flat, local_y.contiguous(), group=group)
    gathered = flat.view(world, M, S)
    if M == 1:
        return gathered.reshape(1, world * S)[:, :N]
    return gathered.permute(1, 0, 2).reshape(M, world * S)[:, :N]


@dataclass
class RowShardedWeight:
    """This rank's shard of an N x K quantized weight.

    blocks: the full GGUF tensor (host bytes, [N][row bytes]) -- each rank
    keeps only its slice -- or, with ``presharded``, this rank's slice only.
    """

    dtype: int
    N: int
    K: int
    group: object = None
    device: Optional[int] = None
    local_fn: Optional[Callable] = None

    def load(self, blocks: np.ndarray, presharded: bool = False) -> "RowShardedWeight":
        import torch.distributed as dist

        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.lo, self.hi, self.S = shard_rows(self.N, self.world, self.rank)
        part = np.ascontiguousarray(blocks).reshape(-1) if presharded else \
            shard_blocks(blocks, self.dtype, self.N, self.K, self.world, self.rank)
        self.rows = self.hi - self.lo
        if self.local_fn is not None:
            self.shard = part
        elif self.rows > 0:
            from . import DeviceWeight, QuantWeight

            self.shard = DeviceWeight(QuantWeight(self.dtype, (self.K, self.rows), part))
        else:
            self.shard = None
        return self

    def matmul(self, x, act_mode: Optional[int] = None):
        """y[M, N] = x[M, K] . W^T on every rank (x replicated)."""
        import torch

        M = x.shape[0]
        full = self.rows == self.S  # no padding rows: compute straight into the send buffer
        local = (torch.empty if full else torch.zeros)((M, self.S), dtype=torch.float32, device=x.device)
        if self.rows > 0:
            if self.local_fn is not None:
                local[:, : self.rows] = self.local_fn(self.dtype, self.shard, x, self.rows, self.K)
            elif full:
                self.shard.matmul(x, local, act_mode=act_mode)
            else:
                local[:, : self.rows] = self.shard.matmul(x, act_mode=act_mode)
        return gather_rows(local, self.N, self.S, self.group)
