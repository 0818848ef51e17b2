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

``fused=True`` replaces the NCCL all-gather: each rank's GEMV stores its
slice straight into every rank's gathered buffer over NVLink and signals
per-rank arrival counters (odi_cuda_matmul_scatter); a one-block kernel
waits for all ranks before the result is used (odi_cuda_wait_peers).
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


class _DevArray:
    """A raw device pointer exposed through __cuda_array_interface__ so torch
    can view it without a copy."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class SymmetricBuffer:
    """One device buffer per rank, each mapped into every rank (IPC handles
    exchanged over the process group).  ``ptrs[p]`` is rank p's buffer as
    this rank addresses it."""

    def __init__(self, nbytes: int, group=None):
        import ctypes

        import torch.distributed as dist

        from . import IPC_HANDLE_BYTES, check, lib

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        L = lib()
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * IPC_HANDLE_BYTES)()
        check(L.odi_cuda_sym_alloc(nbytes, ctypes.byref(own), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs, self._opened = [], []
        for p, hb in enumerate(handles):
            if p == self.rank:
                self.ptrs.append(own.value)
                continue
            q = ctypes.c_void_p()
            check(L.odi_cuda_ipc_open(ctypes.create_string_buffer(hb, IPC_HANDLE_BYTES), ctypes.byref(q)))
            self.ptrs.append(q.value)
            self._opened.append(q.value)
        self._own = own.value

    def close(self):
        from . import lib

        for q in self._opened:
            lib().odi_cuda_ipc_close(q)
        self._opened = []
        if self._own:
            lib().odi_cuda_sym_free(self._own)
            self._own = None


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
    fused: bool = False  # scatter from the GEMV epilogue instead of an NCCL all-gather
    max_tokens: int = 8  # fused: largest M per call (GEMV path: M < ODI_CUDA_TC_MIN_TOKENS)

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
        if self.fused:
            self._setup_fused()
        return self

    # Layout of each rank's symmetric buffer: counters[8] u64, consumed[8]
    # u64, then two output buffers [max_tokens][N] fp32 used alternately
    # (a rank can be at most one call ahead of another: its wait needs the
    # other's scatter of the previous call, issued after that rank's own
    # use of the older result).
    _HDR = 256

    def _setup_fused(self):
        import torch

        from . import new_workspace

        self._obuf = self.max_tokens * self.N * 4
        self.sym = SymmetricBuffer(self._HDR + 2 * self._obuf, self.group)
        self.calls = 0
        self._spans = [shard_rows(self.N, self.world, p) for p in range(self.world)]
        self._ws = new_workspace(256, torch.device("cuda", torch.cuda.current_device()))

    def _increments(self, M: int, act_mode: int):
        import ctypes

        from . import lib

        inc = (ctypes.c_uint64 * self.world)()
        for p, (lo, hi, _) in enumerate(self._spans):
            n = lib().odi_cuda_scatter_signals(self.dtype, M, hi - lo, self.K, act_mode) if hi > lo else 0
            if n < 0:
                raise ValueError("this shape / mode has no fused scatter (tensor-core path)")
            inc[p] = n
        return inc

    def _matmul_fused(self, x, act_mode: int):
        import ctypes

        import torch

        from . import Scatter, _ptr, _stream, check, lib

        M = x.shape[0]
        if M > self.max_tokens:
            raise ValueError(f"M={M} > max_tokens={self.max_tokens}")
        self.calls += 1
        off = self._HDR + (self.calls & 1) * self._obuf
        sc = Scatter()
        for p in range(self.world):
            sc.out[p] = self.sym.ptrs[p] + off
            sc.counters[p] = self.sym.ptrs[p]
        sc.nranks, sc.rank, sc.row0, sc.ld = self.world, self.rank, self.lo, self.N
        stream = _stream(None)
        ws = self.shard._ws_for(M, act_mode, x.device) if self.rows > 0 else self._ws
        if self.rows > 0:
            check(lib().odi_cuda_matmul_scatter(self.dtype, self.shard.data_ptr, _ptr(x), M, self.rows, self.K,
                                                act_mode, _ptr(ws), ws.numel(), 0, ctypes.byref(sc), stream))
        own = self.sym.ptrs[self.rank]
        check(lib().odi_cuda_wait_peers(own, own + 64, self._increments(M, act_mode), self.world, _ptr(ws), stream))
        return torch.as_tensor(_DevArray(own + off, (M, self.N)), device=x.device)

    def matmul(self, x, act_mode: Optional[int] = None):
        """y[M, N] = x[M, K] . W^T on every rank (x replicated).  In fused
        mode the result is a view of this rank's gathered buffer, valid until
        the call after next."""
        import torch

        M = x.shape[0]
        if self.fused and self.local_fn is None:
            from . import ACT_Q8

            return self._matmul_fused(x, ACT_Q8 if act_mode is None else act_mode)
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
