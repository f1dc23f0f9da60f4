"""Column-sharded multi-GPU plumbing for vkflame_quant_linear_gather.

One process per GPU.  Every rank allocates, for each sharded linear, the
gathered output as two buffers (by step parity) of 8-byte words {two fp16
values, epoch}; the buffers are mapped into every other rank with CUDA IPC,
so that the decode GEMV of rank r stores its slice (columns [r * N / W,
(r + 1) * N / W)) into all ranks' buffers directly over NVLink, and a later
GEMV that reads the buffer as X waits inside its kernel for the words of the
current step (include/vkflame_rt.h, vkf_gather_t).  The handle exchange uses
torch.distributed (all_gather_object); nothing on the data path does.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import rt, shard


@dataclass
class GatheredBuffer:
    tensor: object       # torch int32 [2][M][N / 2][2] on this rank's GPU
    ptrs: list           # every rank's buffer 0 (mapped in this process), rank-ordered
    N: int
    M: int

    @property
    def stride(self) -> int:
        return self.M * (self.N // 2) * 8


class GatherGroup:
    """This rank's view of the gathered buffers of one group of ranks.
    `buffer` must be called in the same order on every rank, and every rank
    must pass a host barrier after the last call and before the first
    gathered launch (buffers are zero, epochs 0)."""

    def __init__(self, dist, world: int, rank: int, device: str = "cuda"):
        import torch
        if not 1 <= world <= rt.MAX_RANKS:
            raise ValueError(f"world {world} outside 1..{rt.MAX_RANKS}")
        self.dist, self.world, self.rank, self.device = dist, world, rank, device
        self.done = torch.zeros(1, dtype=torch.int32, device=device)
        self.epochs = []  # one run counter per call site (op)
        self._opened: dict[bytes, int] = {}

    def _share(self, ptr: int) -> list[int]:
        if self.world == 1:
            return [ptr]
        h, off = rt.ipc_handle(ptr)
        allh = [None] * self.world
        self.dist.all_gather_object(allh, (h, off))
        out = []
        for q, (hq, offq) in enumerate(allh):
            if q == self.rank:
                out.append(ptr)
                continue
            base = self._opened.get(hq)
            if base is None:
                base = rt.ipc_open(hq)
                self._opened[hq] = base
            out.append(base + offq)
        return out

    def buffer(self, N: int, M: int = 1) -> GatheredBuffer:
        import torch
        if N % (2 * self.world):
            raise ValueError(f"N = {N} must split into even slices over {self.world} ranks")
        t = torch.zeros((2, M, N // 2, 2), dtype=torch.int32, device=self.device)
        return GatheredBuffer(t, self._share(t.data_ptr()), N, M)

    def op(self, out: GatheredBuffer, x: GatheredBuffer | None = None) -> "rt.Gather":
        """vkf_gather_t of one call site: this rank's linear writing `out`,
        reading X from the gathered buffer `x` (None: X is an ordinary fp16
        row).  Every call site must run once per step."""
        import torch
        ep = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epochs.append(ep)
        r0, _ = shard.row_range(out.N, self.world, self.rank)
        g = rt.Gather()
        g.world, g.rank = self.world, self.rank
        for q in range(self.world):
            g.y_rank[q] = out.ptrs[q] + (r0 // 2) * 8
        g.stride = out.stride
        g.epoch = ep.data_ptr()
        g.done = self.done.data_ptr()
        g.x_gathered = int(x is not None)
        g.x_stride = x.stride if x is not None else 0
        return g

    def chain_linear(self, W: int, wtype: int, K: int, n: int, out: GatheredBuffer | None = None,
                     x_src: int = -1, x_plain: int = 0, y_plain: int = 0) -> "rt.ChainLinear":
        """vkf_chain_linear_t of one link of a chain: this rank's n rows of W
        (ggml blocks, K values each), writing its slice of `out` (gathered)
        or, at world size 1, the plain fp16 row `y_plain`; reading the
        gathered output of chain entry `x_src`, or the fp16 row `x_plain`."""
        c = rt.ChainLinear()
        c.W, c.wtype, c.K, c.N, c.x_src, c.x_plain = W, wtype, K, n, x_src, x_plain
        c.y_plain = y_plain
        if out is not None:
            r0, _ = shard.row_range(out.N, self.world, self.rank)
            if r0 != self.rank * n or out.N != n * self.world:
                raise ValueError("shard rows do not match the gathered buffer")
            for q in range(self.world):
                c.y_rank[q] = out.ptrs[q] + (r0 // 2) * 8
            c.y_stride = out.stride
        return c

    def close(self) -> None:
        for base in self._opened.values():
            rt.ipc_close(base)
        self._opened.clear()


def unpack(words: np.ndarray, epoch: int) -> np.ndarray:
    """[2][M][N/2][2] int32 gathered buffer (host copy) -> the fp16 [M][N] of
    the run whose words carry `epoch` (buffer epoch & 1).  Raises if any
    word carries another epoch."""
    b = np.asarray(words)[epoch & 1]
    if not (b[..., 1] == epoch).all():
        raise ValueError("gathered buffer holds words of another step")
    return np.ascontiguousarray(b[..., 0]).view(np.float16).reshape(b.shape[0], -1)
