"""Pool storage and row sharding.

Reference: ``VectorPool`` holds one ``(N, D)`` bf16 parameter created per
device shard (src/model/pool.py:19-40), and the 1-D ``'tp'`` mesh shards it by
rows, ``P('tp', None)`` (src/training/sharding.py:57-58): rank r owns the
contiguous rows ``[r * N / P, (r + 1) * N / P)``.

On B200 each rank keeps its shard resident in HBM as a row-major bf16
``[N_local, d]`` tensor (16-byte aligned rows, the layout TMA and the gather
kernel read).  ``init_normal`` fills a shard from a counter-based generator so
any shard of any shard count equals the matching rows of the unsharded pool.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from .tiled_topk import _stream_handle


@dataclass(frozen=True)
class ShardSpec:
    """Contiguous row block of a pool of ``n_total`` rows owned by ``rank`` of ``world``."""

    n_total: int
    rank: int
    world: int

    def __post_init__(self):
        if self.world < 1 or not (0 <= self.rank < self.world):
            raise ValueError(f"bad rank/world {self.rank}/{self.world}")
        if self.n_total % self.world != 0:
            # The reference computes global indices as local + chip * N_local
            # (retrieval.py:292-293), which presumes equal shards.
            raise ValueError(f"pool rows {self.n_total} must divide evenly over {self.world} shards")

    @property
    def n_local(self) -> int:
        return self.n_total // self.world

    @property
    def row_begin(self) -> int:
        return self.rank * self.n_local

    @property
    def row_end(self) -> int:
        return self.row_begin + self.n_local


def init_normal(out: torch.Tensor, seed: int, stddev: float = 1.0, row_offset: int = 0) -> torch.Tensor:
    """Fill bf16 ``out`` [rows, cols] with stddev * N(0,1) keyed by (seed, row_offset + r, c)."""
    if out.dtype != torch.bfloat16 or out.dim() != 2 or out.stride(1) != 1:
        raise ValueError("out must be a 2-D bf16 tensor with unit column stride")
    if out.device.type != "cuda":
        raise ValueError("out must live on a CUDA device")
    lib = _lib.load()
    with torch.cuda.device(out.device):
        st = lib.dwa_pool_init_normal(out.data_ptr(), out.shape[0], out.shape[1], out.stride(0),
                                      int(row_offset), int(seed) & (2**64 - 1), float(stddev),
                                      _stream_handle(out.device))
    _lib.check(st, "dwa_pool_init_normal")
    return out


def new_normal(rows: int, cols: int, seed: int, stddev: float = 1.0, row_offset: int = 0,
               device=None) -> torch.Tensor:
    """Allocate and fill a bf16 [rows, cols] tensor (see ``init_normal``)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    out = torch.empty((rows, cols), dtype=torch.bfloat16, device=dev)
    return init_normal(out, seed, stddev, row_offset)
