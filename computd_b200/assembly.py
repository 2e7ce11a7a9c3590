"""Alpha normalisation + gathered pool-row weighted sum (the value side of the path).

Reference: ``alpha = top_vals / (sum(top_vals) + 1e-8)`` (src/model/retrieval.py:326)
and WeightAssembler's gather + alpha-weighted sum
``selected = vectors[idx]; b_delta = einsum('...k,...kj->...j', alpha, selected)``
(src/model/assembly.py:104,127).  The B200 kernel never materialises the
gathered ``[M, k, d]`` rows.

On a row-sharded pool each rank sums only the rows it owns (owner-computes) and
the partial sums are added with one all-reduce, instead of the reference's
GSPMD all-gather of the whole pool (src/model/dwa.py:190-192).
"""
from __future__ import annotations

import torch

from . import _lib
from .tiled_topk import _stream_handle


def _check_values(values: torch.Tensor) -> torch.Tensor:
    if values.device.type != "cuda":
        raise ValueError("values must live on a CUDA device")
    if values.dim() != 2:
        raise ValueError("values must be 2-D [rows, d]")
    if values.dtype != torch.bfloat16:
        values = values.to(torch.bfloat16)
    if values.stride(1) != 1 or values.stride(0) % 8 != 0 or values.data_ptr() % 16 != 0:
        values = values.contiguous()
    return values


def weighted_gather_into(vals: torch.Tensor, gidx: torch.Tensor, values: torch.Tensor,
                         out: torch.Tensor, alpha_out: torch.Tensor | None = None,
                         row_begin: int = 0, row_end: int | None = None) -> None:
    """Launch ``dwa_weighted_gather`` into caller-owned ``out`` [M, d] f32 (no allocation)."""
    M, k = vals.shape
    d = out.shape[1]
    if row_end is None:
        row_end = row_begin + values.shape[0]
    lib = _lib.load()
    with torch.cuda.device(vals.device):
        st = lib.dwa_weighted_gather(
            vals.data_ptr(), gidx.data_ptr(), M, k, values.data_ptr(), int(row_begin),
            int(row_end), values.stride(0), d, out.data_ptr(),
            alpha_out.data_ptr() if alpha_out is not None else None, _stream_handle(vals.device))
    _lib.check(st, "dwa_weighted_gather")


def weighted_value_sum(top_vals: torch.Tensor, top_idx: torch.Tensor, values: torch.Tensor,
                       row_begin: int = 0, return_alpha: bool = True
                       ) -> tuple[torch.Tensor, torch.Tensor | None]:
    """out[m] = sum_j alpha[m, j] * values[top_idx[m, j] - row_begin] over owned rows.

    top_vals f32 [M, k] (fused scores), top_idx i32 [M, k] (global rows),
    values bf16 [rows, d] holding global rows [row_begin, row_begin + rows).
    Returns (out f32 [M, d], alpha f32 [M, k] or None).
    """
    values = _check_values(values)
    if top_vals.shape != top_idx.shape or top_vals.dim() != 2:
        raise ValueError("top_vals and top_idx must both be [M, k]")
    top_vals = top_vals.to(torch.float32).contiguous()
    top_idx = top_idx.to(torch.int32).contiguous()
    M, k = top_vals.shape
    d = values.shape[1]
    dev = top_vals.device
    out = torch.empty((M, d), dtype=torch.float32, device=dev)
    alpha = torch.empty((M, k), dtype=torch.float32, device=dev) if return_alpha else None
    weighted_gather_into(top_vals, top_idx, values, out, alpha, row_begin,
                         row_begin + values.shape[0])
    return out, alpha


def normalise_alpha(top_vals: torch.Tensor, out: torch.Tensor | None = None,
                    idx: torch.Tensor | None = None) -> torch.Tensor:
    """alpha = top_vals / (sum(top_vals) + 1e-8) over the last axis (reference retrieval.py:326),
    computed by the gather kernel with an empty owned row range (no value rows read).
    ``idx`` (i32 [M, k], e.g. the top-k indices) fills the kernel's index operand; it
    is not read for values."""
    if top_vals.dim() != 2:
        raise ValueError("top_vals must be [M, k]")
    top_vals = top_vals.to(torch.float32).contiguous()
    M, k = top_vals.shape
    if out is None:
        out = torch.empty((M, k), dtype=torch.float32, device=top_vals.device)
    if idx is None or idx.shape != top_vals.shape or idx.dtype != torch.int32:
        idx = torch.zeros((M, k), dtype=torch.int32, device=top_vals.device)
    lib = _lib.load()
    with torch.cuda.device(top_vals.device):
        st = lib.dwa_weighted_gather(top_vals.data_ptr(), idx.contiguous().data_ptr(), M, k, None, 0,
                                     0, 8, 8, None, out.data_ptr(), _stream_handle(top_vals.device))
    _lib.check(st, "dwa_weighted_gather")
    return out
