"""Fused score + top-k over one pool shard, with the reference's call signature.

Mirrors ``src/kernels/tiled_topk.py`` of the reference:

* ``tiled_topk_fused(queries, keys, k_max, lambda_sharp, tau, T, use_sigmoid,
  tile_bt=128, tile_n=128) -> (top_vals f32 [BT, k], top_idx i32 [BT, k])``
  (reference lines 86-153), and
* ``tiled_topk_fallback(...)`` with the same contract minus the tile sizes
  (reference lines 160-176, the path the reference actually executes).

Both run the same sm_100a kernel through the C ABI (``dwa_score_topk``):
``top_vals`` are the fused scores ``sigmoid(lambda (s - tau)) * exp(s / T)``
(or ``exp(s / T)``), sorted descending with lower index first among equal
values, exactly the ``jax.lax.top_k`` contract; ``top_idx`` index the shard's
rows (plus ``idx_offset``).  ``tile_bt``/``tile_n`` are accepted for
signature compatibility and ignored: the B200 kernel has a fixed 128 x 256
tile.  There is no CPU or PyTorch fallback; invalid arguments raise
``DWAArgumentError`` (a ``ValueError``) before anything is launched.
"""
from __future__ import annotations

import torch

from . import _lib


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _as_bf16_rows(x: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if x.device.type != "cuda":
        raise ValueError(f"{name} must live on a CUDA device (got {x.device}); "
                         "the retrieval path has no CPU implementation")
    if x.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(x.shape)}")
    if x.dtype != torch.bfloat16:
        # The kernel computes bf16 x bf16 with fp32 accumulation; other inputs
        # are rounded to bf16 first (round-to-nearest-even).
        x = x.to(torch.bfloat16)
    if x.stride(1) != 1 or x.stride(0) % 8 != 0 or x.data_ptr() % 16 != 0:
        x = x.contiguous()
        if x.shape[1] % 8 != 0:
            raise _lib.DWAArgumentError(_lib.DWA_ERR_UNSUPPORTED_SHAPE, "tiled_topk_fused",
                                        f"{name} width {x.shape[1]} must be a multiple of 8")
    return x


def _scalar(v) -> float:
    if isinstance(v, torch.Tensor):
        return float(v.detach().reshape(()).item())
    return float(v)


def workspace_bytes(M: int, N_local: int, d: int, k: int, device=None) -> int:
    """Device workspace ``dwa_score_topk`` needs for this shape on ``device``."""
    lib = _lib.load()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        return int(lib.dwa_score_topk_workspace(M, N_local, d, k))


def score_topk_into(queries: torch.Tensor, keys: torch.Tensor, k_max: int, lambda_sharp, tau, T,
                    use_sigmoid: bool, out_vals: torch.Tensor, out_idx: torch.Tensor,
                    workspace: torch.Tensor, idx_offset: int = 0) -> None:
    """Launch ``dwa_score_topk`` into caller-owned outputs and workspace (no allocation)."""
    lib = _lib.load()
    M, d = queries.shape
    N = keys.shape[0]
    with torch.cuda.device(queries.device):
        st = lib.dwa_score_topk(
            queries.data_ptr(), M, queries.stride(0), keys.data_ptr(), N, keys.stride(0), d,
            int(k_max), _scalar(lambda_sharp), _scalar(tau), _scalar(T), int(bool(use_sigmoid)),
            int(idx_offset), out_vals.data_ptr(), out_idx.data_ptr(), workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), _stream_handle(queries.device))
    _lib.check(st, "dwa_score_topk")


def tiled_topk_fused(queries: torch.Tensor, keys: torch.Tensor, k_max: int, lambda_sharp, tau, T,
                     use_sigmoid: bool, tile_bt: int = 128, tile_n: int = 128, *,
                     idx_offset: int = 0, workspace: torch.Tensor | None = None
                     ) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused tiled GEMM + gate/exp + top_k on one pool shard (reference tiled_topk.py:86-153).

    queries: [BT, d_k], keys: [N_local, d_k] on the same CUDA device.
    Returns (top_vals f32 [BT, k_max], top_idx i32 [BT, k_max]).
    """
    del tile_bt, tile_n  # fixed 128 x 256 tiles on B200
    queries = _as_bf16_rows(queries, "queries")
    keys = _as_bf16_rows(keys, "keys")
    if keys.device != queries.device:
        raise ValueError("queries and keys must be on the same device")
    if queries.shape[1] != keys.shape[1]:
        raise ValueError(f"d_k mismatch: queries {tuple(queries.shape)} vs keys {tuple(keys.shape)}")
    M, d = queries.shape
    N = keys.shape[0]
    k = int(k_max)
    dev = queries.device
    out_vals = torch.empty((M, k), dtype=torch.float32, device=dev)
    out_idx = torch.empty((M, k), dtype=torch.int32, device=dev)
    if M == 0:
        return out_vals, out_idx
    if workspace is None:
        nbytes = workspace_bytes(M, N, d, k, dev)
        workspace = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    score_topk_into(queries, keys, k, lambda_sharp, tau, T, use_sigmoid, out_vals, out_idx,
                    workspace, idx_offset)
    return out_vals, out_idx


def tiled_topk_fallback(queries: torch.Tensor, keys: torch.Tensor, k_max: int, lambda_sharp, tau, T,
                        use_sigmoid: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Same contract as reference tiled_topk.py:160-176; runs the same B200 kernel."""
    return tiled_topk_fused(queries, keys, k_max, lambda_sharp, tau, T, use_sigmoid)


def merge_topk(cand_vals: torch.Tensor, cand_idx: torch.Tensor, k_max: int | None = None
               ) -> tuple[torch.Tensor, torch.Tensor]:
    """Global top-k of per-shard lists [P, M, k] (reference retrieval.py:299-302)."""
    if cand_vals.dim() != 3 or cand_idx.shape != cand_vals.shape:
        raise ValueError("candidate lists must both be [P, M, k]")
    if cand_vals.dtype != torch.float32 or cand_idx.dtype != torch.int32:
        raise ValueError("candidate lists must be float32 scores and int32 indices")
    P, M, k = cand_vals.shape
    if k_max is not None and int(k_max) != k:
        raise ValueError("k_max must equal the candidate list length")
    cand_vals = cand_vals.contiguous()
    cand_idx = cand_idx.contiguous()
    dev = cand_vals.device
    out_v = torch.empty((M, k), dtype=torch.float32, device=dev)
    out_i = torch.empty((M, k), dtype=torch.int32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.dwa_merge_topk(cand_vals.data_ptr(), cand_idx.data_ptr(), P, M, k,
                                out_v.data_ptr(), out_i.data_ptr(), _stream_handle(dev))
    _lib.check(st, "dwa_merge_topk")
    return out_v, out_i
