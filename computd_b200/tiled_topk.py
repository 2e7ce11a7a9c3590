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
signature compatibility and ignored: the B200 kernel has fixed 256 x 256
tiles (a CTA pair of 128 query rows each against 256 keys).  There is no CPU or PyTorch fallback; invalid arguments raise
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


def score_params(lambda_sharp, tau, T, device) -> torch.Tensor:
    """Device array {lambda_sharp, tau, T} (f32 [3]) for the entry points that read
    the runtime scalars on the device (``dwa_score_topk_dev``, ``dwa_seq_scores``,
    ``dwa_score_backward_dev``).  Tensor arguments stay on the device and Python
    numbers are written by a fill kernel, so building it never waits for the GPU
    (the reference's (1,)-operand convention, tiled_topk.py:26-29, 112-115)."""
    parts = []
    for v in (lambda_sharp, tau, T):
        if isinstance(v, torch.Tensor):
            parts.append(v.detach().to(device=device, dtype=torch.float32).reshape(()))
        else:
            parts.append(torch.full((), float(v), dtype=torch.float32, device=device))
    return torch.stack(parts)


def _any_tensor(*xs) -> bool:
    return any(isinstance(x, torch.Tensor) for x in xs)


def workspace_bytes(M: int, N_local: int, d: int, k: int, device=None) -> int:
    """Device workspace ``dwa_score_topk`` needs for this shape on ``device``."""
    lib = _lib.load()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        return int(lib.dwa_score_topk_workspace(M, N_local, d, k))


def score_topk_into(queries: torch.Tensor, keys: torch.Tensor, k_max: int, lambda_sharp, tau, T,
                    use_sigmoid: bool, out_vals: torch.Tensor, out_idx: torch.Tensor,
                    workspace: torch.Tensor, idx_offset: int = 0,
                    params: torch.Tensor | None = None) -> None:
    """Launch ``dwa_score_topk`` into caller-owned outputs and workspace (no allocation).

    With ``params`` (device f32 [3] from ``score_params``) the kernels read
    lambda_sharp, tau and T from it (``dwa_score_topk_dev``) and the scalar
    arguments are ignored: nothing waits for the host."""
    lib = _lib.load()
    M, d = queries.shape
    N = keys.shape[0]
    with torch.cuda.device(queries.device):
        if params is not None:
            st = lib.dwa_score_topk_dev(
                queries.data_ptr(), M, queries.stride(0), keys.data_ptr(), N, keys.stride(0), d,
                int(k_max), params.data_ptr(), int(bool(use_sigmoid)), int(idx_offset),
                out_vals.data_ptr(), out_idx.data_ptr(), workspace.data_ptr(),
                workspace.numel() * workspace.element_size(), _stream_handle(queries.device))
            _lib.check(st, "dwa_score_topk_dev")
            return
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
    ``lambda_sharp``, ``tau`` and ``T`` may be Python numbers or 0-d/(1,) tensors,
    as in the reference; when any is a tensor the kernels read all three from
    the device (no host read of a learned tau).
    """
    del tile_bt, tile_n  # fixed 256 x 256 CTA-pair tiles on B200
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
    params = (score_params(lambda_sharp, tau, T, dev) if _any_tensor(lambda_sharp, tau, T)
              else None)
    score_topk_into(queries, keys, k, lambda_sharp, tau, T, use_sigmoid, out_vals, out_idx,
                    workspace, idx_offset, params=params)
    return out_vals, out_idx


def score_topk_seqmean(queries: torch.Tensor, keys: torch.Tensor, k_max: int, lambda_sharp, tau, T,
                       use_sigmoid: bool, seq: int, *, idx_offset: int = 0,
                       workspace: torch.Tensor | None = None
                       ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused score + top-k plus the per-sequence mean of the fused scores over every key
    (``dwa_score_topk_seqmean``): the queries are ``M / seq`` sequences of ``seq`` rows.

    Returns (top_vals f32 [M, k], top_idx i32 [M, k], fused_mean f32 [M / seq, N]),
    fused_mean[b, n] = mean over the rows t of sequence b of v(q[b seq + t] . keys[n]),
    i.e. hybrid_forward's ``alpha_raw.mean(axis=1)`` (reference retrieval.py:176-181).
    The scalars are read on the device."""
    queries = _as_bf16_rows(queries, "queries")
    keys = _as_bf16_rows(keys, "keys")
    if queries.shape[1] != keys.shape[1] or keys.device != queries.device:
        raise ValueError("queries and keys must have the same width and device")
    M, d = queries.shape
    N = keys.shape[0]
    seq = int(seq)
    if seq < 1 or M % seq:
        raise ValueError(f"seq={seq} must divide the {M} query rows")
    dev = queries.device
    k = int(k_max)
    out_vals = torch.empty((M, k), dtype=torch.float32, device=dev)
    out_idx = torch.empty((M, k), dtype=torch.int32, device=dev)
    fused_mean = torch.empty((M // seq, N), dtype=torch.float32, device=dev)
    if M == 0:
        return out_vals, out_idx, fused_mean
    if workspace is None:
        workspace = torch.empty(max(workspace_bytes(M, N, d, k, dev), 256), dtype=torch.uint8,
                                device=dev)
    params = score_params(lambda_sharp, tau, T, dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.dwa_score_topk_seqmean(
            queries.data_ptr(), M, queries.stride(0), keys.data_ptr(), N, keys.stride(0), d, k,
            params.data_ptr(), int(bool(use_sigmoid)), int(idx_offset), seq, fused_mean.data_ptr(),
            fused_mean.stride(0), out_vals.data_ptr(), out_idx.data_ptr(), workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), _stream_handle(dev))
    _lib.check(st, "dwa_score_topk_seqmean")
    return out_vals, out_idx, fused_mean


def seq_scores(q: torch.Tensor, keys: torch.Tensor, lambda_sharp, tau, T, use_sigmoid: bool,
               sims: torch.Tensor | None = None, fused: torch.Tensor | None = None,
               status: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Sequence-mean auxiliary scores (reference retrieval.py:332-341) on one key shard:
    ``sims = q @ keys.T`` (q f32 [B, d], keys bf16 [N, d], fp32 accumulation) and the
    fused scores ``sigmoid(lambda (sims - tau)) * exp(sims / T)`` (or ``exp(sims / T)``),
    both f32 [B, N], by the HBM-bound ``dwa_seq_scores`` kernel (keys read once
    per 8 query rows).  Scalars may be tensors (read on the device)."""
    keys = _as_bf16_rows(keys, "keys")
    dev = keys.device
    q = q.to(device=dev, dtype=torch.float32)
    if q.dim() != 2 or q.shape[1] != keys.shape[1]:
        raise ValueError(f"q must be [B, {keys.shape[1]}], got {tuple(q.shape)}")
    if q.stride(1) != 1:
        q = q.contiguous()
    B, d = q.shape
    N = keys.shape[0]
    if sims is None:
        sims = torch.empty((B, N), dtype=torch.float32, device=dev)
    if fused is None:
        fused = torch.empty((B, N), dtype=torch.float32, device=dev)
    params = score_params(lambda_sharp, tau, T, dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.dwa_seq_scores(q.data_ptr(), B, q.stride(0), keys.data_ptr(), N, keys.stride(0), d,
                                params.data_ptr(), int(bool(use_sigmoid)), sims.data_ptr(),
                                sims.stride(0), fused.data_ptr(), fused.stride(0),
                                status.data_ptr() if status is not None else None,
                                _stream_handle(dev))
    _lib.check(st, "dwa_seq_scores")
    return sims, fused


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
    if cand_vals.device.type != "cuda" or cand_idx.device != cand_vals.device:
        raise ValueError("candidate lists must live on one CUDA device")
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
