"""The DWA LM block's fused elementwise steps on this library's kernels
(include/dwa_lm.h): the rotary embedding of the attention's queries and keys
(reference src/model/parts.py:17-25) and the packed aspect queries with the
retrieval's device scalars (src/model/retrieval.py:159-168)."""
from __future__ import annotations

import torch

from . import _lib
from .tiled_topk import _stream_handle


def rope_qk(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_heads: int,
            head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotary embedding of the q and k parts of the QKV projection.

    ``qkv`` bf16 [B, S, W] with rows of uniform stride (q in columns
    [0, H dh), k in [H dh, 2 H dh)); ``cos`` / ``sin`` bf16 [>= S, dh / 2].
    Returns q, k bf16 [B, H, S, dh] with
    [x1 cos - x2 sin, x1 sin + x2 cos] for x1 = x[..., 0::2], x2 = x[..., 1::2],
    every step rounded to bf16 as the elementwise bf16 tensor ops round it; both
    are (1, 2)-transposed views of token-major [B, S, H, dh] buffers, the layout
    attention then also writes its output in."""
    if qkv.dtype != torch.bfloat16 or qkv.dim() != 3 or not qkv.is_cuda:
        raise ValueError("qkv must be a bf16 [B, S, W] CUDA tensor")
    B, S, W = qkv.shape
    H, dh = int(n_heads), int(head_dim)
    if qkv.stride(2) != 1 or (B > 1 and qkv.stride(0) != S * qkv.stride(1)):
        raise ValueError("qkv rows must be contiguous with one row stride")
    if W < 2 * H * dh:
        raise ValueError(f"qkv has {W} columns, q and k need {2 * H * dh}")
    for t in (cos, sin):
        if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1 or t.shape[0] < S \
                or t.shape[1] < dh // 2 or t.device != qkv.device:
            raise ValueError("cos / sin must be bf16 [>= S, dh / 2] on the qkv device")
    if cos.stride(0) != sin.stride(0):
        raise ValueError("cos and sin must share a row stride")
    q = torch.empty((B, S, H, dh), dtype=torch.bfloat16, device=qkv.device)
    k = torch.empty_like(q)
    lib = _lib.load()
    with torch.cuda.device(qkv.device):
        st = lib.dwa_lm_rope_qk(qkv.data_ptr(), B, S, H, dh, qkv.stride(1), cos.data_ptr(),
                                sin.data_ptr(), cos.stride(0), q.data_ptr(), k.data_ptr(),
                                _stream_handle(qkv.device))
    _lib.check(st, "dwa_lm_rope_qk")
    return q.transpose(1, 2), k.transpose(1, 2)


def aspect_queries(q_raw: torch.Tensor, S: int, d_k: int, aspect_logits: torch.Tensor,
                   tau_param: torch.Tensor | None, lambda_sharp: float, T: float,
                   use_sigmoid: bool, params_out: torch.Tensor | None = None
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Packed aspect queries [sqrt(w_s) q_s / (|q_s| + 1e-8)]_s (bf16 [M, S d_k]) from the
    per-aspect projections ``q_raw`` (bf16 [M, >= S d_k]), w = softmax(aspect_logits).

    Returns (queries, w f32 [S], params f32 [3] = {lambda_sharp, w . tau_param or 0, T},
    the device scalars of the fused score); ``params_out`` receives the params when
    given.  One kernel, nothing read back to the host."""
    if q_raw.dtype != torch.bfloat16 or q_raw.dim() != 2 or q_raw.stride(1) != 1 or not q_raw.is_cuda:
        raise ValueError("q_raw must be a bf16 [M, S d_k] CUDA tensor with contiguous rows")
    S, d_k = int(S), int(d_k)
    M = q_raw.shape[0]
    if q_raw.shape[1] < S * d_k:
        raise ValueError(f"q_raw has {q_raw.shape[1]} columns, S d_k = {S * d_k}")
    dev = q_raw.device
    logits = aspect_logits.to(device=dev, dtype=torch.float32).contiguous()
    if logits.numel() != S:
        raise ValueError(f"aspect_logits must have {S} entries")
    tau = None
    if use_sigmoid:
        if tau_param is None:
            raise ValueError("the gate needs tau_param")
        tau = tau_param.to(device=dev, dtype=torch.float32).contiguous()
        if tau.numel() != S:
            raise ValueError(f"tau_param must have {S} entries")
    out = torch.empty((M, S * d_k), dtype=torch.bfloat16, device=dev)
    w = torch.empty(S, dtype=torch.float32, device=dev)
    params = params_out if params_out is not None else torch.empty(3, dtype=torch.float32,
                                                                   device=dev)
    if params.dtype != torch.float32 or params.numel() != 3 or not params.is_contiguous():
        raise ValueError("params_out must be a contiguous f32 tensor of 3 entries")
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = lib.dwa_lm_aspect_queries(q_raw.data_ptr(), M, S, d_k, q_raw.stride(0),
                                       logits.data_ptr(), tau.data_ptr() if tau is not None else None,
                                       float(lambda_sharp), float(T), 1 if use_sigmoid else 0,
                                       out.data_ptr(), out.stride(0), w.data_ptr(),
                                       params.data_ptr(), _stream_handle(dev))
    _lib.check(st, "dwa_lm_aspect_queries")
    return out, w, params
