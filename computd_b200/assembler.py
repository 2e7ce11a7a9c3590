"""Low-rank weight assembly on the retrieved pool rows, and the pool-usage EMA.

Host mirror of the reference's ``WeightAssembler`` (src/model/assembly.py:7-128)
for per-position (hybrid) retrieval.  Each pool row holds the blocks
[U (d_B x r) | V (r x d_A) | b (d_B)]; for a token h with retrieved rows j
and weights alpha_j the block output is

    h_mid = LayerNorm(residual + gamma * (h W_base^T + b_base
                                          + sum_j alpha_j (U_j (V_j h) + b_j)))

(assembly.py:104, 110-128), residual = h when d_A == d_B.  The sum never forms
the reference's gathered [.., k, D] tensor.  When rows are selected by two or
more tokens on average it runs row-stationary (``dwa_lowrank_delta_rows``:
each selected row read about once and applied to all its tokens); otherwise
one fused kernel per token streams each selected row (``dwa_lowrank_delta``).
The base GEMM is cuBLAS; residual, gamma and the LayerNorm are one more
kernel (``dwa_assemble_finish``).  On a row-sharded pool each rank sums the rows it
owns and the partial sums are added with one all-reduce before the
LayerNorm.

``usage_ema_update`` is the pool-usage EMA of the training step
(src/training/trainer.py:227-233 with src/model/pool.py:52-55).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .retrieval import _group_rank_world
from .tiled_topk import _stream_handle


def _rows(x: torch.Tensor, name: str) -> tuple[torch.Tensor, int]:
    if x.device.type != "cuda":
        raise ValueError(f"{name} must live on a CUDA device")
    if x.dtype not in (torch.bfloat16, torch.float32):
        x = x.to(torch.float32)
    if x.stride(-1) != 1 or x.data_ptr() % 16 != 0:
        x = x.contiguous()
    return x, 1 if x.dtype == torch.bfloat16 else 0


_ROWS_WORKSPACE: dict[tuple[int, int], torch.Tensor] = {}


def lowrank_rows_workspace(M: int, k: int, n_rows: int, d_B: int,
                           device: torch.device) -> torch.Tensor:
    """The row-stationary path's scratch (``dwa_lowrank_delta_rows_workspace``
    bytes): one buffer per (device, current stream) that grows on demand and is
    shared by the calls on that stream, which the stream orders (the blocks of
    a forward).  Calls on other streams get buffers of their own; a CUDA-graph
    capture allocates its buffer from the graph's pool."""
    need = int(_lib.load().dwa_lowrank_delta_rows_workspace(M, k, n_rows, d_B))
    dev = torch.device(device)
    index = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (index, torch.cuda.current_stream(index).cuda_stream)
    ws = _ROWS_WORKSPACE.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=torch.device("cuda", index))
        _ROWS_WORKSPACE[key] = ws
    return ws


def _rows_path_fits(M: int, k: int, n_rows: int, d_A: int, d_B: int, r: int) -> bool:
    """Row-stationary when rows are selected by >= 4 tokens on average and its
    limits hold (one row's U | V | b in 200 KB of shared memory).  Measured at
    d 1280, r 8, k 16: 8 tokens per row 0.71 vs 1.36 ms for the per-token
    kernel; 2 per row 0.44 vs 0.36 ms; 1 per row 1.65 vs 1.36 ms (the slots'
    write and read cost more than the rows saved)."""
    return (n_rows > 0 and M * k >= 4 * n_rows and M * k <= 2**31 - 1
            and (d_B * r + r * d_A + d_B) * 2 <= 200 * 1024)


def lowrank_delta(h: torch.Tensor, alpha: torch.Tensor, idx: torch.Tensor, vectors: torch.Tensor,
                  d_A: int, d_B: int, r: int, row_begin: int = 0,
                  out: torch.Tensor | None = None, rows: bool | None = None,
                  workspace: torch.Tensor | None = None) -> torch.Tensor:
    """delta[m] = sum_j alpha[m, j] (U_j (V_j h[m]) + b_j) over the pool rows this shard owns.

    h [M, d_A] (bf16 or f32), alpha f32 [M, k], idx i32 [M, k] (global pool rows),
    vectors bf16 [rows, ld] = global rows [row_begin, row_begin + rows).
    ``rows``: True for the row-stationary kernels (``dwa_lowrank_delta_rows``,
    scratch from ``workspace`` or the shared per-device buffer), False for the
    per-token kernel, None to choose by the average number of tokens per row.
    Returns f32 [M, d_B] (``out`` when given).
    """
    h, h_bf16 = _rows(h, "h")
    if h.dim() != 2 or h.shape[1] != d_A:
        raise ValueError(f"h must be [M, {d_A}]")
    M = h.shape[0]
    alpha = alpha.to(torch.float32).contiguous()
    idx = idx.to(torch.int32).contiguous()
    if alpha.shape != idx.shape or alpha.dim() != 2 or alpha.shape[0] != M:
        raise ValueError("alpha and idx must both be [M, k]")
    if vectors.dtype != torch.bfloat16 or vectors.dim() != 2:
        raise ValueError("vectors must be bf16 [rows, D]")
    if vectors.stride(1) != 1 or vectors.stride(0) % 8 != 0 or vectors.data_ptr() % 16 != 0:
        vectors = vectors.contiguous()
    k = alpha.shape[1]
    if out is None:
        out = torch.empty((M, d_B), dtype=torch.float32, device=h.device)
    lib = _lib.load()
    n_rows = vectors.shape[0]
    if rows is None:
        rows = (_rows_path_fits(M, k, n_rows, d_A, d_B, r)
                and h.stride(0) % (8 if h_bf16 else 4) == 0 and out.data_ptr() % 16 == 0)
    with torch.cuda.device(h.device):
        if rows:
            if workspace is None:
                workspace = lowrank_rows_workspace(M, k, n_rows, d_B, h.device)
            st = lib.dwa_lowrank_delta_rows(
                h.data_ptr(), h_bf16, h.stride(0), alpha.data_ptr(), idx.data_ptr(), M, k,
                vectors.data_ptr(), int(row_begin), int(row_begin) + n_rows, vectors.stride(0), d_A,
                d_B, r, out.data_ptr(), workspace.data_ptr(), workspace.numel(),
                _stream_handle(h.device))
            _lib.check(st, "dwa_lowrank_delta_rows")
        else:
            st = lib.dwa_lowrank_delta(h.data_ptr(), h_bf16, h.stride(0), alpha.data_ptr(),
                                       idx.data_ptr(), M, k, vectors.data_ptr(), int(row_begin),
                                       int(row_begin) + n_rows, vectors.stride(0), d_A, d_B, r,
                                       out.data_ptr(), _stream_handle(h.device))
            _lib.check(st, "dwa_lowrank_delta")
    return out


def assemble_finish(delta: torch.Tensor, base: torch.Tensor | None, residual: torch.Tensor | None,
                    gamma: float, ln_scale: torch.Tensor | None, ln_bias: torch.Tensor | None,
                    eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm(residual + gamma * (base + delta)) over the last axis (f32 [M, d_B])."""
    M, d_B = delta.shape
    delta = delta.to(torch.float32).contiguous()
    if base is not None:
        base = base.to(torch.float32).contiguous()
    res_bf16, ldr = 0, 0
    if residual is not None:
        residual, res_bf16 = _rows(residual, "residual")
        ldr = residual.stride(0)
    f32 = lambda t: t.to(torch.float32).contiguous() if t is not None else None
    ln_scale, ln_bias = f32(ln_scale), f32(ln_bias)
    if out is None:
        out = torch.empty((M, d_B), dtype=torch.float32, device=delta.device)
    ptr = lambda t: t.data_ptr() if t is not None else None
    lib = _lib.load()
    with torch.cuda.device(delta.device):
        st = lib.dwa_assemble_finish(ptr(residual), res_bf16, ldr, ptr(base), delta.data_ptr(), M,
                                     d_B, float(gamma), ptr(ln_scale), ptr(ln_bias), float(eps),
                                     out.data_ptr(), _stream_handle(delta.device))
    _lib.check(st, "dwa_assemble_finish")
    return out


def usage_ema_update(ema: torch.Tensor, alpha: torch.Tensor, idx: torch.Tensor, beta: float = 0.99,
                     row_begin: int = 0, n_total: int | None = None) -> torch.Tensor:
    """In place: ema = beta * ema + (1 - beta) * alpha_sum, alpha_sum[g] = sum of
    alpha / n_total over the entries with idx == g (trainer.py:227-233, pool.py:52-55).

    ``ema`` f32 holds global rows [row_begin, row_begin + len); ``n_total`` defaults to
    idx.numel() (the reference divides by all_idx.size)."""
    if ema.dtype != torch.float32 or not ema.is_contiguous():
        raise ValueError("ema must be a contiguous f32 tensor")
    alpha = alpha.to(torch.float32).contiguous()
    idx = idx.to(torch.int32).contiguous()
    n = idx.numel()
    if alpha.numel() != n:
        raise ValueError("alpha and idx must have the same number of entries")
    weight = (1.0 - beta) / float(n_total if n_total is not None else n)
    lib = _lib.load()
    with torch.cuda.device(ema.device):
        st = lib.dwa_usage_ema(alpha.data_ptr(), idx.data_ptr(), n, int(row_begin),
                               int(row_begin) + ema.numel(), weight, float(beta), ema.data_ptr(),
                               _stream_handle(ema.device))
    _lib.check(st, "dwa_usage_ema")
    return ema


class WeightAssembler:
    """The reference's WeightAssembler (assembly.py:7-46) for per-position idx.

    Parameters keep the reference's names: ``W_base`` [d_B, d_A] and ``b_base``
    [d_B] (zero-initialised, as at assembly.py:38-39), ``gamma`` (1.0,
    assembly.py:42) and the LayerNorm ``norm_scale`` / ``norm_bias`` (flax
    LayerNorm defaults: ones / zeros, epsilon 1e-6).
    """

    def __init__(self, d_A: int, d_B: int, r: int, device=None, dtype=torch.bfloat16):
        self.d_A, self.d_B, self.r = int(d_A), int(d_B), int(r)
        self._off_V = self.d_B * self.r
        self._off_b = self._off_V + self.r * self.d_A
        self._end_b = self._off_b + self.d_B
        self.W_base = torch.zeros((self.d_B, self.d_A), dtype=dtype, device=device)
        self.b_base = torch.zeros(self.d_B, dtype=dtype, device=device)
        self.gamma = 1.0
        self.norm_scale = torch.ones(self.d_B, dtype=torch.float32, device=device)
        self.norm_bias = torch.zeros(self.d_B, dtype=torch.float32, device=device)
        self.eps = 1e-6

    def __call__(self, h_A: torch.Tensor, alpha: torch.Tensor, idx: torch.Tensor,
                 vectors: torch.Tensor, group=None) -> torch.Tensor:
        """h_mid (..., d_B) f32 for h_A (..., d_A), alpha / idx (..., k) per position.

        ``vectors`` are this rank's pool rows (the whole pool without ``group``);
        with a row-sharded pool every rank passes the same h_A / alpha / idx and
        gets the same h_mid."""
        if idx is None:
            raise NotImplementedError("soft mode (alpha over the whole pool) is not on this path")
        lead = h_A.shape[:-1]
        if alpha.shape[:-1] != lead or idx.shape != alpha.shape:
            raise ValueError("per-position alpha / idx must be (..., k) over h_A's leading dims")
        rank, world = _group_rank_world(group)
        n_local = vectors.shape[0]
        h = h_A.reshape(-1, self.d_A)
        k = alpha.shape[-1]
        delta = lowrank_delta(h, alpha.reshape(-1, k), idx.reshape(-1, k), vectors, self.d_A,
                              self.d_B, self.r, row_begin=rank * n_local)
        if world > 1:
            dist.all_reduce(delta, group=group)
        return self.finish(h, delta).reshape(*lead, self.d_B)

    def finish(self, h: torch.Tensor, delta: torch.Tensor) -> torch.Tensor:
        """LayerNorm(residual + gamma * (h W_base^T + b_base + delta)) (assembly.py:128)
        for h [M, d_A] and the summed delta f32 [M, d_B] of the retrieved rows
        (h_delta + b_delta; b_delta alone when the pool rows hold only b)."""
        if h.dtype == torch.bfloat16 and self.W_base.dtype == torch.bfloat16:
            # bf16 operands, fp32 result: the tensor-core GEMM (exact products, fp32
            # sums), the f32 bias added in its epilogue
            base = torch.addmm(self.b_base.to(torch.float32), h, self.W_base.t(),
                               out_dtype=torch.float32)
        else:
            base = torch.addmm(self.b_base.to(torch.float32), h.to(torch.float32),
                               self.W_base.to(torch.float32).t())
        residual = h if self.d_A == self.d_B else None
        return assemble_finish(delta, base, residual, self.gamma, self.norm_scale, self.norm_bias,
                               self.eps)
