"""Differentiable retrieval: forward and backward on the B200 kernels.

The reference trains through its plain-jnp retrieval because the Pallas
kernel has no VJP (src/model/retrieval.py:268-271).  ``retrieve`` is the
same op as ``Retriever`` (top-k of gate(s) * exp(s / T), alpha normalisation,
alpha-weighted sum of the gathered value rows) with a backward pass.  The
selected indices are constants of the backward, exactly as for
``jax.lax.top_k``; gradients flow to the queries, the key and value rows that
were selected, and lambda_sharp / tau / T when they are tensors that require
grad.  On a row-sharded pool (``group``) each rank computes the partial
products of the rows it owns, partial sums are all-reduced, and each rank's
key/value gradients cover its own rows only.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .assembly import _check_values, weighted_gather_into
from .retrieval import _group_rank_world, chip_topk, reduce_partials
from .tiled_topk import _as_bf16_rows, _stream_handle


def _f(x):
    return float(x.detach().reshape(()).item()) if isinstance(x, torch.Tensor) else float(x)


def _vec_args(a: torch.Tensor):
    if a.dtype == torch.bfloat16:
        return a.data_ptr(), 1, a.stride(0)
    if a.dtype != torch.float32:
        raise TypeError("row vectors must be float32 or bfloat16")
    return a.data_ptr(), 0, a.stride(0)


def gather_dot(a: torch.Tensor, idx: torch.Tensor, rows: torch.Tensor, row_begin: int) -> torch.Tensor:
    """out[m, j] = <a[m], rows[idx[m, j] - row_begin]> over owned rows (else 0)."""
    M, k = idx.shape
    out = torch.empty((M, k), dtype=torch.float32, device=a.device)
    pa, abf, lda = _vec_args(a)
    lib = _lib.load()
    with torch.cuda.device(a.device):
        st = lib.dwa_gather_dot(pa, abf, lda, idx.data_ptr(), M, k, rows.data_ptr(), row_begin,
                                row_begin + rows.shape[0], rows.stride(0), rows.shape[1],
                                out.data_ptr(), _stream_handle(a.device))
    _lib.check(st, "dwa_gather_dot")
    return out


def _row_gradient(w: torch.Tensor, idx: torch.Tensor, a: torch.Tensor, row_begin: int, n_rows: int,
                  d: int, dtype: torch.dtype, stream) -> torch.Tensor:
    """grad [n_rows, d] of the owned rows: sum of w[m, j] a[m] over the entries
    that selected each row, zero elsewhere (dwa_row_gradient), bf16 or f32."""
    M, k = idx.shape
    dev = a.device
    out_dtype = dtype if dtype in (torch.bfloat16, torch.float32) else torch.float32
    grad = torch.empty((n_rows, d), dtype=out_dtype, device=dev)
    lib = _lib.load()
    ws = torch.empty(max(int(lib.dwa_row_gradient_workspace(M, k, n_rows)), 256), dtype=torch.uint8,
                     device=dev)
    pa, abf, lda = _vec_args(a)
    with torch.cuda.device(dev):
        st = lib.dwa_row_gradient(w.data_ptr(), idx.data_ptr(), M, k, pa, abf, lda, row_begin,
                                  row_begin + n_rows, grad.data_ptr(),
                                  1 if out_dtype == torch.bfloat16 else 0, grad.stride(0), d,
                                  ws.data_ptr(), ws.numel(), stream)
    _lib.check(st, "dwa_row_gradient")
    return grad.to(dtype)


class _RetrievalFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, queries, keys, values, lam, tau, T, k, use_sigmoid, group):
        rank, world = _group_rank_world(group)
        q = _as_bf16_rows(queries.detach(), "queries")
        kk = _as_bf16_rows(keys.detach(), "keys")
        vv = _check_values(values.detach())
        n_local = kk.shape[0]
        row_begin = rank * n_local
        tv, ti = chip_topk(q, kk, k, _f(lam), _f(tau), _f(T), use_sigmoid, group=group)
        M = q.shape[0]
        out = torch.empty((M, vv.shape[1]), dtype=torch.float32, device=q.device)
        alpha = torch.empty((M, k), dtype=torch.float32, device=q.device)
        weighted_gather_into(tv, ti, vv, out, alpha, row_begin, row_begin + n_local)
        reduce_partials(out, group)
        ctx.save_for_backward(q, kk, vv, tv, ti, alpha)
        ctx.params = (_f(lam), _f(tau), _f(T), bool(use_sigmoid), row_begin, group)
        ctx.param_tensors = tuple(isinstance(x, torch.Tensor) for x in (lam, tau, T))
        ctx.in_dtypes = (queries.dtype, keys.dtype, values.dtype)
        ctx.mark_non_differentiable(ti)
        return out, tv, ti

    @staticmethod
    def backward(ctx, dout, _dtv, _dti):
        q, kk, vv, tv, ti, alpha = ctx.saved_tensors
        lam, tau, T, use_sigmoid, row_begin, group = ctx.params
        _, world = _group_rank_world(group)
        lib = _lib.load()
        dev = q.device
        sh = _stream_handle(dev)
        M, k = ti.shape
        d_k, d_v = kk.shape[1], vv.shape[1]
        dout = dout.to(torch.float32).contiguous()
        ds = torch.empty((M, k), dtype=torch.float32, device=dev)
        dparams = torch.zeros(3, dtype=torch.float32, device=dev)
        dq = grad_k = grad_v = None
        if world == 1 and k <= 128:
            # the whole pool here: s, dalpha, ds and dq in one launch, each
            # selected row read once (dwa_retrieval_backward)
            dq = torch.empty((M, d_k), dtype=torch.float32, device=dev)
            pq, qbf, ldq = _vec_args(q)
            with torch.cuda.device(dev):
                st = lib.dwa_retrieval_backward(
                    pq, qbf, ldq, dout.data_ptr(), dout.stride(0), kk.data_ptr(), kk.stride(0),
                    d_k, vv.data_ptr(), vv.stride(0), d_v, tv.data_ptr(), ti.data_ptr(), M, k,
                    row_begin, row_begin + kk.shape[0], lam, tau, T, None, int(use_sigmoid),
                    ds.data_ptr(), dq.data_ptr(), dparams.data_ptr(), None, sh)
            _lib.check(st, "dwa_retrieval_backward")
            if not ctx.needs_input_grad[0]:
                dq = None
        else:
            # dalpha = <dout, V[idx]>, s = <q, K[idx]>: owned partial dots, summed over ranks
            dalpha = gather_dot(dout, ti, vv, row_begin)
            s = gather_dot(q, ti, kk, row_begin)
            if world > 1:
                dist.all_reduce(dalpha, group=group)
                dist.all_reduce(s, group=group)
            with torch.cuda.device(dev):
                st = lib.dwa_score_backward(tv.data_ptr(), s.data_ptr(), dalpha.data_ptr(), M, k,
                                            lam, tau, T, int(use_sigmoid), ds.data_ptr(),
                                            dparams.data_ptr(), sh)
                _lib.check(st, "dwa_score_backward")
                if ctx.needs_input_grad[0]:
                    dq = torch.empty((M, d_k), dtype=torch.float32, device=dev)
                    st = lib.dwa_gather_rows(ds.data_ptr(), ti.data_ptr(), M, k, kk.data_ptr(),
                                             row_begin, row_begin + kk.shape[0], kk.stride(0), d_k,
                                             dq.data_ptr(), 0, sh)
                    _lib.check(st, "dwa_gather_rows")
        qd, kd, vd = ctx.in_dtypes
        # dK[r] = sum ds q over the entries that selected row r, dV[r] = sum alpha dout:
        # the whole owned gradient written once, in the parameter's dtype
        if ctx.needs_input_grad[1]:
            grad_k = _row_gradient(ds, ti, q, row_begin, kk.shape[0], d_k, kd, sh)
        if ctx.needs_input_grad[2]:
            grad_v = _row_gradient(alpha, ti, dout, row_begin, vv.shape[0], d_v, vd, sh)
        if dq is not None and world > 1:
            dist.all_reduce(dq, group=group)
        grads_p = [dparams[i].clone() if ctx.param_tensors[i] and ctx.needs_input_grad[3 + i] else None
                   for i in range(3)]
        return (dq.to(qd) if dq is not None else None,
                grad_k.to(kd) if grad_k is not None else None,
                grad_v.to(vd) if grad_v is not None else None,
                grads_p[0], grads_p[1], grads_p[2], None, None, None)


def retrieve(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, k_max: int,
             lambda_sharp=1.0, tau=0.0, T=1.0, use_sigmoid: bool = False, group=None):
    """Differentiable retrieval over a (possibly row-sharded) pool.

    Returns (out f32 [M, d_v], top_vals f32 [M, k], top_idx i32 [M, k]); ``out``
    carries gradients to queries, keys, values and tensor-valued
    lambda_sharp / tau / T.
    """
    return _RetrievalFn.apply(queries, keys, values, lambda_sharp, tau, T, int(k_max),
                              bool(use_sigmoid), group)
