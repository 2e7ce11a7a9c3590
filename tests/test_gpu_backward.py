"""GPU: gradients of the retrieval path against a plain PyTorch fp32
autograd reference with the same (fixed) selected indices.  Tolerance: rel
1e-2 of the gradient's scale (bf16 inputs, fp32 accumulation)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(got, want, rtol=1e-2):
    got, want = got.detach().float(), want.detach().float()
    scale = want.abs().max().clamp_min(1e-12)
    err = (got - want).abs().max()
    assert float(err) <= rtol * float(scale), f"max err {float(err):.3e} vs scale {float(scale):.3e}"


@pytest.mark.parametrize("M,N,d,dv,k,sig", [(64, 3000, 64, 48, 8, True), (200, 9000, 128, 128, 32, False),
                                            (37, 777, 40, 16, 5, True)])
def test_retrieval_gradients(M, N, d, dv, k, sig):
    import computd_b200 as cb
    from computd_b200.autograd import retrieve

    dev = torch.device("cuda", 0)
    torch.manual_seed(M + N)
    q = (torch.randn(M, d, device=dev)).to(torch.bfloat16).requires_grad_()
    K = (torch.randn(N, d, device=dev) * d ** -0.5).to(torch.bfloat16).requires_grad_()
    V = torch.randn(N, dv, device=dev).to(torch.bfloat16).requires_grad_()
    lam = torch.tensor(2.0, device=dev, requires_grad=True)
    tau = torch.tensor(0.3, device=dev, requires_grad=True)
    T = torch.tensor(0.9, device=dev, requires_grad=True)
    W = torch.randn(M, dv, device=dev)
    out, tv, ti = retrieve(q, K, V, k, lam, tau, T, use_sigmoid=sig)
    (out * W).sum().backward()
    torch.cuda.synchronize()

    # fp32 reference on the same selection
    idx = ti.long()
    qf = q.detach().float().requires_grad_()
    Kf = K.detach().float().requires_grad_()
    Vf = V.detach().float().requires_grad_()
    lf = lam.detach().clone().requires_grad_()
    tf = tau.detach().clone().requires_grad_()
    Tf = T.detach().clone().requires_grad_()
    s = (qf[:, None, :] * Kf[idx]).sum(-1)
    v = torch.exp(s / Tf)
    if sig:
        v = torch.sigmoid(lf * (s - tf)) * v
    alpha = v / (v.sum(-1, keepdim=True) + 1e-8)
    ref = (alpha[..., None] * Vf[idx]).sum(1)
    _close(out, ref.detach())
    (ref * W).sum().backward()
    _close(q.grad, qf.grad)
    _close(K.grad, Kf.grad)
    _close(V.grad, Vf.grad)
    _close(T.grad, Tf.grad)
    if sig:
        _close(lam.grad, lf.grad)
        _close(tau.grad, tf.grad)


@pytest.mark.parametrize("M,N,d,dv,k,sig,q_bf16,dev_params",
                         [(300, 5000, 1024, 512, 64, False, True, False),
                          (129, 2000, 128, 64, 100, True, True, True),
                          (33, 700, 40, 24, 7, True, False, False)])
def test_fused_backward_equals_the_four_kernel_path(M, N, d, dv, k, sig, q_bf16, dev_params):
    """dwa_retrieval_backward (one launch, each selected row read once) gives
    the dscores, dq and scalar-parameter sums of dwa_gather_dot x 2 +
    dwa_score_backward + dwa_gather_rows bit for bit (the same sums in the
    same order)."""
    from computd_b200 import _lib
    from computd_b200.tiled_topk import _stream_handle

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + k)
    q = torch.randn(M, d, device=dev, generator=g)
    q = q.to(torch.bfloat16) if q_bf16 else q
    K = (torch.randn(N, d, device=dev, generator=g) * d ** -0.5).to(torch.bfloat16)
    V = torch.randn(N, dv, device=dev, generator=g).to(torch.bfloat16)
    dout = torch.randn(M, dv, device=dev, generator=g)
    idx = torch.stack([torch.randperm(N, device=dev, generator=g)[:k] for _ in range(M)]).to(
        torch.int32)
    v = torch.rand(M, k, device=dev, generator=g) + 0.05   # fused scores of the forward
    lam, tau, T = 3.0, 0.1, 0.7
    sh = _stream_handle(dev)
    qbf = 1 if q_bf16 else 0
    # the four-kernel path
    s = torch.empty(M, k, device=dev)
    dalpha = torch.empty(M, k, device=dev)
    ds_ref = torch.empty(M, k, device=dev)
    dq_ref = torch.empty(M, d, device=dev)
    dp_ref = torch.zeros(3, device=dev)
    assert lib.dwa_gather_dot(dout.data_ptr(), 0, dv, idx.data_ptr(), M, k, V.data_ptr(), 0, N,
                              dv, dv, dalpha.data_ptr(), sh) == 0
    assert lib.dwa_gather_dot(q.data_ptr(), qbf, d, idx.data_ptr(), M, k, K.data_ptr(), 0, N, d, d,
                              s.data_ptr(), sh) == 0
    assert lib.dwa_score_backward(v.data_ptr(), s.data_ptr(), dalpha.data_ptr(), M, k, lam, tau, T,
                                  int(sig), ds_ref.data_ptr(), dp_ref.data_ptr(), sh) == 0
    assert lib.dwa_gather_rows(ds_ref.data_ptr(), idx.data_ptr(), M, k, K.data_ptr(), 0, N, d, d,
                               dq_ref.data_ptr(), 0, sh) == 0
    # one launch
    ds = torch.empty(M, k, device=dev)
    dq = torch.empty(M, d, device=dev)
    dp = torch.zeros(3, device=dev)
    params = torch.tensor([lam, tau, T], device=dev) if dev_params else None
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    assert lib.dwa_retrieval_backward(
        q.data_ptr(), qbf, d, dout.data_ptr(), dv, K.data_ptr(), d, d, V.data_ptr(), dv, dv,
        v.data_ptr(), idx.data_ptr(), M, k, 0, N, lam, tau, T,
        params.data_ptr() if dev_params else None, int(sig), ds.data_ptr(), dq.data_ptr(),
        dp.data_ptr(), status.data_ptr() if dev_params else None, sh) == 0
    torch.cuda.synchronize()
    assert torch.equal(ds, ds_ref)
    assert torch.equal(dq, dq_ref)
    torch.testing.assert_close(dp, dp_ref, rtol=1e-5, atol=1e-6)  # atomics: order varies
    assert int(status.item()) == 0


@pytest.mark.parametrize("out_bf16", [False, True])
def test_row_gradient_equals_zero_fill_and_scatter(out_bf16):
    """dwa_row_gradient (one write of the owned rows) against zero-filled f32 +
    dwa_scatter_add_rows and an fp64 sum: the same sums (their order may differ:
    the atomics' order is not fixed, so both are held to the fp32 summation
    bound (n - 1) 2^-24 sum |w a| of the fp64 value), untouched rows exactly
    zero, an owned sub-range, bf16 output = the f32 result rounded."""
    from computd_b200 import _lib
    from computd_b200.tiled_topk import _stream_handle

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    M, k, N, d = 500, 16, 3000, 96
    a = torch.randn(M, d, device=dev, generator=g).to(torch.bfloat16)
    w = torch.randn(M, k, device=dev, generator=g)
    idx = torch.randint(0, N, (M, k), device=dev, generator=g, dtype=torch.int32)
    idx[:, 0] = 11                         # one row selected by every query
    sh = _stream_handle(dev)
    for rb, re in ((0, N), (1000, 2200)):
        n = re - rb
        ref = torch.zeros(n, d, device=dev)
        assert lib.dwa_scatter_add_rows(w.data_ptr(), idx.data_ptr(), M, k, a.data_ptr(), 1, d, rb,
                                        re, ref.data_ptr(), d, d, sh) == 0
        out = torch.full((n, d), float("nan"), device=dev,
                         dtype=torch.bfloat16 if out_bf16 else torch.float32)
        ws = torch.empty(max(int(lib.dwa_row_gradient_workspace(M, k, n)), 256), dtype=torch.uint8,
                         device=dev)
        assert lib.dwa_row_gradient(w.data_ptr(), idx.data_ptr(), M, k, a.data_ptr(), 1, d, rb, re,
                                    out.data_ptr(), int(out_bf16), d, d, ws.data_ptr(), ws.numel(),
                                    sh) == 0
        torch.cuda.synchronize()
        sel = torch.zeros(n, dtype=torch.bool, device=dev)
        own = (idx >= rb) & (idx < re)
        sel[(idx[own] - rb).long()] = True
        assert bool((out[~sel] == 0).all())       # untouched rows written as zeros
        rows = (idx[own] - rb).long()
        terms = (w[own][:, None].double() * a[own.nonzero()[:, 0]].double())
        ref64 = torch.zeros(n, d, device=dev, dtype=torch.float64).index_add_(0, rows, terms)
        bound = torch.zeros(n, d, device=dev, dtype=torch.float64).index_add_(0, rows, terms.abs())
        tol = (M - 1) * 2.0 ** -24 * bound + 1e-7
        assert bool(((ref.double() - ref64).abs() <= tol).all())   # the scatter reference itself
        if out_bf16:
            assert bool(((out.double() - ref64).abs() <= 2.0 ** -8 * ref64.abs() + tol).all())
        else:
            assert bool(((out.double() - ref64).abs() <= tol).all())
    # no queries: the whole owned gradient is zero
    out = torch.full((N, d), 1.0, device=dev)
    assert lib.dwa_row_gradient(w.data_ptr(), idx.data_ptr(), 0, k, a.data_ptr(), 1, d, 0, N,
                                out.data_ptr(), 0, d, d, None, 0, sh) == 0
    torch.cuda.synchronize()
    assert bool((out == 0).all())
