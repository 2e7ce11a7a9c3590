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
