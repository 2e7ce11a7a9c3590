"""GPU: the LM block's fused elementwise kernels (include/dwa_lm.h) against
the torch tensor operations they replace: RoPE bit for bit (the kernel rounds
every step to bf16 as the elementwise ops do), the packed aspect queries and
the retrieval's device scalars against the fp32 formulas."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


@pytest.mark.parametrize("B,S,H,dh", [(2, 64, 4, 16), (3, 37, 6, 64), (1, 128, 16, 80),
                                      (2, 16, 2, 128)])
def test_rope_qk_matches_tensor_ops(B, S, H, dh):
    from computd_b200.dwa_lm import _rope
    from computd_b200.lm_ops import rope_qk

    dev = _dev()
    g = torch.Generator(device=dev).manual_seed(B * 100 + dh)
    C = H * dh
    qkv = torch.randn((B, S, 3 * C), device=dev, generator=g).to(torch.bfloat16)
    theta = 1.0 / (10000.0 ** (torch.arange(0, dh, 2, device=dev) / dh))
    f = torch.outer(torch.arange(S + 5, device=dev, dtype=torch.float32), theta)
    cos, sin = f.cos().to(torch.bfloat16), f.sin().to(torch.bfloat16)
    q, k = rope_qk(qkv, cos, sin, H, dh)
    torch.cuda.synchronize()
    q_ref = _rope(qkv[..., :C].view(B, S, H, dh).transpose(1, 2), cos[:S], sin[:S])
    k_ref = _rope(qkv[..., C:2 * C].view(B, S, H, dh).transpose(1, 2), cos[:S], sin[:S])
    assert q.shape == (B, H, S, dh) and q.transpose(1, 2).is_contiguous()
    assert torch.equal(q, q_ref) and torch.equal(k, k_ref)


@pytest.mark.parametrize("M,S,d_k,sig", [(100, 8, 64, True), (37, 6, 64, False), (5, 1, 8, True),
                                         (300, 16, 128, True)])
def test_aspect_queries_match_fp32(M, S, d_k, sig):
    from computd_b200.lm_ops import aspect_queries

    dev = _dev()
    g = torch.Generator(device=dev).manual_seed(M + S)
    q_raw = torch.randn((M, S * d_k + 8), device=dev, generator=g).to(torch.bfloat16)[:, :S * d_k]
    q_raw[0, :d_k] = 0  # a zero aspect: scale 1 / 1e-8 times zeros stays zero
    logits = torch.randn(S, device=dev, generator=g)
    tau = torch.randn(S, device=dev, generator=g) * 0.1
    q, w, params = aspect_queries(q_raw, S, d_k, logits, tau, 2.5, 0.7, sig)
    torch.cuda.synchronize()
    w_ref = torch.softmax(logits, dim=0)
    torch.testing.assert_close(w, w_ref, rtol=1e-6, atol=0)
    qf = q_raw.float().view(M, S, d_k)
    want = qf * (w_ref.sqrt()[None, :, None] / (qf.norm(dim=-1, keepdim=True) + 1e-8))
    got = q.float().view(M, S, d_k)
    # one bf16 rounding of an fp32 value that differs from torch's in the last fp32 bits
    assert float((got - want).abs().max()) <= float(want.abs().max()) * 2.0 ** -8
    assert float(got[0, 0].abs().max()) == 0.0
    tau_ref = float(torch.dot(w_ref, tau)) if sig else 0.0
    assert params[0].item() == 2.5 and abs(params[1].item() - tau_ref) <= 1e-6
    assert abs(params[2].item() - 0.7) < 1e-7
