"""GPU tests of the stream-ordered boundary: the runtime scalars (lambda_sharp,
tau, T) read by the kernels from device memory, as the reference passes them
to its kernel as (1,)-shaped operands (src/kernels/tiled_topk.py:26-29,
112-115), and the sequence-mean auxiliary scores (src/model/retrieval.py:
332-341).

* dwa_score_topk_dev returns exactly what dwa_score_topk returns for the same
  values (same kernels, the scalars only come from elsewhere);
* scalars that fail the checks (T <= 0, a negative lambda with the gate) are
  caught on the device: DWA_ERR_DEVICE_CHECK in the status word, NaN / -1
  outputs, and the next call on the same workspace is clean;
* dwa_score_backward_dev equals dwa_score_backward;
* dwa_seq_scores against an fp64 recomputation (tolerance 1e-5 relative: an
  fp32-accumulated dot product of bf16-exact keys and f32 queries).
"""
import ctypes

import numpy as np
import pytest
import torch

from computd_b200 import _lib
from oracle import dwa_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cb():
    import computd_b200

    computd_b200.load_library()
    return computd_b200


def _dev():
    return torch.device("cuda", 0)


def _ws_status(ws) -> int:
    v = ctypes.c_int32(0)
    st = _lib.load().dwa_workspace_status(ws.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream,
                                          ctypes.byref(v))
    _lib.check(st, "dwa_workspace_status")
    return int(v.value)


@pytest.mark.parametrize("M,N,d,k,sig", [(700, 30000, 256, 32, True), (300, 9000, 1024, 64, False),
                                         (129, 4097, 200, 128, True)])
def test_device_scalars_match_host_scalars(cb, M, N, d, k, sig):
    dev = _dev()
    q = cb.new_normal(M, d, seed=M, stddev=1.0, device=dev)
    keys = cb.new_normal(N, d, seed=N, stddev=d ** -0.5, device=dev)
    lam, tau, T = 2.5, 0.15, 0.8
    v_h, i_h = cb.tiled_topk_fused(q, keys, k, lam, tau, T, sig, idx_offset=11)
    params = torch.tensor([lam, tau, T], dtype=torch.float32, device=dev)
    # tensor scalars route through dwa_score_topk_dev (read on the device)
    v_d, i_d = cb.tiled_topk_fused(q, keys, k, params[0], params[1], params[2], sig, idx_offset=11)
    torch.cuda.synchronize()
    assert torch.equal(i_d, i_h)
    assert torch.equal(v_d, v_h)


@pytest.mark.parametrize("bad", [(1.0, 0.0, 0.0), (1.0, 0.0, float("nan")), (-1.0, 0.0, 1.0),
                                 (1.0, float("inf"), 1.0)])
def test_device_check_catches_bad_scalars(cb, bad):
    dev = _dev()
    M, N, d, k = 300, 5000, 128, 16
    q = cb.new_normal(M, d, seed=1, device=dev)
    keys = cb.new_normal(N, d, seed=2, stddev=d ** -0.5, device=dev)
    ws = torch.empty(cb.workspace_bytes(M, N, d, k, dev), dtype=torch.uint8, device=dev)
    out_v = torch.zeros((M, k), dtype=torch.float32, device=dev)
    out_i = torch.zeros((M, k), dtype=torch.int32, device=dev)
    params = torch.tensor(bad, dtype=torch.float32, device=dev)
    cb.score_topk_into(q, keys, k, 0, 0, 0, True, out_v, out_i, ws, params=params)
    assert _ws_status(ws) == _lib.DWA_ERR_DEVICE_CHECK
    assert bool(torch.isnan(out_v).all()) and bool((out_i == -1).all())
    # the context and the workspace stay usable: a good call comes back clean
    good = torch.tensor([1.0, 0.0, 1.0], dtype=torch.float32, device=dev)
    cb.score_topk_into(q, keys, k, 0, 0, 0, True, out_v, out_i, ws, params=good)
    assert _ws_status(ws) == 0
    qn, kn = q.float().cpu().numpy(), keys.float().cpu().numpy()
    rv, ri = O.tiled_topk(qn, kn, k, 1.0, 0.0, 1.0, True)
    errs = O.compare_topk(out_v.cpu().numpy(), out_i.cpu().numpy(), rv, ri, qn, kn, 1.0, 0.0, 1.0,
                          True)
    assert errs == [], errs


def test_score_backward_dev_matches_host_scalars(cb):
    dev = _dev()
    g = torch.Generator(device=dev).manual_seed(3)
    M, k = 500, 32
    s = torch.randn((M, k), device=dev, generator=g)
    lam, tau, T = 3.0, 0.2, 0.7
    v = torch.sigmoid(lam * (s - tau)) * torch.exp(s / T)
    dalpha = torch.randn((M, k), device=dev, generator=g)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    ds_h = torch.empty_like(s)
    dp_h = torch.zeros(3, device=dev)
    _lib.check(lib.dwa_score_backward(v.data_ptr(), s.data_ptr(), dalpha.data_ptr(), M, k, lam,
                                      tau, T, 1, ds_h.data_ptr(), dp_h.data_ptr(), stream),
               "dwa_score_backward")
    ds_d = torch.empty_like(s)
    dp_d = torch.zeros(3, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    params = torch.tensor([lam, tau, T], dtype=torch.float32, device=dev)
    _lib.check(lib.dwa_score_backward_dev(v.data_ptr(), s.data_ptr(), dalpha.data_ptr(), M, k,
                                          params.data_ptr(), 1, ds_d.data_ptr(), dp_d.data_ptr(),
                                          status.data_ptr(), stream), "dwa_score_backward_dev")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(ds_d, ds_h)
    torch.testing.assert_close(dp_d, dp_h, rtol=1e-5, atol=1e-5)
    # a bad T is caught on the device
    params_bad = torch.tensor([lam, tau, -1.0], dtype=torch.float32, device=dev)
    _lib.check(lib.dwa_score_backward_dev(v.data_ptr(), s.data_ptr(), dalpha.data_ptr(), M, k,
                                          params_bad.data_ptr(), 1, ds_d.data_ptr(), None,
                                          status.data_ptr(), stream), "dwa_score_backward_dev")
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.DWA_ERR_DEVICE_CHECK
    assert bool(torch.isnan(ds_d).all())


@pytest.mark.parametrize("B,N,d,sig", [(1, 1000, 64, True), (3, 5000, 128, False),
                                       (4, 70000, 384, True), (5, 3001, 1024, True),
                                       (9, 20000, 4096, False), (16, 777, 136, True),
                                       (2, 4099, 12800, True), (8, 3000, 4096, True),
                                       (4, 5000, 4096, True), (7, 1500, 1000, True),
                                       (1, 999, 12800, False), (8, 600, 12800, True)])
def test_seq_scores_vs_fp64(cb, B, N, d, sig):
    """sims = q . keys^T and v(sims) for the per-sequence mean queries
    (retrieval.py:332-341), every entry, against fp64."""
    dev = _dev()
    g = torch.Generator(device=dev).manual_seed(B * 1000 + d)
    q = torch.randn((B, d), device=dev, generator=g) * d ** -0.5
    keys = cb.new_normal(N, d, seed=N + d, stddev=d ** -0.5, device=dev)
    lam, tau, T = 4.0, 0.05, 0.9
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    sims, fused = cb.seq_scores(q, keys, lam, tau, T, sig, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want = (q.double() @ keys.double().T).cpu().numpy()
    got = sims.cpu().numpy()
    scale = np.abs(q.double().cpu().numpy()) @ np.abs(keys.double().cpu().numpy()).T
    assert np.all(np.abs(got - want) <= 1e-5 * scale + 1e-7), float(np.max(np.abs(got - want)))
    fw = O.fused_score(want, lam, tau, T, sig)
    np.testing.assert_allclose(fused.cpu().numpy(), fw, rtol=1e-5, atol=1e-7)


def test_seq_scores_strided_and_device_check(cb):
    dev = _dev()
    B, N, d = 6, 2000, 256
    q_big = torch.randn((B, d + 40), device=dev)
    kb = cb.new_normal(N, d + 64, seed=5, stddev=0.1, device=dev)
    q, keys = q_big[:, :d], kb[:, :d]
    sims = torch.full((B, N + 8), -7.0, device=dev)
    fused = torch.full((B, N + 8), -7.0, device=dev)
    cb.seq_scores(q, keys, 1.0, 0.0, 1.0, False, sims=sims[:, :N], fused=fused[:, :N])
    want = (q.double() @ keys.double().T).float()
    torch.testing.assert_close(sims[:, :N], want, rtol=1e-5, atol=1e-5)
    assert bool((sims[:, N:] == -7.0).all()) and bool((fused[:, N:] == -7.0).all())
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    cb.seq_scores(q, keys, 1.0, 0.0, 0.0, True, sims=sims[:, :N], fused=fused[:, :N],
                  status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.DWA_ERR_DEVICE_CHECK
    assert bool(torch.isnan(fused[:, :N]).all())
