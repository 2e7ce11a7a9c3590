"""dwa_score_topk_noalloc: the entry point for callers that cannot allocate.

A caller embedded in a framework that already owns the GPU's memory (or a
binding with no way to pass a scratch buffer) cannot give dwa_score_topk a
workspace.  dwa_score_topk_noalloc uses a scratch array built into the
library instead.  These tests call it through the C ABI and check, on two
calls in a row with different queries (the second call finds the first
call's leftovers in the shared scratch), that it returns what the workspace
entry point returns, within the parity tolerance of the other GPU tests.
The file is named to be collected last so that a failure here does not stop
an `-x` run before the other tests.
"""
import numpy as np
import pytest
import torch

from computd_b200 import _lib
from oracle import dwa_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-2


def _call_noalloc(q, keys, k, lam, tau, T, sig, idx_offset=0):
    lib = _lib.load()
    M, d = q.shape
    N = keys.shape[0]
    vals = torch.empty((M, k), dtype=torch.float32, device=q.device)
    idx = torch.empty((M, k), dtype=torch.int32, device=q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    st = lib.dwa_score_topk_noalloc(q.data_ptr(), M, q.stride(0), keys.data_ptr(), N,
                                    keys.stride(0), d, k, lam, tau, T, int(sig), idx_offset,
                                    vals.data_ptr(), idx.data_ptr(), stream)
    _lib.check(st, "dwa_score_topk_noalloc")
    return vals, idx


@pytest.mark.parametrize("M,N,d,k,sig", [(700, 50000, 256, 32, True), (8192, 1 << 20, 1024, 64, False)])
def test_noalloc_matches_workspace_entry_point(M, N, d, k, sig):
    import computd_b200 as cb

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    keys = cb.new_normal(N, d, seed=21, stddev=d ** -0.5, device=dev)
    lam, tau, T = 2.0, 0.1, 1.0
    for call in range(2):
        q = cb.new_normal(M, d, seed=500 + call, stddev=1.0, device=dev)
        v_ref, i_ref = cb.tiled_topk_fused(q, keys, k, lam, tau, T, sig, idx_offset=7)
        v_new, i_new = _call_noalloc(q, keys, k, lam, tau, T, sig, idx_offset=7)
        torch.cuda.synchronize()
        # same kernels on the same inputs: identical indices, values within tolerance
        np.testing.assert_array_equal(i_new.cpu().numpy(), i_ref.cpu().numpy())
        np.testing.assert_allclose(v_new.cpu().numpy(), v_ref.cpu().numpy(), rtol=RTOL)
        if M * N <= 10**8:
            qn, kn = q.float().cpu().numpy(), keys.float().cpu().numpy()
            rv, ri = O.tiled_topk(qn, kn, k, lam, tau, T, sig)
            errs = O.compare_topk(v_new.cpu().numpy(), i_new.cpu().numpy() - 7, rv, ri, qn, kn,
                                  lam, tau, T, sig, rtol=RTOL)
            assert errs == [], errs


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    M, N, d, k = 1 << 17, 1 << 20, 128, 128   # needs ~1 GB of scratch
    need = lib.dwa_score_topk_workspace(M, N, d, k)
    assert need > (128 << 20)
    FAKE = 0x10000  # never dereferenced: the call is refused before any launch
    st = lib.dwa_score_topk_noalloc(FAKE, M, d, FAKE, N, d, d, k, 1.0, 0.0, 1.0, 0, 0, FAKE, FAKE,
                                    None)
    assert st == _lib.DWA_ERR_UNSUPPORTED_SHAPE
    assert b"built-in" in lib.dwa_last_error()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_noalloc_refuses_a_stream_of_another_device():
    """The scratch used is the current device's: a stream of another GPU is
    refused before anything is launched."""
    lib = _lib.load()
    torch.cuda.set_device(0)
    other = torch.cuda.Stream(device=torch.device("cuda", 1))
    FAKE = 0x10000  # never dereferenced: the call is refused before any launch
    st = lib.dwa_score_topk_noalloc(FAKE, 256, 128, FAKE, 4096, 128, 128, 16, 1.0, 0.0, 1.0, 0, 0,
                                    FAKE, FAKE, other.cuda_stream)
    assert st == _lib.DWA_ERR_INVALID_ARG
    assert b"belongs to device 1" in lib.dwa_last_error()
