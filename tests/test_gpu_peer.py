"""NVLink peer exchange primitives on one GPU (through the C ABI): a one-rank
exchange returns its own list, and the merge's wait for a step nobody
signalled ends after the limit the call gives (here 1 s) with DWA_ERR_TIMEOUT
in the status word, -inf / -1 outputs and a context that stays usable.  Multi-rank parity against
the NCCL all-gather path is in test_gpu_multi.py."""
import ctypes
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DWA_ERR_TIMEOUT = 4


@pytest.fixture(scope="module")
def lib():
    import computd_b200
    from computd_b200 import _lib

    computd_b200.load_library()
    return _lib.load()


def test_single_rank_exchange_and_bounded_wait(lib):
    from computd_b200 import _lib
    from computd_b200.retrieval import _DeviceBuffer

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M, k = 40, 16
    hdr, list_bytes = 256, M * k * 8
    own = ctypes.c_void_p()
    handle = (ctypes.c_char * 64)()
    _lib.check(lib.dwa_peer_alloc(hdr + 2 * list_bytes, ctypes.byref(own), handle), "dwa_peer_alloc")
    try:
        base = own.value
        packed = torch.as_tensor(_DeviceBuffer(base + hdr, (M, k, 2), "<i4"), device=dev)
        header = torch.as_tensor(_DeviceBuffer(base, (hdr // 4,), "<i4"), device=dev)
        rng = np.random.default_rng(0)
        vals = -np.sort(-rng.random((M, k)).astype(np.float32), axis=1)
        idx = rng.integers(0, 1 << 20, (M, k)).astype(np.int32)
        packed[..., 0].copy_(torch.from_numpy(vals).to(dev).view(torch.int32))
        packed[..., 1].copy_(torch.from_numpy(idx).to(dev))
        flags = (ctypes.c_void_p * 1)(base)
        lists = (ctypes.c_void_p * 1)(base + hdr)
        out_v = torch.empty((M, k), dtype=torch.float32, device=dev)
        out_i = torch.empty((M, k), dtype=torch.int32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.dwa_peer_signal(flags, 1, 0, 1, stream), "dwa_peer_signal")
        _lib.check(lib.dwa_merge_topk_peers(lists, 1, M, k, base, 1, 0, out_v.data_ptr(),
                                            out_i.data_ptr(), base + 192, stream), "merge")
        torch.cuda.synchronize()
        assert int(header[0].item()) == 1
        assert int(header[48].item()) == 0
        np.testing.assert_array_equal(out_v.cpu().numpy(), vals)
        np.testing.assert_array_equal(out_i.cpu().numpy(), idx)
        # step 2 was never signalled: every warp gives up after its bounded wait
        t0 = time.time()
        _lib.check(lib.dwa_merge_topk_peers(lists, 1, M, k, base, 2, 1_000_000_000,
                                            out_v.data_ptr(), out_i.data_ptr(), base + 192, stream),
                   "merge")
        torch.cuda.synchronize()
        waited = time.time() - t0
        assert int(header[48].item()) == DWA_ERR_TIMEOUT
        assert 0.9 < waited < 20.0
        assert bool((out_i == -1).all()) and bool(torch.isneginf(out_v).all())
        # the context is still usable
        x = torch.arange(1000, device=dev, dtype=torch.float32)
        assert float(x.sum().item()) == 499500.0
    finally:
        lib.dwa_peer_free(own.value)


def test_peer_exchange_timeout_raises_until_resync(lib, tmp_path):
    """PeerExchange in a one-rank NCCL group: a merge whose step nobody signals
    runs out of its (1 s) wait; the next check raises DWAError, keeps raising,
    and resync() makes the exchange usable again with correct results."""
    import torch.distributed as dist

    from computd_b200 import DWAError
    from computd_b200.retrieval import PeerExchange

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"file://{tmp_path}/pg", rank=0, world_size=1,
                            device_id=dev)
    try:
        M, k = 64, 16
        rng = np.random.default_rng(1)
        vals = torch.from_numpy(-np.sort(-rng.random((M, k)).astype(np.float32), axis=1)).to(dev)
        idx = torch.from_numpy(rng.integers(0, 1 << 20, (M, k)).astype(np.int32)).to(dev)
        ex = PeerExchange(M, k, None, dev, wait_s=1.0)
        ov = torch.empty((M, k), dtype=torch.float32, device=dev)
        oi = torch.empty((M, k), dtype=torch.int32, device=dev)
        ex.publish(vals, idx)
        ex.merge(ov, oi)
        ex.check()
        assert torch.equal(oi, idx) and torch.equal(ov, vals)
        ex.step += 1          # a step nobody publishes
        t0 = time.time()
        ex.merge(ov, oi)
        with pytest.raises(DWAError, match="did not arrive"):
            ex.check()
        assert time.time() - t0 > 0.9
        assert bool((oi == -1).all())
        with pytest.raises(DWAError, match="resync"):
            ex.check()
        ex.resync()
        assert ex.status() == 0
        ex.publish(vals, idx)
        ex.merge(ov, oi)
        ex.check()
        assert torch.equal(oi, idx) and torch.equal(ov, vals)
        ex.close()
    finally:
        dist.destroy_process_group()
