"""Multi-rank host logic on CPU (gloo, world size 2 and 4).

The device kernels cannot run here, so each rank produces its shard's local
top-k with the oracle (the checker); what is under test is the host side the
GPU path uses unchanged: ShardSpec row ranges and global offsets,
exchange_candidates (all-gather order = shard order), the merge contract on
the gathered [P, M, k] lists, and reduce_partials (owner-computes sums).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from computd_b200.pool import ShardSpec
from computd_b200.retrieval import exchange_candidates, reduce_partials


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    from oracle import dwa_oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(1234)            # same pool on every rank
        M, N, d, k = 37, 240, 16, 9
        q = rng.integers(-3, 4, size=(M, d)).astype(np.float32)
        keys = rng.integers(-3, 4, size=(N, d)).astype(np.float32)
        values = rng.standard_normal((N, d)).astype(np.float32)
        spec = ShardSpec(N, rank, world)
        kl = keys[spec.row_begin:spec.row_end]
        lv, li = O.tiled_topk(q, kl, k, 1.0, 0.0, 8.0, False)
        li = li + spec.row_begin                      # retrieval.py:292-293
        cv, ci = exchange_candidates(torch.from_numpy(lv), torch.from_numpy(li))
        assert cv.shape == (world, M, k)
        fv, fi = O.chip_merge(cv.numpy(), ci.numpy())   # the merge dwa_merge_topk implements
        # owner-computes: each rank sums its own rows, all-reduce adds them
        alpha = O.normalise(fv)
        own = (fi >= spec.row_begin) & (fi < spec.row_end)
        part = np.einsum("mk,mkd->md", np.where(own, alpha, 0.0),
                         values[np.where(own, fi, 0)]).astype(np.float32)
        out = reduce_partials(torch.from_numpy(part)).numpy()
        rv, ri = O.tiled_topk(q, keys, k, 1.0, 0.0, 8.0, False)
        ro = O.weighted_sum(O.normalise(rv), ri, values)
        result_q.put((rank, bool(np.array_equal(fi, ri)), bool(np.allclose(fv, rv)),
                      float(np.abs(out - ro).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_retrieval_host_logic(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, idx_ok, val_ok, err in results:
        assert idx_ok and val_ok, f"rank {rank}: merged top-k differs from the unsharded one"
        assert err < 1e-4, f"rank {rank}: reduced partial sums differ by {err}"


def test_shard_spec():
    s = ShardSpec(1 << 20, 3, 8)
    assert (s.n_local, s.row_begin, s.row_end) == (131072, 393216, 524288)
    with pytest.raises(ValueError):
        ShardSpec(10, 0, 3)
    with pytest.raises(ValueError):
        ShardSpec(8, 4, 4)
