"""GPU parity at the per-GPU shard shapes of the LM configurations.

The headline scaling numbers run the fused score + top-k on one GPU's shard of
a row-sharded pool:
  * 1B-scale LM: 16384 queries x 524,288 keys (4,194,304 / 8) x d 2048, k = 64
  * 7B-scale LM: 16384 queries x 2,097,152 keys (16,777,216 / 8) x d 4096, k = 128
    (queries of 128 MiB: the kernel runs its query-tile-grouped unit order)
Both run here at full size.  Every row is checked by size-independent
properties (sorted, in range, no duplicates, each returned score equal to the
recomputed score of its index); 32 sampled rows are checked against an exact
top-k over the whole shard (fp64 scores on the GPU, the oracle's top_k on the
host) with the parity comparator: values rank-wise within RTOL and index sets
equal up to near-ties of the k-th value (tiled_topk.py:160-176 semantics).
"""
import numpy as np
import pytest
import torch

from oracle import dwa_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-2


@pytest.fixture(scope="module")
def cb():
    import computd_b200

    computd_b200.load_library()
    return computd_b200


def _exact_scores(q_rows: torch.Tensor, keys: torch.Tensor, chunk: int = 1 << 16) -> np.ndarray:
    """fp64 q_rows . keys^T over the whole shard, on the GPU in key chunks."""
    out = torch.empty((q_rows.shape[0], keys.shape[0]), dtype=torch.float64, device=keys.device)
    qd = q_rows.double()
    for c0 in range(0, keys.shape[0], chunk):
        out[:, c0:c0 + chunk] = qd @ keys[c0:c0 + chunk].double().T
    return out.cpu().numpy()


def _check_shard(cb, M, N, d, k, lam, tau, T, sig, n_rows=32):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q = cb.new_normal(M, d, seed=M + 7, stddev=1.0, device=dev)
    keys = cb.new_normal(N, d, seed=N + 9, stddev=d ** -0.5, device=dev)
    tv, ti = cb.tiled_topk_fused(q, keys, k, lam, tau, T, sig)
    torch.cuda.synchronize()
    # every row: sorted, in range, distinct indices
    assert bool((tv[:, 1:] <= tv[:, :-1]).all())
    assert int(ti.min()) >= 0 and int(ti.max()) < N
    s_idx, _ = torch.sort(ti, dim=1)
    assert not bool((s_idx[:, 1:] == s_idx[:, :-1]).any())
    # every row: each returned value is the fused score of its index (fp32 recompute)
    for r0 in range(0, M, 1024):
        qi = q[r0:r0 + 1024].float()
        s_true = torch.einsum("md,mkd->mk", qi, keys[ti[r0:r0 + 1024].long()].float())
        v_true = torch.exp(s_true / T)
        if sig:
            v_true = v_true * torch.sigmoid(lam * (s_true - tau))
        torch.testing.assert_close(tv[r0:r0 + 1024], v_true, rtol=1e-4, atol=0)
    # sampled rows (spread over every query tile group): exact top-k over the whole shard
    rows = torch.linspace(0, M - 1, n_rows, device=dev).round().long()
    s = _exact_scores(q[rows], keys)
    rv, ri = O.top_k(O.fused_score(s, lam, tau, T, sig), k)
    errs = O.compare_topk_from_scores(tv[rows].cpu().numpy(), ti[rows].cpu().numpy(), rv, ri, s,
                                      lam, tau, T, sig, rtol=RTOL)
    assert errs == [], errs


def test_lm1b_shard_vs_exact_rows(cb):
    """One GPU's shard of the 1B-scale LM's pool: 16384 x 524,288 x 2048, k = 64."""
    _check_shard(cb, 16384, 524288, 2048, 64, 1.0, 0.0, 1.0, False)


def test_lm7b_shard_vs_exact_rows(cb):
    """One GPU's shard of the 16M-entry pool: 16384 x 2,097,152 x 4096, k = 128
    (query-tile-grouped unit order), with the sigmoid gate on."""
    _check_shard(cb, 16384, 2097152, 4096, 128, 2.0, 0.1, 1.0, True)
