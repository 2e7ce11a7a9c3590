"""GPU parity of the low-rank assembly consumer and the pool-usage EMA
(dwa_lowrank_delta, dwa_assemble_finish, dwa_usage_ema through the C ABI)
against the oracle and against fixtures computed by the reference's own
WeightAssembler.__call__ / VectorPool.update_ema.

Tolerance: bf16 inputs, fp32 accumulation; outputs within rel 1e-2 of the
largest magnitude (the parity contract); the fixtures use bf16-representable
inputs on both sides, so the observed error there is far smaller.
"""
import numpy as np
import pytest
import torch

from oracle import dwa_oracle as O

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


def _bf16(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(O.bf16_bits(x)).view(np.int16)).to(_dev()).view(
        torch.bfloat16)


def _close(got: np.ndarray, want: np.ndarray, rtol=1e-2):
    err = np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64)).max()
    assert err <= rtol * max(np.abs(want).max(), 1e-12), f"max abs err {err} vs max {np.abs(want).max()}"


@pytest.fixture(scope="module")
def lib():
    import computd_b200

    computd_b200.load_library()
    return computd_b200


@pytest.mark.parametrize("name", ["asm_eq", "asm_ne"])
def test_assembler_matches_reference_call(lib, golden, name):
    d_A, d_B, r, D = (int(x) for x in golden[f"{name}/dims"])
    asm = lib.WeightAssembler(d_A, d_B, r, device=_dev())
    asm.W_base = _bf16(golden[f"{name}/W_base"])
    asm.b_base = _bf16(golden[f"{name}/b_base"])
    asm.gamma = float(golden[f"{name}/gamma"])
    asm.norm_scale = torch.from_numpy(golden[f"{name}/ln_scale"]).to(_dev())
    asm.norm_bias = torch.from_numpy(golden[f"{name}/ln_bias"]).to(_dev())
    h = _bf16(O.bits_to_f32(golden[f"{name}/h"]))
    vectors = _bf16(O.bits_to_f32(golden[f"{name}/vectors"]))
    alpha = torch.from_numpy(golden[f"{name}/alpha"]).to(_dev())
    idx = torch.from_numpy(golden[f"{name}/idx"]).to(_dev())
    got = asm(h.reshape(2, -1, d_A), alpha.reshape(2, -1, alpha.shape[-1]),
              idx.reshape(2, -1, idx.shape[-1]), vectors)
    _close(got.reshape(-1, d_B).cpu().numpy(), golden[f"{name}/h_mid"], rtol=1e-4)


@pytest.mark.parametrize("M,N,d_A,d_B,r,k,extra", [
    (300, 2000, 256, 256, 8, 16, 0),     # the 1B configuration's layout at reduced width
    (97, 777, 64, 40, 4, 7, 24),         # d_A != d_B, scalar U path, padded rows
    (64, 500, 128, 128, 3, 5, 8),        # odd rank
    (33, 400, 512, 256, 16, 32, 16),     # r = 16, k = 32
])
@pytest.mark.parametrize("rows", [False, True])   # per-token / row-stationary kernels
def test_lowrank_delta_vs_oracle(lib, M, N, d_A, d_B, r, k, extra, rows):
    rng = np.random.default_rng(M + N + r)
    D = d_B * r + r * d_A + d_B + extra
    vectors = O.bf16_round((rng.standard_normal((N, D)) * 0.2).astype(np.float32))
    h = O.bf16_round(rng.standard_normal((M, d_A)).astype(np.float32))
    alpha = rng.random((M, k)).astype(np.float32)
    idx = np.stack([rng.choice(N, size=k, replace=False) for _ in range(M)]).astype(np.int32)
    got = lib.lowrank_delta(_bf16(h), torch.from_numpy(alpha).to(_dev()),
                            torch.from_numpy(idx).to(_dev()), _bf16(vectors), d_A, d_B, r,
                            rows=rows)
    _close(got.cpu().numpy(), O.lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r))
    # f32 rows of h give the same result
    got32 = lib.lowrank_delta(torch.from_numpy(h).to(_dev()), torch.from_numpy(alpha).to(_dev()),
                              torch.from_numpy(idx).to(_dev()), _bf16(vectors), d_A, d_B, r,
                              rows=rows)
    torch.testing.assert_close(got32, got, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("d_A,d_B", [(128, 96), (256, 128)])
@pytest.mark.parametrize("rows", [False, True])
def test_lowrank_delta_owner_computes_partials_add_up(lib, rows, d_A, d_B):
    rng = np.random.default_rng(7)
    M, N, r, k, P = 120, 900, 8, 12, 3
    D = d_B * r + r * d_A + d_B
    vectors = _bf16((rng.standard_normal((N, D)) * 0.2).astype(np.float32))
    h = _bf16(rng.standard_normal((M, d_A)).astype(np.float32))
    alpha = torch.from_numpy(rng.random((M, k)).astype(np.float32)).to(_dev())
    idx = torch.from_numpy(rng.integers(0, N, (M, k)).astype(np.int32)).to(_dev())
    full = lib.lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r, rows=rows)
    n = N // P
    parts = sum(lib.lowrank_delta(h, alpha, idx, vectors[p * n:(p + 1) * n], d_A, d_B, r,
                                  row_begin=p * n, rows=rows) for p in range(P))
    torch.testing.assert_close(parts, full, rtol=1e-4, atol=1e-4)
    # a shard that owns none of the rows contributes exactly zero
    none = lib.lowrank_delta(h, alpha, idx, vectors[:8], d_A, d_B, r, row_begin=N + 10,
                             rows=rows)
    assert torch.count_nonzero(none) == 0


@pytest.mark.parametrize("d_B", [192, 256])
def test_lowrank_rows_skewed_rows_and_determinism(lib, d_B):
    """Row-stationary path: a few rows selected by every token (their pairs span
    many 32-pair chunks), repeated rows inside a token, the per-token kernel as
    the reference, and two runs bit-identical (no float atomics)."""
    rng = np.random.default_rng(21)
    M, N, d_A, r, k = 700, 3000, 256, 8, 16
    D = d_B * r + r * d_A + d_B
    vectors = _bf16((rng.standard_normal((N, D)) * 0.2).astype(np.float32))
    h = _bf16(rng.standard_normal((M, d_A)).astype(np.float32))
    alpha = torch.from_numpy(rng.random((M, k)).astype(np.float32)).to(_dev())
    idx_np = rng.integers(0, N, (M, k)).astype(np.int32)
    idx_np[:, 0] = 5            # every token selects row 5 ...
    idx_np[:, 1] = 2999         # ... and the last row
    idx_np[::3, 2] = 5          # a third of them select row 5 twice
    idx = torch.from_numpy(idx_np).to(_dev())
    ref = lib.lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r, rows=False)
    a1 = lib.lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r, rows=True)
    a2 = lib.lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r, rows=True)
    torch.testing.assert_close(a1, ref, rtol=1e-4, atol=1e-4)
    assert torch.equal(a1, a2)
    # h as a column slice of a wider activation (row stride 320 > d_A)
    wide = torch.zeros((M, d_A + 64), dtype=torch.bfloat16, device=_dev())
    wide[:, 32:32 + d_A] = h
    a3 = lib.lowrank_delta(wide[:, 32:32 + d_A], alpha, idx, vectors, d_A, d_B, r, rows=True)
    assert torch.equal(a3, a1)


def test_lowrank_rows_reference_1b_layout(lib):
    """The reference's 1B layout (d 1280, r 8, 16,384 pool rows of [U | V | b],
    k 16) at 2048 tokens: the row-stationary path against the per-token kernel
    on all tokens and against the oracle on 48 sampled tokens."""
    rng = np.random.default_rng(5)
    M, N, d, r, k = 2048, 16384, 1280, 8, 16
    D = d * r + r * d + d
    g = torch.Generator(device=_dev()).manual_seed(3)
    vectors = (torch.randn(N, D, device=_dev(), generator=g) * 0.02).to(torch.bfloat16)
    h = torch.randn(M, d, device=_dev(), generator=g).to(torch.bfloat16)
    alpha = torch.softmax(torch.randn(M, k, device=_dev(), generator=g), -1)
    idx = torch.stack([torch.randperm(N, device=_dev(), generator=g)[:k] for _ in range(M)]).to(
        torch.int32)
    ref = lib.lowrank_delta(h, alpha, idx, vectors, d, d, r, rows=False)
    got = lib.lowrank_delta(h, alpha, idx, vectors, d, d, r, rows=True)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)
    rows_m = rng.choice(M, size=48, replace=False)
    sel = torch.from_numpy(rows_m).to(_dev())
    i_s = idx[sel].cpu().numpy()
    uniq, inv = np.unique(i_s, return_inverse=True)
    vec_s = vectors[torch.from_numpy(uniq).to(_dev())].float().cpu().numpy()
    want = O.lowrank_delta(h[sel].float().cpu().numpy(), alpha[sel].cpu().numpy(),
                           inv.reshape(i_s.shape).astype(np.int32), vec_s, d, d, r)
    _close(got[sel].cpu().numpy(), want)


@pytest.mark.parametrize("M,d", [(77, 200), (300, 1280), (33, 128), (9, 2048)])
def test_assemble_finish_vs_oracle(lib, M, d):
    """The generic kernel (d = 200) and the register-resident one (d a multiple
    of 128 up to 2048, 16-byte aligned rows)."""
    rng = np.random.default_rng(11 + d)
    delta = rng.standard_normal((M, d)).astype(np.float32)
    base = rng.standard_normal((M, d)).astype(np.float32)
    res = O.bf16_round(rng.standard_normal((M, d)).astype(np.float32))
    scale = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(d)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(_dev())
    got = lib.assemble_finish(t(delta), t(base), _bf16(res), 0.5, t(scale), t(bias), 1e-6)
    want = O.layer_norm(res + 0.5 * (base + delta), scale, bias, 1e-6)
    _close(got.cpu().numpy(), want, rtol=1e-4)
    got0 = lib.assemble_finish(t(delta), None, None, 1.0, None, None, 1e-6)
    _close(got0.cpu().numpy(), O.layer_norm(delta, 1.0, 0.0, 1e-6), rtol=1e-4)


@pytest.mark.parametrize("name", ["asm_eq", "asm_ne"])
def test_usage_ema_matches_reference(lib, golden, name):
    ema = torch.from_numpy(golden[f"{name}/ema0"].copy()).to(_dev())
    lib.usage_ema_update(ema, torch.from_numpy(golden[f"{name}/alpha"]).to(_dev()),
                         torch.from_numpy(golden[f"{name}/idx"]).to(_dev()), beta=0.99)
    np.testing.assert_allclose(ema.cpu().numpy(), golden[f"{name}/ema1"], rtol=1e-5, atol=1e-8)


def test_usage_ema_sharded_rows(lib):
    rng = np.random.default_rng(5)
    N, n, P = 1000, 4000, 4
    alpha = rng.random(n).astype(np.float32)
    idx = rng.integers(0, N, n).astype(np.int32)
    ema0 = rng.random(N).astype(np.float32) * 0.01
    want = O.usage_ema(ema0, alpha, idx, 0.9)
    t = lambda a: torch.from_numpy(a).to(_dev())
    shards = []
    for p in range(P):
        e = t(ema0[p * N // P:(p + 1) * N // P].copy())
        lib.usage_ema_update(e, t(alpha), t(idx), beta=0.9, row_begin=p * N // P)
        shards.append(e.cpu().numpy())
    np.testing.assert_allclose(np.concatenate(shards), want, rtol=1e-5, atol=1e-8)
