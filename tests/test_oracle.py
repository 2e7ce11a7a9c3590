"""CPU tests of the oracle: pinned against fixtures computed by the reference's
own code (tests/golden/make_golden.py), the lax.top_k contract, Philox KATs,
and the comparator's ability to catch planted mistakes."""
import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import dwa_oracle as O


def _case(golden, name):
    k, lam, tau, T, sig = golden[f"{name}/params"]
    return (O.bits_to_f32(golden[f"{name}/q"]), O.bits_to_f32(golden[f"{name}/keys"]), int(k),
            float(lam), float(tau), float(T), bool(sig))


@pytest.mark.parametrize("name", ["c1_exp", "c1_gate", "odd", "ties"])
def test_oracle_matches_reference_tiled_topk(golden, name):
    q, keys, k, lam, tau, T, sig = _case(golden, name)
    # The reference ran jnp.dot in float32 on these bf16-valued inputs.
    v, i = O.tiled_topk(q, keys, k, lam, tau, T, sig, accum=np.float32)
    np.testing.assert_array_equal(i, golden[f"{name}/idx"])
    np.testing.assert_allclose(v, golden[f"{name}/vals"], rtol=1e-6)


def test_oracle_f64_agrees_with_reference_within_tolerance(golden):
    q, keys, k, lam, tau, T, sig = _case(golden, "c1_gate")
    v, i = O.tiled_topk(q, keys, k, lam, tau, T, sig, accum=np.float64)
    errs = O.compare_topk(v, i, golden["c1_gate/vals"], golden["c1_gate/idx"], q, keys, lam, tau, T,
                          sig)
    assert errs == []


def test_ties_put_lower_index_first(golden):
    vals, idx = golden["ties/vals"], golden["ties/idx"]
    for r in range(vals.shape[0]):
        for j in range(vals.shape[1] - 1):
            if vals[r, j] == vals[r, j + 1]:
                assert idx[r, j] < idx[r, j + 1]
    assert (np.diff(vals, axis=1) == 0).any(), "fixture must contain exact ties"


def test_oracle_sharded_path_matches_reference(golden):
    q, keys, k, lam, tau, T, sig = _case(golden, "sharded")
    P = int(golden["sharded/n_chips"])
    n_local = keys.shape[0] // P
    # per-chip lists (retrieval.py:288-291)
    for p in range(P):
        v, i = O.tiled_topk(q, keys[p * n_local:(p + 1) * n_local], k, lam, tau, T, sig,
                            accum=np.float32)
        np.testing.assert_array_equal(i, golden["sharded/local_idx"][p])
        np.testing.assert_allclose(v, golden["sharded/local_vals"][p], rtol=1e-6)
    # merge (retrieval.py:292-302) and alpha (326)
    gi = golden["sharded/local_idx"] + (np.arange(P) * n_local)[:, None, None]
    fv, fi = O.chip_merge(golden["sharded/local_vals"], gi.astype(np.int32))
    np.testing.assert_array_equal(fi, golden["sharded/idx"])
    np.testing.assert_allclose(O.normalise(fv), golden["sharded/alpha"], rtol=1e-6)
    fv2, fi2 = O.sharded_topk(q, keys, k, P, lam, tau, T, sig, accum=np.float32)
    np.testing.assert_array_equal(fi2, golden["sharded/idx"])


def test_oracle_weighted_sum_matches_reference_assembly(golden):
    vectors = O.bits_to_f32(golden["sharded/vectors"])
    b0, b1 = golden["sharded/b_slice"]
    out = O.weighted_sum(golden["sharded/alpha"], golden["sharded/idx"], vectors[:, b0:b1])
    np.testing.assert_allclose(out, golden["sharded/b_delta"], rtol=1e-5, atol=1e-6)


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 6), st.integers(1, 40), st.data())
def test_top_k_contract(M, n, data):
    k = data.draw(st.integers(1, n))
    # few distinct values => many ties
    v = np.array(data.draw(st.lists(st.integers(-3, 3), min_size=M * n, max_size=M * n)),
                 dtype=np.float32).reshape(M, n)
    tv, ti = O.top_k(v, k)
    for r in range(M):
        want = sorted(range(n), key=lambda j: (-v[r, j], j))[:k]
        assert ti[r].tolist() == want
        np.testing.assert_array_equal(tv[r], v[r, want])


@settings(max_examples=25, deadline=None)
@given(st.integers(1, 4), st.sampled_from([1, 2, 4]), st.integers(1, 6), st.data())
def test_sharded_equals_unsharded(M, P, k, data):
    rng = np.random.default_rng(data.draw(st.integers(0, 10**6)))
    n_local = data.draw(st.integers(k, 12))
    q = rng.integers(-2, 3, size=(M, 8)).astype(np.float32)
    keys = rng.integers(-2, 3, size=(P * n_local, 8)).astype(np.float32)
    a = O.tiled_topk(q, keys, k, 1.0, 0.0, 4.0, False)
    b = O.sharded_topk(q, keys, k, P, 1.0, 0.0, 4.0, False)
    np.testing.assert_array_equal(a[1], b[1])
    np.testing.assert_array_equal(a[0], b[0])


def test_philox_known_answers():
    kat = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
           ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF),
            (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
           ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
            (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in kat:
        got = O.philox4x32_10(np.array(ctr, dtype=np.uint32), key)
        assert [int(x) for x in got] == list(want)


def test_pool_init_is_shard_invariant_and_normal():
    full = O.pool_init_normal(64, 36, seed=7, stddev=0.5)
    part = O.pool_init_normal(16, 36, seed=7, stddev=0.5, row_offset=32)
    np.testing.assert_array_equal(full[32:48], part)
    big = O.pool_init_normal(512, 256, seed=3)
    assert abs(big.mean()) < 0.02 and abs(big.std() - 1.0) < 0.02


def test_comparator_catches_planted_mistakes(golden):
    q, keys, k, lam, tau, T, sig = _case(golden, "c1_gate")
    v, i = O.tiled_topk(q, keys, k, lam, tau, T, sig)
    assert O.compare_topk(v, i, v, i, q, keys, lam, tau, T, sig) == []
    # wrong index (a key that is far from the top)
    i2 = i.copy()
    s = O.fused_score(O.scores(q[:1], keys), lam, tau, T, sig)[0]
    i2[0, 3] = int(np.argmin(s))
    assert O.compare_topk(v, i2, v, i, q, keys, lam, tau, T, sig)
    # value perturbed beyond tolerance
    v2 = v.copy()
    v2[5, 0] *= 1.05
    assert O.compare_topk(v2, i, v, i, q, keys, lam, tau, T, sig)
    # order broken
    v3, i3 = v.copy(), i.copy()
    v3[2, [0, 1]] = v3[2, [1, 0]]
    i3[2, [0, 1]] = i3[2, [1, 0]]
    assert O.compare_topk(v3, i3, v, i, q, keys, lam, tau, T, sig)
    # duplicate index
    i4 = i.copy()
    i4[1, 1] = i4[1, 0]
    assert O.compare_topk(v, i4, v, i, q, keys, lam, tau, T, sig)


def test_score_lookup_comparator_agrees_with_recomputing_one(golden):
    """compare_topk_from_scores (precomputed f64 scores, for pools too large to
    recompute on the host) gives the same verdicts as compare_topk."""
    q, keys, k, lam, tau, T, sig = _case(golden, "c1_gate")
    v, i = O.tiled_topk(q, keys, k, lam, tau, T, sig)
    s = O.scores(q, keys)
    assert O.compare_topk_from_scores(v, i, v, i, s, lam, tau, T, sig) == []
    i2 = i.copy()
    i2[0, 3] = int(np.argmin(s[0]))
    v2 = v.copy()
    v2[5, 0] *= 1.05
    for gv, gi in ((v, i2), (v2, i)):
        a = O.compare_topk(gv, gi, v, i, q, keys, lam, tau, T, sig)
        b = O.compare_topk_from_scores(gv, gi, v, i, s, lam, tau, T, sig)
        assert a and b and len(a) == len(b)


def test_compare_rows():
    rng = np.random.default_rng(0)
    ref = rng.standard_normal((8, 16))
    assert O.compare_rows(ref * (1 + 1e-4), ref) == []
    bad = ref.copy()
    bad[3, 3] += 0.5
    assert O.compare_rows(bad, ref)


def _asm_case(golden, name):
    d_A, d_B, r, D = (int(x) for x in golden[f"{name}/dims"])
    return dict(h=O.bits_to_f32(golden[f"{name}/h"]), alpha=golden[f"{name}/alpha"],
                idx=golden[f"{name}/idx"], vectors=O.bits_to_f32(golden[f"{name}/vectors"]),
                W_base=golden[f"{name}/W_base"], b_base=golden[f"{name}/b_base"],
                gamma=float(golden[f"{name}/gamma"]), ln_scale=golden[f"{name}/ln_scale"],
                ln_bias=golden[f"{name}/ln_bias"], d_A=d_A, d_B=d_B, r=r)


@pytest.mark.parametrize("name", ["asm_eq", "asm_ne"])
def test_oracle_assembler_matches_reference_call(golden, name):
    """WeightAssembler.__call__ (per-position idx, residual when d_A == d_B) as run
    by the reference's own code."""
    c = _asm_case(golden, name)
    got = O.assemble_forward(c["h"], c["alpha"], c["idx"], c["vectors"], c["W_base"], c["b_base"],
                             c["gamma"], c["ln_scale"], c["ln_bias"], c["d_A"], c["d_B"], c["r"])
    np.testing.assert_allclose(got, golden[f"{name}/h_mid"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["asm_eq", "asm_ne"])
def test_oracle_usage_ema_matches_reference(golden, name):
    got = O.usage_ema(golden[f"{name}/ema0"], golden[f"{name}/alpha"], golden[f"{name}/idx"], 0.99)
    np.testing.assert_allclose(got, golden[f"{name}/ema1"], rtol=1e-6, atol=1e-9)


def test_lowrank_delta_catches_planted_factor_swap(golden):
    """A restatement that swapped the U and V blocks of the pool rows must not pass."""
    c = _asm_case(golden, "asm_eq")
    good = O.lowrank_delta(c["h"], c["alpha"], c["idx"], c["vectors"], c["d_A"], c["d_B"], c["r"])
    d_A, d_B, r = c["d_A"], c["d_B"], c["r"]
    swapped = c["vectors"].copy()
    nU = d_B * r
    swapped[:, :nU], swapped[:, nU:2 * nU] = c["vectors"][:, nU:2 * nU], c["vectors"][:, :nU]
    bad = O.lowrank_delta(c["h"], c["alpha"], c["idx"], swapped, d_A, d_B, r)
    assert np.abs(bad - good).max() > 1e-2 * np.abs(good).max()


@pytest.mark.parametrize("name", ["hybrid_gate", "hybrid_exp"])
def test_oracle_hybrid_forward_matches_reference(golden, name):
    """oracle.hybrid_forward against the reference's own hybrid_forward run
    (retrieval.py:131-181): identical indices, values and means within 1e-5."""
    B, seq, d_A, S, d_k, k, N, D = (int(x) for x in golden[f"{name}/dims"])
    lam, T, sig = golden[f"{name}/params"]
    alpha, idx, sims_seq, raw_seq, top_vals = O.hybrid_forward(
        O.bits_to_f32(golden[f"{name}/z"]), O.bits_to_f32(golden[f"{name}/vectors"]),
        O.bits_to_f32(golden[f"{name}/W_Q"]), O.bits_to_f32(golden[f"{name}/W_K"]),
        golden[f"{name}/aspect_logits"], golden[f"{name}/tau_param"], k, float(T), float(lam),
        bool(sig))
    np.testing.assert_array_equal(idx, golden[f"{name}/idx"])
    np.testing.assert_allclose(top_vals, golden[f"{name}/top_vals"], rtol=1e-5)
    np.testing.assert_allclose(alpha, golden[f"{name}/alpha"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(sims_seq, golden[f"{name}/sims_seq"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(raw_seq, golden[f"{name}/alpha_raw_seq"], rtol=1e-5)
