"""GPU parity: the sm_100a kernels (through the C ABI) against the oracle and
against fixtures computed by the reference's own code.

Tolerance (the parity contract): bf16 inputs, fp32 accumulation; scores and
outputs within rel 1e-2; top-k index sets identical except at near-ties of
the k-th value (oracle.compare_topk).  Exact ties must come back lower index
first, like jax.lax.top_k.
"""
import numpy as np
import pytest
import torch

from oracle import dwa_oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-2


def _dev():
    return torch.device("cuda", 0)


def to_dev_bf16(bits: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(_dev())
    return t.view(torch.bfloat16)


def from_f32(x: np.ndarray) -> torch.Tensor:
    return to_dev_bf16(O.bf16_bits(x))


def _status_ok():
    torch.cuda.synchronize()


@pytest.fixture(scope="module")
def lib():
    import computd_b200

    computd_b200.load_library()
    return computd_b200


def _case(golden, name):
    k, lam, tau, T, sig = golden[f"{name}/params"]
    return (O.bits_to_f32(golden[f"{name}/q"]), O.bits_to_f32(golden[f"{name}/keys"]), int(k),
            float(lam), float(tau), float(T), bool(sig))


@pytest.mark.parametrize("name", ["c1_exp", "c1_gate", "odd", "ties"])
def test_golden_tiled_topk(lib, golden, name):
    q, keys, k, lam, tau, T, sig = _case(golden, name)
    v, i = lib.tiled_topk_fused(to_dev_bf16(golden[f"{name}/q"]),
                                to_dev_bf16(golden[f"{name}/keys"]), k, lam, tau, T, sig)
    v, i = v.cpu().numpy(), i.cpu().numpy()
    errs = O.compare_topk(v, i, golden[f"{name}/vals"], golden[f"{name}/idx"], q, keys, lam, tau,
                          T, sig, rtol=RTOL)
    assert errs == [], errs
    if name == "ties":
        # integer-valued inputs: every dot product is exact, so the indices
        # (tie order included) must match bit for bit; the fp32 exp may differ
        # from NumPy's by an ulp.
        np.testing.assert_array_equal(i, golden["ties/idx"])
        np.testing.assert_allclose(v, golden["ties/vals"], rtol=1e-6)


def test_golden_sharded_merge_and_assembly(lib, golden):
    q, keys, k, lam, tau, T, sig = _case(golden, "sharded")
    P = int(golden["sharded/n_chips"])
    n_local = keys.shape[0] // P
    qd = to_dev_bf16(golden["sharded/q"])
    kd = to_dev_bf16(golden["sharded/keys"])
    loc_v, loc_i = [], []
    for p in range(P):
        v, i = lib.tiled_topk_fused(qd, kd[p * n_local:(p + 1) * n_local], k, lam, tau, T, sig,
                                    idx_offset=p * n_local)
        loc_v.append(v)
        loc_i.append(i)
        errs = O.compare_topk(v.cpu().numpy(), i.cpu().numpy() - p * n_local,
                              golden["sharded/local_vals"][p], golden["sharded/local_idx"][p], q,
                              keys[p * n_local:(p + 1) * n_local], lam, tau, T, sig, rtol=RTOL)
        assert errs == [], (p, errs)
    fv, fi = lib.merge_topk(torch.stack(loc_v), torch.stack(loc_i))
    fv, fi = fv.cpu().numpy(), fi.cpu().numpy()
    errs = O.compare_topk(fv, fi, O.chip_merge(golden["sharded/local_vals"],
                                               (golden["sharded/local_idx"] + (np.arange(P) * n_local)[:, None, None]).astype(np.int32))[0],
                          golden["sharded/idx"], q, keys, lam, tau, T, sig, rtol=RTOL)
    assert errs == [], errs
    np.testing.assert_allclose(O.normalise(fv), golden["sharded/alpha"], rtol=RTOL)
    # value side through the reference's own assembly output (b_delta block)
    vectors = to_dev_bf16(golden["sharded/vectors"])
    b0, b1 = (int(x) for x in golden["sharded/b_slice"])
    out, alpha = lib.weighted_value_sum(torch.from_numpy(golden["sharded/alpha"]).to(_dev()),
                                        torch.from_numpy(golden["sharded/idx"]).to(_dev()),
                                        vectors[:, b0:b1])
    assert O.compare_rows(out.cpu().numpy(), golden["sharded/b_delta"], rtol=RTOL) == []


SHAPES = [
    # M, N, d, k, use_sigmoid
    (1, 300, 64, 1, False),
    (1, 256, 8, 8, True),
    (5, 17, 16, 17, False),          # k == N
    (127, 1000, 128, 16, False),
    (129, 4097, 200, 32, True),      # ragged M, N and d (d not a multiple of 64)
    (300, 20000, 384, 32, False),
    (256, 9000, 1024, 64, True),
    (200, 6000, 512, 128, False),    # largest supported k
    (64, 3000, 40, 100, True),
]


@pytest.mark.parametrize("M,N,d,k,sig", SHAPES)
def test_random_shapes_vs_oracle(lib, M, N, d, k, sig):
    rng = np.random.default_rng(M * 7919 + N * 31 + d + k)
    q = O.bf16_round(rng.standard_normal((M, d), dtype=np.float32))
    keys = O.bf16_round(rng.standard_normal((N, d), dtype=np.float32) / np.float32(np.sqrt(d)))
    lam, tau, T = 3.0, 0.2, 0.9
    v, i = lib.tiled_topk_fused(from_f32(q), from_f32(keys), k, lam, tau, T, sig)
    rv, ri = O.tiled_topk(q, keys, k, lam, tau, T, sig)
    errs = O.compare_topk(v.cpu().numpy(), i.cpu().numpy(), rv, ri, q, keys, lam, tau, T, sig,
                          rtol=RTOL)
    assert errs == [], errs


def test_strided_inputs_and_offset(lib):
    rng = np.random.default_rng(5)
    M, N, d, k = 70, 3000, 96, 10
    qb = from_f32(rng.standard_normal((M, 128), dtype=np.float32))
    kb = from_f32(rng.standard_normal((N, 160), dtype=np.float32) / 10)
    q, keys = qb[:, :d], kb[:, :d]   # row strides 128 and 160 elements
    v, i = lib.tiled_topk_fused(q, keys, k, 1.0, 0.0, 1.0, False, idx_offset=12345)
    qn = q.float().cpu().numpy()
    kn = keys.float().cpu().numpy()
    rv, ri = O.tiled_topk(qn, kn, k)
    errs = O.compare_topk(v.cpu().numpy(), i.cpu().numpy() - 12345, rv, ri, qn, kn, rtol=RTOL)
    assert errs == [], errs


@pytest.mark.parametrize("P,M,k", [(8, 333, 64), (40, 100, 32), (100, 50, 16), (40, 70, 64),
                                   (128, 20, 128), (1, 17, 5)])
def test_merge_matches_oracle(lib, P, M, k):
    """The k-way merge on every path: lists staged in shared memory with one,
    two or four lists per lane (n_lists x k <= 2048), and the register-cursor
    kernel for longer list sets."""
    rng = np.random.default_rng(11 + P)
    vals = -np.sort(-rng.standard_normal((P, M, k)).astype(np.float32), axis=2)
    vals[:, :, 10:14] = vals[:, :, 10:11]   # ties inside and across lists
    vals = -np.sort(-vals, axis=2)
    idx = (np.arange(P)[:, None, None] * 1000 + rng.integers(0, 1000, (P, M, k))).astype(np.int32)
    for p in range(P):  # sorted lists, lower index first on ties (as dwa_score_topk emits)
        for m in range(M):
            o = np.lexsort((idx[p, m], -vals[p, m]))
            idx[p, m], vals[p, m] = idx[p, m][o], vals[p, m][o]
    fv, fi = lib.merge_topk(torch.from_numpy(vals).to(_dev()), torch.from_numpy(idx).to(_dev()))
    rv, ri = O.chip_merge(vals, idx)
    np.testing.assert_array_equal(fi.cpu().numpy(), ri)
    np.testing.assert_array_equal(fv.cpu().numpy(), rv)


@pytest.mark.parametrize("M,N,d,k", [(1, 10, 8, 1), (77, 500, 128, 16), (64, 4096, 1024, 64),
                                     (33, 700, 264, 128)])
def test_weighted_gather_vs_oracle(lib, M, N, d, k):
    rng = np.random.default_rng(M + N + d + k)
    vals = np.abs(rng.standard_normal((M, k))).astype(np.float32) + 0.1
    idx = rng.integers(0, N, (M, k)).astype(np.int32)
    values = O.bf16_round(rng.standard_normal((N, d), dtype=np.float32))
    out, alpha = lib.weighted_value_sum(torch.from_numpy(vals).to(_dev()),
                                        torch.from_numpy(idx).to(_dev()), from_f32(values))
    ra = O.normalise(vals)
    np.testing.assert_allclose(alpha.cpu().numpy(), ra, rtol=1e-5)
    assert O.compare_rows(out.cpu().numpy(), O.weighted_sum(ra, idx, values), rtol=RTOL) == []


def test_owner_computes_partials_add_up(lib):
    rng = np.random.default_rng(3)
    M, N, d, k, P = 50, 800, 64, 16, 4
    vals = np.abs(rng.standard_normal((M, k))).astype(np.float32)
    idx = rng.integers(0, N, (M, k)).astype(np.int32)
    values = from_f32(rng.standard_normal((N, d), dtype=np.float32))
    vd, idd = torch.from_numpy(vals).to(_dev()), torch.from_numpy(idx).to(_dev())
    full, _ = lib.weighted_value_sum(vd, idd, values)
    n = N // P
    parts = sum(lib.weighted_value_sum(vd, idd, values[p * n:(p + 1) * n], row_begin=p * n)[0]
                for p in range(P))
    torch.testing.assert_close(parts, full, rtol=1e-5, atol=1e-5)


def test_pool_init_matches_oracle_generator(lib):
    rows, cols, seed = 300, 72, 123456789
    dev = lib.new_normal(rows, cols, seed, stddev=0.5, row_offset=1000)
    got = dev.float().cpu().numpy()
    want = O.bf16_round(O.pool_init_normal(rows, cols, seed, 0.5, row_offset=1000))
    ulp = np.abs(got.view(np.int32) - want.view(np.int32)) >> 16
    assert ulp.max() <= 1
    assert (ulp == 0).mean() > 0.99
    # shard invariance on the device
    a = lib.new_normal(64, 72, seed, 0.5, row_offset=1000)
    torch.testing.assert_close(a, dev[:64], rtol=0, atol=0)


def test_c1_config_full(lib):
    """C1: queries [2048,128] ~N(0,1), keys [16384,128] ~N(0,1/128), values ~N(0,1),
    k=16, softmax over the 16 scores, weighted sum (seed 0; bf16-rounded on the GPU)."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2048, 128), dtype=np.float32)
    keys = rng.standard_normal((16384, 128), dtype=np.float32) / np.float32(np.sqrt(128))
    values = rng.standard_normal((16384, 128), dtype=np.float32)
    qb, kb, vb = O.bf16_round(q), O.bf16_round(keys), O.bf16_round(values)
    r = lib.Retriever(from_f32(kb), from_f32(vb), 2048, 16)
    out, alpha, tv, ti = r(from_f32(qb))
    torch.cuda.synchronize()
    assert r.status() == 0
    ro, ra, rv, ri = O.retrieve(qb, kb, vb, 16)
    errs = O.compare_topk(tv.cpu().numpy(), ti.cpu().numpy(), rv, ri, qb, kb, rtol=RTOL)
    assert errs == [], errs
    # value side checked on the GPU's own selection (a near-tie swap changes rows legitimately)
    ti_n = ti.cpu().numpy()
    want = O.weighted_sum(O.normalise(tv.cpu().numpy()), ti_n, vb)
    assert O.compare_rows(out.cpu().numpy(), want, rtol=RTOL) == []
    assert O.compare_rows(out.cpu().numpy(), ro, rtol=RTOL) == [] or \
        (ti_n != ri).any()


def test_op_at_scale_properties(lib):
    """C3 shape (8192 x 1,048,576 x 1024, k=64): sampled rows against an exact
    recomputation, plus size-independent properties on every row."""
    dev = _dev()
    M, N, d, k = 8192, 1 << 20, 1024, 64
    q = lib.new_normal(M, d, seed=1, stddev=1.0)
    keys = lib.new_normal(N, d, seed=2, stddev=d ** -0.5)
    values = lib.new_normal(N, d, seed=3, stddev=1.0)
    r = lib.Retriever(keys, values, M, k)
    out, alpha, tv, ti = r(q)
    torch.cuda.synchronize()
    assert r.status() == 0
    # every row: sorted, in range, no duplicates, alpha sums to 1
    assert bool((tv[:, 1:] <= tv[:, :-1]).all())
    assert int(ti.min()) >= 0 and int(ti.max()) < N
    s_idx, _ = torch.sort(ti, dim=1)
    assert not bool((s_idx[:, 1:] == s_idx[:, :-1]).any())
    torch.testing.assert_close(alpha.sum(1), torch.ones(M, device=dev), rtol=1e-5, atol=1e-5)
    # returned scores equal the recomputed dot products of the returned indices
    s_true = torch.einsum("md,mkd->mk", q.float(), keys[ti.long()].float())
    torch.testing.assert_close(tv, torch.exp(s_true), rtol=1e-4, atol=0)
    # sampled rows: exact top-k over the whole pool (fp32 scores on the GPU, oracle top_k)
    rows = torch.arange(0, M, M // 24, device=dev)
    s = (q[rows].float() @ keys.float().T).double().cpu().numpy()
    rv, ri = O.top_k(np.exp(s), k)
    got_v, got_i = tv[rows].cpu().numpy(), ti[rows].cpu().numpy()
    qn, kn = q[rows].float().cpu().numpy(), None
    bad = 0
    for j in range(len(rows)):
        gs, rs_ = set(got_i[j].tolist()), set(ri[j].tolist())
        if gs != rs_:
            extra = np.array(sorted(gs - rs_))
            vext = np.exp(s[j, extra])
            if (vext < rv[j, -1] * (1 - RTOL)).any():
                bad += 1
    assert bad == 0
    np.testing.assert_allclose(got_v, rv, rtol=RTOL)
    # value side on the sampled rows
    want = torch.einsum("mk,mkd->md", alpha[rows].double(), values[ti[rows].long()].double())
    assert O.compare_rows(out[rows].cpu().numpy(), want.cpu().numpy(), rtol=RTOL) == []


@pytest.mark.parametrize("M,N,d,k", [(300, 40000, 64, 16), (512, 70000, 128, 64), (100, 9000, 32, 128)])
def test_exact_ties_across_key_splits(lib, M, N, d, k):
    """Integer-valued inputs make every score exact, and duplicated key rows
    spread over the whole pool create ties between key-range splits; the
    shared admission bound must still return exactly lax.top_k's indices
    (lower index first among equal scores)."""
    rng = np.random.default_rng(M + N + k)
    q = rng.integers(-2, 3, size=(M, d)).astype(np.float32)
    base = rng.integers(-2, 3, size=(N // 8, d)).astype(np.float32)
    keys = base[rng.integers(0, base.shape[0], size=N)]
    T = 64.0  # keeps exp(s / T) finite and exactly ordered
    v, i = lib.tiled_topk_fused(from_f32(q), from_f32(keys), k, 1.0, 0.0, T, False)
    torch.cuda.synchronize()
    rv, ri = O.tiled_topk(q, keys, k, 1.0, 0.0, T, False)
    np.testing.assert_array_equal(i.cpu().numpy(), ri)
    np.testing.assert_allclose(v.cpu().numpy(), rv, rtol=1e-6)


@pytest.mark.parametrize("k", [32, 64, 128])
def test_exact_ties_grouped_unit_order(lib, k):
    """Queries larger than half of L2 (9651 x 4096 bf16, 79 MB) switch the
    score kernel to query-tile groups: here 38 query tiles x 3 key splits, in
    groups of 24 and 14 query tiles (a ragged last group, ragged M and N).
    Integer inputs keep every score exact (|s| <= 4 * 4096 < 2^24), and
    duplicated key rows tie across splits and groups; indices must equal the
    oracle's top_k on exactly recomputed scores, lower index first on ties."""
    dev = _dev()
    M, N, d = 9651, 8205, 4096
    g = torch.Generator(device=dev).manual_seed(k)
    q = torch.randint(-2, 3, (M, d), generator=g, device=dev).to(torch.bfloat16)
    base = torch.randint(-2, 3, (N // 8, d), generator=g, device=dev).to(torch.bfloat16)
    keys = base[torch.randint(0, N // 8, (N,), generator=g, device=dev)].contiguous()
    T = 64.0  # s / T is exact and exp(s / T) stays finite and strictly ordered
    v, i = lib.tiled_topk_fused(q, keys, k, 1.0, 0.0, T, False)
    torch.cuda.synchronize()
    got_v, got_i = v.cpu().numpy(), i.cpu().numpy()
    kf = keys.float()
    for r0 in range(0, M, 1024):
        s = (q[r0:r0 + 1024].float() @ kf.T).double().cpu().numpy()
        rv, ri = O.top_k(O.fused_score(s, 1.0, 0.0, T, False), k)
        np.testing.assert_array_equal(got_i[r0:r0 + 1024], ri)
        np.testing.assert_allclose(got_v[r0:r0 + 1024], rv, rtol=1e-5)


def _hybrid_mirror(lib, golden, dtype):
    dev = _dev()
    W_Q, W_K = golden["sharded/W_Q"], golden["sharded/W_K"]
    S, d_k, d_A = W_Q.shape
    vectors = to_dev_bf16(golden["sharded/vectors"])
    m = lib.MultiAspectRetrieval(D=W_K.shape[2], d_A=d_A, S=S, d_k=d_k, N=vectors.shape[0],
                                 device=dev, dtype=dtype)
    m.W_Q = torch.from_numpy(W_Q).to(dev).to(dtype)
    m.W_K = torch.from_numpy(W_K).to(dev).to(dtype)
    m.aspect_logits = torch.from_numpy(golden["sharded/aspect_logits"]).to(dev)
    m.tau = torch.from_numpy(golden["sharded/tau_param"]).to(dev)
    return m, vectors, torch.from_numpy(golden["sharded/z"]).to(dev)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pallas_hybrid_forward_matches_reference(lib, golden, dtype):
    """MultiAspectRetrieval.pallas_hybrid_forward with the parameters the
    reference ran with (its own 4-chip shard_map run produced the fixture).

    Every row goes through the parity comparator: the returned indices' fused
    scores are recomputed in fp64 from the collapsed bf16 queries / keys the
    score kernel saw, the values must match the reference's merged top-k
    rank-wise within RTOL, and an index set may differ from the reference's
    only by swaps inside a near-tie of the k-th value.  alpha and the aux
    outputs are then compared on all rows.  fp32 parameters take the fp32
    projection; bf16 parameters (the reference's own dtype, retrieval.py:37,41)
    take the fused tcgen05 key projection."""
    k, lam, tau, T, sig = golden["sharded/params"]
    k, lam, T, sig = int(k), float(lam), float(T), bool(sig)
    m, vectors, z = _hybrid_mirror(lib, golden, dtype)
    p = m.pallas_hybrid_parts(z, vectors, k, T, lam, sig, tp_axis=None)
    torch.cuda.synchronize()
    B, seq = z.shape[:2]
    assert p.alpha.shape == (B, seq, k) and p.top_idx.shape == (B, seq, k)
    assert abs(float(p.tau) - float(tau)) <= 1e-6 * max(1.0, abs(float(tau)))
    P = int(golden["sharded/n_chips"])
    n_local = vectors.shape[0] // P
    ref_v, ref_i = O.chip_merge(golden["sharded/local_vals"],
                                (golden["sharded/local_idx"] + (np.arange(P) * n_local)[:, None, None]
                                 ).astype(np.int32))
    np.testing.assert_array_equal(ref_i, golden["sharded/idx"])
    qf = p.queries_flat.float().cpu().numpy()
    kw = p.keys_w.float().cpu().numpy()
    got_v, got_i = p.top_vals.cpu().numpy(), p.top_idx.reshape(-1, k).cpu().numpy()
    errs = O.compare_topk(got_v, got_i, ref_v, ref_i, qf, kw, lam, float(p.tau), T, sig, rtol=RTOL)
    assert errs == [], errs
    # alpha rank-wise on every row (a near-tie swap changes a value by < RTOL)
    np.testing.assert_allclose(p.alpha.reshape(-1, k).cpu().numpy(), golden["sharded/alpha"],
                               rtol=RTOL, atol=1e-4)
    np.testing.assert_allclose(p.sims_seq.cpu().numpy(), golden["sharded/sims_seq"], rtol=RTOL,
                               atol=1e-3)
    np.testing.assert_allclose(p.alpha_raw_seq.cpu().numpy(), golden["sharded/alpha_raw_seq"],
                               rtol=RTOL, atol=1e-3)


def test_host_pipeline_matches_retriever(lib):
    """HostPipeline (pinned host in, pinned host out, copies overlapped with the
    neighbouring batches' kernels) returns, batch by batch, exactly what a
    direct Retriever call returns for the same queries."""
    M, N, d, k = 600, 40000, 256, 32
    keys = lib.new_normal(N, d, seed=21, stddev=d ** -0.5, device=_dev())
    values = lib.new_normal(N, d, seed=22, device=_dev())
    batches = [lib.new_normal(M, d, seed=30 + i, device=_dev()) for i in range(5)]
    ref = lib.Retriever(keys, values, M, k, lambda_sharp=2.0, tau=0.1, T=0.9, use_sigmoid=True)
    want = []
    for q in batches:
        out, alpha, _, idx = ref(q)
        want.append((out.cpu().clone(), alpha.cpu().clone(), idx.cpu().clone()))
    pipe = lib.HostPipeline(keys, values, M, k, lambda_sharp=2.0, tau=0.1, T=0.9,
                            use_sigmoid=True)
    q_host = [q.cpu().pin_memory() for q in batches]
    got = [(torch.empty((M, d), dtype=torch.float32).pin_memory(),
            torch.empty((M, k), dtype=torch.float32).pin_memory(),
            torch.empty((M, k), dtype=torch.int32).pin_memory()) for _ in batches]
    for qh, (oh, ah, ih) in zip(q_host, got):
        pipe.submit(qh, oh, ah, ih)
    pipe.synchronize()
    assert pipe.status() == 0
    for (oh, ah, ih), (ow, aw, iw) in zip(got, want):
        assert torch.equal(ih, iw)
        assert torch.equal(ah, aw)
        assert torch.equal(oh, ow)


@pytest.mark.parametrize("N,D,S,d_k", [
    (1000, 88, 2, 32),      # the reference-run fixture's shape (one padded projection tile)
    (5000, 1024, 16, 64),   # four full projection tiles
    (700, 520, 3, 128),     # d_k = 128, D tail of 8 columns, padded tile
    (300, 4096, 8, 128),
])
def test_project_keys_vs_fp32(lib, N, D, S, d_k):
    """dwa_project_keys (fused projection + L2 normalisation + aspect collapse)
    against a plain fp32 PyTorch restatement on the same bf16 inputs."""
    dev = _dev()
    g = torch.Generator(device=dev)
    g.manual_seed(N + D)
    v = torch.randn((N, D), device=dev, generator=g).to(torch.bfloat16)
    wk = (torch.randn((S, d_k, D), device=dev, generator=g) * D ** -0.5).to(torch.bfloat16)
    w = torch.softmax(torch.randn(S, device=dev, generator=g), 0)
    got = lib.project_keys(v, wk, w).float()
    ks = torch.einsum("skd,nd->snk", wk.float(), v.float())
    ks = ks / (ks.norm(dim=-1, keepdim=True) + 1e-8)
    want = torch.einsum("s,snk->nk", w, ks)
    err = float((got - want).abs().max())
    assert err <= RTOL * float(want.abs().max()), f"max abs err {err}"


@pytest.mark.parametrize("name", ["hybrid_gate", "hybrid_exp"])
def test_hybrid_forward_matches_reference(lib, golden, name):
    """MultiAspectRetrieval.hybrid_forward (retrieval.py:131-181) against the
    reference's own run: packed per-aspect keys from the tcgen05 projection,
    the aspect-weighted score through the fused score + top-k kernel, and the
    seq mean of the fused scores from that kernel's epilogue.  hybrid_exp has
    seq = 40, so warps straddle two sequences (the per-lane accumulation path)."""
    dev = _dev()
    B, seq, d_A, S, d_k, k, N, D = (int(x) for x in golden[f"{name}/dims"])
    lam, T, sig = (float(x) for x in golden[f"{name}/params"])
    sig = bool(sig)
    m = lib.MultiAspectRetrieval(D=D, d_A=d_A, S=S, d_k=d_k, N=N, device=dev, dtype=torch.bfloat16)
    m.W_Q = to_dev_bf16(golden[f"{name}/W_Q"])
    m.W_K = to_dev_bf16(golden[f"{name}/W_K"])
    m.aspect_logits = torch.from_numpy(golden[f"{name}/aspect_logits"]).to(dev)
    m.tau = torch.from_numpy(golden[f"{name}/tau_param"]).to(dev)
    z = to_dev_bf16(golden[f"{name}/z"])
    vectors = to_dev_bf16(golden[f"{name}/vectors"])
    p = m.hybrid_parts(z, vectors, k, T, lam, sig)
    alpha, idx, sims_seq, raw_seq = m.hybrid_forward(z, vectors, k, T, lam, sig)
    torch.cuda.synchronize()
    assert alpha.shape == (B, seq, k) and idx.shape == (B, seq, k)
    assert sims_seq.shape == (B, N) and raw_seq.shape == (B, N)
    qf = p.queries_flat.float().cpu().numpy()
    kp = p.keys_w.float().cpu().numpy()
    errs = O.compare_topk(p.top_vals.cpu().numpy(), p.top_idx.reshape(-1, k).cpu().numpy(),
                          golden[f"{name}/top_vals"].reshape(-1, k),
                          golden[f"{name}/idx"].reshape(-1, k), qf, kp, lam, float(p.tau), T, sig,
                          rtol=RTOL)
    assert errs == [], errs
    np.testing.assert_allclose(alpha.cpu().numpy(), golden[f"{name}/alpha"], rtol=RTOL, atol=1e-4)
    np.testing.assert_allclose(sims_seq.cpu().numpy(), golden[f"{name}/sims_seq"], rtol=RTOL,
                               atol=1e-3)
    np.testing.assert_allclose(raw_seq.cpu().numpy(), golden[f"{name}/alpha_raw_seq"], rtol=RTOL)
    # the second call (no state kept between calls) returns the same selection
    assert torch.equal(idx, p.top_idx)


@pytest.mark.parametrize("B,seq,N,d,k,sig", [(4, 256, 20000, 512, 16, True),
                                             (3, 96, 9000, 2048, 32, False),
                                             (2, 300, 5000, 256, 64, True)])
def test_score_topk_seqmean_vs_fp64(lib, B, seq, N, d, k, sig):
    """The fused seq-mean epilogue (dwa_score_topk_seqmean) against fp64 means of
    every (position, key) score on the same bf16 inputs, and its top-k output
    equal to dwa_score_topk_dev's (the epilogue only adds work)."""
    dev = _dev()
    M = B * seq
    q = lib.new_normal(M, d, seed=d + seq, stddev=d ** -0.5, device=dev)
    keys = lib.new_normal(N, d, seed=N + k, stddev=d ** -0.5, device=dev)
    lam, tau, T = 3.0, 0.05, 0.6
    tv, ti, mean = lib.score_topk_seqmean(q, keys, k, lam, tau, T, sig, seq)
    params = lib.score_params(lam, tau, T, dev)
    tv2, ti2 = lib.tiled_topk_fused(q, keys, k, params[0], params[1], params[2], sig)
    torch.cuda.synchronize()
    assert torch.equal(ti, ti2) and torch.equal(tv, tv2)
    s = q.double() @ keys.double().T
    v = torch.exp(s / T)
    if sig:
        v = v * torch.sigmoid(lam * (s - tau))
    want = v.view(B, seq, N).mean(1)
    torch.testing.assert_close(mean.double(), want, rtol=1e-4, atol=0)


@pytest.mark.parametrize("M,N,d,k,seq", [(600, 30000, 512, 128, 200),       # whole-heap list
                                          (18944, 524288, 512, 128, 256)])  # two-level list
def test_score_topk_seqmean_k128(lib, M, N, d, k, seq):
    """The seq-mean epilogue on the k > 64 lists (the whole shared-memory heap for
    short units, the register + heap two-level list for long ones): the top-k equal
    to the plain kernel's and the fused means of sampled sequences against fp64."""
    dev = _dev()
    q = lib.new_normal(M, d, seed=M + k, stddev=d ** -0.5, device=dev)
    keys = lib.new_normal(N, d, seed=N + d, stddev=d ** -0.5, device=dev)
    lam, tau, T = 2.0, 0.02, 0.5
    tv, ti, mean = lib.score_topk_seqmean(q, keys, k, lam, tau, T, True, seq)
    params = lib.score_params(lam, tau, T, dev)
    tv2, ti2 = lib.tiled_topk_fused(q, keys, k, params[0], params[1], params[2], True)
    torch.cuda.synchronize()
    assert torch.equal(ti, ti2) and torch.equal(tv, tv2)
    kd = keys.double()
    B = M // seq
    for b in sorted({0, B // 2, B - 1}):
        s = q[b * seq:(b + 1) * seq].double() @ kd.T
        v = torch.exp(s / T) * torch.sigmoid(lam * (s - tau))
        torch.testing.assert_close(mean[b].double(), v.mean(0), rtol=1e-4, atol=0)


@pytest.mark.parametrize("k", [100, 128])
def test_exact_ties_two_level_list(lib, k):
    """k > 64 over units whose key tiles x d reach 2^20 takes the two-level list
    (best 64 in registers, the rest in a shared-memory heap).  18944 queries =
    74 query tiles, one unit per CTA pair, each over all 2048 key tiles of
    524,288 duplicated integer keys of width 512: every score is exact and ties
    abound.  Every row's indices must equal lax.top_k's (values descending,
    lower index first), computed on the GPU from composite integer keys
    (score, -index)."""
    dev = _dev()
    M, N, d = 18944, 524288, 512
    g = torch.Generator(device=dev).manual_seed(k)
    q = torch.randint(-2, 3, (M, d), generator=g, device=dev).to(torch.bfloat16)
    base = torch.randint(-2, 3, (N // 16, d), generator=g, device=dev).to(torch.bfloat16)
    keys = base[torch.randint(0, N // 16, (N,), generator=g, device=dev)].contiguous()
    T = 512.0  # |s| <= 2048: s / T is exact, exp(s / T) finite and strictly increasing in s
    v, i = lib.tiled_topk_fused(q, keys, k, 1.0, 0.0, T, False)
    torch.cuda.synchronize()
    kf = keys.float()
    ar = torch.arange(N, device=dev, dtype=torch.int64)
    for r0 in range(0, M, 512):
        s = (q[r0:r0 + 512].float() @ kf.T).to(torch.int64)     # exact integer scores
        comp = s * (1 << 26) - ar                                # higher score, then lower index
        ref = torch.topk(comp, k, dim=1, sorted=True).indices.to(torch.int32)
        assert torch.equal(i[r0:r0 + 512], ref), r0
        want_v = torch.exp(torch.gather(s, 1, ref.long()).double() / T).float()
        torch.testing.assert_close(v[r0:r0 + 512], want_v, rtol=1e-6, atol=0)


@pytest.mark.parametrize("N,d,k", [(64, 64, 8), (300, 128, 16), (5000, 64, 32)])
def test_identity_keys_one_hot_queries_known_answer(lib, N, d, k):
    """Known answer: key n = c_n e_n for n < d (c_n = 1 + n / 64, exact in bf16),
    zero rows beyond; query m = e_{m mod d}.  Query e_j scores c_j on key j and
    exactly 0 on every other key, so its top-k is j followed by the zero-score
    keys in ascending index order (lower index first among ties); the values
    are the fused scores exp(s / T) of those raw scores."""
    M = 2 * d + 3
    keys = np.zeros((N, d), np.float32)
    c = 1.0 + np.arange(d, dtype=np.float32) / 64.0
    keys[np.arange(d), np.arange(d)] = c
    q = np.zeros((M, d), np.float32)
    q[np.arange(M), np.arange(M) % d] = 1.0
    T = 0.5
    v, i = lib.tiled_topk_fused(from_f32(q), from_f32(keys), k, 1.0, 0.0, T, False)
    v, i = v.cpu().numpy(), i.cpu().numpy()
    for m in range(M):
        j = m % d
        want = [j] + [n for n in range(k) if n != j][:k - 1]
        assert list(i[m]) == want, (m, list(i[m]), want)
        assert np.isclose(v[m, 0], np.exp(c[j] / T), rtol=1e-6)
        assert np.allclose(v[m, 1:], 1.0)
