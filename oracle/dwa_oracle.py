"""CPU restatement of computd's DWA retrieval path — TEST INFRASTRUCTURE, not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` legs may import this module, and only as the checker or
as the timed CPU baseline.  The product path (``computd_b200``) never calls it.

Every function restates one piece of the reference (file:line in the
reference tree):

* ``fused_score``      — src/kernels/tiled_topk.py:172-175 (gate * exp, or exp)
* ``top_k``            — jax.lax.top_k as used at tiled_topk.py:176: values
                         descending, lower index first among equal values
                         (jaxlib 0.10.0, not vendored; published contract)
* ``tiled_topk``       — src/kernels/tiled_topk.py:160-176 (tiled_topk_fallback)
* ``chip_merge``       — src/model/retrieval.py:292-302 (global offset,
                         all_gather stacking, transpose/reshape, top_k, take)
* ``sharded_topk``     — retrieval.py:280-313 (shard_map over a row-sharded pool)
* ``normalise``        — retrieval.py:326 (alpha = v / (sum v + 1e-8))
* ``hybrid_forward``   — retrieval.py:131-181 (MultiAspectRetrieval.hybrid_forward:
                         per-aspect scores weighted by softmax(aspect_logits),
                         gate/exp, top_k per position, seq means of sims and scores)
* ``weighted_sum``     — src/model/assembly.py:104,127 (vectors[idx], alpha-weighted sum)
* ``lowrank_delta``    — src/model/assembly.py:110-127 (U/V/b split, hV, h_delta, b_delta)
* ``assemble_forward`` — assembly.py:75-128, WeightAssembler.__call__ per-position path
                         (+ flax nnx.LayerNorm, eps 1e-6)
* ``usage_ema``        — src/training/trainer.py:227-233 (scatter of alpha / idx.size)
                         + src/model/pool.py:52-55 (EMA with beta)
* ``pool_init_normal`` — the counter-based generator of computd_b200/csrc/pool_init.cu
                         (Philox4x32-10, Salmon et al. SC'11, + Box-Muller)

Parity pin: the reference ships no tests or golden vectors for this path and
JAX cannot be installed here, so the restatement is pinned against fixtures
produced by executing the reference's own functions (tiled_topk_fallback,
MultiAspectRetrieval.pallas_hybrid_forward with a 4-way shard_map,
WeightAssembler.assemble) over a NumPy stand-in for jax/flax
(tests/golden/make_golden.py).  The jax primitives themselves (jnp.dot,
lax.top_k, all_gather) are the stand-in's restatement of their published
contracts, so the pin covers the reference's composition, not jaxlib.
"""
from __future__ import annotations

import numpy as np

try:  # bf16 rounding on the CPU
    import ml_dtypes

    BF16 = ml_dtypes.bfloat16
except ImportError:  # pragma: no cover - ml_dtypes ships with the image
    BF16 = None


# --------------------------------------------------------------------------- dtypes
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bf16 (ties to even); returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    if BF16 is not None:
        return x.astype(BF16).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) of float32 values (rounded to nearest even)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------- scores
def fused_score(s: np.ndarray, lambda_sharp: float, tau: float, T: float,
                use_sigmoid: bool) -> np.ndarray:
    """src/kernels/tiled_topk.py:172-175."""
    s = np.asarray(s)
    with np.errstate(over="ignore"):
        e = np.exp(s / np.asarray(T, dtype=s.dtype))
        if not use_sigmoid:
            return e
        g = 1.0 / (1.0 + np.exp(-(np.asarray(lambda_sharp, dtype=s.dtype) * (s - np.asarray(tau, dtype=s.dtype)))))
    return g * e


def top_k(v: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """jax.lax.top_k along the last axis: (values desc, int32 indices); among
    equal values the lower index comes first."""
    v = np.asarray(v)
    n = v.shape[-1]
    if not 1 <= k <= n:
        raise ValueError(f"top_k needs 1 <= k <= {n}, got {k}")
    lead = v.shape[:-1]
    v2 = v.reshape(-1, n)
    kth = -np.partition(-v2, k - 1, axis=1)[:, k - 1]
    gt = v2 > kth[:, None]
    eq = v2 == kth[:, None]
    need = k - gt.sum(axis=1)
    sel = gt | (eq & (np.cumsum(eq, axis=1) <= need[:, None]))
    rows, cols = np.nonzero(sel)
    idx = cols.reshape(-1, k)                      # ascending index within each row
    vals = np.take_along_axis(v2, idx, axis=1)
    order = np.argsort(-vals, axis=1, kind="stable")  # stable: lower index first on ties
    idx = np.take_along_axis(idx, order, axis=1)
    vals = np.take_along_axis(vals, order, axis=1)
    return vals.reshape(*lead, k), idx.astype(np.int32).reshape(*lead, k)


def scores(q: np.ndarray, keys: np.ndarray, accum=np.float64) -> np.ndarray:
    """s = q . keys^T accumulated in `accum` (inputs taken as given)."""
    return np.asarray(q, dtype=accum) @ np.asarray(keys, dtype=accum).T


def tiled_topk(q: np.ndarray, keys: np.ndarray, k: int, lambda_sharp: float = 1.0, tau: float = 0.0,
               T: float = 1.0, use_sigmoid: bool = False, *, accum=np.float64,
               chunk_rows: int = 256) -> tuple[np.ndarray, np.ndarray]:
    """tiled_topk_fallback (src/kernels/tiled_topk.py:160-176) on one shard.

    Returns (vals f32 [M, k] fused scores, idx i32 [M, k]).  Selection uses the
    fused score in `accum` precision; rows are processed in chunks.
    """
    M = q.shape[0]
    out_v = np.empty((M, k), dtype=np.float32)
    out_i = np.empty((M, k), dtype=np.int32)
    kf = np.asarray(keys, dtype=accum)
    for r0 in range(0, M, chunk_rows):
        s = np.asarray(q[r0:r0 + chunk_rows], dtype=accum) @ kf.T
        v = fused_score(s, lambda_sharp, tau, T, use_sigmoid)
        tv, ti = top_k(v, k)
        out_v[r0:r0 + chunk_rows] = tv
        out_i[r0:r0 + chunk_rows] = ti
    return out_v, out_i


def chip_merge(cand_v: np.ndarray, cand_i: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """retrieval.py:299-302: [P, BT, k] -> transpose(1,0,2) -> [BT, P*k] -> top_k -> take."""
    P, BT, k = cand_v.shape
    cv = cand_v.transpose(1, 0, 2).reshape(BT, P * k)
    ci = cand_i.transpose(1, 0, 2).reshape(BT, P * k)
    fv, sel = top_k(cv, k)
    fi = np.take_along_axis(ci, sel, axis=1)
    return fv, fi.astype(np.int32)


def sharded_topk(q: np.ndarray, keys: np.ndarray, k: int, P: int, lambda_sharp: float = 1.0,
                 tau: float = 0.0, T: float = 1.0, use_sigmoid: bool = False, *,
                 accum=np.float64) -> tuple[np.ndarray, np.ndarray]:
    """retrieval.py:280-313: per-shard top-k + global offset (292-293) + merge."""
    N = keys.shape[0]
    if N % P:
        raise ValueError("pool rows must divide evenly over the shards")
    n_local = N // P
    cv, ci = [], []
    for p in range(P):
        tv, li = tiled_topk(q, keys[p * n_local:(p + 1) * n_local], k, lambda_sharp, tau, T,
                            use_sigmoid, accum=accum)
        cv.append(tv)
        ci.append(li + p * n_local)
    return chip_merge(np.stack(cv), np.stack(ci).astype(np.int32))


def normalise(vals: np.ndarray) -> np.ndarray:
    """retrieval.py:326: alpha = v / (sum(v) + 1e-8) over the last axis."""
    vals = np.asarray(vals, dtype=np.float32)
    return vals / (np.sum(vals, axis=-1, keepdims=True) + np.float32(1e-8))


def weighted_sum(alpha: np.ndarray, idx: np.ndarray, values: np.ndarray,
                 accum=np.float64) -> np.ndarray:
    """assembly.py:104,127: sum_j alpha[..., j] * values[idx[..., j]]."""
    sel = np.asarray(values, dtype=accum)[idx]          # [..., k, d]
    return np.einsum("...k,...kd->...d", np.asarray(alpha, dtype=accum), sel)


def retrieve(q, keys, values, k, lambda_sharp=1.0, tau=0.0, T=1.0, use_sigmoid=False, P=1,
             accum=np.float64):
    """Full path: (out [M, d] f64, alpha f32 [M, k], vals f32 [M, k], idx i32 [M, k])."""
    if P == 1:
        v, i = tiled_topk(q, keys, k, lambda_sharp, tau, T, use_sigmoid, accum=accum)
    else:
        v, i = sharded_topk(q, keys, k, P, lambda_sharp, tau, T, use_sigmoid, accum=accum)
    a = normalise(v)
    return weighted_sum(a, i, values, accum=accum), a, v, i


def _l2n(x: np.ndarray) -> np.ndarray:
    return x / (np.linalg.norm(x, axis=-1, keepdims=True) + 1e-8)


def hybrid_forward(z, vectors, W_Q, W_K, aspect_logits, tau_param, k, T=1.0, lambda_sharp=1.0,
                   use_sigmoid=True, accum=np.float64):
    """MultiAspectRetrieval.hybrid_forward (retrieval.py:131-181), computed in `accum`.

    keys_s = normalise(W_K[s] . vectors), queries_s = normalise(W_Q[s] . z) per
    aspect; sims_w[b, t, n] = sum_s w_s <queries_s[b, t], keys_s[n]> with
    w = softmax(aspect_logits); alpha_raw = gate * exp(sims_w / T) (gate =
    sigmoid(lambda (sims_w - w . tau)) when use_sigmoid); top_k per position;
    alpha = top_vals / (sum + 1e-8); seq means of sims_w and alpha_raw.
    Returns (alpha f32 [B, seq, k], idx i32 [B, seq, k], sims_seq f64 [B, N],
    alpha_raw_seq f64 [B, N], top_vals f32 [B, seq, k])."""
    W_Q = np.asarray(W_Q, accum)
    W_K = np.asarray(W_K, accum)
    keys = _l2n(np.einsum("skd,nd->snk", W_K, np.asarray(vectors, accum)))        # 155-156
    queries = _l2n(np.einsum("skd,btd->sbtk", W_Q, np.asarray(z, accum)))        # 159-160
    al = np.asarray(aspect_logits, accum)
    w = np.exp(al - al.max())
    w = w / w.sum()                                                               # 164
    sims_w = np.einsum("s,sbtn->btn", w, np.einsum("sbtk,snk->sbtn", queries, keys))  # 163-165
    tau = float(w @ np.asarray(tau_param, accum)) if use_sigmoid else 0.0          # 168
    alpha_raw = fused_score(sims_w, lambda_sharp, tau, T, use_sigmoid)             # 168-172
    top_vals, top_idx = top_k(alpha_raw, k)                                       # 175
    top_vals = top_vals.astype(np.float32)
    alpha = normalise(top_vals)                                                   # 178
    return alpha, top_idx, sims_w.mean(axis=1), alpha_raw.mean(axis=1), top_vals  # 181


# --------------------------------------------------------------------------- low-rank assembly
def split_vectors(sel: np.ndarray, d_A: int, d_B: int, r: int):
    """assembly.py:61-63 / 110-112: pool vector = [U (d_B x r) | V (r x d_A) | b (d_B)]."""
    off_V, off_b = d_B * r, d_B * r + r * d_A
    U = sel[..., :off_V].reshape(*sel.shape[:-1], d_B, r)
    V = sel[..., off_V:off_b].reshape(*sel.shape[:-1], r, d_A)
    b = sel[..., off_b:off_b + d_B]
    return U, V, b


def lowrank_delta(h: np.ndarray, alpha: np.ndarray, idx: np.ndarray, vectors: np.ndarray,
                  d_A: int, d_B: int, r: int, accum=np.float64) -> np.ndarray:
    """assembly.py:123-127 (per-position idx): h_delta + b_delta for rows h [M, d_A].

    hV = h . V_j (r values per selected vector), h_delta = sum_j alpha_j U_j hV_j,
    b_delta = sum_j alpha_j b_j.
    """
    sel = np.asarray(vectors, dtype=accum)[idx]            # [M, k, D]
    U, V, b = split_vectors(sel, d_A, d_B, r)
    h = np.asarray(h, dtype=accum)
    a = np.asarray(alpha, dtype=accum)
    hV = np.einsum("md,mkrd->mkr", h, V)
    h_delta = np.einsum("mkr,mkir->mi", hV * a[..., None], U)
    b_delta = np.einsum("mk,mkj->mj", a, b)
    return h_delta + b_delta


def layer_norm(x: np.ndarray, scale: np.ndarray, bias: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """flax.nnx.LayerNorm over the last axis (the norm of assembly.py:52): mean and
    variance of x, (x - mean) / sqrt(var + eps) * scale + bias."""
    x = np.asarray(x, dtype=np.float64)
    mean = x.mean(axis=-1, keepdims=True)
    var = np.maximum((x * x).mean(axis=-1, keepdims=True) - mean * mean, 0.0)
    return (x - mean) / np.sqrt(var + eps) * scale + bias


def assemble_forward(h: np.ndarray, alpha: np.ndarray, idx: np.ndarray, vectors: np.ndarray,
                     W_base: np.ndarray, b_base: np.ndarray, gamma: float, ln_scale: np.ndarray,
                     ln_bias: np.ndarray, d_A: int, d_B: int, r: int, eps: float = 1e-6) -> np.ndarray:
    """WeightAssembler.__call__, per-position path (assembly.py:75-82, 84-85, 104, 110-128):
    LayerNorm(residual + gamma * (h W_base^T + b_base + h_delta + b_delta)),
    residual = h when d_A == d_B, else 0."""
    h64 = np.asarray(h, dtype=np.float64)
    base = h64 @ np.asarray(W_base, np.float64).T + np.asarray(b_base, np.float64)
    x = gamma * (base + lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r))
    if d_A == d_B:
        x = x + h64
    return layer_norm(x, ln_scale, ln_bias, eps)


def usage_ema(ema: np.ndarray, alpha: np.ndarray, idx: np.ndarray, beta: float = 0.99) -> np.ndarray:
    """trainer.py:227-233 + pool.py:52-55 (per-position idx): alpha_sum = zeros(N) with
    alpha / idx.size scatter-added at idx; ema' = beta * ema + (1 - beta) * alpha_sum."""
    alpha_sum = np.zeros(ema.shape[0], dtype=np.float64)
    np.add.at(alpha_sum, np.asarray(idx).reshape(-1),
              np.asarray(alpha, np.float64).reshape(-1) / np.asarray(idx).size)
    return beta * np.asarray(ema, np.float64) + (1.0 - beta) * alpha_sum


# --------------------------------------------------------------------------- comparator
def true_fused(q, keys, rows, idx, lambda_sharp=1.0, tau=0.0, T=1.0, use_sigmoid=False):
    """Fused score of (row, key idx) pairs in float64; idx < 0 gives -inf."""
    rows = np.asarray(rows)
    idx = np.asarray(idx)
    safe = np.where(idx >= 0, idx, 0)
    s = np.einsum("...d,...d->...", np.asarray(q, np.float64)[rows],
                  np.asarray(keys, np.float64)[safe])
    v = fused_score(s, lambda_sharp, tau, T, use_sigmoid)
    return np.where(idx >= 0, v, -np.inf)


def compare_topk(got_v, got_i, ref_v, ref_i, q, keys, lambda_sharp=1.0, tau=0.0, T=1.0,
                 use_sigmoid=False, rtol=1e-2, row_ids=None) -> list[str]:
    """Tie-tolerant top-k comparison (the tolerance rule of the parity contract).

    * values rank-wise within rtol (both lists sorted descending),
    * each returned index really has the returned value (recomputed in f64),
    * no duplicate indices, values non-increasing,
    * index sets equal except for near-ties at the k-th boundary: an index only
      in `got` must score within rtol of ref's k-th value, an index only in
      `ref` within rtol of got's k-th value.
    Returns a list of failure messages (empty = pass).
    """
    M = np.asarray(got_v).shape[0]
    rows = np.arange(M) if row_ids is None else np.asarray(row_ids)

    def true_of(r, idx):  # r: row positions in the compared arrays, idx: key indices
        return true_fused(q, keys, rows[r], idx, lambda_sharp, tau, T, use_sigmoid)

    return _compare_core(got_v, got_i, ref_v, ref_i, true_of, rtol)


def compare_topk_from_scores(got_v, got_i, ref_v, ref_i, s, lambda_sharp=1.0, tau=0.0, T=1.0,
                             use_sigmoid=False, rtol=1e-2) -> list[str]:
    """``compare_topk`` with the raw scores given: row r of ``s`` (f64 [R, N]) holds
    q[row] . keys[n] for every key n of the compared rows, so a pool too large to
    convert to f64 on the host can still be checked on sampled rows."""
    s = np.asarray(s, np.float64)

    def true_of(r, idx):
        idx = np.asarray(idx)
        safe = np.where(idx >= 0, idx, 0)
        v = fused_score(s[np.broadcast_to(r, safe.shape), safe], lambda_sharp, tau, T, use_sigmoid)
        return np.where(idx >= 0, v, -np.inf)

    return _compare_core(got_v, got_i, ref_v, ref_i, true_of, rtol)


def _compare_core(got_v, got_i, ref_v, ref_i, true_of, rtol) -> list[str]:
    got_v = np.asarray(got_v, np.float64)
    ref_v = np.asarray(ref_v, np.float64)
    got_i = np.asarray(got_i)
    ref_i = np.asarray(ref_i)
    errs: list[str] = []
    if got_v.shape != ref_v.shape or got_i.shape != ref_i.shape:
        return [f"shape mismatch {got_v.shape} vs {ref_v.shape}"]
    M, k = got_v.shape
    scale = np.maximum(np.abs(ref_v), 1e-30)
    bad = np.abs(got_v - ref_v) > rtol * scale
    if bad.any():
        r, c = np.argwhere(bad)[0]
        errs.append(f"{bad.sum()} values outside rtol={rtol}; first row {r} rank {c}: "
                    f"got {got_v[r, c]!r} ref {ref_v[r, c]!r}")
    if (np.diff(got_v, axis=1) > 0).any():
        errs.append("returned values are not sorted descending")
    srt = np.sort(got_i, axis=1)
    if (srt[:, 1:] == srt[:, :-1]).any():
        errs.append("duplicate indices in a row")
    if (got_i < 0).any():
        errs.append("negative (sentinel) index returned")
    tv = true_of(np.arange(M)[:, None], got_i)
    inc = np.abs(tv - got_v) > rtol * np.maximum(np.abs(tv), 1e-30)
    if inc.any():
        r, c = np.argwhere(inc)[0]
        errs.append(f"{inc.sum()} returned values do not match their index's true score; first "
                    f"row {r} rank {c}: returned {got_v[r, c]!r} true {tv[r, c]!r}")
    n_extra = 0
    for r in range(M):
        gs, rs = set(got_i[r].tolist()), set(ref_i[r].tolist())
        if gs == rs:
            continue
        only_g = np.array(sorted(gs - rs), dtype=np.int64)
        only_r = np.array(sorted(rs - gs), dtype=np.int64)
        vg = true_of(np.full(only_g.shape, r), only_g)
        vr = true_of(np.full(only_r.shape, r), only_r)
        if (vg < ref_v[r, -1] - rtol * abs(ref_v[r, -1])).any() or \
           (vr > got_v[r, -1] + rtol * abs(got_v[r, -1])).any():
            n_extra += 1
            if n_extra == 1:
                errs.append(f"row {r}: index sets differ beyond a near-tie at the k-th value "
                            f"(only got {only_g[:4]}, only ref {only_r[:4]})")
    return errs


def compare_rows(got, ref, rtol=1e-2) -> list[str]:
    """Row-wise closeness for [M, d] outputs: |got - ref| <= rtol * (|ref| + rms(ref row))."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if got.shape != ref.shape:
        return [f"shape mismatch {got.shape} vs {ref.shape}"]
    rms = np.sqrt(np.mean(ref * ref, axis=-1, keepdims=True)) + 1e-30
    bad = np.abs(got - ref) > rtol * (np.abs(ref) + rms)
    if bad.any():
        r = np.argwhere(bad)[0]
        return [f"{bad.sum()} elements outside rtol={rtol}; first at {tuple(r)}: "
                f"got {got[tuple(r)]!r} ref {ref[tuple(r)]!r}"]
    return []


# --------------------------------------------------------------------------- Philox
_PHILOX_M0 = np.uint64(0xD2511F53)
_PHILOX_M1 = np.uint64(0xCD9E8D57)
_PHILOX_W0 = np.uint32(0x9E3779B9)
_PHILOX_W1 = np.uint32(0xBB67AE85)
_COUNTER_TAG = 0x706F6F6C
_MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr: np.ndarray, key) -> np.ndarray:
    """Philox4x32 with 10 rounds.  ctr: uint32 [..., 4]; key: two uint32 words."""
    c = [np.asarray(ctr[..., j], dtype=np.uint64) for j in range(4)]
    k0 = np.uint32(key[0])
    k1 = np.uint32(key[1])
    for r in range(10):
        if r:
            k0 = np.uint32((int(k0) + int(_PHILOX_W0)) & 0xFFFFFFFF)
            k1 = np.uint32((int(k1) + int(_PHILOX_W1)) & 0xFFFFFFFF)
        p0 = _PHILOX_M0 * c[0]
        p1 = _PHILOX_M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & _MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _MASK32
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
    return np.stack([x.astype(np.uint32) for x in c], axis=-1)


def _unit_open(x: np.ndarray) -> np.ndarray:
    return ((x >> np.uint32(8)).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -24)


def pool_init_normal(rows: int, cols: int, seed: int, stddev: float = 1.0,
                     row_offset: int = 0) -> np.ndarray:
    """Same draws as dwa_pool_init_normal, returned as float32 (before bf16 rounding)."""
    groups = (cols + 3) // 4
    r = np.arange(rows, dtype=np.uint64)[:, None] + np.uint64(row_offset)
    g = np.arange(groups, dtype=np.uint64)[None, :]
    ctr = np.empty((rows, groups, 4), dtype=np.uint32)
    ctr[..., 0] = g.astype(np.uint32)
    ctr[..., 1] = (r & _MASK32).astype(np.uint32)
    ctr[..., 2] = (r >> np.uint64(32)).astype(np.uint32)
    ctr[..., 3] = _COUNTER_TAG
    x = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    out = np.empty((rows, groups, 4), dtype=np.float32)
    for pair in range(2):
        u1 = _unit_open(x[..., 2 * pair])
        u2 = _unit_open(x[..., 2 * pair + 1])
        rad = np.sqrt(np.float32(-2.0) * np.log(u1))
        ang = 2.0 * np.pi * u2.astype(np.float64)
        out[..., 2 * pair] = rad * np.cos(ang).astype(np.float32)
        out[..., 2 * pair + 1] = rad * np.sin(ang).astype(np.float32)
    return (out.reshape(rows, groups * 4)[:, :cols] * np.float32(stddev)).astype(np.float32)
