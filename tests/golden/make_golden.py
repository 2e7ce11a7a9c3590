"""Generate tests/golden/dwa_golden.npz by executing the reference's own code.

The reference (computd) is JAX; JAX is not installable here, so its modules
are imported over ``jax_standin`` (NumPy restatements of jnp.dot, lax.top_k,
all_gather, shard_map, ...).  What runs is the reference's own source:

* ``src/kernels/tiled_topk.py``  ``tiled_topk_fallback``            (lines 160-176)
* ``src/model/retrieval.py``     ``MultiAspectRetrieval.pallas_hybrid_forward``
                                  with a 4-device ``shard_map``         (lines 204-343)
* ``src/model/assembly.py``      ``WeightAssembler.assemble``        (lines 47-73)
                                  ``WeightAssembler.__call__``, per-position idx
                                  with a flax-LayerNorm stand-in       (lines 75-128)
* ``src/model/pool.py``          ``VectorPool.update_ema``           (lines 52-55)
* ``src/model/retrieval.py``     ``MultiAspectRetrieval.hybrid_forward`` (lines 131-181)

Inputs are float32 arrays holding bf16-representable values (the B200 kernel
takes bf16, so both sides see identical inputs).  Run from the repository
root:  ``python tests/golden/make_golden.py --reference PATH`` (or with
``COMPUTD_REFERENCE=PATH`` in the environment).
The reference tree is read only; nothing from it is copied into the fixture
except the computed outputs.
"""
from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1]))

import jax_standin  # noqa: E402
from oracle.dwa_oracle import bf16_bits, bf16_round  # noqa: E402


def _bits(x):
    return bf16_bits(x)


def case_tiled_topk(ref_tk, name, rng, M, N, d, k, lam, tau, T, use_sigmoid, out, q_scale=1.0,
                    k_scale=None):
    """tiled_topk_fallback on C1-distributed inputs (q ~ N(0,1), keys ~ N(0,1/d))."""
    k_scale = (1.0 / np.sqrt(d)) if k_scale is None else k_scale
    q = bf16_round(rng.standard_normal((M, d), dtype=np.float32) * q_scale)
    keys = bf16_round(rng.standard_normal((N, d), dtype=np.float32) * np.float32(k_scale))
    vals, idx = ref_tk.tiled_topk_fallback(q, keys, k, np.float32(lam), np.float32(tau),
                                           np.float32(T), use_sigmoid)
    out[f"{name}/q"] = _bits(q)
    out[f"{name}/keys"] = _bits(keys)
    out[f"{name}/params"] = np.array([k, lam, tau, T, float(use_sigmoid)], dtype=np.float64)
    out[f"{name}/vals"] = np.asarray(vals, np.float32)
    out[f"{name}/idx"] = np.asarray(idx, np.int32)


def case_ties(ref_tk, rng, out):
    """Exact score ties: small-integer inputs make every dot product exact in fp32,
    and duplicated key rows tie; lax.top_k must put the lower index first."""
    M, N, d, k = 64, 600, 64, 12
    q = rng.integers(-2, 3, size=(M, d)).astype(np.float32) * np.float32(0.25)
    base = rng.integers(-2, 3, size=(N // 4, d)).astype(np.float32) * np.float32(0.25)
    keys = np.concatenate([base, base[::-1], base, base[::2], base[1::2]], axis=0)[:N]
    perm = rng.permutation(N)
    keys = np.ascontiguousarray(keys[perm])
    vals, idx = ref_tk.tiled_topk_fallback(q, keys, k, np.float32(1.0), np.float32(0.0),
                                           np.float32(8.0), False)
    out["ties/q"] = _bits(q)
    out["ties/keys"] = _bits(keys)
    out["ties/params"] = np.array([k, 1.0, 0.0, 8.0, 0.0], dtype=np.float64)
    out["ties/vals"] = np.asarray(vals, np.float32)
    out["ties/idx"] = np.asarray(idx, np.int32)


def case_sharded(ref_tk, ref_ret, ref_asm, rng, out, n_chips=4):
    """pallas_hybrid_forward over a 4-device mesh + WeightAssembler.assemble."""
    B, seq, d_A, S, d_k, k = 2, 48, 32, 2, 32, 8
    d_B, r = 8, 2
    N = n_chips * 250
    D = d_B * r + r * d_A + d_B  # 88: U, V and b blocks of each pool vector
    lam, T, use_sigmoid = 5.0, 0.8, True

    recorded = {"q": None, "keys": [None] * n_chips, "local": [None] * n_chips}
    orig = ref_tk.tiled_topk_fallback

    def recording_fallback(queries, keys, k_max, lambda_sharp, tau, T_, use_sig):
        # bf16 inputs, as the B200 kernel receives them
        qb = bf16_round(np.asarray(queries, np.float32))
        kb = bf16_round(np.asarray(keys, np.float32))
        chip = int(jax_standin._ctx.index)
        recorded["q"] = qb
        recorded["keys"][chip] = kb
        recorded["tau"] = float(tau)
        res = orig(qb, kb, k_max, lambda_sharp, tau, T_, use_sig)
        recorded["local"][chip] = res
        return res

    ref_tk.tiled_topk_fallback = recording_fallback
    try:
        self = types.SimpleNamespace()
        self.S, self.d_k, self.N = S, d_k, N
        self.W_Q = types.SimpleNamespace(value=(rng.standard_normal((S, d_k, d_A)) * d_A ** -0.5).astype(np.float32))
        self.W_K = types.SimpleNamespace(value=(rng.standard_normal((S, d_k, D)) * D ** -0.5).astype(np.float32))
        self.aspect_logits = types.SimpleNamespace(value=rng.standard_normal(S).astype(np.float32))
        self.tau = types.SimpleNamespace(value=(0.1 * rng.standard_normal(S)).astype(np.float32))
        z = rng.standard_normal((B, seq, d_A)).astype(np.float32)
        vectors = bf16_round(rng.standard_normal((N, D)).astype(np.float32) * np.float32(0.02 * 50))
        mesh = jax_standin.Mesh(np.arange(n_chips), ("tp",))
        alpha, top_idx, sims_seq, alpha_raw_seq = ref_ret.MultiAspectRetrieval.pallas_hybrid_forward(
            self, z, vectors, k, T, lam, use_sigmoid, tp_axis="tp", mesh=mesh)
    finally:
        ref_tk.tiled_topk_fallback = orig

    asm = types.SimpleNamespace(d_A=d_A, d_B=d_B, r=r, _off_V=d_B * r, _off_b=d_B * r + r * d_A,
                                _end_b=d_B * r + r * d_A + d_B)
    asm.W_base = types.SimpleNamespace(value=np.zeros((d_B, d_A), np.float32))
    asm.b_base = types.SimpleNamespace(value=np.zeros(d_B, np.float32))
    W, b = ref_asm.WeightAssembler.assemble(asm, alpha, top_idx, vectors)

    out["sharded/q"] = _bits(recorded["q"])
    out["sharded/keys"] = _bits(np.concatenate(recorded["keys"], axis=0))
    out["sharded/params"] = np.array([k, lam, recorded["tau"], T, float(use_sigmoid)], dtype=np.float64)
    out["sharded/n_chips"] = np.array(n_chips)
    out["sharded/alpha"] = np.asarray(alpha, np.float32).reshape(B * seq, k)
    out["sharded/idx"] = np.asarray(top_idx, np.int32).reshape(B * seq, k)
    out["sharded/local_vals"] = np.stack([np.asarray(v, np.float32) for v, _ in recorded["local"]])
    out["sharded/local_idx"] = np.stack([np.asarray(i, np.int32) for _, i in recorded["local"]])
    out["sharded/vectors"] = _bits(vectors)
    out["sharded/b_slice"] = np.array([asm._off_b, asm._end_b])
    out["sharded/b_delta"] = np.asarray(b, np.float32).reshape(B * seq, d_B)
    # raw inputs and aux outputs of pallas_hybrid_forward itself
    out["sharded/z"] = z.astype(np.float32)
    out["sharded/W_Q"] = self.W_Q.value
    out["sharded/W_K"] = self.W_K.value
    out["sharded/aspect_logits"] = self.aspect_logits.value
    out["sharded/tau_param"] = self.tau.value
    out["sharded/sims_seq"] = np.asarray(sims_seq, np.float32)
    out["sharded/alpha_raw_seq"] = np.asarray(alpha_raw_seq, np.float32)


def case_hybrid(ref_ret, rng, out, name, B, seq, d_A, S, d_k, k, N, D, lam, T, use_sigmoid):
    """MultiAspectRetrieval.hybrid_forward (retrieval.py:131-181), single device:
    per-position top-k over all N with the aspect-weighted score, plus the seq
    means of sims and of the fused scores.  Parameters and inputs hold
    bf16-representable values (the reference's parameter dtype); the top_k
    call is recorded for its values."""
    self = types.SimpleNamespace()
    self.S, self.d_k, self.N = S, d_k, N
    self.W_Q = types.SimpleNamespace(value=bf16_round(rng.standard_normal((S, d_k, d_A)) * d_A ** -0.5))
    self.W_K = types.SimpleNamespace(value=bf16_round(rng.standard_normal((S, d_k, D)) * D ** -0.5))
    self.aspect_logits = types.SimpleNamespace(value=rng.standard_normal(S).astype(np.float32))
    self.tau = types.SimpleNamespace(value=(0.1 * rng.standard_normal(S)).astype(np.float32))
    z = bf16_round(rng.standard_normal((B, seq, d_A)).astype(np.float32))
    vectors = bf16_round(rng.standard_normal((N, D)).astype(np.float32))
    recorded = {}
    lax = ref_ret.jax.lax
    orig = lax.top_k

    def recording_top_k(x, kk):
        res = orig(x, kk)
        recorded["top_vals"] = np.asarray(res[0], np.float32)
        return res

    lax.top_k = recording_top_k
    try:
        alpha, top_idx, sims_seq, alpha_raw_seq = ref_ret.MultiAspectRetrieval.hybrid_forward(
            self, z, vectors, k, T, lam, use_sigmoid)
    finally:
        lax.top_k = orig
    out[f"{name}/dims"] = np.array([B, seq, d_A, S, d_k, k, N, D])
    out[f"{name}/params"] = np.array([lam, T, float(use_sigmoid)], dtype=np.float64)
    out[f"{name}/z"] = _bits(z)
    out[f"{name}/vectors"] = _bits(vectors)
    out[f"{name}/W_Q"] = _bits(self.W_Q.value)
    out[f"{name}/W_K"] = _bits(self.W_K.value)
    out[f"{name}/aspect_logits"] = self.aspect_logits.value
    out[f"{name}/tau_param"] = self.tau.value
    out[f"{name}/alpha"] = np.asarray(alpha, np.float32)
    out[f"{name}/idx"] = np.asarray(top_idx, np.int32)
    out[f"{name}/top_vals"] = recorded["top_vals"]
    out[f"{name}/sims_seq"] = np.asarray(sims_seq, np.float32)
    out[f"{name}/alpha_raw_seq"] = np.asarray(alpha_raw_seq, np.float32)


def case_assembler(ref_asm, ref_pool, rng, out, name, d_A, d_B, r):
    """WeightAssembler.__call__ on per-position (hybrid) idx, non-zero W_base / b_base /
    gamma / LayerNorm parameters, pool rows wider than U|V|b; then VectorPool.update_ema
    on the per-position usage scatter."""
    B, seq, k, N = 2, 24, 6, 300
    D = d_B * r + r * d_A + d_B + 8
    vectors = bf16_round((rng.standard_normal((N, D)) * 0.3).astype(np.float32))
    h = bf16_round(rng.standard_normal((B, seq, d_A)).astype(np.float32))
    raw = np.exp(rng.standard_normal((B, seq, k))).astype(np.float32)
    alpha = (raw / (raw.sum(-1, keepdims=True) + np.float32(1e-8))).astype(np.float32)
    idx = np.stack([rng.choice(N, size=k, replace=False) for _ in range(B * seq)])
    idx = idx.reshape(B, seq, k).astype(np.int32)
    W_base = bf16_round((rng.standard_normal((d_B, d_A)) * d_A ** -0.5).astype(np.float32))
    b_base = bf16_round((0.1 * rng.standard_normal(d_B)).astype(np.float32))
    gamma = np.float32(0.7)
    ln_scale = (1.0 + 0.1 * rng.standard_normal(d_B)).astype(np.float32)
    ln_bias = (0.1 * rng.standard_normal(d_B)).astype(np.float32)
    asm = types.SimpleNamespace(d_A=d_A, d_B=d_B, r=r, _off_V=d_B * r, _off_b=d_B * r + r * d_A,
                                _end_b=d_B * r + r * d_A + d_B)
    asm.W_base = types.SimpleNamespace(value=W_base)
    asm.b_base = types.SimpleNamespace(value=b_base)
    asm.gamma = types.SimpleNamespace(value=gamma)
    asm.norm = jax_standin.LayerNorm(d_B, scale=ln_scale, bias=ln_bias)
    h_mid = ref_asm.WeightAssembler.__call__(asm, h, alpha, idx, vectors)
    out[f"{name}/dims"] = np.array([d_A, d_B, r, D])
    out[f"{name}/vectors"] = _bits(vectors)
    out[f"{name}/h"] = _bits(h.reshape(B * seq, d_A))
    out[f"{name}/alpha"] = alpha.reshape(B * seq, k)
    out[f"{name}/idx"] = idx.reshape(B * seq, k)
    out[f"{name}/W_base"] = W_base
    out[f"{name}/b_base"] = b_base
    out[f"{name}/gamma"] = np.array(gamma)
    out[f"{name}/ln_scale"] = ln_scale
    out[f"{name}/ln_bias"] = ln_bias
    out[f"{name}/h_mid"] = np.asarray(h_mid, np.float32).reshape(B * seq, d_B)
    # usage EMA: trainer.py:227-233 scatter restated here, pool.py:52-55 executed
    ema0 = np.abs(rng.standard_normal(N)).astype(np.float32) * 0.01
    alpha_sum = np.zeros(N, np.float32)
    np.add.at(alpha_sum, idx.reshape(-1), alpha.reshape(-1) / np.float32(idx.size))
    pool = types.SimpleNamespace(ema_usage=types.SimpleNamespace(value=ema0.copy()))
    ref_pool.VectorPool.update_ema(pool, alpha_sum, 0.99)
    out[f"{name}/ema0"] = ema0
    out[f"{name}/ema1"] = np.asarray(pool.ema_usage.value, np.float32)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("COMPUTD_REFERENCE"),
                    help="path of the reference checkout, read only (default: the "
                         "COMPUTD_REFERENCE environment variable)")
    ap.add_argument("--out", default=str(HERE / "dwa_golden.npz"))
    args = ap.parse_args(argv)
    if not args.reference or not os.path.isdir(os.path.join(args.reference, "src")):
        ap.error("give the reference checkout with --reference PATH or COMPUTD_REFERENCE")

    jax_standin.install()
    sys.path.insert(0, args.reference)
    from src.kernels import tiled_topk as ref_tk  # noqa: E402  (reference code)
    from src.model import assembly as ref_asm  # noqa: E402
    from src.model import pool as ref_pool  # noqa: E402
    from src.model import retrieval as ref_ret  # noqa: E402

    rng = np.random.default_rng(20261201)
    out: dict[str, np.ndarray] = {}
    case_tiled_topk(ref_tk, "c1_exp", rng, 128, 2000, 128, 16, 1.0, 0.0, 1.0, False, out)
    case_tiled_topk(ref_tk, "c1_gate", rng, 96, 1500, 128, 16, 5.0, 0.5, 0.7, True, out)
    case_tiled_topk(ref_tk, "odd", rng, 33, 777, 40, 5, 2.0, -0.25, 1.3, True, out)
    case_ties(ref_tk, rng, out)
    case_sharded(ref_tk, ref_ret, ref_asm, rng, out)
    case_assembler(ref_asm, ref_pool, rng, out, "asm_eq", 48, 48, 4)
    case_assembler(ref_asm, ref_pool, rng, out, "asm_ne", 40, 24, 8)
    # appended after the cases above so that their arrays stay as they were
    case_hybrid(ref_ret, rng, out, "hybrid_gate", 2, 64, 48, 3, 32, 8, 700, 96, 4.0, 0.9, True)
    case_hybrid(ref_ret, rng, out, "hybrid_exp", 3, 40, 40, 2, 64, 12, 500, 72, 1.0, 0.7, False)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
