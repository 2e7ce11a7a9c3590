"""GPU: the DWA LM forward (the retrieval path's call site) runs, and one
block's pieces match the oracle on the inputs that block built:

* the packed aspect queries -> fused score + top-k (oracle tiled_topk /
  compare_topk),
* r > 0 (the reference's [U | V | b] pool layout): the block's packed keys
  from the tcgen05 projection against fp32 torch, and the block output against
  the oracle's WeightAssembler (assemble_forward, assembly.py:75-128) on the
  block's own alpha / idx,
* r == 0 (value rows): the block output against the same formula with the
  value rows as the b vectors,
* CUDA-graph replay of the whole forward equal to eager, bit for bit.
"""
import numpy as np
import pytest
import torch

from oracle import dwa_oracle as O

pytestmark = pytest.mark.gpu


def _model(cfg, seed):
    import computd_b200 as cb
    from computd_b200.dwa_lm import DWALM

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if cfg.r > 0:
        vectors = cb.new_normal(cfg.pool_rows, cfg.D, seed=seed, stddev=0.3, device=dev)
        return DWALM(cfg, None, vectors), None, vectors
    keys = cb.new_normal(cfg.pool_rows, cfg.key_width, seed=seed, stddev=cfg.key_width ** -0.5,
                         device=dev)
    values = cb.new_normal(cfg.pool_rows, cfg.d_model, seed=seed + 1,
                           stddev=cfg.d_model ** -0.5, device=dev)
    return DWALM(cfg, keys, values), keys, values


def _capture_block0(model, tokens):
    """Run the forward, recording block 0's input to query_proj (h after the
    attention), its packed queries and its output."""
    blk = model.blocks[0]
    rec = {}
    h1 = blk.query_proj.register_forward_hook(
        lambda m, inp, out: rec.setdefault("h", inp[0].detach().clone()))
    h2 = blk.register_forward_hook(lambda m, inp, out: rec.setdefault("out", out.detach().clone()))
    orig = blk.queries

    def queries(z):
        q, w = orig(z)
        rec.setdefault("q", q.detach().clone())
        rec.setdefault("w", w.detach().clone())
        return q, w

    blk.queries = queries
    try:
        logits = model(tokens)
    finally:
        blk.queries = orig
        h1.remove()
        h2.remove()
    torch.cuda.synchronize()
    return logits, rec


# (r, pool rows): value rows; [U | V | b] rows read per token (192 tokens x 8 over
# 4096 rows); [U | V | b] rows shared by ~6 tokens each, so the assembler takes
# the row-stationary path
@pytest.mark.parametrize("r,pool", [(0, 4096), (2, 4096), (2, 256)])
def test_dwa_lm_block_matches_oracle(r, pool):
    import computd_b200 as cb
    from computd_b200.dwa_lm import DWALMConfig

    cfg = DWALMConfig(vocab=65, d_model=64, n_layers=2, n_heads=4, seq_len=64, batch=3,
                      pool_rows=pool, top_k=8, S=2, d_k=32, r=r)
    model, keys, pool = _model(cfg, seed=11 + r)
    tokens = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=pool.device,
                           generator=torch.Generator(device=pool.device).manual_seed(r))
    logits, rec = _capture_block0(model, tokens)
    assert logits.shape == (cfg.batch, cfg.seq_len, cfg.vocab)
    assert bool(torch.isfinite(logits).all())
    blk = model.blocks[0]
    if r > 0:
        # this block's keys, projected from the pool vectors by the tcgen05 kernel
        keys = cb.project_keys_packed(pool, blk.retrieval.W_K, rec["w"])
        ks = torch.einsum("skd,nd->nsk", blk.retrieval.W_K.float(), pool.float())
        ks = ks / (ks.norm(dim=-1, keepdim=True) + 1e-8) * rec["w"].sqrt()[None, :, None]
        want = ks.reshape(cfg.pool_rows, -1)
        assert float((keys.float() - want).abs().max()) <= 1e-2 * float(want.abs().max())
    q = rec["q"]
    ret = cb.Retriever(keys, None, cfg.tokens, cfg.top_k)
    _, alpha, tv, ti = ret(q)
    torch.cuda.synchronize()
    qn, kn = q.float().cpu().numpy(), keys.float().cpu().numpy()
    rv, ri = O.tiled_topk(qn, kn, cfg.top_k)
    assert O.compare_topk(tv.cpu().numpy(), ti.cpu().numpy(), rv, ri, qn, kn, rtol=1e-2) == []
    # the block output: WeightAssembler on the block's own selection
    asm = blk.assembler
    h = rec["h"].reshape(cfg.tokens, cfg.d_model)
    want = O.assemble_forward(h.float().cpu().numpy(), alpha.cpu().numpy(), ti.cpu().numpy(),
                              pool.float().cpu().numpy(), asm.W_base.float().cpu().numpy(),
                              asm.b_base.float().cpu().numpy(), asm.gamma,
                              asm.norm_scale.cpu().numpy(), asm.norm_bias.cpu().numpy(),
                              cfg.d_model, cfg.d_model, cfg.r)
    got = rec["out"].reshape(cfg.tokens, cfg.d_model).float().cpu().numpy()
    assert O.compare_rows(got, want, rtol=2e-2) == []


@pytest.mark.parametrize("r,pool", [(0, 4096), (2, 4096), (2, 256)])
def test_dwa_lm_graph_replay_matches_eager(r, pool):
    from computd_b200.assembler import _rows_path_fits
    from computd_b200.dwa_lm import DWALMConfig, GraphedForward

    cfg = DWALMConfig(vocab=65, d_model=128, n_layers=3, n_heads=4, seq_len=64, batch=2,
                      pool_rows=pool, top_k=8, S=4, d_k=32, r=r)
    if r > 0:  # the parametrisation covers both assembly paths
        assert _rows_path_fits(cfg.tokens, cfg.top_k, pool, cfg.d_model, cfg.d_model, r) == (
            pool == 256)
    model, _, pool = _model(cfg, seed=21 + r)
    dev = pool.device
    g = torch.Generator(device=dev).manual_seed(5)
    t1 = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=dev, generator=g)
    t2 = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=dev, generator=g)
    eager1, eager2 = model(t1).clone(), model(t2).clone()
    gf = GraphedForward(model, t1)
    g1 = gf(t1).clone()
    g2 = gf(t2).clone()
    torch.cuda.synchronize()
    torch.testing.assert_close(g1, eager1, rtol=0, atol=0)
    torch.testing.assert_close(g2, eager2, rtol=0, atol=0)
    assert model.retriever.status() == 0
