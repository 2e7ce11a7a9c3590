"""GPU: the DWA LM forward (the retrieval path's call site) runs, and the
retrieval inside a block matches the oracle for the queries that block built."""
import numpy as np
import pytest
import torch

from oracle import dwa_oracle as O

pytestmark = pytest.mark.gpu


def test_dwa_lm_forward_and_block_retrieval():
    import computd_b200 as cb
    from computd_b200.dwa_lm import DWALM, DWALMConfig

    dev = torch.device("cuda", 0)
    cfg = DWALMConfig(vocab=65, d_model=128, n_layers=2, n_heads=4, seq_len=64, batch=3,
                      pool_rows=8192, top_k=16)
    keys = cb.new_normal(cfg.pool_rows, cfg.d_model, seed=11, stddev=cfg.d_model ** -0.5, device=dev)
    values = cb.new_normal(cfg.pool_rows, cfg.d_model, seed=12, stddev=cfg.d_model ** -0.5, device=dev)
    model = DWALM(cfg, keys, values)
    captured = {}

    def grab(mod, inp, out):
        captured.setdefault("z", out.detach().clone())

    h = model.blocks[0].query_proj.register_forward_hook(grab)
    tokens = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=dev)
    logits = model(tokens)
    h.remove()
    torch.cuda.synchronize()
    assert logits.shape == (cfg.batch, cfg.seq_len, cfg.vocab)
    assert bool(torch.isfinite(logits).all())
    z = captured["z"].reshape(-1, cfg.d_model)
    r = cb.Retriever(keys, values, cfg.tokens, cfg.top_k)
    out, alpha, tv, ti = r(z)
    torch.cuda.synchronize()
    qn, kn, vn = z.float().cpu().numpy(), keys.float().cpu().numpy(), values.float().cpu().numpy()
    rv, ri = O.tiled_topk(qn, kn, cfg.top_k)
    assert O.compare_topk(tv.cpu().numpy(), ti.cpu().numpy(), rv, ri, qn, kn, rtol=1e-2) == []
    want = O.weighted_sum(O.normalise(tv.cpu().numpy()), ti.cpu().numpy(), vn)
    assert O.compare_rows(out.cpu().numpy(), want, rtol=1e-2) == []


def test_dwa_lm_graph_replay_matches_eager():
    import computd_b200 as cb
    from computd_b200.dwa_lm import DWALM, DWALMConfig, GraphedForward

    dev = torch.device("cuda", 0)
    cfg = DWALMConfig(vocab=65, d_model=128, n_layers=3, n_heads=4, seq_len=64, batch=2,
                      pool_rows=4096, top_k=8)
    keys = cb.new_normal(cfg.pool_rows, cfg.d_model, seed=21, stddev=cfg.d_model ** -0.5, device=dev)
    values = cb.new_normal(cfg.pool_rows, cfg.d_model, seed=22, stddev=cfg.d_model ** -0.5, device=dev)
    model = DWALM(cfg, keys, values)
    t1 = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=dev)
    t2 = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=dev)
    eager1, eager2 = model(t1).clone(), model(t2).clone()
    gf = GraphedForward(model, t1)
    g1 = gf(t1).clone()
    g2 = gf(t2).clone()
    torch.cuda.synchronize()
    torch.testing.assert_close(g1, eager1, rtol=0, atol=0)
    torch.testing.assert_close(g2, eager2, rtol=0, atol=0)
    assert model.retriever.status() == 0
