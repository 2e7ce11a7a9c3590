"""Multi-GPU parity: the row-sharded path (one process per GPU, NCCL) returns
the same top-k and value sums as the single-GPU path on the same pool.

Runs only when 2 or more CUDA devices are visible.  Each rank generates its
own shard with the counter-based generator, so every shard count sees the
same pool; rank 0 also runs the unsharded retrieval on its GPU as the
reference and compares.  The process group has a short timeout, so a rank
that fails ends the others' next collective with an error instead of a hang.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    from datetime import timedelta

    import torch.distributed as dist

    import computd_b200 as cb
    from oracle import dwa_oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        M, N, d, k = 1000, 96 * 1024, 256, 32
        spec = cb.ShardSpec(N, rank, world)
        keys = cb.new_normal(spec.n_local, d, seed=2, stddev=d ** -0.5, row_offset=spec.row_begin,
                             device=dev)
        values = cb.new_normal(spec.n_local, d, seed=3, row_offset=spec.row_begin, device=dev)
        queries = cb.new_normal(M, d, seed=4, device=dev)
        r = cb.Retriever(keys, values, M, k, lambda_sharp=3.0, tau=0.5, T=0.8, use_sigmoid=True)
        out, alpha, tv, ti = r(queries)
        # chip_topk (the shard_map body) must agree with the Retriever
        cv, ci = cb.chip_topk(queries, keys, k, 3.0, 0.5, 0.8, True)
        torch.cuda.synchronize()
        same_chip = bool(torch.equal(ci, ti))
        msg = "ok"
        g0 = dist.new_group([0])  # every rank takes part in group creation
        if rank == 0:
            full_k = cb.new_normal(N, d, seed=2, stddev=d ** -0.5, device=dev)
            full_v = cb.new_normal(N, d, seed=3, device=dev)
            r1 = cb.Retriever(full_k, full_v, M, k, lambda_sharp=3.0, tau=0.5, T=0.8,
                              use_sigmoid=True, group=g0)
            o1, a1, v1, i1 = r1(queries)
            torch.cuda.synchronize()
            qn = queries.float().cpu().numpy()
            kn = full_k.float().cpu().numpy()
            errs = O.compare_topk(tv.cpu().numpy(), ti.cpu().numpy(), v1.cpu().numpy(),
                                  i1.cpu().numpy(), qn, kn, 3.0, 0.5, 0.8, True, rtol=1e-2)
            if errs:
                msg = "; ".join(errs)
            elif not torch.equal(ti, i1):
                msg = "sharded indices differ from the single-GPU indices"
            else:
                errs = O.compare_rows(out.cpu().numpy(), o1.cpu().numpy(), rtol=1e-2)
                if errs:
                    msg = "; ".join(errs)
        # sharded backward: dq equal on every rank; dK/dV = this rank's rows of the full grads
        from computd_b200.autograd import retrieve
        qg = queries.clone().requires_grad_()
        kg = keys.clone().requires_grad_()
        vg = values.clone().requires_grad_()
        W = cb.new_normal(M, d, seed=9, device=dev).float()
        out_s, _, ti_s = retrieve(qg, kg, vg, k, 3.0, 0.5, 0.8, True)
        (out_s * W).sum().backward()
        if rank == 0 and msg == "ok":
            full_k = cb.new_normal(N, d, seed=2, stddev=d ** -0.5, device=dev).requires_grad_()
            full_v = cb.new_normal(N, d, seed=3, device=dev).requires_grad_()
            q1 = queries.clone().requires_grad_()
            out_1, _, ti_1 = retrieve(q1, full_k, full_v, k, 3.0, 0.5, 0.8, True, group=g0)
            (out_1 * W).sum().backward()
            torch.cuda.synchronize()
            if not torch.equal(ti_1, ti_s):
                msg = "backward: selections differ"
            else:
                def close(a, b):
                    a, b = a.float(), b.float()
                    return float((a - b).abs().max()) <= 1e-2 * float(b.abs().max().clamp_min(1e-12))
                if not close(qg.grad, q1.grad):
                    msg = "backward: dq differs from the single-GPU dq"
                elif not close(kg.grad, full_k.grad[:spec.n_local]):
                    msg = "backward: dK rows differ"
                elif not close(vg.grad, full_v.grad[:spec.n_local]):
                    msg = "backward: dV rows differ"
        # NVLink peer exchange vs the NCCL all-gather path: identical results over
        # three steps (both parity buffers, step flags reused).  Every rank runs the
        # same collective sequence whatever its own checks found.
        rp = cb.Retriever(keys, values, M, k, lambda_sharp=3.0, tau=0.5, T=0.8,
                          use_sigmoid=True, exchange="nvlink")
        rn = cb.Retriever(keys, values, M, k, lambda_sharp=3.0, tau=0.5, T=0.8,
                          use_sigmoid=True, exchange="nccl")
        same = rp.peer is not None and rn.peer is None
        for step in range(3):
            qs = cb.new_normal(M, d, seed=50 + step, device=dev)
            op, ap, vp, ip = (t.clone() for t in rp(qs))
            on, an, vn, in_ = rn(qs)
            torch.cuda.synchronize()
            # selections and scores bit for bit; the fp32 sums of P partials may be added
            # in another order than NCCL's ring (equal only up to rounding)
            same = (same and torch.equal(ip, in_) and torch.equal(vp, vn)
                    and torch.allclose(op, on, rtol=1e-5, atol=1e-5))
        st_p = rp.status()
        rp.close()
        # sharded WeightAssembler (owner-computes delta + all-reduce + LayerNorm)
        # against the unsharded one on rank 0; every rank runs the same collectives
        d_A = d_B = 64
        r_lr = 8
        D = d_B * r_lr + r_lr * d_A + d_B
        vec_l = cb.new_normal(spec.n_local, D, seed=61, stddev=0.2, row_offset=spec.row_begin,
                              device=dev)
        h = cb.new_normal(M, d_A, seed=62, device=dev)
        asm = cb.WeightAssembler(d_A, d_B, r_lr, device=dev)
        asm.W_base = cb.new_normal(d_B, d_A, seed=63, stddev=d_A ** -0.5, device=dev)
        asm.gamma = 0.8
        hm = asm(h, alpha, ti, vec_l)
        if rank == 0 and msg == "ok":
            vec_full = cb.new_normal(N, D, seed=61, stddev=0.2, device=dev)
            asm1 = cb.WeightAssembler(d_A, d_B, r_lr, device=dev)
            asm1.W_base, asm1.gamma = asm.W_base, asm.gamma
            h1 = asm1(h, alpha, ti, vec_full, group=g0)
            torch.cuda.synchronize()
            err = float((hm - h1).abs().max()) / max(float(h1.abs().max()), 1e-12)
            if err > 1e-3:
                msg = f"sharded WeightAssembler differs from the single-GPU one (rel {err:.2e})"
        # the DWA LM on the sharded pool against the same model on one GPU (rank 0),
        # both pool layouts; every rank runs the same collectives
        from computd_b200.dwa_lm import DWALM, DWALMConfig
        for r_lm in (0, 2):
            cfg = DWALMConfig(vocab=65, d_model=64, n_layers=2, n_heads=4, seq_len=64, batch=2,
                              pool_rows=8192, top_k=8, S=2, d_k=32, r=r_lm)
            lspec = cb.ShardSpec(cfg.pool_rows, rank, world)

            def pools(rows, off):
                if r_lm:
                    return None, cb.new_normal(rows, cfg.D, seed=71, stddev=0.3, row_offset=off,
                                               device=dev)
                return (cb.new_normal(rows, cfg.key_width, seed=72, stddev=cfg.key_width ** -0.5,
                                      row_offset=off, device=dev),
                        cb.new_normal(rows, cfg.d_model, seed=73, stddev=cfg.d_model ** -0.5,
                                      row_offset=off, device=dev))

            lk, lv = pools(lspec.n_local, lspec.row_begin)
            lm = DWALM(cfg, lk, lv)
            tokens = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=dev,
                                   generator=torch.Generator(device=dev).manual_seed(3))
            logits = lm(tokens)
            st_lm = lm.retriever.status()
            if rank == 0 and msg == "ok":
                fk, fv = pools(cfg.pool_rows, 0)
                lm1 = DWALM(cfg, fk, fv, group=g0)
                logits1 = lm1(tokens)
                torch.cuda.synchronize()
                err = float((logits.float() - logits1.float()).abs().max())
                scale = float(logits1.float().abs().max())
                if st_lm != 0 or not err <= 2e-2 * scale:
                    msg = f"sharded LM (r={r_lm}) differs from one GPU: {err:.3g} of {scale:.3g}"
            lm.retriever.close()
        if msg == "ok" and not same:
            msg = "nvlink exchange differs from the NCCL path"
        if msg == "ok" and st_p != 0:
            msg = f"nvlink exchange status {st_p}"

        q.put((rank, same_chip, msg, r.status()))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same_chip, msg, status in sorted(results):
        assert status == 0, f"rank {rank}: device status {status}"
        assert same_chip, f"rank {rank}: chip_topk differs from Retriever.topk"
        assert msg == "ok", f"rank {rank}: {msg}"
