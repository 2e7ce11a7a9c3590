"""Benchmark of the DWA retrieval hot path on B200.

Workload (the op-at-scale configuration): queries [8192, 1024] bf16 ~N(0,1);
pool keys [1,048,576, 1024] bf16 ~N(0, 1/1024) and values ~N(0,1) (2 GiB
each, resident in HBM); top-k = 64, fp32 accumulate, softmax over the k
scores (no gate), weighted sum of the gathered value rows -> [8192, 1024] f32.
One step = one retrieval of all 8192 queries.  Inputs are synthetic (seeded
counter-based generator on the device).

Multi-GPU (torchrun, one process per GPU, NCCL): the same pool is row-sharded
over the N ranks (strong scaling): each rank runs the fused score + top-k on
its shard, the per-rank candidates are all-gathered over NVLink and merged on
the device, each rank sums the value rows it owns and one all-reduce combines
them.  Time = max over ranks of the CUDA-event step time.

Reported: queries/s (value, device-resident inputs), e2e queries/s through the
public API with pinned host buffers (H2D of queries + D2H of out/alpha/idx
inside the timed region), the fused kernel's roofline fraction, the CPU
baseline (NumPy restatement on the host cores, bounded sample), clocks.

``--impl reference`` times the reference's CPU path restated in NumPy
(oracle/dwa_oracle.py) on the host cores on a bounded sample of the same
workload and prints the same JSON line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (M queries, N pool rows, d, k, use_sigmoid)
    "op_at_scale": dict(M=8192, N=1 << 20, d=1024, k=64, use_sigmoid=False,
                        desc="queries [8192,1024] bf16 ~N(0,1); pool 1,048,576x1024 bf16 keys "
                             "~N(0,1/1024), values ~N(0,1); top-k 64; softmax-weighted value sum"),
    "profile_small": dict(M=8192, N=131072, d=1024, k=64, use_sigmoid=False,
                          desc="profiling case: queries [8192,1024]; pool 131,072x1024 (256 MiB "
                               "keys, larger than L2); top-k 64"),
    "lm_small_layer": dict(M=4096, N=65536, d=384, k=32, use_sigmoid=False,
                           desc="small DWA LM, one layer's retrieval: 16x256 tokens against a "
                                "65,536x384 pool, top-k 32"),
    "lm1b_shard8": dict(M=16384, N=524288, d=2048, k=64, use_sigmoid=False,
                        desc="1B-scale DWA LM, one layer's retrieval on one GPU of 8: 8x2048 "
                             "tokens against a 524,288x2048 shard (4,194,304 rows / 8), top-k 64"),
    "lm7b_shard8": dict(M=16384, N=2097152, d=4096, k=128, use_sigmoid=False,
                        desc="7B-scale DWA LM, one layer's retrieval on one GPU of 8: 4x4096 "
                             "tokens against a 2,097,152x4096 shard (16,777,216 rows / 8), top-k 128"),
    "op_16m": dict(M=16384, N=1 << 24, d=4096, k=128, use_sigmoid=False,
                   desc="the 16M-entry pool of the 7B layout: queries [16384,4096] bf16; pool "
                        "16,777,216x4096 bf16 keys ~N(0,1/4096), values ~N(0,1) (256 GiB in all: "
                        "2 or more GPUs); top-k 128; softmax-weighted value sum"),
    "c1_op": dict(M=2048, N=16384, d=128, k=16, use_sigmoid=False,
                  desc="queries [2048,128]; pool [16384,128]; top-k 16; softmax-weighted sum"),
}
METRIC = "fused score+top-k retrieval queries/s"

# dram__bytes_read.sum + dram__bytes_write.sum of one full-size launch of the
# fused score + top-k kernel, from a separate ncu capture of the same workload
# (one pass, after the plain command exited 0).  External evidence, not
# measured by the run that prints it; the profile file holds the command.
NCU_TRAFFIC = {
    "op_at_scale": {"bytes_per_launch": 3042590000,
                    "source": "profiles/score_topk_op_at_scale.md (ncu, one full-size launch)",
                    "captured": "2026-12-02"},
}


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["bf16_tflops_sustained"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""
        return False

    def summary(self):
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU legs
def cpu_sample(keys_rows_fn, n_total, d, k, q_host, use_sigmoid, chunk_rows=131072):
    """NumPy restatement of the reference path for the sampled queries against
    the whole pool, streamed in chunks: scores, fused score, running top-k,
    normalisation, gather + weighted sum.  Returns seconds spent on CPU work."""
    import numpy as np

    from oracle import dwa_oracle as O

    t_cpu = 0.0
    best_v = best_i = None
    for r0 in range(0, n_total, chunk_rows):
        kf = keys_rows_fn(r0, min(n_total, r0 + chunk_rows))  # float32 [rows, d], untimed fetch
        t0 = time.perf_counter()
        s = q_host @ kf.T
        v = O.fused_score(s, 1.0, 0.0, 1.0, use_sigmoid)
        tv, ti = O.top_k(v, k)
        ti = ti + r0
        if best_v is None:
            best_v, best_i = tv, ti
        else:
            best_v, sel = O.top_k(np.concatenate([best_v, tv], 1), k)
            best_i = np.take_along_axis(np.concatenate([best_i, ti], 1), sel, 1)
        t_cpu += time.perf_counter() - t0
    t0 = time.perf_counter()
    alpha = O.normalise(best_v)
    t_cpu += time.perf_counter() - t0
    return t_cpu, alpha, best_i


def _jax_probe() -> str:
    """Whether the reference's own runtime (JAX) exists on this host."""
    try:
        import jax  # noqa: F401

        return f"jax {jax.__version__} importable (the reference source is not on this host)"
    except Exception:
        return "absent"


def run_reference(args, wl):
    """--impl reference: NumPy restatement of the reference's CPU path, host cores.

    Each step scores ``--cpu-queries`` sampled queries against a contiguous
    slice of the pool sized so that all warm-up + timed steps end in about
    ``--reference-budget-s`` seconds; the per-step time is scaled to the whole
    pool linearly in pool rows (the scan's cost is proportional to the rows it
    reads), so the line reports full-pool queries/s."""
    import numpy as np

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = len(os.sched_getaffinity(0))
    M, N, d, k = wl["M"], wl["N"], wl["d"], wl["k"]
    mq = args.cpu_queries
    rng = np.random.default_rng(0)
    from oracle import dwa_oracle as O

    def make_rows(n):
        keys = O.bf16_round(rng.standard_normal((n, d), dtype=np.float32) / np.float32(np.sqrt(d)))
        values = O.bf16_round(rng.standard_normal((n, d), dtype=np.float32))
        return keys, values

    def step(keys, values):
        q = O.bf16_round(rng.standard_normal((mq, d), dtype=np.float32))
        t_cpu, alpha, idx = cpu_sample(lambda a, b: keys[a:b], keys.shape[0], d, k, q,
                                       wl["use_sigmoid"])
        t0 = time.perf_counter()
        O.weighted_sum(alpha, idx, values, accum=np.float32)
        return t_cpu + time.perf_counter() - t0

    # calibrate on a small slice, then size the slice of the timed steps
    n_cal = min(N, max(k, 65536))
    keys, values = make_rows(n_cal)
    t_cal = step(keys, values) * N / n_cal
    n_steps = args.warmup + args.steps
    frac = min(1.0, args.reference_budget_s / max(1e-9, n_steps * t_cal))
    n_s = int(min(N, max(k, frac * N)))
    t0 = time.perf_counter()
    keys, values = make_rows(n_s)   # pool sample generated once on the host, untimed
    gen_s = time.perf_counter() - t0
    step_times = []
    for i in range(n_steps):
        t = step(keys, values)
        if i >= args.warmup:
            step_times.append(t * N / n_s)
    per_step = sum(step_times) / len(step_times)
    qps = mq / per_step
    sample = (f"{mq} queries per step against a {n_s}-row slice of the {N}-row pool, time scaled "
              f"to the full pool linearly in rows (NumPy restatement of tiled_topk_fallback + "
              f"normalise + gather-sum; pool slice generation {gen_s:.1f}s untimed)")
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (bf16-valued inputs)", "data": "synthetic",
        "config": {"workload": args.workload, "M": M, "N": N, "d": d, "k": k,
                   "desc": wl["desc"], "sample_queries_per_step": mq, "sample_pool_rows": n_s},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "jax": _jax_probe(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- GPU arm
def run_ours(args, wl):
    import torch
    import torch.distributed as dist

    import computd_b200 as cb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cb.load_library()

    M, N, d, k = wl["M"], wl["N"], wl["d"], wl["k"]
    spec = cb.ShardSpec(N, rank, world)
    keys = cb.new_normal(spec.n_local, d, seed=2, stddev=d ** -0.5, row_offset=spec.row_begin,
                         device=dev)
    values = cb.new_normal(spec.n_local, d, seed=3, stddev=1.0, row_offset=spec.row_begin,
                           device=dev)
    queries = [cb.new_normal(M, d, seed=100 + i, stddev=1.0, device=dev) for i in range(2)]
    r = cb.Retriever(keys, values, M, k, use_sigmoid=wl["use_sigmoid"], group=group)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    # ------------------------------------------------ device-resident timing
    for i in range(args.warmup):
        r(queries[i % 2])
    barrier()
    n_ph = 6  # start | local score+top-k | exchange | merge | gather | reduce
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ph)] for _ in range(args.steps)]
    with ClockSampler(local_rank) as clocks:
        barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record()
        for i in range(args.steps):
            e = ev[i]
            e[0].record()
            r.topk_local(queries[i % 2])     # fused kernel + split merge on this rank
            e[1].record()
            r.exchange()                     # all-gather of [M, k] candidates (N > 1)
            e[2].record()
            r.merge()                        # global top-k merge (N > 1)
            e[3].record()
            r.gather()                       # alpha + owner-computes gathered sum
            e[4].record()
            r.reduce()                       # all-reduce of the partial sums (N > 1)
            e[5].record()
        t_end.record()
        barrier()
    status = r.status()
    total_ms = t_start.elapsed_time(t_end)
    phase_ms = [sum(e[j].elapsed_time(e[j + 1]) for e in ev) / args.steps for j in range(n_ph - 1)]
    t = torch.tensor([total_ms] + phase_ms, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t[0])
    phases = dict(zip(["score_topk_local", "exchange", "merge", "gather", "reduce"],
                      [round(float(x), 4) for x in t[1:]]))
    topk_avg_ms = phases["score_topk_local"]
    ms_per_step = total_ms / args.steps

    # ------------------------------------------------ end to end (host buffers)
    # The queries arrive in pinned host memory at rank 0, are copied to its GPU
    # and broadcast over NVLink to the other ranks; the replicated result
    # (out, alpha, top_idx) is read back to pinned host memory at rank 0.  The
    # public HostPipeline overlaps a batch's copies with its neighbours'
    # kernels; every step still uploads its own queries and reads back its
    # own result inside the timed region.
    pipe = cb.HostPipeline(keys, values, M, k, use_sigmoid=wl["use_sigmoid"], group=group)
    q_host = [queries[i].cpu().pin_memory() for i in range(2)]
    out_host = [torch.empty((M, d), dtype=torch.float32).pin_memory() for _ in range(2)]
    alpha_host = [torch.empty((M, k), dtype=torch.float32).pin_memory() for _ in range(2)]
    idx_host = [torch.empty((M, k), dtype=torch.int32).pin_memory() for _ in range(2)]

    def e2e_step(i):
        b = i % 2
        pipe.submit(q_host[b] if rank == 0 else None, out_host[b], alpha_host[b], idx_host[b])

    for i in range(args.warmup):
        e2e_step(i)
    pipe.synchronize()
    barrier()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record()
    for i in range(args.steps):
        e2e_step(i)
    pipe.join()
    e_end.record()
    barrier()
    status = max(status, pipe.status())
    te = torch.tensor([e_start.elapsed_time(e_end)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te[0]) / args.steps
    h2d = q_host[0].numel() * q_host[0].element_size()
    d2h = (out_host[0].numel() * 4 + alpha_host[0].numel() * 4 + idx_host[0].numel() * 4)
    del pipe

    # ------------------------------------------------ roofline of the fused kernel
    burst, sustained, hbm, peak_src = _peaks()
    n_local = spec.n_local
    flops = 2.0 * M * n_local * d
    achieved_tflops = flops / (topk_avg_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved_tflops, "peak": burst,
                "unit": "TFLOP/s", "frac": achieved_tflops / burst,
                "frac_of_sustained": achieved_tflops / sustained,
                "peak_source": f"{peak_src} bf16 dense burst (MEASURED_PEAKS.json)",
                "kernel": "score_topk_kernel + split merge (dwa_score_topk) on this GPU's shard",
                "flops_per_launch": flops, "ms_per_launch": topk_avg_ms,
                # DRAM bytes are not measurable inside a timed run: null here, and the
                # figure of a separate ncu capture of this workload, when one exists, is
                # reported beside it as external evidence with where it came from
                "traffic": None,
                "traffic_external": NCU_TRAFFIC.get(args.workload) if world == 1 else None,
                "algorithmic_bytes_per_launch": 2.0 * n_local * d + 2.0 * M * d + 8.0 * M * k}

    line = {
        "metric": METRIC, "value": M / (ms_per_step * 1e-3), "unit": "queries/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 in, f32 accumulate", "data": "synthetic",
        "config": {"workload": args.workload, "M": M, "N": N, "d": d, "k": k,
                   "n_local": n_local, "desc": wl["desc"],
                   "parallelism": f"pool rows sharded x{world}" if world > 1 else "single GPU",
                   "l2": (f"inputs larger than L2 ({n_local * d * 2 / 2**30:.2f} GiB keys + "
                          f"{n_local * d * 2 / 2**30:.2f} GiB values per GPU)")},
        "e2e": {"value": M / (e2e_ms * 1e-3), "unit": "queries/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "path": ("pinned host -> rank 0 -> NCCL broadcast; result read back at rank 0;"
                         " HostPipeline overlaps each batch's copies with the neighbouring"
                         " batches' kernels")},
        "roofline": roofline,
        "phase_ms": phases,
        "gpu_launches": r.kernels_per_call * args.steps,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = _cpu_baseline(args, wl, keys, values, queries[0])
    if args.lm or not args.no_assembly:
        del r, keys, values, queries
        torch.cuda.empty_cache()
    if not args.no_assembly:
        line["assembly"] = measure_assembly(world, rank, local_rank, group)
        line["key_projection"] = measure_key_projection(world, rank, local_rank)
        if world == 1:
            line["hybrid"] = measure_hybrid(local_rank)
            line["backward"] = measure_backward(local_rank)
    if args.lm:
        names = [n for n in args.lm.split(",") if n and (n != "small_char" or world == 1)]
        line["lm"] = [measure_lm(n, world, rank, local_rank, group) for n in names]
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def measure_assembly(world, rank, local_rank, group, warmup=3, steps=10):
    """WeightAssembler (per-position low-rank consumer of the retrieved rows,
    assembly.py:75-128) on the reference's 1B layout: d_A = d_B = 1280, r = 8,
    D = 21760, k = 16, pool of 16384 rows row-sharded over the ranks, 8192
    tokens per step (batch 8 x seq 1024).  Indices are synthetic, uniform over
    the pool, distinct per token; alpha normalised random weights."""
    import torch
    import torch.distributed as dist

    import computd_b200 as cb

    d_A = d_B = 1280
    r, k, N, M = 8, 16, 16384, 8192
    D = d_B * r + r * d_A + d_B
    dev = torch.device("cuda", local_rank)
    spec = cb.ShardSpec(N, rank, world)
    vectors = cb.new_normal(spec.n_local, D, seed=41, stddev=0.02, row_offset=spec.row_begin,
                            device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(43)
    h = torch.randn((M, d_A), device=dev, generator=g).to(torch.bfloat16)
    idx = torch.argsort(torch.rand((M, N), device=dev, generator=g), dim=1)[:, :k].to(torch.int32)
    alpha = torch.rand((M, k), device=dev, generator=g)
    alpha = alpha / alpha.sum(-1, keepdim=True)
    asm = cb.WeightAssembler(d_A, d_B, r, device=dev)
    asm.W_base = (torch.randn((d_B, d_A), device=dev, generator=g) * d_A ** -0.5).to(torch.bfloat16)
    grp = group if world > 1 else None

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    for _ in range(warmup):
        asm(h, alpha, idx, vectors, group=grp)
    barrier()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record()
    for _ in range(steps):
        asm(h, alpha, idx, vectors, group=grp)
    e1.record()
    barrier()
    # the delta alone (this rank's owned rows), on the path WeightAssembler takes
    # (row-stationary when rows are shared by >= 4 tokens), then the per-token
    # kernel for comparison
    from computd_b200.assembler import _rows_path_fits
    rows = _rows_path_fits(M, k, spec.n_local, d_A, d_B, r)
    for _ in range(steps):
        cb.lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r, row_begin=spec.row_begin, rows=rows)
    e2.record()
    e3 = torch.cuda.Event(enable_timing=True)
    for _ in range(steps):
        cb.lowrank_delta(h, alpha, idx, vectors, d_A, d_B, r, row_begin=spec.row_begin, rows=False)
    e3.record()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1) / steps, e1.elapsed_time(e2) / steps,
                      e2.elapsed_time(e3) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_delta, ms_token = float(t[0]), float(t[1]), float(t[2])
    own = (idx >= spec.row_begin) & (idx < spec.row_end)
    owned = float(own.sum())
    uniq = float(torch.unique(idx[own]).numel())
    # algorithmic bytes.  Per-token kernel: each owned selected row's U, V and b
    # blocks once per (token, entry), h once per token, delta written once.
    # Row-stationary: each distinct owned row once, each pair's d_B-float slot
    # written and read back once, h and delta once.
    bytes_token = owned * (D * 2.0) + M * (d_A * 2.0 + d_B * 4.0)
    bytes_rows = uniq * (D * 2.0) + owned * d_B * 8.0 + M * (d_A * 2.0 + d_B * 4.0)
    bytes_delta = bytes_rows if rows else bytes_token
    hbm = _peaks()[2]
    del vectors, h, idx, alpha, asm
    torch.cuda.empty_cache()
    return {"config": "reference 1B assembly layout (d_A=d_B=1280, r=8, D=21760, k=16, N=16384)",
            "tokens_per_step": M, "tokens_per_s": M / (ms * 1e-3), "unit": "tokens/s",
            "ms_per_step": ms, "pool_rows_per_gpu": spec.n_local,
            "roofline": {"bound": "hbm",
                         "kernel": ("lowrank_rows: pair sort + row kernel + per-token slot sum"
                                    if rows else "lowrank_delta_staged_kernel"),
                         "ms_per_launch": ms_delta,
                         "achieved": bytes_delta / (ms_delta * 1e-3) / 1e9, "peak": hbm,
                         "unit": "GB/s", "frac": bytes_delta / (ms_delta * 1e-3) / 1e9 / hbm,
                         "algorithmic_bytes_per_launch": bytes_delta},
            "per_token_kernel": {"ms_per_launch": ms_token,
                                 "algorithmic_bytes_per_launch": bytes_token,
                                 "frac": bytes_token / (ms_token * 1e-3) / 1e9 / hbm},
            "data": "synthetic: uniform distinct indices per token, random weights"}


def measure_key_projection(world, rank, local_rank, warmup=2, steps=5):
    """Pool keys (projection + L2 normalisation + aspect collapse, retrieval.py:241-262)
    on the reference's 7B layout: S = 16 aspects, d_k = 128, D = 69632, a pool of
    32768 rows sharded over the ranks; one fused tcgen05 launch per step."""
    import torch
    import torch.distributed as dist

    import computd_b200 as cb

    S, d_k, D, N = 16, 128, 69632, 32768
    dev = torch.device("cuda", local_rank)
    spec = cb.ShardSpec(N, rank, world)
    vectors = cb.new_normal(spec.n_local, D, seed=71, stddev=0.02, row_offset=spec.row_begin,
                            device=dev)
    wk = cb.new_normal(S * d_k, D, seed=72, stddev=D ** -0.5, device=dev).view(S, d_k, D)
    w = torch.softmax(torch.linspace(-1.0, 1.0, S, device=dev), 0)
    out = torch.empty((spec.n_local, d_k), dtype=torch.bfloat16, device=dev)
    for _ in range(warmup):
        cb.project_keys(vectors, wk, w, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        cb.project_keys(vectors, wk, w, out=out)
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    flops = 2.0 * spec.n_local * D * S * d_k
    burst = _peaks()[0]
    del vectors, wk, out
    torch.cuda.empty_cache()
    return {"config": "reference 7B key layout (S=16, d_k=128, D=69632, N=32768)",
            "pool_rows_per_gpu": spec.n_local, "ms_per_launch": ms,
            "rows_per_s": N / (ms * 1e-3), "unit": "pool rows/s",
            "roofline": {"bound": "tensor", "kernel": "key_project_kernel",
                         "achieved": flops / (ms * 1e-3) / 1e12, "peak": burst, "unit": "TFLOP/s",
                         "frac": flops / (ms * 1e-3) / 1e12 / burst, "flops_per_launch": flops}}


def measure_hybrid(local_rank, warmup=3, steps=10):
    """MultiAspectRetrieval.hybrid_forward (retrieval.py:131-181) on the reference's
    1B layout (configs/large_1b.py: d_A 1280, S = 8 aspects of d_k = 64, pool
    16384 x 21760, k = 16, batch 8 x seq 1024), one GPU: packed key projection,
    fused score + top-k with the seq-mean epilogue, seq scores, alpha.  Also the
    fused kernel with and without the seq-mean epilogue on the same packed
    inputs, and the seq-scores kernel on one GPU's shard of the 7B LM pool
    (4 sequence-mean queries against 2,097,152 x 4096 keys) against HBM."""
    import torch

    import computd_b200 as cb

    dev = torch.device("cuda", local_rank)
    B, seq, d_A, S, d_k, N, D, k = 8, 1024, 1280, 8, 64, 16384, 21760, 16
    m = cb.MultiAspectRetrieval(D=D, d_A=d_A, S=S, d_k=d_k, N=N, device=dev, seed=5)
    vectors = cb.new_normal(N, D, seed=81, stddev=0.02, device=dev)
    z = cb.new_normal(B * seq, d_A, seed=82, device=dev).view(B, seq, d_A)

    def timed(fn, n):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    ms_eager = timed(lambda: m.hybrid_forward(z, vectors, k, 1.0, 1.0, True), steps)
    # The same call captured once in a CUDA graph and replayed: the device time
    # without the host's per-op launch overhead (what a jitted caller sees).
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        m.hybrid_forward(z, vectors, k, 1.0, 1.0, True)
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        m.hybrid_forward(z, vectors, k, 1.0, 1.0, True)
    ms_fwd = timed(graph.replay, steps)
    del graph
    p = m.hybrid_parts(z, vectors, k, 1.0, 1.0, True)
    q, keys = p.queries_flat, p.keys_w
    params = cb.score_params(1.0, p.tau, 1.0, dev)
    ms_aux = timed(lambda: cb.score_topk_seqmean(q, keys, k, params[0], params[1], params[2], True,
                                                 seq), steps)
    ms_plain = timed(lambda: cb.tiled_topk_fused(q, keys, k, params[0], params[1], params[2], True),
                     steps)
    burst, _, hbm, _ = _peaks()
    flops = 2.0 * B * seq * N * S * d_k
    del m, vectors, z, p, q, keys
    torch.cuda.empty_cache()
    # seq scores at the 7B shard: HBM-bound
    Ns, ds, Bs = 2097152, 4096, 4
    ks = cb.new_normal(Ns, ds, seed=83, stddev=ds ** -0.5, device=dev)
    qm = torch.randn((Bs, ds), device=dev) * ds ** -0.5
    sims = torch.empty((Bs, Ns), dtype=torch.float32, device=dev)
    fused = torch.empty_like(sims)
    ms_seq = timed(lambda: cb.seq_scores(qm, ks, 1.0, 0.0, 1.0, True, sims=sims, fused=fused), 5)
    bytes_seq = Ns * ds * 2.0 + 2.0 * Bs * Ns * 4 + Bs * ds * 4.0
    del ks, qm, sims, fused
    torch.cuda.empty_cache()
    return {"config": "reference 1B hybrid layout: batch 8 x seq 1024, d_A 1280, S 8 x d_k 64, "
                      "pool 16384 x 21760, k 16, gate on",
            "hybrid_forward_ms": ms_fwd, "timing": "CUDA-graph replay of the whole call",
            "hybrid_forward_eager_ms": ms_eager, "tokens_per_s": B * seq / (ms_fwd * 1e-3),
            "score_topk_seqmean_ms": ms_aux, "score_topk_plain_ms": ms_plain,
            "seqmean_overhead": ms_aux / ms_plain - 1.0,
            "roofline_score": {"bound": "tensor", "flops_per_launch": flops,
                               "achieved": flops / (ms_aux * 1e-3) / 1e12, "peak": burst,
                               "unit": "TFLOP/s",
                               "frac": flops / (ms_aux * 1e-3) / 1e12 / burst},
            "seq_scores": {"shape": f"{Bs} x {Ns} x {ds}", "ms_per_launch": ms_seq,
                           "roofline": {"bound": "hbm", "algorithmic_bytes": bytes_seq,
                                        "achieved": bytes_seq / (ms_seq * 1e-3) / 1e9,
                                        "peak": hbm, "unit": "GB/s",
                                        "frac": bytes_seq / (ms_seq * 1e-3) / 1e9 / hbm}}}


def measure_backward(local_rank, warmup=2, steps=5):
    """The custom VJP of the retrieval op (computd_b200.autograd.retrieve; the
    reference trains through its plain-jnp path, retrieval.py:268-271) at the
    op-at-scale shape: 8192 queries x 1,048,576-row pool, d 1024, k 64.

    Two timings: the backward with only the queries requiring grad (one
    launch of dwa_retrieval_backward: <dout, V[idx]> and <q, K[idx]>, the
    score derivative and the ds-weighted key-row sum), and the full backward,
    which also writes the dense bf16 key and value gradients of the whole pool
    (dwa_row_gradient: 2 GiB each, every row written once)."""
    import torch

    import computd_b200 as cb
    from computd_b200.autograd import retrieve

    M, N, d, k = 8192, 1 << 20, 1024, 64
    dev = torch.device("cuda", local_rank)
    keys = cb.new_normal(N, d, seed=51, stddev=d ** -0.5, device=dev)
    values = cb.new_normal(N, d, seed=52, stddev=1.0, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(53)
    q0 = torch.randn((M, d), device=dev, generator=g).to(torch.bfloat16)
    dout = torch.randn((M, d), device=dev, generator=g)
    res = {"config": "op-at-scale retrieval backward: 8192 x 1,048,576 x 1024, k 64, bf16 pool",
           "data": "synthetic"}
    for name, kv_grad in (("queries_only", False), ("all_inputs", True)):
        q = q0.clone().requires_grad_(True)
        kk = keys.requires_grad_(kv_grad)
        vv = values.requires_grad_(kv_grad)
        ts = []
        for it in range(warmup + steps):
            out, _, _ = retrieve(q, kk, vv, k)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out.backward(dout)
            e1.record()
            torch.cuda.synchronize()
            if it >= warmup:
                ts.append(e0.elapsed_time(e1))
            q.grad = None
            kk.grad = None
            vv.grad = None
            del out
        res[f"{name}_ms"] = sorted(ts)[len(ts) // 2]
    keys.requires_grad_(False)
    values.requires_grad_(False)
    # algorithmic bytes of the queries-only backward (one fused launch on one
    # GPU): each selected key and value row once (M k bf16 rows each), q and
    # dout once, dq written
    b = 2.0 * M * k * d * 2 + M * d * 2 + M * d * 4 + M * d * 4
    hbm = _peaks()[2]
    res["roofline_queries_only"] = {"bound": "hbm", "algorithmic_bytes": b,
                                    "achieved": b / (res["queries_only_ms"] * 1e-3) / 1e9,
                                    "peak": hbm, "unit": "GB/s",
                                    "frac": b / (res["queries_only_ms"] * 1e-3) / 1e9 / hbm}
    del keys, values, q0, dout
    torch.cuda.empty_cache()
    return res


def measure_lm(cfg_name, world, rank, local_rank, group=None, warmup=3, steps=3):
    """DWA LM forward tokens/s (all ranks run the same forward; the pool is row-sharded)."""
    import torch
    import torch.distributed as dist

    import computd_b200 as cb
    from computd_b200 import dwa_lm

    cfg = dwa_lm.CONFIGS[cfg_name]
    if cfg_name == "large_7b":
        if world < 4:
            # 16,777,216 rows x 4096 of keys and of values: 256 GiB, more than one or two B200s
            return {"config": cfg_name, "skipped": "the 256 GiB pool needs 4 or more GPUs"}
        steps = 2  # ~8.6 s (8 GPUs) to ~17 s (4 GPUs) per forward; warm-up stays at 3
    dev = torch.device("cuda", local_rank)
    spec = cb.ShardSpec(cfg.pool_rows, rank, world)
    if cfg.r > 0:
        # the reference's pool: N(0, 1) * 0.02 rows of [U | V | b] (pool.py:34, 39)
        keys = None
        values = cb.new_normal(spec.n_local, cfg.D, seed=33, stddev=0.02,
                               row_offset=spec.row_begin, device=dev)
    else:
        keys = cb.new_normal(spec.n_local, cfg.key_width, seed=31, stddev=cfg.key_width ** -0.5,
                             row_offset=spec.row_begin, device=dev)
        values = cb.new_normal(spec.n_local, cfg.d_model, seed=32, stddev=cfg.d_model ** -0.5,
                               row_offset=spec.row_begin, device=dev)
    model = dwa_lm.DWALM(cfg, keys, values, group=group if world > 1 else None)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    tokens = torch.randint(0, cfg.vocab, (cfg.batch, cfg.seq_len), device=dev, generator=g)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    # one process: replay the whole forward as one CUDA graph; sharded: eager
    # (the blocks' collectives stay outside graphs)
    fwd = dwa_lm.GraphedForward(model, tokens) if world == 1 else model
    for _ in range(warmup):
        fwd(tokens)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fwd(tokens)
    e1.record()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    d, n_tok, kw = cfg.d_model, cfg.tokens, cfg.key_width
    # tensor-core work per forward on one GPU: the fused score GEMM over this
    # GPU's shard, the key projection of the shard (r > 0), and the dense
    # layers (QKV + proj 8 d^2, query_proj 2 d^2, aspect query projection
    # 2 d S d_k, W_base 2 d^2 per token; attention 4 seq d; PartA 2 d^2,
    # PartB 8 d^2 + 8 d vocab).  HBM-bound parts (gathers, low-rank delta) are
    # not in the bound.
    retr = cfg.n_layers * 2.0 * n_tok * spec.n_local * kw
    keyproj = cfg.n_layers * 2.0 * spec.n_local * kw * cfg.D if cfg.r > 0 else 0.0
    dense = n_tok * (cfg.n_layers * (12.0 * d * d + 2.0 * d * kw + 4.0 * cfg.seq_len * d)
                     + 10.0 * d * d + 8.0 * d * cfg.vocab)
    burst = _peaks()[0]
    t_roof = (retr + keyproj + dense) / (burst * 1e12)
    status = model.retriever.status()
    graphed = fwd is not model
    del fwd, model, keys, values
    torch.cuda.empty_cache()
    return {"config": cfg_name, "tokens_per_s": n_tok / (ms * 1e-3),
            "unit": "tokens/s", "ms_per_forward": ms, "tokens_per_forward": n_tok,
            "layers": cfg.n_layers, "d_model": d, "pool_rows": cfg.pool_rows,
            "pool_rows_per_gpu": spec.n_local, "top_k": cfg.top_k,
            "aspects": cfg.S, "d_k": cfg.d_k, "lowrank_r": cfg.r,
            "pool_layout": ("reference [U|V|b] rows, keys projected per block and forward"
                            if cfg.r > 0 else "packed keys [N, S d_k] + value rows [N, d]"),
            "roofline": {"t_roof_ms": t_roof * 1e3, "frac": t_roof * 1e3 / ms,
                         "flops_retrieval_per_gpu": retr, "flops_key_projection_per_gpu": keyproj,
                         "flops_dense": dense, "peak": "bf16 burst (MEASURED_PEAKS.json)"},
            "warmup": warmup, "steps": steps, "device_status": status,
            "cuda_graph": graphed}


def _cpu_baseline(args, wl, keys_dev, values_dev, q_dev):
    import numpy as np
    import torch

    from oracle import dwa_oracle as O

    threads = len(os.sched_getaffinity(0))
    N, d, k = wl["N"], wl["d"], wl["k"]
    mq = args.cpu_queries
    q = q_dev[:mq].float().cpu().numpy()
    cache = {}

    def rows(a, b):
        return keys_dev[a:b].float().cpu().numpy()

    t_cpu, alpha, idx = cpu_sample(rows, N, d, k, q, wl["use_sigmoid"])
    vals = values_dev[torch.from_numpy(idx.reshape(-1).astype(np.int64)).to(values_dev.device)]
    vals = vals.float().cpu().numpy().reshape(mq, k, d)
    t0 = time.perf_counter()
    np.einsum("mk,mkd->md", alpha, vals)
    t_cpu += time.perf_counter() - t0
    return {"value": mq / t_cpu, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{mq} queries against the full {N}-row pool, NumPy restatement of the "
                      f"reference jnp path (matmul, gate/exp, top_k, normalise, gather-sum), "
                      f"{t_cpu:.2f}s of CPU work"}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=320,
                    help="timed steps (the default gives a timed region of ~4 s at one GPU, "
                         ">= 20 clock samples)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="op_at_scale")
    ap.add_argument("--cpu-queries", type=int, default=64,
                    help="queries per CPU sample (CPU baseline / reference arm)")
    ap.add_argument("--reference-budget-s", type=float, default=60.0,
                    help="CPU seconds the reference arm spends on all its steps")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-assembly", action="store_true",
                    help="skip the WeightAssembler (low-rank consumer) measurement")
    ap.add_argument("--shape", default="",
                    help="MxNxDxK: run the chosen workload's step at these sizes instead "
                         "(profiling and sweeps; the workload is then named by its sizes)")
    ap.add_argument("--lm", default="small_char,ref_1b,large_1b,large_7b",
                    help="DWA LM forwards to time after the op (comma list; empty to skip); "
                         "large_7b runs on 4 or more GPUs")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    wl = WORKLOADS[args.workload]
    if args.shape:
        try:
            M, N, d, k = (int(x) for x in args.shape.lower().split("x"))
        except ValueError:
            ap.error("--shape must be MxNxDxK, e.g. 16384x262144x4096x64")
        wl = dict(wl, M=M, N=N, d=d, k=k,
                  desc=f"queries [{M},{d}] bf16 ~N(0,1); pool {N}x{d} bf16 keys ~N(0,1/{d}), "
                       f"values ~N(0,1); top-k {k}; softmax-weighted value sum")
        args.workload = f"shape_{M}x{N}x{d}x{k}"
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_ours(args, wl)


if __name__ == "__main__":
    raise SystemExit(main())
