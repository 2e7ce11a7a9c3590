"""CPU tests of the C ABI: the library loads, exports exactly what
include/*.h (dwa_retrieval.h, dwa_lm.h) declare, and rejects invalid
arguments on the host without launching anything (no GPU is touched by these
calls)."""
import ctypes
import re
from pathlib import Path

import pytest

from computd_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols():
    text = "\n".join(h.read_text() for h in HEADERS)
    return sorted(set(re.findall(r"DWA_API\s+[\w\s\*]+?\b(dwa_\w+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.dwa_abi_version() == 2


def test_only_dwa_symbols_are_exported():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    text_syms = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert sorted(text_syms) == declared_symbols()


def test_status_strings():
    lib = _lib.load()
    names = {s: lib.dwa_status_string(s).decode() for s in range(7)}
    assert names[0] == "DWA_OK" and names[4] == "DWA_ERR_TIMEOUT"
    assert lib.dwa_status_string(99).decode() == "DWA_ERR_UNKNOWN"


FAKE = 0x10000  # 16-byte aligned, never dereferenced: validation fails before any launch


def score_topk(**kw):
    lib = _lib.load()
    a = dict(q=FAKE, M=128, ldq=128, keys=FAKE, N=1000, ldk=128, d=128, k=16, lam=1.0, tau=0.0,
             T=1.0, sig=0, off=0, ov=FAKE, oi=FAKE, ws=FAKE, ws_bytes=0, stream=None)
    a.update(kw)
    st = lib.dwa_score_topk(a["q"], a["M"], a["ldq"], a["keys"], a["N"], a["ldk"], a["d"], a["k"],
                            a["lam"], a["tau"], a["T"], a["sig"], a["off"], a["ov"], a["oi"],
                            a["ws"], a["ws_bytes"], a["stream"])
    return st, lib.dwa_last_error().decode()


@pytest.mark.parametrize("kw,status", [
    (dict(q=None), _lib.DWA_ERR_INVALID_ARG),
    (dict(ov=None), _lib.DWA_ERR_INVALID_ARG),
    (dict(M=-1), _lib.DWA_ERR_INVALID_ARG),
    (dict(N=0), _lib.DWA_ERR_INVALID_ARG),
    (dict(k=0), _lib.DWA_ERR_INVALID_ARG),
    (dict(k=1001), _lib.DWA_ERR_INVALID_ARG),          # k > N (lax.top_k raises too)
    (dict(k=129, N=5000), _lib.DWA_ERR_UNSUPPORTED_SHAPE),
    (dict(d=100, ldq=128, ldk=128), _lib.DWA_ERR_UNSUPPORTED_SHAPE),
    (dict(d=4, ldq=8, ldk=8), _lib.DWA_ERR_UNSUPPORTED_SHAPE),
    (dict(ldq=64), _lib.DWA_ERR_INVALID_ARG),
    (dict(ldk=132), _lib.DWA_ERR_UNSUPPORTED_SHAPE),
    (dict(q=FAKE + 8), _lib.DWA_ERR_INVALID_ARG),      # misaligned
    (dict(off=-1), _lib.DWA_ERR_INVALID_ARG),
    (dict(off=2**31 - 10), _lib.DWA_ERR_INVALID_ARG),  # global index overflows int32
    (dict(T=0.0), _lib.DWA_ERR_UNSUPPORTED_SHAPE),
    (dict(T=float("nan")), _lib.DWA_ERR_UNSUPPORTED_SHAPE),
    (dict(sig=1, lam=-1.0), _lib.DWA_ERR_UNSUPPORTED_SHAPE),  # non-monotone gate
    (dict(ws=None), _lib.DWA_ERR_WORKSPACE),
    (dict(ws=FAKE + 16), _lib.DWA_ERR_WORKSPACE),      # not 256-aligned
    (dict(ws_bytes=1024), _lib.DWA_ERR_WORKSPACE),     # too small
])
def test_score_topk_rejects_before_launch(kw, status):
    st, msg = score_topk(**kw)
    assert st == status, msg
    assert msg


def test_score_topk_empty_batch_is_a_noop():
    st, msg = score_topk(M=0, q=None)
    assert st == _lib.DWA_OK and msg == ""


def test_workspace_plan():
    lib = _lib.load()
    # 8192 queries x 1M keys (the op-at-scale shape): 64 query tiles, 4096 key tiles
    nbytes = lib.dwa_score_topk_workspace(8192, 1 << 20, 1024, 64)
    # status block + per-row admission bounds (16 int32 slots) + one partial list per key split
    assert nbytes > 0 and (nbytes - 256 - 8192 * 64) % (64 * 8192 * 8) == 0
    assert lib.dwa_score_topk_workspace(8192, 1 << 20, 1024, 129) == 0
    assert lib.dwa_score_topk_workspace(0, 10, 8, 1) == 0


def test_merge_and_gather_validation():
    lib = _lib.load()
    assert lib.dwa_merge_topk(FAKE, FAKE, 0, 8, 4, FAKE + 256, FAKE + 512, None) == 1
    assert lib.dwa_merge_topk(FAKE, FAKE, 2, 8, 4, FAKE, FAKE + 512, None) == 1  # aliasing
    assert lib.dwa_merge_topk(FAKE, FAKE, 2, 8, 200, FAKE + 256, FAKE + 512, None) == 2
    assert lib.dwa_weighted_gather(FAKE, FAKE, 8, 4, FAKE, 0, 10, 64, 60, FAKE, None, None) == 2
    assert lib.dwa_weighted_gather(FAKE, FAKE, 8, 4, FAKE, 5, 2, 64, 64, FAKE, None, None) == 1
    assert lib.dwa_weighted_gather(FAKE, FAKE, 8, 4, FAKE + 8, 0, 10, 64, 64, FAKE, None, None) == 1
    assert lib.dwa_weighted_gather(FAKE, FAKE, 8, 4, FAKE, 0, 10, 60, 64, FAKE, None, None) == 1
    assert lib.dwa_pool_init_normal(FAKE, 4, 8, 4, 0, 1, 1.0, None) == 1
    assert lib.dwa_workspace_status(None, None, ctypes.byref(ctypes.c_int32())) == 1


def test_python_api_refuses_cpu_tensors():
    import torch

    from computd_b200 import tiled_topk_fused

    q = torch.zeros(4, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        tiled_topk_fused(q, q, 2, 1.0, 0.0, 1.0, False)


def _ptrs(*vals):
    return (ctypes.c_void_p * len(vals))(*vals)


def test_nvlink_and_projection_entry_points_validate_before_launch():
    """The NVLink exchange / value-sum, key projection, assembly and EMA entry points
    reject bad arguments on the host, before any CUDA call (runs without a GPU)."""
    lib = _lib.load()
    nul = ctypes.c_void_p()
    # peer buffers and signals
    assert lib.dwa_peer_alloc(0, ctypes.byref(nul), FAKE) == 1
    assert lib.dwa_peer_open(None, ctypes.byref(nul)) == 1
    assert lib.dwa_peer_signal(_ptrs(FAKE, FAKE), 0, 0, 1, None) == 1
    assert lib.dwa_peer_signal(_ptrs(FAKE, FAKE), 2, 2, 1, None) == 1          # rank >= P
    assert lib.dwa_peer_signal(_ptrs(FAKE, FAKE), 17, 0, 1, None) == 1         # P > 16
    # peer merge: odd k (16-byte staging), P range, list alignment
    out_v, out_i, st = FAKE + 4096, FAKE + 8192, FAKE + 12288
    assert lib.dwa_merge_topk_peers(_ptrs(FAKE, FAKE), 2, 8, 5, FAKE, 1, 0, out_v, out_i, st, None) == 2
    assert lib.dwa_merge_topk_peers(_ptrs(FAKE), 0, 8, 4, FAKE, 1, 0, out_v, out_i, st, None) == 1
    assert lib.dwa_merge_topk_peers(_ptrs(FAKE + 8, FAKE), 2, 8, 4, FAKE, 1, 0, out_v, out_i, st,
                                    None) == 1
    # peer value sum: blocks must cover M, d % 8
    assert lib.dwa_weighted_gather_peers(FAKE, FAKE, 100, 4, FAKE, 0, 10, 64, 64, _ptrs(FAKE, FAKE),
                                         2, 0, 40, None, None) == 1
    assert lib.dwa_weighted_gather_peers(FAKE, FAKE, 100, 4, FAKE, 0, 10, 64, 60, _ptrs(FAKE, FAKE),
                                         2, 0, 50, None, None) == 2
    assert lib.dwa_weighted_gather_peers(FAKE, FAKE, 100, 4, FAKE, 0, 10, 64, 64, _ptrs(FAKE, FAKE),
                                         2, 2, 50, None, None) == 1
    assert lib.dwa_reduce_broadcast_peers(FAKE, 2, 0, 40, 100, 64, _ptrs(FAKE, FAKE), FAKE, 1, 0, st,
                                          None) == 1
    assert lib.dwa_reduce_broadcast_peers(FAKE, 2, 0, 50, 100, 60, _ptrs(FAKE, FAKE), FAKE, 1, 0, st,
                                          None) == 2
    assert lib.dwa_peer_wait(None, 2, 1, 0, st, None) == 1
    assert lib.dwa_peer_wait(FAKE, 0, 1, 0, st, None) == 1
    # key projection: d_k, D, S, strides
    assert lib.dwa_project_keys(FAKE, 10, 64, 64, FAKE, 64, 2, 48, FAKE, FAKE, 64, None, None) == 2
    assert lib.dwa_project_keys(FAKE, 10, 64, 12, FAKE, 64, 2, 32, FAKE, FAKE, 64, None, None) == 2
    assert lib.dwa_project_keys(FAKE, 10, 64, 64, FAKE, 64, 0, 32, FAKE, FAKE, 64, None, None) == 2
    assert lib.dwa_project_keys(None, 10, 64, 64, FAKE, 64, 2, 32, FAKE, FAKE, 64, None, None) == 1
    assert lib.dwa_project_keys(FAKE, 10, 60, 64, FAKE, 64, 2, 32, FAKE, FAKE, 64, None, None) == 1
    assert lib.dwa_project_keys(FAKE, 10, 68, 64, FAKE, 64, 2, 32, FAKE, FAKE, 64, None, None) == 2
    # low-rank assembly and EMA
    assert lib.dwa_lowrank_delta(FAKE, 1, 64, FAKE, FAKE, 4, 2, FAKE, 0, 10, 2048, 12, 16, 8, FAKE,
                                 None) == 2
    assert lib.dwa_lowrank_delta(FAKE, 1, 64, FAKE, FAKE, 4, 2, FAKE, 0, 10, 2048, 64, 16, 0, FAKE,
                                 None) == 2
    assert lib.dwa_lowrank_delta(FAKE, 1, 64, FAKE, FAKE, 4, 2, FAKE, 0, 10, 100, 64, 16, 8, FAKE,
                                 None) == 1
    # dense row gradient: workspace and limits checked before any launch
    assert lib.dwa_row_gradient_workspace(8192, 64, 1 << 20) >= 8192 * 64 * 4 + (1 << 20) * 8
    rg = lambda **kw: lib.dwa_row_gradient(FAKE, FAKE, kw.get("M", 4), 8, FAKE, 1, 64, 0, 100, FAKE,
                                           1, 64, kw.get("d", 64), kw.get("ws", FAKE),
                                           kw.get("ws_bytes", 1 << 30), None)
    assert rg(ws=None) == _lib.DWA_ERR_WORKSPACE
    assert rg(ws_bytes=16) == _lib.DWA_ERR_WORKSPACE
    assert rg(d=12) == 2
    assert rg(M=1 << 29) == 2                  # M k above INT32_MAX
    # fused backward: limits checked before any launch
    bwd = lambda **kw: lib.dwa_retrieval_backward(
        kw.get("q", FAKE), 1, 64, FAKE, 64, FAKE, 64, 64, FAKE, 64, 64, FAKE, FAKE, 4,
        kw.get("k", 8), 0, 100, 1.0, 0.0, kw.get("T", 1.0), kw.get("params", None), 0,
        FAKE, kw.get("dq", FAKE), None, kw.get("status", None), None)
    assert bwd(k=129) == 2                     # k above 128
    assert bwd(T=0.0) == 2                     # host temperature must be > 0
    assert bwd(params=FAKE) == 1               # device params need a status word
    assert bwd(dq=FAKE + 4) == 1               # dq not 16-byte aligned
    assert bwd(q=None) == 1
    # row-stationary low-rank assembly: same checks, then its own limits
    need = lib.dwa_lowrank_delta_rows_workspace(8192, 16, 16384, 1280)
    assert need >= 8192 * 16 * 1280 * 4 + 8192 * 16 * 4 + 16384 * 8
    assert lib.dwa_lowrank_delta_rows_workspace(-1, 16, 16384, 1280) == 0
    D = 1280 * 8 + 8 * 1280 + 1280
    rows = lambda M, k, d_A, d_B, r, ldv, ws, ws_bytes: lib.dwa_lowrank_delta_rows(
        FAKE, 1, d_A, FAKE, FAKE, M, k, FAKE, 0, 16384, ldv, d_A, d_B, r, FAKE, ws, ws_bytes, None)
    assert rows(4, 2, 1280, 1280, 8, D, None, 0) == _lib.DWA_ERR_WORKSPACE
    assert rows(4, 2, 1280, 1280, 8, D, FAKE, 16) == _lib.DWA_ERR_WORKSPACE
    assert rows(4, 2, 1280, 1280, 0, D, FAKE, 1 << 40) == 2          # r outside [1, 32]
    assert rows(4, 2, 1280, 1280, 8, 100, FAKE, 1 << 40) == 1        # ldv below the row
    D_big = 8192 * 8 + 8 * 8192 + 8192                               # 272 KB of U | V | b
    assert rows(4, 2, 8192, 8192, 8, D_big, FAKE, 1 << 40) == 2
    assert rows(1 << 27, 32, 1280, 1280, 8, D, FAKE, 1 << 62) == 2   # M k above INT32_MAX
    assert rows(0, 2, 1280, 1280, 8, D, None, 0) == 0                # empty batch: no-op
    assert lib.dwa_assemble_finish(None, 0, 0, None, None, 4, 16, 1.0, None, None, 1e-6, FAKE,
                                   None) == 1
    assert lib.dwa_usage_ema(FAKE, FAKE, -1, 0, 10, 0.01, 0.99, FAKE, None) == 1


def test_device_scalar_and_seq_entry_points_validate_before_launch():
    """dwa_score_topk_dev / dwa_score_backward_dev / dwa_seq_scores: the host
    checks what it can see (pointers, shapes, alignment) and launches nothing on
    failure; the scalars themselves are checked on the device."""
    lib = _lib.load()
    args = [FAKE, 128, 128, FAKE, 1000, 128, 128, 16]
    tail = [0, 0, FAKE, FAKE, FAKE, 0, None]
    # null params, misaligned params, and the shape checks dwa_score_topk makes
    assert lib.dwa_score_topk_dev(*args, None, *tail) == 1
    assert lib.dwa_score_topk_dev(*args, FAKE + 2, *tail) == 1
    assert lib.dwa_score_topk_dev(FAKE, 128, 128, FAKE, 1000, 128, 128, 129, FAKE, *tail) == 2
    assert lib.dwa_score_topk_dev(*args, FAKE, 0, 0, FAKE, FAKE, None, 0, None) == 6  # workspace
    assert lib.dwa_score_topk_dev(FAKE, 0, 128, FAKE, 1000, 128, 128, 16, None, *tail) == 0
    assert lib.dwa_score_backward_dev(FAKE, FAKE, FAKE, 8, 4, None, 1, FAKE, None, None, None) == 1
    assert lib.dwa_score_backward_dev(FAKE, FAKE, FAKE, 8, 0, FAKE, 1, FAKE, None, None, None) == 1
    # seq scores: d range, strides, fused without params, key alignment
    seq = lambda **kw: lib.dwa_seq_scores(*[kw.get(n, v) for n, v in [
        ("q", FAKE), ("B", 4), ("ldq", 128), ("keys", FAKE), ("N", 1000), ("ldk", 128),
        ("d", 128), ("params", FAKE), ("sig", 1), ("sims", FAKE), ("lds", 1000),
        ("fused", FAKE), ("ldf", 1000), ("status", None), ("stream", None)]])
    assert seq(d=100, ldq=128, ldk=128) == 2
    assert seq(d=12808, ldq=12808, ldk=12808) == 2
    assert seq(lds=999) == 1
    assert seq(params=None) == 1
    assert seq(keys=FAKE + 8) == 2
    assert seq(sims=None) == 1
    assert seq(B=0) == 0 and seq(N=0) == 0


def test_lm_helpers_reject_bad_arguments_on_host():
    lib = _lib.load()
    rope = lambda **kw: lib.dwa_lm_rope_qk(*[kw.get(n, v) for n, v in [
        ("qkv", FAKE), ("B", 2), ("S", 64), ("H", 4), ("dh", 64), ("ld", 768), ("cos", FAKE),
        ("sin", FAKE), ("ldcs", 32), ("q", FAKE), ("k", FAKE), ("stream", None)]])
    assert rope(dh=60, ld=720) == 2                    # dh % 8
    assert rope(ld=511) == 1                           # row shorter than q and k
    assert rope(ld=516) == 2                           # ld_qkv % 8
    assert rope(ldcs=31) == 1
    assert rope(ldcs=34) == 2                          # ld_cs % 4
    assert rope(qkv=FAKE + 8) == 2 and rope(sin=FAKE + 4) == 2
    assert rope(q=None) == 1 and rope(H=0) == 1
    assert rope(B=0) == 0 and rope(S=0) == 0
    asp = lambda **kw: lib.dwa_lm_aspect_queries(*[kw.get(n, v) for n, v in [
        ("q", FAKE), ("M", 100), ("S", 8), ("dk", 64), ("ldq", 512), ("logits", FAKE),
        ("tau", FAKE), ("lam", 1.0), ("T", 1.0), ("sig", 1), ("out", FAKE), ("ldo", 512),
        ("w", None), ("params", None), ("stream", None)]])
    assert asp(S=0) == 2 and asp(S=65, ldq=65 * 64, ldo=65 * 64) == 2
    assert asp(dk=60) == 2
    assert asp(ldq=504) == 1 and asp(ldo=504) == 1
    assert asp(ldq=520, ldo=516) == 2
    assert asp(tau=None) == 1 and asp(logits=None) == 1
    assert asp(out=None) == 1 and asp(q=FAKE + 8) == 2
    assert asp(params=FAKE + 2) == 1
