"""Pool-parallel retrieval: local fused top-k, all-gather, merge, owner-computes value sum.

Mirrors the reference's multi-chip retrieval, ``MultiAspectRetrieval.pallas_hybrid_forward``
(src/model/retrieval.py:204-343) and its ``shard_map`` body ``_chip_topk``
(retrieval.py:285-303):

    tv, li     = tiled_topk_fallback(q, keys_local, k, lambda, tau, T, use_sigmoid)
    gidx       = li + axis_index * N_local                        (292-293)
    cand_v/i   = all_gather(tv / gidx)  -> [P, BT, k]             (295-296)
    fv, fi     = top_k over the P*k candidates per row            (299-302)
    alpha      = fv / (sum(fv) + 1e-8)                            (326)

On B200 the ``shard_map`` becomes one process per GPU (torch.distributed over
NCCL): queries are replicated and rank r holds pool rows [r*N/P, (r+1)*N/P) in
HBM.  The candidate exchange and merge run as one kernel that reads the
other GPUs' lists over NVLink (``PeerExchange``: CUDA IPC buffers, a
system-scope release flag per rank and step, a bounded wait in the merge);
an NCCL all-gather + device merge remains selectable.  The value side
(assembly.py:104-128) sums only owned rows per rank and adds the partial sums
with one all-reduce.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch
import torch.distributed as dist

from . import _lib
from .assembly import _check_values, normalise_alpha, weighted_gather_into
from .pool import ShardSpec
from .tiled_topk import (_as_bf16_rows, _stream_handle, merge_topk, score_topk_into,
                         score_topk_seqmean, seq_scores, tiled_topk_fused, workspace_bytes)


def _group_rank_world(group) -> tuple[int, int]:
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


class _DeviceBuffer:
    """A raw device range seen by torch as a tensor (``__cuda_array_interface__``, no copy)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class PeerExchange:
    """Cross-shard candidate exchange + merge over NVLink peer memory.

    The reference's all_gather of every chip's [M, k] candidates followed by the
    top_k merge (src/model/retrieval.py:295-302) becomes: each rank writes its
    packed (score bits, global index) lists into its own CUDA-IPC buffer and
    raises flag[rank] = step on every rank (``dwa_peer_signal``: system fence +
    release stores); then every rank's merge kernel (``dwa_merge_topk_peers``)
    waits for all flags of this step and merges the P lists straight from the
    other GPUs' memory.

    Every wait for another rank is bounded by ``wait_s`` (default 30 s, well
    above the longest layer, so a rank whose host falls behind for a while is
    still waited for).  A wait that runs out writes -inf / -1 for its rows and
    DWA_ERR_TIMEOUT in the status word.  The status word is copied to pinned
    host memory after each waiting launch, and ``check`` (run at the start of
    every ``Retriever`` call) raises ``DWAError`` once it shows an error: so
    the failed call's outputs are never used by a following call.  From then
    on the exchange refuses work until every rank has called ``resync``.

    Buffers alternate by step parity.  A rank rewrites the buffer of step s at
    step s + 2 only after its own merge of step s + 1, which waited for every
    rank's step-(s + 1) flag, raised after that rank's merge of step s: so no
    list is overwritten while a peer still reads it.  Construction is
    collective over ``group`` (all ranks, same order).

    With ``d`` the buffer also carries the value side (owner-computes sum over
    NVLink): an inbox [P][block_rows][d] f32 receiving every rank's partial
    sums of this rank's row block, and the replicated output [M, d] f32 that
    the block owners write into.  A rank's partials of step s + 1 reach an
    inbox only after its wait for every block of step s, raised after the
    owner finished reading that inbox.
    """

    _HDR = 256            # bytes: int32 flag words: [0, 16) lists, [16, 32) partials,
    _STATUS_OFF = 192     # [32, 48) blocks done; status word at byte 192

    def __init__(self, M: int, k: int, group, device: torch.device, d: int | None = None,
                 wait_s: float = 30.0):
        self.rank, self.world = _group_rank_world(group)
        if not 0.0 < float(wait_s) <= 600.0:
            raise ValueError("wait_s must be in (0, 600] seconds")
        self.wait_ns = int(float(wait_s) * 1e9)
        if self.world > 16:
            raise _lib.DWAArgumentError(_lib.DWA_ERR_UNSUPPORTED_SHAPE, "PeerExchange",
                                        "more than 16 ranks")
        self.M, self.k, self.group, self.device = int(M), int(k), group, device
        self._list_bytes = self.M * self.k * 8
        self.d = int(d) if d is not None else 0
        self.block_rows = -(-self.M // self.world)
        self._inbox_off = self._HDR + 2 * self._list_bytes
        self._inbox_bytes = self.world * self.block_rows * self.d * 4
        self._out_off = self._inbox_off + self._inbox_bytes
        nbytes = self._out_off + self.M * self.d * 4
        lib = _lib.load()
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        # Set-up failures are collective: every rank takes part in the same
        # exchanges, and all of them raise together if any rank could not
        # allocate or map (a rank raising alone would leave the others waiting
        # in the next collective).
        err = ""
        with torch.cuda.device(device):
            st = lib.dwa_peer_alloc(nbytes, ctypes.byref(own), handle)
        if st != 0:
            err = f"dwa_peer_alloc: {_lib.last_error()}"
        self._own = own.value if st == 0 else None
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle) if st == 0 else b"", group=group)
        self._opened = []
        bases = []
        with torch.cuda.device(device):
            for p in range(self.world):
                if err:
                    break
                if p == self.rank:
                    bases.append(self._own)
                    continue
                if not handles[p]:
                    err = f"rank {p} has no exchange buffer"
                    break
                q = ctypes.c_void_p()
                if lib.dwa_peer_open(handles[p], ctypes.byref(q)) != 0:
                    err = f"dwa_peer_open of rank {p}: {_lib.last_error()}"
                    break
                self._opened.append(q.value)
                bases.append(q.value)
        ok = torch.tensor([0 if err else 1], dtype=torch.int32, device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            with torch.cuda.device(device):
                for q in self._opened:
                    lib.dwa_peer_close(q)
                if self._own is not None:
                    lib.dwa_peer_free(self._own)
            self._opened, self._own = [], None
            raise _lib.DWAError(_lib.DWA_ERR_CUDA, "PeerExchange",
                                err or "a peer rank could not set up its exchange buffer")
        self._bases = bases
        self._flag_table = (ctypes.c_void_p * self.world)(*bases)
        self._list_tables = [(ctypes.c_void_p * self.world)(
            *[b + self._HDR + par * self._list_bytes for b in bases]) for par in range(2)]
        self._packed = [torch.as_tensor(_DeviceBuffer(self._own + self._HDR + par * self._list_bytes,
                                                      (self.M, self.k, 2), "<i4"), device=device)
                        for par in range(2)]
        self._hdr = torch.as_tensor(_DeviceBuffer(self._own, (self._HDR // 4,), "<i4"), device=device)
        if self.d:
            self._part_flags = (ctypes.c_void_p * self.world)(*[b + 64 for b in bases])
            self._done_flags = (ctypes.c_void_p * self.world)(*[b + 128 for b in bases])
            self._inboxes = (ctypes.c_void_p * self.world)(*[b + self._inbox_off for b in bases])
            self._outs = (ctypes.c_void_p * self.world)(*[b + self._out_off for b in bases])
            self.out = torch.as_tensor(_DeviceBuffer(self._own + self._out_off, (self.M, self.d), "<f4"),
                                       device=device)
        self.step = 0
        # the status word as last copied back (pinned), and the copy's completion
        self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._status_event = torch.cuda.Event()
        self._status_pending = False
        self.failed = 0
        dist.barrier(group=group, device_ids=[device.index])

    def _copy_status(self) -> None:
        """Enqueue a copy of the status word to pinned host memory (after this stream's
        waits); ``check`` reads it."""
        self._status_host.copy_(self._hdr[self._STATUS_OFF // 4:self._STATUS_OFF // 4 + 1],
                                non_blocking=True)
        self._status_event.record(torch.cuda.current_stream(self.device))
        self._status_pending = True

    def check(self) -> None:
        """Raise ``DWAError`` if a wait of an earlier step ran out (waits for the
        status copy of the last step, which normally finished long ago)."""
        if self.failed:
            raise _lib.DWAError(self.failed, "PeerExchange",
                                "an earlier cross-rank wait ran out; call resync() on every rank")
        if not self._status_pending:
            return
        self._status_event.synchronize()
        self._status_pending = False
        v = int(self._status_host[0])
        if v != 0:
            self.failed = v
            raise _lib.DWAError(v, "PeerExchange",
                                f"a peer's flags did not arrive within {self.wait_ns / 1e9:.1f} s "
                                f"by step {self.step}; that step's outputs are -inf / -1.  Call "
                                "resync() on every rank before the next call")

    def resync(self) -> None:
        """Collective: after a run-out wait, wait for every rank, clear the flags and
        the status word and restart the step count, so the exchange is usable again."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group, device_ids=[self.device.index])
        self._hdr.zero_()
        torch.cuda.synchronize(self.device)
        self.step = 0
        self.failed = 0
        self._status_pending = False
        dist.barrier(group=self.group, device_ids=[self.device.index])

    def publish(self, local_vals: torch.Tensor, local_idx: torch.Tensor) -> None:
        """Pack this rank's [M, k] lists into its buffer and raise its flag on every rank."""
        self.step += 1
        buf = self._packed[self.step & 1]
        buf[..., 0].copy_(local_vals.view(torch.int32))
        buf[..., 1].copy_(local_idx)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            st = lib.dwa_peer_signal(self._flag_table, self.world, self.rank, self.step,
                                     _stream_handle(self.device))
        _lib.check(st, "dwa_peer_signal")

    def merge(self, out_vals: torch.Tensor, out_idx: torch.Tensor) -> None:
        """Global top-k of this step's lists of all ranks, read over NVLink."""
        lib = _lib.load()
        with torch.cuda.device(self.device):
            st = lib.dwa_merge_topk_peers(self._list_tables[self.step & 1], self.world, self.M,
                                          self.k, self._own, self.step, self.wait_ns,
                                          out_vals.data_ptr(), out_idx.data_ptr(),
                                          self._own + self._STATUS_OFF,
                                          _stream_handle(self.device))
            _lib.check(st, "dwa_merge_topk_peers")
            self._copy_status()

    def gather_partials(self, top_vals: torch.Tensor, top_idx: torch.Tensor, values: torch.Tensor,
                        row_begin: int, row_end: int, alpha_out: torch.Tensor) -> None:
        """alpha (all rows) and this shard's partial sums, stored into the owners' inboxes
        over NVLink; then this rank's "partials ready" flag on every rank."""
        lib = _lib.load()
        sh = _stream_handle(self.device)
        with torch.cuda.device(self.device):
            st = lib.dwa_weighted_gather_peers(top_vals.data_ptr(), top_idx.data_ptr(), self.M, self.k,
                                               values.data_ptr(), int(row_begin), int(row_end),
                                               values.stride(0), self.d, self._inboxes, self.world,
                                               self.rank, self.block_rows, alpha_out.data_ptr(), sh)
            _lib.check(st, "dwa_weighted_gather_peers")
            st = lib.dwa_peer_signal(self._part_flags, self.world, self.rank, self.step, sh)
        _lib.check(st, "dwa_peer_signal")

    def reduce_broadcast(self) -> torch.Tensor:
        """Sum of this rank's row block over the P inboxes, written into every rank's
        output; then wait until every block of this step has arrived here."""
        lib = _lib.load()
        sh = _stream_handle(self.device)
        status = self._own + self._STATUS_OFF
        with torch.cuda.device(self.device):
            st = lib.dwa_reduce_broadcast_peers(self._own + self._inbox_off, self.world, self.rank,
                                                self.block_rows, self.M, self.d, self._outs,
                                                self._own + 64, self.step, self.wait_ns, status, sh)
            _lib.check(st, "dwa_reduce_broadcast_peers")
            st = lib.dwa_peer_signal(self._done_flags, self.world, self.rank, self.step, sh)
            _lib.check(st, "dwa_peer_signal")
            st = lib.dwa_peer_wait(self._own + 128, self.world, self.step, self.wait_ns, status, sh)
            _lib.check(st, "dwa_peer_wait")
            self._copy_status()
        return self.out

    def status(self) -> int:
        """Device status word of the peer waits (0 or DWA_ERR_TIMEOUT); syncs the device."""
        torch.cuda.synchronize(self.device)
        return int(self._hdr[self._STATUS_OFF // 4].item())

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        if self._own is None:
            return
        dist.barrier(group=self.group, device_ids=[self.device.index])
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for q in self._opened:
                lib.dwa_peer_close(q)
            lib.dwa_peer_free(self._own)
        self._opened, self._own = [], None


def exchange_candidates(local_vals: torch.Tensor, local_idx: torch.Tensor, group=None,
                        out_vals: torch.Tensor | None = None, out_idx: torch.Tensor | None = None
                        ) -> tuple[torch.Tensor, torch.Tensor]:
    """All-gather each rank's [M, k] candidates into [P, M, k] (reference retrieval.py:295-296).

    Same collective order on every rank.  NCCL gathers straight into the
    stacked buffer; other backends (gloo, used by the CPU tests) use list
    all_gather.
    """
    _, world = _group_rank_world(group)
    M, k = local_vals.shape
    if out_vals is None:
        out_vals = torch.empty((world, M, k), dtype=local_vals.dtype, device=local_vals.device)
    if out_idx is None:
        out_idx = torch.empty((world, M, k), dtype=local_idx.dtype, device=local_idx.device)
    if world == 1:
        out_vals[0].copy_(local_vals)
        out_idx[0].copy_(local_idx)
        return out_vals, out_idx
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out_vals, local_vals.contiguous(), group=group)
        dist.all_gather_into_tensor(out_idx, local_idx.contiguous(), group=group)
    else:
        dist.all_gather(list(out_vals.unbind(0)), local_vals.contiguous(), group=group)
        dist.all_gather(list(out_idx.unbind(0)), local_idx.contiguous(), group=group)
    return out_vals, out_idx


def reduce_partials(out: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the owner-computes partial value sums over ranks (in place)."""
    _, world = _group_rank_world(group)
    if world > 1:
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out


def chip_topk(queries_flat: torch.Tensor, keys_local: torch.Tensor, k_max: int, lambda_sharp, tau,
              T, use_sigmoid: bool, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """The per-rank body of the reference's shard_map (retrieval.py:285-303).

    Returns the global top-k (fused scores f32, global indices i32), identical
    on every rank of ``group``.
    """
    rank, world = _group_rank_world(group)
    n_local = keys_local.shape[0]
    tv, gi = tiled_topk_fused(queries_flat, keys_local, k_max, lambda_sharp, tau, T, use_sigmoid,
                              idx_offset=rank * n_local)
    if world == 1:
        return tv, gi
    cand_v, cand_i = exchange_candidates(tv, gi, group)
    return merge_topk(cand_v, cand_i)


class Retriever:
    """Pre-planned retrieval over a resident (possibly row-sharded) pool.

    Owns its outputs and workspace so that repeated calls allocate nothing and
    enqueue only kernels and collectives.  One call computes, for queries
    [M, d_k]:

        top_vals, top_idx = global top-k of v(q . key) (fused scores, global rows)
        alpha             = top_vals / (sum + 1e-8)
        out               = sum_j alpha[:, j] * values[top_idx[:, j]]   (f32 [M, d_v])

    ``keys_local`` / ``values_local`` are this rank's rows [row_begin, row_end)
    of the pool (the whole pool when ``group`` is None or has one rank).
    On a sharded pool every wait for another rank gives up after
    ``peer_wait_s`` seconds; the next call then raises ``DWAError`` (see
    ``PeerExchange``) instead of computing on the -1 indices of the failed one.
    """

    def __init__(self, keys_local: torch.Tensor, values_local: torch.Tensor, M: int, k: int, *,
                 lambda_sharp: float = 1.0, tau: float = 0.0, T: float = 1.0,
                 use_sigmoid: bool = False, group=None, exchange: str = "auto",
                 peer_wait_s: float = 30.0):
        self.keys = _as_bf16_rows(keys_local, "keys_local")
        # values_local None: top-k and alpha only (the caller consumes the indices
        # itself, e.g. the low-rank WeightAssembler)
        self.values = _check_values(values_local) if values_local is not None else None
        if self.values is not None and self.values.shape[0] != self.keys.shape[0]:
            raise ValueError("keys_local and values_local must hold the same pool rows")
        self.group = group
        self.rank, self.world = _group_rank_world(group)
        self.n_local = self.keys.shape[0]
        self.shard = ShardSpec(self.n_local * self.world, self.rank, self.world)
        self.M, self.k = int(M), int(k)
        self.d_k = self.keys.shape[1]
        self.d_v = self.values.shape[1] if self.values is not None else 0
        self.lambda_sharp, self.tau, self.T = float(lambda_sharp), float(tau), float(T)
        self.use_sigmoid = bool(use_sigmoid)
        dev = self.keys.device
        self.device = dev
        f32, i32 = torch.float32, torch.int32
        self.local_vals = torch.empty((self.M, self.k), dtype=f32, device=dev)
        self.local_idx = torch.empty((self.M, self.k), dtype=i32, device=dev)
        if self.world > 1:
            self.top_vals = torch.empty((self.M, self.k), dtype=f32, device=dev)
            self.top_idx = torch.empty((self.M, self.k), dtype=i32, device=dev)
        else:
            self.top_vals, self.top_idx = self.local_vals, self.local_idx
        self.alpha = torch.empty((self.M, self.k), dtype=f32, device=dev)
        self.out = (torch.empty((self.M, self.d_v), dtype=f32, device=dev) if self.d_v else None)
        nbytes = workspace_bytes(self.M, self.n_local, self.d_k, self.k, dev)
        if nbytes == 0:
            raise _lib.DWAArgumentError(_lib.DWA_ERR_UNSUPPORTED_SHAPE, "Retriever",
                                        "no workspace plan for this shape")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        # cross-shard exchange: "nvlink" (PeerExchange), "nccl" (all-gather +
        # merge) or "auto" (nvlink for an NCCL group of more than one rank)
        if exchange not in ("auto", "nvlink", "nccl"):
            raise ValueError("exchange must be 'auto', 'nvlink' or 'nccl'")
        if exchange == "nvlink" and self.k % 2:
            raise ValueError("exchange='nvlink' needs an even k (16-byte list staging)")
        use_peer = self.world > 1 and (exchange == "nvlink" or (
            exchange == "auto" and self.k % 2 == 0 and dist.get_backend(self.group) == "nccl"))
        self.peer = None
        if use_peer and self.d_v % 8 == 0:
            try:
                self.peer = PeerExchange(self.M, self.k, self.group, dev, d=self.d_v or None,
                                         wait_s=peer_wait_s)
            except _lib.DWAError:
                # raised on every rank together; "auto" falls back to NCCL everywhere
                if exchange == "nvlink":
                    raise
        if self.peer is not None and self.d_v:
            self.out = self.peer.out  # the owners write the summed blocks straight into it
        if self.world > 1 and self.peer is None:
            self._packed_local = torch.empty((self.M, self.k, 2), dtype=i32, device=dev)
            self._packed_all = torch.empty((self.world, self.M, self.k, 2), dtype=i32, device=dev)

    @property
    def kernels_per_call(self) -> int:
        """Kernels of this library one full call launches (NCCL and torch copy kernels
        not counted).  One GPU: bound reset, fused score + top-k, split merge,
        weighted gather.  NVLink path: those four, plus the list signal, peer merge,
        partials signal, reduce-broadcast, blocks-done signal and wait.  NCCL path:
        the four plus the cross-shard merge."""
        if self.world == 1:
            return 4
        if self.values is None:
            return 7 if self.peer is not None else 5
        return 10 if self.peer is not None else 5

    def topk_local(self, queries: torch.Tensor, params: torch.Tensor | None = None
                   ) -> tuple[torch.Tensor, torch.Tensor]:
        """This rank's shard only: fused score + top-k and the split merge
        (global indices), into ``local_vals`` / ``local_idx``.  ``params``
        (device f32 [3], ``score_params``) overrides the constructor's scalars
        for this call and is read on the device (a learned tau needs no host sync)."""
        if tuple(queries.shape) != (self.M, self.d_k):
            raise ValueError(f"queries must be [{self.M}, {self.d_k}], got {tuple(queries.shape)}")
        if self.peer is not None:
            self.peer.check()  # raises if a cross-rank wait of an earlier call ran out
        score_topk_into(queries, self.keys, self.k, self.lambda_sharp, self.tau, self.T,
                        self.use_sigmoid, self.local_vals, self.local_idx, self.workspace,
                        idx_offset=self.shard.row_begin, params=params)
        return self.local_vals, self.local_idx

    def exchange(self) -> None:
        """All-gather every rank's [M, k] candidates into [P, M, k] (retrieval.py:295-296).

        Scores and indices travel together as one int32 [M, k, 2] buffer, so
        the exchange is a single collective.
        """
        if self.world == 1:
            return
        if self.peer is not None:
            self.peer.publish(self.local_vals, self.local_idx)
            return
        self._packed_local[..., 0].copy_(self.local_vals.view(torch.int32))
        self._packed_local[..., 1].copy_(self.local_idx)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self._packed_all, self._packed_local, group=self.group)
        else:
            dist.all_gather(list(self._packed_all.unbind(0)), self._packed_local, group=self.group)

    def merge(self) -> None:
        """Global top-k of the gathered [P, M, k] lists (retrieval.py:299-302), on the device."""
        if self.world == 1:
            return
        if self.peer is not None:
            self.peer.merge(self.top_vals, self.top_idx)
            return
        lib = _lib.load()
        with torch.cuda.device(self.device):
            st = lib.dwa_merge_topk_strided(
                self._packed_all.data_ptr(), self._packed_all.data_ptr() + 4, self.world,
                self.M, self.k, 2 * self.M * self.k, 2, 2 * self.k,
                self.top_vals.data_ptr(), self.top_idx.data_ptr(), _stream_handle(self.device))
        _lib.check(st, "dwa_merge_topk_strided")

    def _merge_shards(self) -> None:
        self.exchange()
        self.merge()

    def gather(self) -> None:
        """Owner-computes alpha-weighted sum over this rank's pool rows (alpha only
        when the retriever has no value rows)."""
        if self.values is None:
            normalise_alpha(self.top_vals, self.alpha, idx=self.top_idx)
            return
        if self.peer is not None:
            self.peer.gather_partials(self.top_vals, self.top_idx, self.values, self.shard.row_begin,
                                      self.shard.row_end, self.alpha)
            return
        weighted_gather_into(self.top_vals, self.top_idx, self.values, self.out, self.alpha,
                             self.shard.row_begin, self.shard.row_end)

    def reduce(self) -> None:
        if self.values is None:
            return
        if self.peer is not None:
            self.peer.reduce_broadcast()
            return
        reduce_partials(self.out, self.group)

    def topk(self, queries: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Global top-k only (fused scores f32, global indices i32), same on every rank."""
        self.topk_local(queries)
        self._merge_shards()
        return self.top_vals, self.top_idx

    def finish(self):
        """After ``topk_local``: cross-shard merge, alpha, owner-computes weighted
        sum and the all-reduce of the partial sums."""
        self.exchange()
        self.merge()
        self.gather()
        self.reduce()
        return self.out, self.alpha, self.top_vals, self.top_idx

    def __call__(self, queries: torch.Tensor, params: torch.Tensor | None = None):
        """Returns (out f32 [M, d_v] or None without value rows, alpha f32 [M, k],
        top_vals f32 [M, k], top_idx i32 [M, k])."""
        self.topk_local(queries, params)
        return self.finish()

    def status(self) -> int:
        """Device status word the fused kernel left in the workspace (syncs the stream)."""
        import ctypes
        lib = _lib.load()
        v = ctypes.c_int32(0)
        with torch.cuda.device(self.device):
            st = lib.dwa_workspace_status(self.workspace.data_ptr(), _stream_handle(self.device),
                                          ctypes.byref(v))
        _lib.check(st, "dwa_workspace_status")
        peer = self.peer.status() if self.peer is not None else 0
        return int(v.value) or peer

    def close(self) -> None:
        """Collective on a sharded pool: releases the NVLink exchange buffers (every
        rank calls it, after its last call).  The retriever is unusable afterwards."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None


class HostPipeline:
    """Retrieval batches streamed from pinned host memory and back, for serving.

    Each ``submit`` copies one batch of queries [M, d_k] from pinned host
    memory to the device of rank ``src`` (broadcast to the other ranks when
    the pool is sharded), runs the retrieval and copies (out, alpha, top_idx)
    back to the caller's pinned host buffers on rank ``src``.  The upload of a
    batch and the read-back of the previous one run on their own streams
    (PCIe carries both directions at once) while the previous / next batch
    computes, so the copies overlap the kernels instead of adding to them.
    Two ``Retriever`` instances over the same resident shard alternate, so a
    batch's result buffers stay untouched until their read-back has finished.

    Host buffers passed to ``submit`` must stay alive and unmodified until
    ``synchronize`` (or until the result of that batch has been waited for).
    """

    def __init__(self, keys_local: torch.Tensor, values_local: torch.Tensor, M: int, k: int, *,
                 src: int = 0, **retriever_kwargs):
        self.ret = [Retriever(keys_local, values_local, M, k, **retriever_kwargs) for _ in range(2)]
        r0 = self.ret[0]
        self.device = r0.device
        self.group, self.rank, self.world = r0.group, r0.rank, r0.world
        self.src = int(src)
        self.q_dev = [torch.empty((r0.M, r0.d_k), dtype=torch.bfloat16, device=self.device)
                      for _ in range(2)]
        self.h2d_stream = torch.cuda.Stream(self.device)
        self.d2h_stream = torch.cuda.Stream(self.device)
        ev = lambda: torch.cuda.Event()
        self.h2d_done = [ev(), ev()]
        self.compute_done = [ev(), ev()]
        self.d2h_done = [ev(), ev()]
        self.n = 0

    def submit(self, q_host: torch.Tensor | None, out_host: torch.Tensor | None = None,
               alpha_host: torch.Tensor | None = None, idx_host: torch.Tensor | None = None):
        """Enqueue one batch; returns the device results (out, alpha, top_vals, top_idx)
        of this batch, valid on the current stream."""
        b, n = self.n % 2, self.n
        is_src = self.rank == self.src
        cs = torch.cuda.current_stream(self.device)
        q = self.q_dev[b]
        if is_src:
            if q_host is None:
                raise ValueError("the source rank needs host queries")
            with torch.cuda.stream(self.h2d_stream):
                if n >= 2:  # batch n - 2 read this query buffer
                    self.h2d_stream.wait_event(self.compute_done[b])
                q.copy_(q_host, non_blocking=True)
                self.h2d_done[b].record(self.h2d_stream)
            cs.wait_event(self.h2d_done[b])
        if self.world > 1:
            dist.broadcast(q, src=dist.get_global_rank(self.group, self.src)
                           if self.group is not None else self.src, group=self.group)
        if n >= 2:  # batch n - 2's read-back of this retriever's buffers
            cs.wait_event(self.d2h_done[b])
        res = self.ret[b](q)
        self.compute_done[b].record(cs)
        if is_src:
            out, alpha, _, top_idx = res
            with torch.cuda.stream(self.d2h_stream):
                self.d2h_stream.wait_event(self.compute_done[b])
                for dst, srct in ((out_host, out), (alpha_host, alpha), (idx_host, top_idx)):
                    if dst is not None:
                        dst.copy_(srct, non_blocking=True)
                self.d2h_done[b].record(self.d2h_stream)
        else:
            self.d2h_done[b].record(cs)
        self.n += 1
        return res

    def join(self) -> None:
        """Make the current stream wait for every enqueued copy (no host sync)."""
        cs = torch.cuda.current_stream(self.device)
        cs.wait_stream(self.h2d_stream)
        cs.wait_stream(self.d2h_stream)

    def synchronize(self) -> None:
        self.join()
        torch.cuda.current_stream(self.device).synchronize()

    def status(self) -> int:
        return max(r.status() for r in self.ret)

    def close(self) -> None:
        """Collective on a sharded pool: waits for the enqueued work, then releases both
        retrievers' NVLink buffers."""
        self.synchronize()
        for r in self.ret:
            r.close()


class HybridParts(NamedTuple):
    """Outputs and intermediates of one ``pallas_hybrid_forward`` call."""
    alpha: torch.Tensor           # f32 [B, seq, k]
    top_idx: torch.Tensor         # i32 [B, seq, k] global pool rows
    sims_seq: torch.Tensor        # f32 [B, N_local]
    alpha_raw_seq: torch.Tensor   # f32 [B, N_local]
    queries_flat: torch.Tensor    # bf16 [B * seq, d_k]: the queries the score kernel saw
    keys_w: torch.Tensor          # bf16 [N_local, d_k]: the keys the score kernel saw
    tau: torch.Tensor             # f32 0-d, device: w . tau (0 without the gate)
    top_vals: torch.Tensor        # f32 [B * seq, k]: fused scores of the global top-k


def project_keys(vectors: torch.Tensor, W_K: torch.Tensor, w: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """keys_w [N, d_k] bf16 = sum_s w[s] k_s / (|k_s| + 1e-8), k_s = W_K[s] @ v, for the
    pool rows ``vectors`` [N, D] (retrieval.py:241-242, 253, 261) in one tcgen05 GEMM
    with the normalisation and aspect collapse in its epilogue (``dwa_project_keys``).

    W_K [S, d_k, D] (converted to bf16), w [S] aspect weights (softmax of the
    aspect logits).  d_k in {32, 64, 128}, D % 8 == 0.
    """
    v = _as_bf16_rows(vectors, "vectors")
    S, d_k, D = W_K.shape
    if v.shape[1] != D:
        raise ValueError(f"vectors must be [N, {D}]")
    wk = W_K.to(device=v.device, dtype=torch.bfloat16).reshape(S * d_k, D).contiguous()
    wv = w.to(device=v.device, dtype=torch.float32).contiguous()
    N = v.shape[0]
    if out is None:
        out = torch.empty((N, d_k), dtype=torch.bfloat16, device=v.device)
    lib = _lib.load()
    with torch.cuda.device(v.device):
        st = lib.dwa_project_keys(v.data_ptr(), N, v.stride(0), D, wk.data_ptr(), wk.stride(0), S,
                                  d_k, wv.data_ptr(), out.data_ptr(), out.stride(0), None,
                                  _stream_handle(v.device))
    _lib.check(st, "dwa_project_keys")
    return out


def project_keys_packed(vectors: torch.Tensor, W_K: torch.Tensor, w: torch.Tensor,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-aspect pool keys side by side, [N, S d_k] bf16:
    out[n, s d_k : (s + 1) d_k] = sqrt(w[s]) k_s / (|k_s| + 1e-8), k_s = W_K[s] @ v
    (``dwa_project_keys_packed``: one tcgen05 GEMM, normalisation and scaling in
    its epilogue).  With queries packed the same way, one dot product of length
    S d_k is hybrid_forward's aspect-weighted score sum_s w_s <q_s, k_s>
    (reference retrieval.py:154-165)."""
    v = _as_bf16_rows(vectors, "vectors")
    S, d_k, D = W_K.shape
    if v.shape[1] != D:
        raise ValueError(f"vectors must be [N, {D}]")
    wk = W_K.to(device=v.device, dtype=torch.bfloat16).reshape(S * d_k, D).contiguous()
    wv = w.to(device=v.device, dtype=torch.float32).contiguous()
    N = v.shape[0]
    if out is None:
        out = torch.empty((N, S * d_k), dtype=torch.bfloat16, device=v.device)
    lib = _lib.load()
    with torch.cuda.device(v.device):
        st = lib.dwa_project_keys_packed(v.data_ptr(), N, v.stride(0), D, wk.data_ptr(),
                                         wk.stride(0), S, d_k, wv.data_ptr(), out.data_ptr(),
                                         out.stride(0), None, _stream_handle(v.device))
    _lib.check(st, "dwa_project_keys_packed")
    return out


class MultiAspectRetrieval:
    """Parameters and ``pallas_hybrid_forward`` of the reference's retrieval
    module (src/model/retrieval.py:7-46, 204-343) on B200.

    The projection, normalisation and aspect collapse (241-263) are dense
    einsums on cuBLAS; the per-shard score + top-k, the cross-shard merge and
    the alpha normalisation (280-326) run on this library's kernels.  ``mesh``
    takes a torch.distributed process group (the reference's ``Mesh``); with
    ``tp_axis`` None or no group the single-chip path is used, as in the
    reference (314-319).  The collapsed ``tau = w . tau`` stays on the device:
    the kernels read it there (``dwa_score_topk_dev``, ``dwa_seq_scores``), as
    the reference passes it to its kernel as an operand.
    """

    def __init__(self, D: int, d_A: int, S: int, d_k: int, N: int, device=None,
                 dtype=torch.bfloat16, seed: int = 0):
        dev = torch.device(device) if device is not None else torch.device("cuda")
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.S, self.d_k, self.N = S, d_k, N
        self.W_Q = (torch.randn(S, d_k, d_A, device=dev, generator=g) * d_A ** -0.5).to(dtype)
        self.W_K = (torch.randn(S, d_k, D, device=dev, generator=g) * D ** -0.5).to(dtype)
        self.aspect_logits = torch.zeros(S, device=dev)
        self.tau = torch.zeros(S, device=dev)

    @staticmethod
    def _normalize(x: torch.Tensor) -> torch.Tensor:
        return x / (torch.linalg.norm(x, dim=-1, keepdim=True) + 1e-8)

    def _project_queries(self, z: torch.Tensor) -> torch.Tensor:
        """sum_d W_Q[s, k, d] z[b, t, d] in fp32 (retrieval.py:159, 247), f32 [B, seq, S, d_k].

        For bf16 z every product with a bf16 weight is exact in fp32, so the fp32
        einsum equals bf16 tensor-core GEMMs with fp32 accumulation: one GEMM for
        bf16 W_Q; for fp32 W_Q, W_Q = hi + mid + lo (three bf16 parts, together
        within 2^-24 of W_Q) and three GEMMs accumulating into one fp32 result.
        fp32 z keeps the fp32 einsum."""
        B, seq, d_A = z.shape
        if z.dtype != torch.bfloat16 or not z.is_cuda:
            return torch.einsum("skd,btd->btsk", self.W_Q.float(), z.float())
        z2 = z.reshape(B * seq, d_A)
        W = self.W_Q.reshape(self.S * self.d_k, d_A)
        if W.dtype == torch.bfloat16:
            q = torch.mm(z2, W.t(), out_dtype=torch.float32)
        else:
            Wf = W.float()
            hi = Wf.to(torch.bfloat16)
            r = Wf - hi.float()
            mid = r.to(torch.bfloat16)
            lo = (r - mid.float()).to(torch.bfloat16)
            q = torch.mm(z2, hi.t(), out_dtype=torch.float32)
            q = torch.addmm(q, z2, mid.t(), out_dtype=torch.float32)
            q = torch.addmm(q, z2, lo.t(), out_dtype=torch.float32)
        return q.view(B, seq, self.S, self.d_k)

    def project_keys(self, vectors: torch.Tensor, w: torch.Tensor, chunk_rows: int = 1 << 18
                     ) -> torch.Tensor:
        """keys_w = sum_s w_s W_K[s] v / (|W_K[s] v| + 1e-8) for every pool row
        (retrieval.py:241-242, 261).  With bf16 W_K (the default) one fused tcgen05
        kernel (``dwa_project_keys``: bf16 operands, fp32 accumulation,
        normalisation and collapse in its epilogue) when d_k is 32, 64 or 128 and
        D % 8 == 0; with fp32 W_K, fp32 cuBLAS GEMMs chunked over rows, so the
        projection keeps the parameters' precision.  The (S, N, d_k) tensor is
        never materialised."""
        N, D = vectors.shape
        if (self.W_K.dtype == torch.bfloat16 and self.d_k in (32, 64, 128) and D % 8 == 0
                and vectors.is_cuda):
            return project_keys(vectors, self.W_K, w)
        out = torch.empty((N, self.d_k), dtype=torch.bfloat16, device=vectors.device)
        WK = self.W_K.float()
        for r0 in range(0, N, chunk_rows):
            v = vectors[r0:r0 + chunk_rows].float()
            acc = torch.zeros((v.shape[0], self.d_k), device=v.device)
            for s in range(self.S):
                acc += w[s] * self._normalize(v @ WK[s].T)
            out[r0:r0 + chunk_rows] = acc.to(torch.bfloat16)
        return out

    def project_keys_packed(self, vectors: torch.Tensor, w: torch.Tensor,
                            chunk_rows: int = 1 << 16) -> torch.Tensor:
        """[sqrt(w_s) W_K[s] v / (|W_K[s] v| + 1e-8)]_s for every pool row, [N, S d_k]
        bf16.  bf16 W_K: the fused tcgen05 kernel (``dwa_project_keys_packed``) when
        d_k is 32, 64 or 128 and D % 8 == 0; fp32 W_K: fp32 GEMMs chunked over
        rows, keeping the parameters' precision."""
        N, D = vectors.shape
        if (self.W_K.dtype == torch.bfloat16 and self.d_k in (32, 64, 128) and D % 8 == 0
                and vectors.is_cuda):
            return project_keys_packed(vectors, self.W_K, w)
        out = torch.empty((N, self.S * self.d_k), dtype=torch.bfloat16, device=vectors.device)
        WK = self.W_K.float()
        sw = w.float().sqrt()
        for r0 in range(0, N, chunk_rows):
            v = vectors[r0:r0 + chunk_rows].float()
            ks = self._normalize(torch.einsum("skd,nd->nsk", WK, v)) * sw[None, :, None]
            out[r0:r0 + chunk_rows] = ks.reshape(v.shape[0], -1).to(torch.bfloat16)
        return out

    def hybrid_parts(self, z: torch.Tensor, vectors: torch.Tensor, k_max: int, T: float = 1.0,
                     lambda_sharp: float = 1.0, use_sigmoid: bool = True) -> "HybridParts":
        """``hybrid_forward`` with its intermediates (queries_flat / keys_w are the
        packed [sqrt(w_s) q_s]_s / [sqrt(w_s) k_s]_s the score kernel saw)."""
        B, seq, d_A = z.shape
        w = torch.softmax(self.aspect_logits.float(), dim=0)                     # 164
        tau = (torch.dot(w, self.tau.float()) if use_sigmoid                    # 168
               else torch.zeros((), dtype=torch.float32, device=w.device))
        keys_p = self.project_keys_packed(vectors, w)                           # 155-156
        queries_s = self._normalize(self._project_queries(z))                  # 159-160
        q_packed = (queries_s * w.sqrt()[None, None, :, None]).reshape(B, seq, -1)
        queries_flat = q_packed.reshape(B * seq, -1).to(torch.bfloat16)
        # 163-175: the aspect-weighted score of every (position, key), its gate/exp,
        # the per-position top-k and the seq mean of the fused scores, in one kernel
        top_vals, top_idx, alpha_raw_seq = score_topk_seqmean(
            queries_flat, keys_p, k_max, lambda_sharp, tau, T, use_sigmoid, seq)
        alpha = normalise_alpha(top_vals).view(B, seq, k_max)                   # 178
        # 181: the seq mean of sims is linear in the query: one skinny product
        sims_seq, _ = seq_scores(q_packed.mean(dim=1), keys_p, lambda_sharp, tau, T, use_sigmoid)
        return HybridParts(alpha, top_idx.view(B, seq, k_max), sims_seq, alpha_raw_seq,
                           queries_flat, keys_p, tau, top_vals)

    def hybrid_forward(self, z: torch.Tensor, vectors: torch.Tensor, k_max: int, T: float = 1.0,
                       lambda_sharp: float = 1.0, use_sigmoid: bool = True):
        """Per-position retrieval over all N with the aspect-weighted score, keeping only
        the top-k (reference retrieval.py:131-181).  Returns (alpha f32 [B, seq, k],
        top_idx i32 [B, seq, k], sims_seq f32 [B, N], alpha_raw_seq f32 [B, N]).

        The score sum_s w_s <q_s, k_s> is one dot product of the packed
        [sqrt(w_s) q_s]_s and [sqrt(w_s) k_s]_s (d = S d_k), so it runs on the same
        fused score + top-k kernel as ``pallas_hybrid_forward``; alpha_raw_seq (the
        seq mean of the fused scores, which needs every score) is summed in that
        kernel's epilogue and never goes through HBM as a [B, seq, N] tensor."""
        p = self.hybrid_parts(z, vectors, k_max, T, lambda_sharp, use_sigmoid)
        return p.alpha, p.top_idx, p.sims_seq, p.alpha_raw_seq

    def pallas_hybrid_parts(self, z: torch.Tensor, vectors: torch.Tensor, k_max: int,
                            T: float = 1.0, lambda_sharp: float = 1.0, use_sigmoid: bool = True,
                            tp_axis: str | None = "tp", mesh=None) -> "HybridParts":
        """``pallas_hybrid_forward`` with its intermediates: the collapsed bf16
        queries and pool keys the score kernel saw, the collapsed tau and the
        global top-k's fused scores (what a parity check recomputes against)."""
        B, seq, d_A = z.shape
        w = torch.softmax(self.aspect_logits.float(), dim=0)                     # 253
        # 254: stays on the device; the kernels read it there (no host sync)
        tau = (torch.dot(w, self.tau.float()) if use_sigmoid
               else torch.zeros((), dtype=torch.float32, device=w.device))
        keys_w = self.project_keys(vectors, w)                                  # 241-242, 261
        zf = z.float()
        queries_s = self._normalize(self._project_queries(z))                  # 247-248
        queries_w = torch.einsum("s,btsk->btk", w, queries_s)                   # 262
        queries_flat = queries_w.reshape(B * seq, self.d_k).to(torch.bfloat16)  # 263
        group = mesh if (tp_axis is not None and mesh is not None) else None
        final_v, final_i = chip_topk(queries_flat, keys_w, k_max, lambda_sharp, tau, T,
                                     use_sigmoid, group=group)                  # 280-319
        alpha = normalise_alpha(final_v).view(B, seq, k_max)                    # 324-326
        top_idx = final_i.view(B, seq, k_max)
        z_mean = zf.mean(dim=1)                                                 # 332-336
        q_mean_s = self._normalize(torch.einsum("skd,bd->sbk", self.W_Q.float(), z_mean))
        q_mean_w = torch.einsum("s,sbk->bk", w, q_mean_s)
        sims_seq, alpha_raw_seq = seq_scores(q_mean_w, keys_w, lambda_sharp, tau, T,
                                             use_sigmoid)                       # 336-341
        return HybridParts(alpha, top_idx, sims_seq, alpha_raw_seq, queries_flat, keys_w, tau,
                           final_v)

    def pallas_hybrid_forward(self, z: torch.Tensor, vectors: torch.Tensor, k_max: int,
                              T: float = 1.0, lambda_sharp: float = 1.0, use_sigmoid: bool = True,
                              tp_axis: str | None = "tp", mesh=None):
        """Returns (alpha [B, seq, k], top_idx [B, seq, k], sims_seq [B, N_local],
        alpha_raw_seq [B, N_local]) like retrieval.py:204-343."""
        p = self.pallas_hybrid_parts(z, vectors, k_max, T, lambda_sharp, use_sigmoid, tp_axis,
                                     mesh)
        return p.alpha, p.top_idx, p.sims_seq, p.alpha_raw_seq
