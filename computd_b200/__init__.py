"""computd_b200 — B200-native (sm_100a) DWA retrieval hot path.

Drop-in for computd's retrieval path (reference: src/kernels/tiled_topk.py,
src/model/retrieval.py, src/model/assembly.py): fused query x pool-key score
GEMM with a streaming top-k epilogue (tcgen05/TMEM/TMA), cross-shard merge,
and the softmax-weighted gather of pool value rows.  All compute runs in
``libdwa_b200.so`` through the C ABI of ``include/dwa_retrieval.h``; PyTorch
provides device memory, streams and torch.distributed plumbing only.
"""
from ._lib import DWA_MAX_K, DWAArgumentError, DWAError, load as load_library
from .assembler import WeightAssembler, assemble_finish, lowrank_delta, usage_ema_update
from .assembly import normalise_alpha, weighted_gather_into, weighted_value_sum
from .pool import ShardSpec, init_normal, new_normal
from .retrieval import (HostPipeline, HybridParts, MultiAspectRetrieval, PeerExchange, Retriever,
                        chip_topk, exchange_candidates, project_keys, project_keys_packed,
                        reduce_partials)
from .tiled_topk import (merge_topk, score_params, score_topk_into, score_topk_seqmean, seq_scores,
                         tiled_topk_fallback, tiled_topk_fused, workspace_bytes)

__all__ = [
    "DWA_MAX_K", "DWAArgumentError", "DWAError", "load_library",
    "WeightAssembler", "assemble_finish", "lowrank_delta", "usage_ema_update",
    "normalise_alpha", "weighted_gather_into", "weighted_value_sum", "MultiAspectRetrieval",
    "ShardSpec", "init_normal", "new_normal",
    "HostPipeline", "HybridParts", "PeerExchange", "Retriever", "chip_topk", "project_keys",
    "project_keys_packed", "exchange_candidates", "reduce_partials",
    "merge_topk", "score_params", "score_topk_into", "score_topk_seqmean", "seq_scores",
    "tiled_topk_fallback", "tiled_topk_fused", "workspace_bytes",
]
