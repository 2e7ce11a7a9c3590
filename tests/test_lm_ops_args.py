"""CPU: Python wrappers (the LM block kernels, the shard merge) reject what
their kernels cannot take before anything reaches the library (no GPU is
touched)."""
import pytest
import torch

from computd_b200.lm_ops import aspect_queries, rope_qk


def test_rope_qk_rejects_bad_inputs():
    cs = torch.zeros((64, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError):       # host tensor
        rope_qk(torch.zeros((2, 64, 48), dtype=torch.bfloat16), cs, cs, 2, 16)
    with pytest.raises(ValueError):       # not bf16
        rope_qk(torch.zeros((2, 64, 48)), cs, cs, 2, 16)
    with pytest.raises(ValueError):       # not [B, S, W]
        rope_qk(torch.zeros((64, 48), dtype=torch.bfloat16), cs, cs, 2, 16)


def test_aspect_queries_rejects_bad_inputs():
    logits = torch.zeros(4)
    with pytest.raises(ValueError):       # host tensor
        aspect_queries(torch.zeros((8, 256), dtype=torch.bfloat16), 4, 64, logits, None, 1.0,
                       1.0, False)
    with pytest.raises(ValueError):       # not bf16
        aspect_queries(torch.zeros((8, 256)), 4, 64, logits, None, 1.0, 1.0, False)
    with pytest.raises(ValueError):       # strided columns
        aspect_queries(torch.zeros((256, 8), dtype=torch.bfloat16).t(), 4, 64, logits, None,
                       1.0, 1.0, False)


def test_merge_topk_rejects_host_lists():
    from computd_b200.tiled_topk import merge_topk

    with pytest.raises(ValueError):
        merge_topk(torch.zeros((2, 4, 8)), torch.zeros((2, 4, 8), dtype=torch.int32))
