"""Drop-in replacement for saf3r.triton.adaptive_block_attention.block_attention.

Same signature, argument meaning and return value as the reference
(saf3r/triton/adaptive_block_attention.py:63-83): inputs contiguous
[H, N, d] bf16/fp16 CUDA tensors, ``indices`` int32 [sparseH, ceil(N/BQ), maxK]
of unique patch-block ids of which the first ``counts[s]`` are read,
``head_ids`` int32 [sparseH]; returns ``(out, evidence)`` where only the rows of
the selected heads of ``out`` are written and ``evidence`` is fp32 with -inf in
unused slots.  A ValueError is raised for non-BF16/FP16 inputs, as in the
reference; unlike the reference, malformed shapes, counts, heads and ids are
also rejected (ValueError) instead of reading out of bounds.
"""
import math

import torch

from . import _lib, ops


def _status_message(bits):
    parts = []
    if bits & _lib.STATUS_BAD_INDEX:
        parts.append("a selected block id is outside [0, n_blocks)")
    if bits & _lib.STATUS_BAD_COUNT:
        parts.append("a count is negative or exceeds indices.shape[-1]")
    if bits & _lib.STATUS_BAD_HEAD:
        parts.append("a head id is outside [0, heads)")
    if bits & _lib.STATUS_TIMEOUT:
        parts.append("a device pipeline wait timed out")
    return "; ".join(parts)


def block_attention(q, patch_k, patch_v, special_k, special_v, indices, counts, head_ids, *,
                    query_block=64, key_block=64, scale=None, out=None, head_dense=None,
                    return_evidence=True, kernel="auto", validate=True):
    """Shared-within-query-block, head-specific exact sparse attention.

    Extensions beyond the reference signature (all keyword-only, defaults
    keep the reference behaviour): ``counts`` may be [sparseH, n_qblocks];
    ``head_dense`` [sparseH] bool routes a slot to the dense path of the same
    kernel; ``return_evidence=False`` skips the evidence pass (evidence is
    then all -inf); ``kernel`` picks 'auto' | 'tcgen05' | 'mma_sync';
    ``validate`` reads back the device status word (one host sync) and raises
    ValueError on a bad id, count or head.
    """
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError('Tensor-core sparse execution requires BF16 or FP16')
    h, n, d = q.shape
    if out is None:
        out = torch.empty_like(q)
    evidence = torch.full(indices.shape, -math.inf, device=q.device, dtype=torch.float32)
    status = torch.zeros(1, device=q.device, dtype=torch.int32) if validate else None
    if special_k is None:
        special_k = q.new_empty((h, 0, d))
        special_v = q.new_empty((h, 0, d))
    ops.launch_block_attention(q, patch_k, patch_v, special_k, special_v, indices, counts,
                               head_ids, head_dense=head_dense, query_block=query_block,
                               key_block=key_block, scale=scale, out=out,
                               evidence=evidence if return_evidence else None, status=status,
                               kernel=kernel)
    if validate:
        bits = int(status.item())
        if bits:
            raise ValueError("block_attention: " + _status_message(bits))
    return out, evidence
