"""Block-mask estimator: the device op that replaces the reference's PyTorch
pooling + routing + mask assembly (saf3r/patch/adaptive_block_value.py:315-362)
with mean-pooled Q/K block scores and on-device selection.
"""
import math
from dataclasses import dataclass

import torch

from . import ops


@dataclass
class BlockMasks:
    """Output of the estimator for the estimated heads (slots).

    indices  int32 [slots, n_qblocks, max_blocks], ascending block ids, -1 padded
    counts   int32 [slots, n_qblocks]  (the per-row extension of the reference's
             per-head counts)
    scores   fp32 [slots, n_qblocks, n_blocks] pooled scores, when exported
    """
    indices: torch.Tensor
    counts: torch.Tensor
    scores: torch.Tensor | None = None


class EstimatorWorkspace:
    """Reusable device scratch for the pooled Q/K rows (sized on first use)."""

    def __init__(self):
        self._buf = None

    def get(self, numel, device):
        if self._buf is None or self._buf.numel() < numel or self._buf.device != device:
            self._buf = torch.empty(numel, device=device, dtype=torch.float32)
        return self._buf[:numel]


def mask_capacity(mode, topk, n_blocks):
    """Slots per row the index tensor needs for a selection rule."""
    return min(int(topk), n_blocks) if mode == "topk" else n_blocks


def block_mask_estimate(q, k_patch, *, head_ids=None, query_block=64, key_block=64, mode="topk",
                        topk=None, tau=None, scale=None, export_scores=False, max_blocks=None,
                        workspace=None, out=None, status=None):
    """Pool, score and select key blocks for every (head, query block).

    q [H, N, d] (all tokens), k_patch [H, NP, d] (patch tokens only), bf16/fp16
    CUDA tensors.  mode 'topk' keeps ``topk`` blocks per row (ties to the lower
    id); mode 'mass' keeps the smallest descending prefix whose softmax mass
    over pooled scores reaches ``tau``.  Specials are not pooled: the
    attention operator always attends them.
    """
    if q.dim() != 3 or k_patch.dim() != 3:
        raise ValueError("q and k_patch must be [heads, tokens, dim]")
    h, n, d = q.shape
    device = q.device
    if head_ids is None:
        head_ids = torch.arange(h, device=device, dtype=torch.int32)
    elif not torch.is_tensor(head_ids):
        head_ids = torch.tensor(list(head_ids), device=device, dtype=torch.int32)
    head_ids = head_ids.to(device=device, dtype=torch.int32).contiguous()
    if mode not in ("topk", "mass"):
        raise ValueError("mode must be 'topk' or 'mass'")
    if mode == "topk" and (topk is None or int(topk) < 1):
        raise ValueError("topk mode needs topk >= 1")
    if mode == "mass" and (tau is None or not 0.0 < float(tau) <= 1.0):
        raise ValueError("mass mode needs 0 < tau <= 1")
    scale = d ** -0.5 if scale is None else float(scale)
    s = head_ids.numel()
    qbc = math.ceil(n / query_block)
    nb = math.ceil(k_patch.shape[1] / key_block)
    cap = mask_capacity(mode, topk, nb) if max_blocks is None else int(max_blocks)
    if out is not None:
        indices, counts = out
    else:
        indices = torch.empty((s, qbc, cap), device=device, dtype=torch.int32)
        counts = torch.empty((s, qbc), device=device, dtype=torch.int32)
    ws = workspace or EstimatorWorkspace()
    # pooled_q rows first, pooled_k rows after; both 16-byte aligned (d % 4 == 0)
    buf = ws.get(s * (qbc + nb) * d, device)
    pooled_q = buf[: s * qbc * d].view(s, qbc, d)
    pooled_k = buf[s * qbc * d:].view(s, nb, d)
    scores = torch.empty((s, qbc, nb), device=device, dtype=torch.float32) if export_scores else None
    ops.launch_block_mask_estimate(q, k_patch, head_ids, query_block=query_block,
                                   key_block=key_block, mode=mode, topk=topk, tau=tau, scale=scale,
                                   pooled_q=pooled_q, pooled_k=pooled_k, indices=indices,
                                   counts=counts, scores=scores, status=status)
    return BlockMasks(indices, counts, scores)


def block_select(scores, *, mode="topk", topk=None, tau=None):
    """Re-run the selection rule on fp32 scores [..., n_blocks] on the device."""
    nb = scores.shape[-1]
    cap = mask_capacity(mode, topk, nb)
    lead = scores.shape[:-1]
    indices = torch.empty((*lead, cap), device=scores.device, dtype=torch.int32)
    counts = torch.empty(lead, device=scores.device, dtype=torch.int32)
    ops.launch_block_select(scores.contiguous(), mode=mode, topk=topk, tau=tau, indices=indices,
                            counts=counts)
    return indices, counts
