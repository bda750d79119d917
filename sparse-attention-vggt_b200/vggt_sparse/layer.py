"""One sparse global-attention layer on the device: the hot path.

``SparseGlobalLayer`` runs the block-mask estimator on the sparse heads and
ONE attention launch that serves sparse heads from their index lists and
dense-profiled heads through the dense path of the same kernel.  It replaces
steps 4-7 of the reference wrapper (saf3r/patch/adaptive_block_value.py:314-404)
for a fixed retention / mass rule: estimator -> masks -> block_attention for
sparse heads, SDPA for dense heads.
"""
import math

import torch

from . import ops
from .estimator import EstimatorWorkspace, block_mask_estimate, mask_capacity
from .profile import split_heads


def topk_budget(rho, n_tokens, n_special, n_blocks, key_block):
    """Blocks kept for retention rho (saf3r/patch/adaptive_block_value.py:187)."""
    return min(n_blocks, max(1, math.ceil((round(rho * n_tokens) - n_special) / key_block)))


class SparseGlobalLayer:
    """Estimator + block-sparse attention for one layer shape.

    mode 'topk' keeps topk_budget(retention) blocks per query block (or an
    explicit ``topk``); mode 'mass' keeps the smallest prefix of pooled-score
    softmax mass >= tau.  ``dense_heads`` go through the dense path.
    ``head_subset`` restricts the layer to some heads (their K/V alone need
    to be in place when it runs).
    """

    def __init__(self, heads, *, mode="topk", retention=0.25, topk=None, tau=0.9,
                 dense_heads=(), block=64, kernel="auto", evidence=False, head_subset=None):
        if mode not in ("topk", "mass"):
            raise ValueError("mode must be 'topk' or 'mass'")
        self.heads = heads
        self.mode, self.retention, self.topk, self.tau = mode, retention, topk, tau
        self.block = block
        self.kernel = kernel
        self.evidence = evidence
        self.sparse_heads, self.dense_heads = split_heads(heads, dense_heads)
        if head_subset is not None:
            # serve only these heads (the others' rows of `out` are not written)
            keep = set(int(h) for h in head_subset)
            if not keep <= set(range(heads)):
                raise ValueError("head_subset must name heads in [0, %d)" % heads)
            self.sparse_heads = [h for h in self.sparse_heads if h in keep]
            self.dense_heads = [h for h in self.dense_heads if h in keep]
        self.workspace = EstimatorWorkspace()
        self._cache = {}
        self.last_masks = None
        # pair query blocks by selection overlap for the 128-row tcgen05 tiles
        self.pair_qblocks = True
        self.last_evidence = None

    def budget(self, n_tokens, n_special, n_blocks):
        if self.mode == "mass":
            return None
        if self.topk is not None:
            return min(int(self.topk), n_blocks)
        return topk_budget(self.retention, n_tokens, n_special, n_blocks, self.block)

    def _buffers(self, device, n_tokens, n_patch, n_special):
        key = (device, n_tokens, n_patch, n_special)
        buf = self._cache.get(key)
        if buf is None:
            qbc = math.ceil(n_tokens / self.block)
            nb = math.ceil(n_patch / self.block)
            k = self.budget(n_tokens, n_special, nb)
            cap = mask_capacity(self.mode, k or nb, nb)
            s = len(self.sparse_heads)
            slots = self.sparse_heads + self.dense_heads
            # a layer of dense slots only still passes one (never read) slot of
            # indices and counts: the C ABI takes no NULL mask pointers
            sa = max(s, 1)
            buf = dict(
                topk=k,
                indices=torch.full((sa, qbc, cap), -1, device=device, dtype=torch.int32),
                counts=torch.zeros((sa, qbc), device=device, dtype=torch.int32),
                sparse_ids=torch.tensor(self.sparse_heads, device=device, dtype=torch.int32),
                slot_ids=torch.tensor(slots, device=device, dtype=torch.int32),
                dense_flags=torch.tensor([0] * s + [1] * len(self.dense_heads), device=device,
                                         dtype=torch.uint8),
                evidence=torch.empty((sa, qbc, cap), device=device, dtype=torch.float32),
            )
            ws = ops.attention_workspace_size(n_tokens, n_patch, len(slots), self.block,
                                              self.block) if s else 0
            buf["attn_ws"] = (torch.empty(ws, device=device, dtype=torch.uint8) if ws else None)
            self._cache[key] = buf
        return buf

    def estimate(self, q, kp, n_special):
        """The block-mask estimator alone (masks kept for ``attend``); needs
        only q and the patch keys, so a caller can run it while V (or the
        specials) are still arriving."""
        h, n, d = q.shape
        if h != self.heads:
            raise ValueError("layer built for %d heads, got %d" % (self.heads, h))
        buf = self._buffers(q.device, n, kp.shape[1], n_special)
        if self.sparse_heads:
            block_mask_estimate(q, kp, head_ids=buf["sparse_ids"], query_block=self.block,
                                key_block=self.block, mode=self.mode, topk=buf["topk"],
                                tau=self.tau, workspace=self.workspace,
                                out=(buf["indices"], buf["counts"]))
        self.last_masks = (buf["indices"], buf["counts"])
        return buf

    def estimate_pooled(self, pooled_q, pooled_k, n_tokens, n_patch, n_special):
        """The estimator's selection from block means of every head (pooled_q
        [H, QB, d], pooled_k [H, NB, d] fp32, e.g. from ``project_qkv``): the
        masks of ``estimate`` without another pass over Q and K."""
        buf = self._buffers(pooled_q.device, n_tokens, n_patch, n_special)
        if self.sparse_heads:
            ops.launch_block_select_pooled(pooled_q, pooled_k, buf["sparse_ids"],
                                           mode=self.mode, topk=buf["topk"], tau=self.tau,
                                           scale=pooled_q.shape[-1] ** -0.5,
                                           indices=buf["indices"], counts=buf["counts"])
        self.last_masks = (buf["indices"], buf["counts"])
        return buf

    def forward_projected(self, qkv, out=None):
        """The layer on the outputs of ``vggt_sparse.project_qkv`` (q, split
        K/V and block means): selection from the means, then attention."""
        n, npatch, nspecial = qkv.q.shape[1], qkv.patch_k.shape[1], qkv.special_k.shape[1]
        self.estimate_pooled(qkv.pooled_q, qkv.pooled_k, n, npatch, nspecial)
        return self.attend(qkv.q, qkv.patch_k, qkv.patch_v, qkv.special_k, qkv.special_v,
                           out=out)

    def attend(self, q, kp, vp, ks, vs, out=None):
        """Block-sparse attention with the masks of the last ``estimate``."""
        h, n, d = q.shape
        buf = self._buffers(q.device, n, kp.shape[1], ks.shape[1])
        if out is None:
            out = torch.empty_like(q)
        evidence = None
        if self.evidence and self.sparse_heads:
            evidence = buf["evidence"]
            evidence.fill_(-math.inf)
        ops.launch_block_attention(q, kp, vp, ks, vs, buf["indices"], buf["counts"],
                                   buf["slot_ids"], head_dense=buf["dense_flags"],
                                   query_block=self.block, key_block=self.block, out=out,
                                   evidence=evidence, kernel=self.kernel,
                                   pair_qblocks=self.pair_qblocks and bool(self.sparse_heads),
                                   workspace=buf["attn_ws"])
        self.last_masks = (buf["indices"], buf["counts"])
        self.last_evidence = evidence
        return out

    def __call__(self, q, kp, vp, ks, vs, out=None, events=None):
        """Run the layer; ``events`` (3 CUDA events) are recorded before the
        estimator, between estimator and attention, and after attention."""
        if events is not None:
            events[0].record()
        self.estimate(q, kp, ks.shape[1])
        if events is not None:
            events[1].record()
        out = self.attend(q, kp, vp, ks, vs, out=out)
        if events is not None:
            events[2].record()
        return out

    def kept_flops(self, n_tokens, n_patch, n_special, dim):
        """Algorithmic FLOPs of the last call: 4*d*sum(valid rows x (kept valid
        keys + specials)) over sparse heads + 4*d*rows*(n_patch + n_special)
        per dense head (4*d*N*N for a whole layer).  ``n_tokens`` is the
        number of query rows of the call (a shard's rows under query-block
        sharding)."""
        bq = bk = self.block
        qbc = math.ceil(n_tokens / bq)
        nb = math.ceil(n_patch / bk)
        total = 0.0
        rows = torch.full((qbc,), float(bq), dtype=torch.float64)
        rows[-1] = n_tokens - (qbc - 1) * bq
        if self.sparse_heads and self.last_masks is not None:
            idx, cnt = (t.cpu() for t in self.last_masks)
            last_cols = n_patch - (nb - 1) * bk
            slot = torch.arange(idx.shape[-1])[None, None, :] < cnt[..., None].long()
            cols = torch.where(idx == nb - 1, float(last_cols), float(bk)).double() * slot
            keys = cols.sum(-1) + n_special
            total += 4.0 * dim * float((keys * rows[None]).sum())
        total += 4.0 * dim * float(n_tokens) * float(n_patch + n_special) * len(self.dense_heads)
        return total
