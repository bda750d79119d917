"""Tensor-level launchers over the C ABI, and their ``torch.ops`` registration.

Launchers take CUDA tensors, pass raw pointers and the current CUDA stream to
``libvggt_sparse.so`` and never synchronise.  ``torch.ops.vggt_sparse.*``
wraps them as functional custom operators (with fake implementations so they
trace under ``torch.library`` tooling).
"""
import math

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16}
KERNELS = {"auto": _lib.ATTN_AUTO, "mma_sync": _lib.ATTN_MMA_SYNC, "tcgen05": _lib.ATTN_TCGEN05}
MODES = {"topk": _lib.SELECT_TOPK, "mass": _lib.SELECT_MASS}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("vggt_sparse operators take CUDA tensors (there is no CPU path)")


def _require_contig(**named):
    for name, t in named.items():
        if t is not None and not t.is_contiguous():
            raise ValueError("%s must be contiguous" % name)


def dtype_code(dtype):
    if dtype not in _DTYPES:
        raise ValueError("Tensor-core sparse execution requires BF16 or FP16")
    return _DTYPES[dtype]


def attention_workspace_size(n_tokens, n_patch, n_slots, query_block=64, key_block=64):
    """Bytes of the query-block pairing workspace (0 when not paired)."""
    return int(_lib.load().vggt_block_attention_workspace_size(n_tokens, n_patch, n_slots,
                                                                 query_block, key_block))


def launch_block_attention(q, patch_k, patch_v, special_k, special_v, indices, counts, head_ids,
                           *, head_dense=None, query_block=64, key_block=64, scale=None, out,
                           evidence=None, status=None, kernel="auto", pair_qblocks=True,
                           workspace=None):
    """Enqueue one block-sparse attention launch (see vggt_block_attention).

    With ``pair_qblocks`` (and a kernel choice other than mma_sync) the call
    goes through vggt_block_attention_ex with a device workspace, so the
    tcgen05 kernel pairs query blocks by selection overlap; ``workspace`` may
    pass a reusable uint8 CUDA buffer of at least the size query's bytes."""
    _require_cuda(q, patch_k, patch_v, special_k, special_v, indices, counts, head_ids, head_dense,
                  out, evidence, status)
    _require_contig(q=q, patch_k=patch_k, patch_v=patch_v, special_k=special_k,
                    special_v=special_v, indices=indices, counts=counts, head_ids=head_ids,
                    out=out, evidence=evidence)
    code = dtype_code(q.dtype)
    for name, t in (("patch_k", patch_k), ("patch_v", patch_v), ("special_k", special_k),
                    ("special_v", special_v), ("out", out)):
        if t is not None and t.dtype != q.dtype:
            raise ValueError("%s dtype %s differs from q dtype %s" % (name, t.dtype, q.dtype))
    if q.dim() != 3:
        raise ValueError("q must be [heads, tokens, dim]")
    h, n, d = q.shape
    npatch, nspecial = patch_k.shape[1], special_k.shape[1] if special_k is not None else 0
    if patch_k.shape != (h, npatch, d) or patch_v.shape != patch_k.shape:
        raise ValueError("patch_k/patch_v must be [heads, n_patch, dim] matching q")
    if special_k is not None and (special_k.shape != (h, nspecial, d) or
                                  special_v.shape != special_k.shape):
        raise ValueError("special_k/special_v must be [heads, n_special, dim] matching q")
    if out.shape != q.shape:
        raise ValueError("out must have the shape of q")
    for name, t in (("indices", indices), ("counts", counts), ("head_ids", head_ids)):
        if t.dtype != torch.int32:
            raise ValueError("%s must be int32" % name)
    n_slots = head_ids.numel()
    qbc = math.ceil(n / query_block)
    if indices.dim() != 3 or indices.shape[1] != qbc:
        raise ValueError("indices must be [slots, ceil(N/query_block), max_blocks]")
    n_sparse = indices.shape[0]
    if counts.dim() == 1:
        per_row = 0
        if counts.numel() < n_sparse:
            raise ValueError("counts must have one entry per indexed slot")
    elif counts.dim() == 2 and counts.shape[1] == qbc:
        per_row = 1
        if counts.shape[0] < n_sparse:
            raise ValueError("counts must have one row per indexed slot")
    else:
        raise ValueError("counts must be [slots] or [slots, ceil(N/query_block)]")
    if head_dense is not None:
        if head_dense.dtype not in (torch.uint8, torch.bool) or head_dense.numel() != n_slots:
            raise ValueError("head_dense must be uint8/bool [slots]")
        head_dense = head_dense.to(torch.uint8)
    if n_sparse < n_slots and head_dense is None:
        raise ValueError("indices has fewer slots than head_ids and no head_dense flags")
    if evidence is not None and (evidence.dtype != torch.float32 or evidence.shape != indices.shape):
        raise ValueError("evidence must be float32 with the shape of indices")
    scale = d ** -0.5 if scale is None else float(scale)
    lib = _lib.load()
    ws_bytes = 0
    if pair_qblocks and kernel != "mma_sync" and indices.shape[2] > 0:
        ws_bytes = int(lib.vggt_block_attention_workspace_size(n, npatch, n_slots, query_block,
                                                               key_block))
    if ws_bytes > 0:
        if workspace is None or workspace.numel() < ws_bytes:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
        _require_cuda(workspace)
    else:
        workspace = None
    rc = lib.vggt_block_attention_ex(
        _ptr(q), _ptr(patch_k), _ptr(patch_v), _ptr(special_k), _ptr(special_v), code, h, n,
        npatch, nspecial, d, _ptr(indices), _ptr(counts), per_row, _ptr(head_ids),
        _ptr(head_dense), n_slots, indices.shape[2], query_block, key_block, scale, _ptr(out),
        _ptr(evidence), _ptr(status), KERNELS[kernel], _stream(q.device), _ptr(workspace),
        ws_bytes)
    _lib.check(rc)
    return out, evidence


def launch_block_mask_estimate(q, k_patch, head_ids, *, query_block, key_block, mode, topk, tau,
                               scale, pooled_q, pooled_k, indices, counts, scores=None,
                               status=None):
    """Enqueue pooling + scoring + selection (see vggt_block_mask_estimate)."""
    _require_cuda(q, k_patch, head_ids, pooled_q, pooled_k, indices, counts, scores, status)
    _require_contig(q=q, k_patch=k_patch, head_ids=head_ids, pooled_q=pooled_q,
                    pooled_k=pooled_k, indices=indices, counts=counts, scores=scores)
    code = dtype_code(q.dtype)
    if k_patch.dtype != q.dtype:
        raise ValueError("k_patch dtype differs from q dtype")
    h, n, d = q.shape
    npatch = k_patch.shape[1]
    lib = _lib.load()
    rc = lib.vggt_block_mask_estimate(
        _ptr(q), _ptr(k_patch), code, h, n, npatch, d, _ptr(head_ids), head_ids.numel(),
        query_block, key_block, MODES[mode], int(topk or 0), float(tau or 0.0), float(scale),
        _ptr(pooled_q), _ptr(pooled_k), _ptr(indices), indices.shape[-1], _ptr(counts),
        _ptr(scores), _ptr(status), _stream(q.device))
    _lib.check(rc)
    return indices, counts, scores


def launch_block_select_pooled(pooled_q, pooled_k, head_ids, *, mode, topk=None, tau=None,
                               scale, indices, counts, scores=None, status=None):
    """Enqueue scores + selection from block means of every head (pooled_q
    [H, QB, d], pooled_k [H, NB, d] fp32); slot s uses head head_ids[s]."""
    _require_cuda(pooled_q, pooled_k, head_ids, indices, counts, scores, status)
    _require_contig(pooled_q=pooled_q, pooled_k=pooled_k, head_ids=head_ids, indices=indices,
                    counts=counts, scores=scores)
    if pooled_q.dtype != torch.float32 or pooled_k.dtype != torch.float32:
        raise ValueError("pooled means must be float32")
    if pooled_q.dim() != 3 or pooled_k.dim() != 3 or pooled_q.shape[0] != pooled_k.shape[0] or \
            pooled_q.shape[2] != pooled_k.shape[2]:
        raise ValueError("pooled_q [H, QB, d] and pooled_k [H, NB, d] expected")
    h, qbc, d = pooled_q.shape
    if indices.shape[:2] != (head_ids.numel(), qbc) or counts.shape != (head_ids.numel(), qbc):
        raise ValueError("indices [slots, QB, max_blocks] and counts [slots, QB] expected")
    lib = _lib.load()
    rc = lib.vggt_block_select_pooled(
        _ptr(pooled_q), _ptr(pooled_k), h, _ptr(head_ids), head_ids.numel(), qbc,
        pooled_k.shape[1], d, MODES[mode], int(topk or 0), float(tau or 0.0), float(scale),
        _ptr(indices), indices.shape[-1], _ptr(counts), _ptr(scores), _ptr(status),
        _stream(pooled_q.device))
    _lib.check(rc)
    return indices, counts


def launch_block_select(scores, *, mode, topk=None, tau=None, indices, counts):
    """Enqueue selection from fp32 scores [..., n_blocks]."""
    _require_cuda(scores, indices, counts)
    _require_contig(scores=scores, indices=indices, counts=counts)
    if scores.dtype != torch.float32:
        raise ValueError("scores must be float32")
    nb = scores.shape[-1]
    rows = scores.numel() // nb
    lib = _lib.load()
    rc = lib.vggt_block_select(_ptr(scores), rows, nb, MODES[mode], int(topk or 0),
                               float(tau or 0.0), _ptr(indices), indices.shape[-1], _ptr(counts),
                               _stream(scores.device))
    _lib.check(rc)
    return indices, counts


# ---------------------------------------------------------------------------
# torch.ops.vggt_sparse.*
# ---------------------------------------------------------------------------
@torch.library.custom_op("vggt_sparse::block_sparse_attn_fwd", mutates_args=(), device_types="cuda")
def block_sparse_attn_fwd(q: torch.Tensor, patch_k: torch.Tensor, patch_v: torch.Tensor,
                          special_k: torch.Tensor, special_v: torch.Tensor, indices: torch.Tensor,
                          counts: torch.Tensor, head_ids: torch.Tensor,
                          head_dense: torch.Tensor | None, scale: float, query_block: int,
                          key_block: int, return_evidence: bool
                          ) -> tuple[torch.Tensor, torch.Tensor]:
    out = torch.empty_like(q)
    evidence = torch.full(indices.shape, -math.inf, device=q.device, dtype=torch.float32)
    launch_block_attention(q, patch_k, patch_v, special_k, special_v, indices, counts, head_ids,
                           head_dense=head_dense, query_block=query_block, key_block=key_block,
                           scale=scale, out=out, evidence=evidence if return_evidence else None)
    return out, evidence


@block_sparse_attn_fwd.register_fake
def _(q, patch_k, patch_v, special_k, special_v, indices, counts, head_ids, head_dense, scale,
      query_block, key_block, return_evidence):
    return torch.empty_like(q), indices.new_empty(indices.shape, dtype=torch.float32)


@torch.library.custom_op("vggt_sparse::block_mask_estimate", mutates_args=(), device_types="cuda")
def block_mask_estimate_op(q: torch.Tensor, k_patch: torch.Tensor, head_ids: torch.Tensor,
                           query_block: int, key_block: int, mode: str, topk: int, tau: float,
                           scale: float, export_scores: bool
                           ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    from .estimator import block_mask_estimate
    res = block_mask_estimate(q, k_patch, head_ids=head_ids, query_block=query_block,
                              key_block=key_block, mode=mode, topk=topk, tau=tau, scale=scale,
                              export_scores=export_scores)
    scores = res.scores if res.scores is not None else q.new_empty((0,), dtype=torch.float32)
    return res.indices, res.counts, scores


@block_mask_estimate_op.register_fake
def _(q, k_patch, head_ids, query_block, key_block, mode, topk, tau, scale, export_scores):
    s = head_ids.shape[0]
    qbc = math.ceil(q.shape[1] / query_block)
    nb = math.ceil(k_patch.shape[1] / key_block)
    maxk = min(topk, nb) if mode == "topk" else nb
    return (q.new_empty((s, qbc, maxk), dtype=torch.int32),
            q.new_empty((s, qbc), dtype=torch.int32),
            q.new_empty((s, qbc, nb) if export_scores else (0,), dtype=torch.float32))
