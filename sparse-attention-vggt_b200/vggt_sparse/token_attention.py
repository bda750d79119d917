"""Per-token sparse attention (vggt_token_sparse_attention).

``token_sparse_attention`` keeps the signature and return value of the
reference's saf3r/triton/sparse_topk_attention.py fused_sparse_topk_attention
(and fused_sparse_topk_attention_2): q [N, D], k [Nk, D], v [Nk, D],
kv_indices [N, TopK] -> out [N, D] in v's dtype.  CUDA tensors only.
"""
import torch

from . import _lib
from .ops import _ptr, _require_cuda, _stream, dtype_code


def token_sparse_attention(q, k, v, kv_indices, scale=None, *, out=None, status=None):
    if q.dim() != 2 or k.dim() != 2 or v.dim() != 2 or kv_indices.dim() != 2:
        raise ValueError("q [N, D], k [Nk, D], v [Nk, D] and kv_indices [N, TopK] expected")
    n, d = q.shape
    if k.shape[1] != d or v.shape != k.shape:
        raise ValueError("k and v must be [Nk, %d]" % d)
    if kv_indices.shape[0] != n:
        raise ValueError("kv_indices needs one row per query")
    code = dtype_code(q.dtype)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must share a dtype")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    idx = kv_indices
    if idx.dtype != torch.int32:
        idx = idx.to(torch.int32)
    # a row-broadcast view (stride 0 on the query dim) stays shared; other
    # layouts are made contiguous
    if idx.stride(1) != 1 or (idx.stride(0) not in (0, idx.shape[1])):
        idx = idx.contiguous()
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        # the kernel writes N * D elements of q's dtype, row by row, from out's first byte
        raise ValueError("out must be a contiguous %s tensor of shape %s"
                         % (q.dtype, tuple(q.shape)))
    if status is not None and (status.dtype != torch.int32 or status.numel() < 1):
        raise ValueError("status must be an int32 tensor with at least one element")
    _require_cuda(q, k, v, kv_indices, out, status)
    scale = d ** -0.5 if scale is None else float(scale)
    lib = _lib.load()
    rc = lib.vggt_token_sparse_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(idx), idx.stride(0), n,
                                         k.shape[0], idx.shape[1], d, code, scale, _ptr(out),
                                         _ptr(status), _stream(q.device))
    _lib.check(rc)
    return out
