"""Per-frame QK top-k (vggt_frame_qk_topk).

``compute_qk_topk_indices_fused`` keeps the signature and return value of
the reference's saf3r/triton/fused_qk_topk.py:128-217: q (B, Nq, D), k
(B, Nk, D), topk per frame, num_toks_per_img tokens per frame -> (B, Nq,
num_imgs * min(topk, num_toks_per_img)) int32 global key indices, frame-major,
each frame's entries in descending score order (ties to the lower index).
Its asserts are kept (AssertionError on the same conditions).  Differences:
CUDA tensors only (the reference answers CPU tensors with a PyTorch path),
and no timing printout.
"""
import torch
import torch.nn.functional as F

from . import _lib
from .ops import _ptr, _require_cuda, _stream


def compute_qk_topk_indices_fused(q, k, topk, num_toks_per_img=None, *, groups=0, status=None):
    assert num_toks_per_img is not None and num_toks_per_img > 0
    assert q.dim() == 3 and k.dim() == 3 and q.shape[0] == k.shape[0] and q.shape[2] == k.shape[2]
    assert k.shape[1] % num_toks_per_img == 0, "Nk must be divisible by num_toks_per_img"
    _require_cuda(q, k, status)
    b, nq, d = q.shape
    assert d <= 128, "this fused impl targets D <= 128 (per-head)"
    n = int(num_toks_per_img)
    frames = k.shape[1] // n
    topk_eff = min(int(topk), n)
    assert topk_eff <= 128, "this impl supports per-frame topk up to 128"
    # the reference computes in bf16 whatever the input dtype
    qb = q.to(torch.bfloat16).contiguous()
    kb = k.to(torch.bfloat16).contiguous()
    dp = 64 if d <= 64 else 128
    if dp != d:  # zero columns add nothing to a dot product
        qb = F.pad(qb, (0, dp - d))
        kb = F.pad(kb, (0, dp - d))
    out = torch.empty((b, nq, frames * topk_eff), dtype=torch.int32, device=q.device)
    if topk_eff <= 0 or out.numel() == 0:
        return out
    lib = _lib.load()
    rc = lib.vggt_frame_qk_topk(_ptr(qb), _ptr(kb), _ptr(out), b, nq, frames, n, dp, topk_eff,
                                int(groups), _ptr(status), _stream(q.device))
    _lib.check(rc)
    return out
