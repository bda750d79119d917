"""CPU restatement of the reference's per-frame QK top-k (test infrastructure
only: the checker for the CUDA path, never called by it).

saf3r/triton/fused_qk_topk.py:128-217 (compute_qk_topk_indices_fused) with
its kernel :24-108: scores s = q . k in fp32 (no scale); keys split into
frames of `tokens` consecutive keys; per (query, frame) the min(topk, tokens)
keys with the largest composite (sortable 32-bit key of s, then the lower key
index), in descending order (bitonic merge, :84-93); returned as global key
indices, frame-major.  The sortable key is topk_utils.py:24-28
(fpval_to_key): bits ^ 0xffffffff for a set sign bit, else bits ^ 0x80000000.

The reference accumulates on the tensor cores; here the scores are the
float64 dot products of the bf16 values rounded once to fp32.  The two agree
exactly when every partial sum is representable (small-integer inputs), and
otherwise within fp32 rounding, which can swap near-tied keys.
"""
import numpy as np


def score_keys32(s):
    """fpval_to_key on fp32 values -> uint32 sortable keys (-0 below +0)."""
    bits = np.ascontiguousarray(s, dtype=np.float32).view(np.uint32)
    neg = (bits >> np.uint32(31)).astype(bool)
    return np.where(neg, bits ^ np.uint32(0xFFFFFFFF), bits ^ np.uint32(0x80000000))


def frame_scores(q, k):
    """(B, Nq, D) x (B, Nk, D) -> (B, Nq, Nk) fp32 scores."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    return np.einsum("bqd,bkd->bqk", q, k).astype(np.float32)


def qk_topk_per_frame(q, k, topk, tokens_per_frame, scores=None):
    """-> (B, Nq, F * min(topk, tokens)) int32 global key indices."""
    s = frame_scores(q, k) if scores is None else np.asarray(scores, dtype=np.float32)
    b, nq, nk = s.shape
    n = int(tokens_per_frame)
    assert nk % n == 0
    frames = nk // n
    te = min(int(topk), n)
    keys = score_keys32(s).reshape(b, nq, frames, n).astype(np.int64)
    # descending key, ascending index: a stable sort of the negated keys
    order = np.argsort(-keys, axis=-1, kind="stable")[..., :te]
    base = (np.arange(frames, dtype=np.int64) * n)[None, None, :, None]
    return (order + base).reshape(b, nq, frames * te).astype(np.int32)
