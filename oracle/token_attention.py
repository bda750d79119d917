"""CPU restatement of the reference's per-token sparse attention (test
infrastructure only: the checker for the CUDA path, never called by it).

saf3r/triton/sparse_topk_attention.py:115-166 (fused_sparse_topk_attention)
and :261-286 (its online-softmax variant for large top-k): every query n
attends to the keys kv_indices[n, :] (duplicates count twice) with an fp32
softmax of q_n . k_j * scale, accumulated in fp32.  Index entries outside
[0, n_keys) are skipped here (the reference reads them unchecked); the CUDA
path skips them too and reports them in its status word.
"""
import numpy as np


def token_sparse_attention(q, k, v, kv_indices, scale=None):
    """q [N, D], k [Nk, D], v [Nk, Dv], kv_indices [N, TopK] -> [N, Dv] fp32."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    idx = np.asarray(kv_indices, dtype=np.int64)
    n, d = q.shape
    scale = d ** -0.5 if scale is None else float(scale)
    out = np.zeros((n, v.shape[1]), dtype=np.float32)
    for r in range(n):
        ids = idx[r]
        ids = ids[(ids >= 0) & (ids < k.shape[0])]
        if ids.size == 0:
            continue
        s = k[ids] @ q[r] * scale
        p = np.exp(s - s.max())
        out[r] = (p @ v[ids] / p.sum()).astype(np.float32)
    return out
