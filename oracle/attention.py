"""Block-sparse attention restatement (oracle; test infrastructure only).

Computes, in float64, the exact softmax attention of each query block over
its selected patch key blocks plus every special key, and the same-pass
evidence (mean over valid query rows of the per-block row log-sum-exp).

Restates the reference CPU branch saf3r/patch/adaptive_block_value.py:371-385
and the known-answer formula of tests/test_adaptive_block_value.py:172-184,
which define what the Triton kernel saf3r/triton/adaptive_block_attention.py:7-60
computes.
"""
import math

import numpy as np


def _lse(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    return (m + np.log(np.sum(np.exp(x - m), axis=axis, keepdims=True))).squeeze(axis)


def block_sparse_attention(q, patch_k, patch_v, special_k, special_v, indices, counts, head_ids,
                           *, query_block=64, key_block=64, scale=None, head_dense=None,
                           qblocks=None):
    """Reference output and evidence of the block-sparse operator.

    q [H, N, d]; patch_k/v [H, NP, d]; special_k/v [H, NS, d];
    indices [S, QB, maxK]; counts [S] or [S, QB]; head_ids [S];
    head_dense [S] bool (a dense slot attends to all patch blocks).
    qblocks: optional iterable of query-block ids to evaluate (others stay NaN).

    Returns (out float32 [H, N, d] with NaN in rows not produced,
    evidence float32 [S, QB, maxK] with -inf in unused slots).
    """
    q = np.asarray(q, dtype=np.float64)
    pk = np.asarray(patch_k, dtype=np.float64)
    pv = np.asarray(patch_v, dtype=np.float64)
    sk = np.asarray(special_k, dtype=np.float64)
    sv = np.asarray(special_v, dtype=np.float64)
    indices = np.asarray(indices)
    counts = np.asarray(counts)
    h, n, d = q.shape
    npatch = pk.shape[1]
    scale = d ** -0.5 if scale is None else float(scale)
    qbc = math.ceil(n / query_block)
    nb = math.ceil(npatch / key_block)
    out = np.full(q.shape, np.nan, dtype=np.float32)
    evidence = np.full(indices.shape, -np.inf, dtype=np.float32)
    blocks = range(qbc) if qblocks is None else qblocks
    for slot, head in enumerate(np.asarray(head_ids).tolist()):
        dense = bool(head_dense[slot]) if head_dense is not None else False
        for block in blocks:
            qr = slice(block * query_block, min((block + 1) * query_block, n))
            if dense:
                ids = np.arange(nb)
            else:
                count = int(counts[slot, block]) if counts.ndim == 2 else int(counts[slot])
                ids = indices[slot, block, :count].astype(np.int64)
            ix = (ids[:, None] * key_block + np.arange(key_block)).reshape(-1)
            ix = ix[ix < npatch]
            logits_p = q[head, qr] @ pk[head, ix].T * scale
            if not dense:
                for j, bid in enumerate(ids):
                    span = (ix // key_block) == bid
                    evidence[slot, block, j] = _lse(logits_p[:, span]).mean()
            keys = np.concatenate((pk[head, ix], sk[head]))
            values = np.concatenate((pv[head, ix], sv[head]))
            logits = q[head, qr] @ keys.T * scale
            p = np.exp(logits - logits.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            out[head, qr] = (p @ values).astype(np.float32)
    return out, evidence


def dense_attention(q, k, v, scale=None, rows=None):
    """Exact dense softmax attention per head (the SDPA dense-head path,
    saf3r/patch/adaptive_block_value.py:399-404).  q [H, N, d], k/v [H, M, d].
    rows: optional index array of query rows to evaluate."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if rows is not None:
        q = q[:, rows]
    logits = np.einsum("hnd,hmd->hnm", q, k) * scale
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.einsum("hnm,hmd->hnd", p, v).astype(np.float32)
