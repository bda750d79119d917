"""Block-mask estimator restatement (oracle; test infrastructure only).

Pooling, pooled scores and the two selection rules of the sparse global
attention path, in numpy.  Each function cites the reference lines it
restates.  The mass rule uses the deterministic weight arithmetic that the
CUDA kernel uses (explicitly rounded fp32 Taylor polynomial of 2^f, weights
quantised to 2^-40, threshold tau quantised to 2^-24), so that given the same
fp32 pooled scores the selected ids agree bit for bit; the reference's literal
fp32 rule (softmax -> sort -> cumsum -> count) agrees with it except where a
cumulative mass lies within fp32 rounding of tau, which the tests measure.
"""
import math

import numpy as np

F32 = np.float32
# c_k = fp32((ln 2)^k / k!), the Taylor coefficients of 2^f = exp(f ln 2)
_C = [np.frombuffer(np.uint32(h).tobytes(), dtype=np.float32)[0] for h in (
    0x3f800000, 0x3f317218, 0x3e75fdf0, 0x3d635847,
    0x3c1d955b, 0x3aaec3ff, 0x39218489, 0x377fe5fe)]
_LOG2E = np.frombuffer(np.uint32(0x3fb8aa3b).tobytes(), dtype=np.float32)[0]
MASS_FRAC_BITS = 40
TAU_BITS = 24


def block_mean(x, block):
    """Mean over consecutive row blocks; the last block uses its real size.

    Restates saf3r/patch/adaptive_block_value.py:16-23 (pad, reshape, sum,
    divide by the per-block population) for an array [..., n, d]; returns
    (means float32 [..., ceil(n/block), d], populations int64).
    """
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-2]
    count = math.ceil(n / block)
    pad = count * block - n
    widths = [(0, 0)] * (x.ndim - 2) + [(0, pad), (0, 0)]
    padded = np.pad(x, widths)
    summed = padded.reshape(*x.shape[:-2], count, block, x.shape[-1]).sum(-2, dtype=np.float32)
    population = np.full((count,), block, dtype=np.int64)
    population[-1] -= pad
    return (summed / population.astype(np.float32)[:, None]).astype(np.float32), population


def pooled_scores(pooled_q, pooled_k, scale):
    """fp32 matched-head scores Qbar . Kbar^T * scale.

    Restates saf3r/patch/coarse_sensing.py:25-31 (relevance_logits: fp32 bmm,
    no cross-head terms, no size prior) with pooled queries in place of probe
    queries.  Shapes [h, qb, d] x [h, nb, d] -> [h, qb, nb].
    """
    pq = np.asarray(pooled_q, dtype=np.float32)
    pk = np.asarray(pooled_k, dtype=np.float32)
    return (np.matmul(pq, np.swapaxes(pk, -1, -2)) * F32(scale)).astype(np.float32)


def score_keys(scores):
    """Monotone uint32 keys of fp32 scores (-0.0 and +0.0 share a key)."""
    s = np.asarray(scores, dtype=np.float32) + F32(0.0)
    b = s.view(np.uint32)
    return np.where(b & np.uint32(0x80000000), ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def _descending_order(row):
    """Ids by score descending, ties -> lower id (a stable descending sort).

    The reference ranks with ``argsort(descending=True, stable=True)``
    (saf3r/patch/adaptive_block_value.py:170) and its Triton top-k selector
    breaks ties toward the lower index (saf3r/triton/fused_qk_topk.py:73-80).
    """
    keys = score_keys(row).astype(np.int64)
    return np.argsort(-keys, kind="stable")


def select_topk(scores, k):
    """k highest blocks per row, returned as ascending ids.

    Restates the fast path of select_block_mask
    (saf3r/patch/adaptive_block_value.py:54-56:
    ``scores.topk(count).indices.sort()``) with deterministic tie-breaking.
    scores [..., nb] -> int32 [..., min(k, nb)].
    """
    s = np.asarray(scores, dtype=np.float32)
    nb = s.shape[-1]
    k = min(int(k), nb)
    flat = s.reshape(-1, nb)
    out = np.empty((flat.shape[0], k), dtype=np.int32)
    for r in range(flat.shape[0]):
        out[r] = np.sort(_descending_order(flat[r])[:k])
    return out.reshape(*s.shape[:-1], k)


def mass_weights(row, rowmax):
    """Quantised softmax weights floor(2^((s - max) log2 e) * 2^40) as uint64.

    Every operation is a separately rounded fp32 multiply or add, in the same
    order as the CUDA kernel, so both produce identical integers.
    """
    s = np.asarray(row, dtype=np.float32)
    x = (s - F32(rowmax)).astype(np.float32)
    t = (x * _LOG2E).astype(np.float32)
    live = t >= F32(-64.0)
    t = np.where(live, t, F32(0.0)).astype(np.float32)
    n = np.rint(t).astype(np.float32)
    f = (t - n).astype(np.float32)
    p = np.full_like(f, _C[7])
    for c in _C[6::-1]:
        p = ((p * f).astype(np.float32) + c).astype(np.float32)
    scale = np.ldexp(np.ones_like(p), n.astype(np.int32)).astype(np.float32)
    w = (p * scale).astype(np.float32)
    wq = (w * F32(2.0 ** MASS_FRAC_BITS)).astype(np.float32)
    q = np.floor(wq).astype(np.uint64)
    q[~live] = 0
    return q


def tau_numerator(tau):
    """tau quantised to units of 2^-24 (what the kernel receives)."""
    num = int(math.floor(float(tau) * (1 << TAU_BITS) + 0.5))
    return max(num, 1)


def mass_target(total, tau_num):
    """ceil(tau_num * total / 2^24) in exact integer arithmetic."""
    return -((-tau_num * int(total)) >> TAU_BITS)


def select_mass(scores, tau, return_counts=True):
    """Cumulative softmax-mass selection per row, ascending ids, -1 padded.

    Restates saf3r/patch/region_history_attention.py:39-42 (concentration):
    probabilities sorted descending, cumulative sum, m = #(cumsum < tau) + 1,
    clamped to the number of blocks; the m highest blocks are kept.  Softmax
    weights use the deterministic quantised arithmetic of ``mass_weights``.
    scores [..., nb] -> (ids int32 [..., nb] -1 padded, counts int32 [...]).
    """
    s = np.asarray(scores, dtype=np.float32)
    nb = s.shape[-1]
    flat = s.reshape(-1, nb)
    ids = np.full((flat.shape[0], nb), -1, dtype=np.int32)
    counts = np.empty((flat.shape[0],), dtype=np.int32)
    tau_num = tau_numerator(tau)
    for r in range(flat.shape[0]):
        row = flat[r]
        w = mass_weights(row, row.max())
        total = int(w.sum(dtype=np.uint64))
        target = mass_target(total, tau_num)
        order = _descending_order(row)
        cum = np.cumsum(w[order], dtype=np.uint64)
        m = 1 + int(np.count_nonzero(cum < np.uint64(target))) if target <= total else nb + 1
        m = min(m, nb)
        counts[r] = m
        ids[r, :m] = np.sort(order[:m])
    ids = ids.reshape(*s.shape[:-1], nb)
    counts = counts.reshape(s.shape[:-1])
    return (ids, counts) if return_counts else ids


def topk_budget(rho, n_tokens, n_special, n_blocks, key_block):
    """Blocks kept for a retention ratio rho.

    Restates saf3r/patch/adaptive_block_value.py:187:
    ``min(nb, max(1, ceil((round(rho * n) - nspecial) / key_block)))``.
    """
    return min(n_blocks, max(1, math.ceil((round(rho * n_tokens) - n_special) / key_block)))


def estimate_masks(q, k_patch, head_ids, block_q, block_k, mode, budget, scale):
    """Full estimator: pool Q and patch K, score, select.

    q [H, N, d], k_patch [H, NP, d] (float arrays); head_ids the heads to
    estimate.  mode 'topk' (budget = k) or 'mass' (budget = tau).  Returns
    (indices int32 [S, QB, max_blocks] -1 padded, counts int32 [S, QB],
    scores float32 [S, QB, NB]).
    """
    q = np.asarray(q, dtype=np.float32)
    kp = np.asarray(k_patch, dtype=np.float32)
    heads = np.asarray(head_ids, dtype=np.int64)
    pq, _ = block_mean(q[heads], block_q)
    pk, _ = block_mean(kp[heads], block_k)
    scores = pooled_scores(pq, pk, scale)
    nb = scores.shape[-1]
    if mode == "topk":
        sel = select_topk(scores, budget)
        counts = np.full(scores.shape[:-1], sel.shape[-1], dtype=np.int32)
        return sel.astype(np.int32), counts, scores
    if mode == "mass":
        ids, counts = select_mass(scores, budget)
        assert ids.shape[-1] == nb
        return ids, counts, scores
    raise ValueError(f"unknown mode {mode!r}")
