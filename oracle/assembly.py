"""CPU restatement of the reference's mask assembly with history and value
order, and of its same-pass history update (test infrastructure only: the
checker for the CUDA path, never called by it).

* ``select_block_mask`` follows saf3r/patch/adaptive_block_value.py:42-91:
  at most half of the attention slots reuse history blocks that still rank in
  the top 2A of the current scores, the rest take the current top scores, and
  the remaining count - A slots are filled in value order with uncovered
  blocks.  Returns ascending ids and the origin code (1 reused, 2 attention,
  0 value fill).
* ``history_update`` follows :389-396: per row, the ``keep`` selected blocks
  with the largest same-pass evidence.

Ties: the reference uses torch.topk, whose order among equal values is not
specified.  Here every ranking breaks ties to the lower index (block id, or
history position), the rule the device path implements; on tie-free inputs
both agree with the reference, which the golden vectors pin.
"""
import numpy as np


def _top_set(values, k):
    """Indices of the k largest values, ties to the lower index."""
    values = np.asarray(values)
    k = int(max(0, min(k, values.shape[0])))
    if k == 0:
        return np.zeros(0, dtype=np.int64)
    order = np.lexsort((np.arange(values.shape[0]), -values.astype(np.float64)))
    return order[:k]


def select_block_mask(scores, value_order, count, attention_count, history=None):
    """scores [rows, blocks] fp32; value_order [blocks]; history [rows, H] or None.
    Returns (ids [rows, count] int64 ascending, origin [rows, count] uint8)."""
    scores = np.asarray(scores, dtype=np.float32)
    rows, blocks = scores.shape
    vo = np.asarray(value_order, dtype=np.int64)
    a_cnt = min(count, max(0, attention_count))
    ids = np.zeros((rows, count), dtype=np.int64)
    origin = np.zeros((rows, count), dtype=np.uint8)
    for r in range(rows):
        s = scores[r]
        a = np.zeros(blocks, bool)
        reused = np.zeros(blocks, bool)
        if a_cnt:
            if history is not None and history.shape[-1] and a_cnt >= 2:
                eligible = min(blocks, 2 * a_cnt)
                cutoff = s[_top_set(s, eligible)[-1]]
                h = np.asarray(history[r], dtype=np.int64)
                valid = h >= 0
                old = np.where(valid, s[np.clip(h, 0, None)], -np.inf).astype(np.float32)
                take = min(a_cnt // 2, h.shape[0])
                for j in _top_set(old, take):
                    if valid[j] and old[j] >= cutoff:
                        reused[h[j]] = True
                a |= reused
            remaining = a_cnt - int(a.sum())
            masked = np.where(a, -np.inf, s).astype(np.float32)
            a[_top_set(masked, remaining)] = True
        fill = np.zeros(blocks, bool)
        quota = count - a_cnt
        for blk in vo:
            if quota <= 0:
                break
            if not a[blk]:
                fill[blk] = True
                quota -= 1
        sel = np.nonzero(a | fill)[0][:count]
        ids[r, :len(sel)] = sel
        origin[r, :len(sel)] = np.where(reused[sel], 1, np.where(a[sel], 2, 0))
    return ids, origin


def history_update(evidence, ids, count, keep):
    """evidence [rows, >= count] fp32, ids [rows, >= count]: the ids of the
    ``keep`` largest evidence values among the first ``count`` slots, in
    ascending id order (the reference keeps them in evidence order; the set is
    what later layers use)."""
    evidence = np.asarray(evidence, dtype=np.float32)
    out = np.zeros((evidence.shape[0], keep), dtype=np.int64)
    for r in range(evidence.shape[0]):
        win = _top_set(evidence[r, :count], keep)
        out[r] = np.sort(np.asarray(ids[r])[win])
    return out
