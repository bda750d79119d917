"""The reference's CPU PyTorch path for one sparse global layer, restated in
torch (fp32, CPU) — the timed CPU baseline of bench.py (test infrastructure;
never part of the product).

Follows the CPU branch of AdaptiveBlockValueAttention.forward:
  pooling     saf3r/patch/adaptive_block_value.py:16-23 (block_mean on K; here
              also on Q, as the mean-Q estimator prescribes)
  scores      saf3r/patch/coarse_sensing.py:25-31 (fp32 bmm * scale)
  selection   top-k: adaptive_block_value.py:54-56 (topk + sort);
              mass: region_history_attention.py:39-42 (softmax, sort, cumsum)
  attention   adaptive_block_value.py:371-385: per (head, query block) gather
              the selected patch rows, concatenate the specials, one SDPA call
  dense heads adaptive_block_value.py:399-404 (SDPA over all keys)
"""
import math

import torch
import torch.nn.functional as F


def block_mean(x, block):
    n = x.shape[-2]
    count = math.ceil(n / block)
    pad = count * block - n
    result = F.pad(x, (0, 0, 0, pad)).reshape(*x.shape[:-2], count, block, x.shape[-1]).sum(-2)
    populations = torch.full((count,), block, dtype=torch.long)
    populations[-1] -= pad
    return result / populations.to(result.dtype)[..., None]


def estimate(q, kp, mode, budget, scale, block=64, qblocks=None):
    """Masks [H, len(qblocks), maxK] (-1 padded) and counts [H, len(qblocks)]."""
    pq = block_mean(q.float(), block)
    pk = block_mean(kp.float(), block)
    if qblocks is not None:
        pq = pq[:, qblocks]
    scores = torch.bmm(pq, pk.transpose(1, 2)) * scale
    nb = scores.shape[-1]
    if mode == "topk":
        k = min(int(budget), nb)
        ids = scores.topk(k, dim=-1).indices.sort(dim=-1).values
        return ids, torch.full(scores.shape[:-1], k, dtype=torch.long)
    p = scores.softmax(-1)
    srt = p.sort(-1, descending=True)
    m = ((srt.values.cumsum(-1) < budget).sum(-1) + 1).clamp_max(nb)
    ids = torch.full(scores.shape, -1, dtype=torch.long)
    for h in range(scores.shape[0]):
        for r in range(scores.shape[1]):
            c = int(m[h, r])
            ids[h, r, :c] = srt.indices[h, r, :c].sort().values
    return ids, m


def sparse_layer(q, kp, vp, ks, vs, ids, counts, sparse_heads, dense_heads, qblocks, scale,
                 block=64, k_full=None, v_full=None):
    """Attention output rows of the sampled query blocks, [H, rows, d].

    Dense heads attend over the layer's full k/v [H, N, d], which the
    reference's dense branch reads as they are (``k_full``/``v_full``); when
    they are not given, patch and special keys are concatenated here."""
    h, n, d = q.shape
    npatch = kp.shape[1]
    rows = [torch.arange(b * block, min((b + 1) * block, n)) for b in qblocks]
    out = torch.empty((h, sum(len(r) for r in rows), d))
    k_all = v_all = None
    if dense_heads:
        hh = torch.tensor(dense_heads)
        if k_full is not None and v_full is not None:
            k_all, v_all = k_full[hh].float(), v_full[hh].float()
        else:
            k_all = torch.cat((kp[hh], ks[hh]), 1).float()
            v_all = torch.cat((vp[hh], vs[hh]), 1).float()
    for head in sparse_heads:
        off = 0
        for j, b in enumerate(qblocks):
            qr = rows[j]
            sel = ids[head, j, :int(counts[head, j])]
            ix = (sel[:, None] * block + torch.arange(block)).flatten()
            ix = ix[ix < npatch]
            keys = torch.cat((kp[head, ix], ks[head])).float()
            values = torch.cat((vp[head, ix], vs[head])).float()
            out[head, off:off + len(qr)] = F.scaled_dot_product_attention(
                q[head, qr].float(), keys, values, scale=scale)
            off += len(qr)
    if dense_heads:
        qr = torch.cat(rows)
        out[hh] = F.scaled_dot_product_attention(q[hh][:, qr].float()[None], k_all[None],
                                                 v_all[None], scale=scale)[0]
    return out


def layer_sample(q, kp, vp, ks, vs, *, mode, budget, dense_heads, qblocks, scale, block=64,
                 k_full=None, v_full=None):
    """Estimator (pooling over the full layer, scores/selection for the
    sampled query blocks) + attention for the sampled query blocks."""
    h = q.shape[0]
    sparse = [x for x in range(h) if x not in set(dense_heads)]
    ids, counts = estimate(q, kp, mode, budget, scale, block, qblocks)
    return sparse_layer(q, kp, vp, ks, vs, ids, counts, sparse, list(dense_heads), qblocks,
                        scale, block, k_full=k_full, v_full=v_full)
