"""Query-block pairing for the tcgen05 kernel (vggt_block_attention_ex).

The GPU pair table matches a numpy restatement of the same greedy rule bit
for bit and covers every query block exactly once.  Pairing changes only
which two query blocks share a 128-row tile, so outputs and evidence are
bit-identical to the adjacent pairing."""
import math

import numpy as np
import pytest
import torch

import vggt_sparse
from vggt_sparse import ops
from vggt_sparse.synthetic import clustered_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _pair_short_selections(monkeypatch):
    """These tests run the pairing and the key-range split on small layers,
    whose short selections would otherwise take the plain launch."""
    monkeypatch.setenv("VGGT_ATTN_PAIR_MIN", "0")

WINDOW = 128


def reference_pairs(ids, counts, nb):
    """Greedy pairing restated: blocks in order; an unpaired block a takes the
    unpaired block c in (a, a + WINDOW] minimising popcount(bm[a] ^ bm[c])
    (clamped to 0xfffe; ties -> smallest c); blocks without a candidate pair
    with each other in order, the last alone when their number is odd."""
    S, QB, _ = ids.shape
    out = np.full((S, (QB + 1) // 2, 2), -1, np.int32)
    for s in range(S):
        bm = np.zeros((QB, nb), bool)
        for q in range(QB):
            c = int(counts[s, q] if counts.ndim == 2 else counts[s])
            row = ids[s, q, :c]
            bm[q, row[(row >= 0) & (row < nb)]] = True
        taken = np.zeros(QB, bool)
        pairs, singles = [], []
        for a in range(QB):
            if taken[a]:
                continue
            taken[a] = True
            cand = np.arange(a + 1, min(QB, a + WINDOW + 1))
            cand = cand[~taken[cand]]
            if len(cand):
                cost = np.minimum((bm[cand] ^ bm[a]).sum(1), 0xfffe)
                b = int(cand[np.argmin(cost)])
                taken[b] = True
                pairs.append((a, b))
            else:
                singles.append(a)
        for i in range(0, len(singles), 2):
            pairs.append((singles[i], singles[i + 1] if i + 1 < len(singles) else -1))
        out[s] = np.asarray(pairs, np.int32)
    return out


def _layer_masks(cuda, frames, mode, dense_heads=(), seed=3):
    x = clustered_layer(frames, centres=64, seed=seed, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode=mode, retention=0.25, tau=0.9,
                                          dense_heads=dense_heads, kernel="mma_sync")
    layer(x.q, x.kp, x.vp, x.ks, x.vs)
    idx, cnt = layer.last_masks
    buf = layer._cache[next(iter(layer._cache))]
    return x, idx, cnt, buf


def _run(x, idx, cnt, buf, *, pair, evidence=False):
    out = torch.zeros_like(x.q)
    ev = torch.full(idx.shape, -math.inf, device=idx.device) if evidence else None
    ws = None
    if pair:
        nbytes = ops.attention_workspace_size(x.shape.n_tokens, x.shape.n_patch,
                                              buf["slot_ids"].numel())
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=x.q.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.q.device)
    ops.launch_block_attention(x.q, x.kp, x.vp, x.ks, x.vs, idx, cnt, buf["slot_ids"],
                               head_dense=buf["dense_flags"], out=out, evidence=ev,
                               status=status, kernel="tcgen05", pair_qblocks=pair, workspace=ws)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, ev, ws


@pytest.mark.parametrize("mode", ["topk", "mass"])
def test_pair_table_matches_restatement_and_covers_every_block(cuda, mode):
    x, idx, cnt, buf = _layer_masks(cuda, 8, mode, dense_heads=(0, 5))
    _, _, ws = _run(x, idx, cnt, buf, pair=True)
    s_idx, qb = idx.shape[0], idx.shape[1]
    npairs = (qb + 1) // 2
    table = ws[: s_idx * npairs * 2 * 4].view(torch.int32).view(s_idx, npairs, 2).cpu().numpy()
    want = reference_pairs(idx.cpu().numpy(), cnt.cpu().numpy(), x.shape.n_blocks)
    np.testing.assert_array_equal(table, want)
    for s in range(s_idx):
        ids = table[s].reshape(-1)
        assert sorted(ids[ids >= 0].tolist()) == list(range(qb))
        assert (ids < 0).sum() == 2 * npairs - qb


@pytest.mark.parametrize("mode", ["topk", "mass"])
@pytest.mark.parametrize("evidence", [False, True])
def test_pairing_leaves_outputs_bit_identical(cuda, mode, evidence, monkeypatch):
    monkeypatch.setenv("VGGT_ATTN_SPLIT", "1")  # no key-range split: same summation order
    x, idx, cnt, buf = _layer_masks(cuda, 8, mode, dense_heads=(0, 5))
    out0, ev0, _ = _run(x, idx, cnt, buf, pair=False, evidence=evidence)
    out1, ev1, _ = _run(x, idx, cnt, buf, pair=True, evidence=evidence)
    assert torch.equal(out0, out1)
    if evidence:
        assert torch.equal(ev0, ev1)


def test_pairing_reduces_union_tiles(cuda):
    """On clustered inputs the chosen pairs share more of their selections
    than adjacent blocks do (fewer tiles in the unions)."""
    x, idx, cnt, buf = _layer_masks(cuda, 8, "topk")
    _, _, ws = _run(x, idx, cnt, buf, pair=True)
    s_idx, qb, _ = idx.shape
    npairs = (qb + 1) // 2
    table = ws[: s_idx * npairs * 2 * 4].view(torch.int32).view(s_idx, npairs, 2).cpu().numpy()
    ids, c = idx.cpu().numpy(), cnt.cpu().numpy()
    sets = [[set(ids[s, q, :c[s, q]].tolist()) for q in range(qb)] for s in range(s_idx)]

    def union_tiles(pairs):
        return sum(len(sets[s][a] | (sets[s][b] if b >= 0 else set()))
                   for s in range(s_idx) for a, b in pairs[s])
    adjacent = [[(2 * p, 2 * p + 1 if 2 * p + 1 < qb else -1) for p in range(npairs)]
                for _ in range(s_idx)]
    assert union_tiles(table) < union_tiles(adjacent)


def test_layer_uses_pairing_by_default(cuda, monkeypatch):
    monkeypatch.setenv("VGGT_ATTN_SPLIT", "1")
    x = clustered_layer(4, centres=64, seed=1, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode="topk", retention=0.25, kernel="tcgen05")
    a = layer(x.q, x.kp, x.vp, x.ks, x.vs).clone()
    assert layer.pair_qblocks
    assert layer._cache[next(iter(layer._cache))]["attn_ws"] is not None
    layer.pair_qblocks = False
    b = layer(x.q, x.kp, x.vp, x.ks, x.vs)
    assert torch.equal(a, b)


def test_work_order_is_a_longest_first_permutation(cuda):
    """The schedule lists every (slot, pair) item once: slots from the last
    (dense) to the first, each slot's pairs by non-increasing union size."""
    x, idx, cnt, buf = _layer_masks(cuda, 8, "mass", dense_heads=(0, 5))
    _, _, ws = _run(x, idx, cnt, buf, pair=True)
    n_slots = buf["slot_ids"].numel()
    s_idx, qb, _ = idx.shape
    npairs = (qb + 1) // 2
    up = lambda b: (b + 255) // 256 * 256
    off = up(n_slots * npairs * 2 * 4)
    order = ws[off: off + n_slots * npairs * 4].view(torch.int32).cpu().numpy()
    assert sorted(order.tolist()) == list(range(n_slots * npairs))
    table = ws[: s_idx * npairs * 2 * 4].view(torch.int32).view(s_idx, npairs, 2).cpu().numpy()
    ids, c = idx.cpu().numpy(), cnt.cpu().numpy()
    nb = x.shape.n_blocks

    def size(item):
        slot, p = divmod(int(item), npairs)
        if slot >= s_idx:
            return nb
        a, b = table[slot, p]
        sa = set(ids[slot, a, :c[slot, a]].tolist())
        sb = set(ids[slot, b, :c[slot, b]].tolist()) if b >= 0 else set()
        return len(sa | sb)
    slots = order // npairs
    assert np.all(np.diff(slots) <= 0)
    for slot in range(n_slots):
        items = order[slots == slot]
        buckets = np.array([size(i) for i in items]) * 1023 // nb
        assert np.all(np.diff(buckets) <= 0), slot


def test_short_selections_take_the_plain_launch(cuda, monkeypatch):
    """With the default threshold (64 selected blocks per query block), a
    4-frame top-k 25 % call with a workspace runs exactly the plain launch:
    no pairing and no key-range split, so the output equals the plain call's
    bit for bit (the 4-way split the grid size would pick sums differently)."""
    monkeypatch.delenv("VGGT_ATTN_PAIR_MIN", raising=False)
    monkeypatch.delenv("VGGT_ATTN_SPLIT", raising=False)
    x = clustered_layer(4, centres=64, seed=2, device=cuda)
    heads = torch.arange(16, device=cuda, dtype=torch.int32)
    k = vggt_sparse.topk_budget(0.25, x.shape.n_tokens, x.shape.n_special, x.shape.n_blocks, 64)
    assert k < 64
    res = vggt_sparse.block_mask_estimate(x.q, x.kp, head_ids=heads, mode="topk", topk=k)
    outs = []
    for pair in (True, False):
        out = torch.empty_like(x.q)
        vggt_sparse.ops.launch_block_attention(x.q, x.kp, x.vp, x.ks, x.vs, res.indices,
                                               res.counts, heads, out=out, kernel="tcgen05",
                                               pair_qblocks=pair)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
