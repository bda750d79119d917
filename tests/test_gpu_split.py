"""Key-range splitting of the tcgen05 work items (small grids, e.g. one rank's
query-block shard): each 128-row item's tiles run on 2-4 CTAs and a second
launch merges the partial results.  Outputs agree with the unsplit kernel to
rounding and with the fp32 oracle at the parity tolerance; evidence (one value
per tile) at 1e-4."""
import numpy as np
import pytest
import torch

import oracle
import vggt_sparse
from vggt_sparse import ops
from vggt_sparse.synthetic import clustered_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _pair_short_selections(monkeypatch):
    """These tests run the pairing and the key-range split on small layers,
    whose short selections would otherwise take the plain launch."""
    monkeypatch.setenv("VGGT_ATTN_PAIR_MIN", "0")


def _run(x, idx, cnt, buf, evidence):
    out = torch.zeros_like(x.q)
    ev = torch.full(idx.shape, -float("inf"), device=x.q.device) if evidence else None
    status = torch.zeros(1, dtype=torch.int32, device=x.q.device)
    ops.launch_block_attention(x.q, x.kp, x.vp, x.ks, x.vs, idx, cnt, buf["slot_ids"],
                               head_dense=buf["dense_flags"], out=out, evidence=ev,
                               status=status, kernel="tcgen05")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, ev


@pytest.mark.parametrize("mode,dense", [("topk", ()), ("mass", (0, 5))])
def test_split_matches_unsplit(cuda, mode, dense, monkeypatch):
    x = clustered_layer(8, centres=64, seed=5, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode=mode, retention=0.25, tau=0.9,
                                          dense_heads=dense, kernel="mma_sync")
    layer(x.q, x.kp, x.vp, x.ks, x.vs)
    idx, cnt = layer.last_masks
    buf = layer._cache[next(iter(layer._cache))]
    results = {}
    for split in ("1", "2", "3", "4"):
        monkeypatch.setenv("VGGT_ATTN_SPLIT", split)
        results[split] = _run(x, idx, cnt, buf, evidence=True)
    base_out, base_ev = results["1"]
    fin = torch.isfinite(base_ev)
    for split in ("2", "3", "4"):
        out, ev = results[split]
        d = (out.float() - base_out.float()).abs()
        assert d.max().item() <= 2e-2 and d.mean().item() <= 1e-3, split
        assert torch.equal(torch.isfinite(ev), fin)
        torch.testing.assert_close(ev[fin], base_ev[fin], rtol=1e-4, atol=1e-4)


def test_split_against_oracle_with_tails(cuda, monkeypatch):
    """Tail query and key blocks, 7 specials, a head with an empty selection
    in some rows: the split path against the fp32 oracle."""
    monkeypatch.setenv("VGGT_ATTN_SPLIT", "4")
    torch.manual_seed(3)
    h, n, d = 3, 300, 64
    npatch, nspec = 250, 7
    q = torch.randn(h, n, d).to(torch.bfloat16)
    kp = torch.randn(h, npatch, d).to(torch.bfloat16)
    vp = torch.randn_like(kp)
    ks = torch.randn(h, nspec, d).to(torch.bfloat16)
    vs = torch.randn_like(ks)
    qb, nb = 5, 4
    idx = torch.full((2, qb, 3), -1, dtype=torch.int32)
    cnt = torch.zeros((2, qb), dtype=torch.int32)
    rng = np.random.default_rng(1)
    for s in range(2):
        for b in range(qb):
            c = int(rng.integers(0, 4)) if s == 1 else 3
            sel = np.sort(rng.permutation(nb)[:c])
            idx[s, b, :c] = torch.tensor(sel, dtype=torch.int32)
            cnt[s, b] = c
    heads = torch.tensor([0, 2], dtype=torch.int32)
    args = [t.to(cuda) for t in (q, kp, vp, ks, vs, idx, cnt, heads)]
    out, _ = vggt_sparse.block_attention(*args, return_evidence=False, kernel="tcgen05")
    want, _ = oracle.block_sparse_attention(q.float().numpy(), kp.float().numpy(),
                                            vp.float().numpy(), ks.float().numpy(),
                                            vs.float().numpy(), idx.numpy(), cnt.numpy(),
                                            heads.numpy())
    for head in heads.tolist():
        a = out[head].float().cpu().numpy()
        e = want[head]
        np.testing.assert_allclose(a, e, rtol=0.02, atol=0.006)
        assert np.abs(a - e).max() <= 2e-2
