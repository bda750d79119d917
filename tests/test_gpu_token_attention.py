"""Per-token sparse attention (vggt_token_sparse_attention) against the fp32
oracle restatement of saf3r/triton/sparse_topk_attention.py, at the parity
tolerance of the block-sparse tests (rtol .02 / atol .006, max-abs 2e-2)."""
import numpy as np
import pytest
import torch

import oracle
import vggt_sparse

pytestmark = pytest.mark.gpu


def _check(got, want):
    a = got.float().cpu().numpy()
    np.testing.assert_allclose(a, want, rtol=0.02, atol=0.006)
    assert np.abs(a - want).max() <= 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dim", [32, 64, 128])
@pytest.mark.parametrize("topk", [1, 7, 64, 300, 2500])
def test_matches_oracle(cuda, dtype, dim, topk):
    g = torch.Generator().manual_seed(dim * 7 + topk)
    n, nk = 97, 3000
    q = torch.randn(n, dim, generator=g).to(dtype)
    k = torch.randn(nk, dim, generator=g).to(dtype)
    v = torch.randn(nk, dim, generator=g).to(dtype)
    idx = torch.randint(0, nk, (n, topk), generator=g, dtype=torch.int32)  # duplicates allowed
    out = vggt_sparse.token_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), idx.to(cuda))
    want = oracle.token_sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                         idx.numpy())
    _check(out, want)


def test_shared_index_row_and_scale(cuda):
    """A stride-zero expanded index view (one list for every query), as the
    reference passes for a uniform pattern; an explicit scale."""
    g = torch.Generator().manual_seed(3)
    n, nk, topk = 200, 800, 129
    q, k, v = (torch.randn(r, 64, generator=g).to(torch.bfloat16) for r in (n, nk, nk))
    row = torch.randperm(nk, generator=g)[:topk].to(torch.int32)
    idx = row[None].expand(n, topk)
    out = vggt_sparse.token_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda),
                                             idx.to(cuda), scale=0.2)
    want = oracle.token_sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                         idx.numpy(), scale=0.2)
    _check(out, want)


def test_invalid_entries_are_skipped_and_reported(cuda):
    g = torch.Generator().manual_seed(4)
    n, nk, topk = 40, 100, 50
    q, k, v = (torch.randn(r, 64, generator=g).to(torch.bfloat16) for r in (n, nk, nk))
    idx = torch.randint(0, nk, (n, topk), generator=g, dtype=torch.int32)
    idx[::3, ::4] = -1
    idx[1, 5] = nk + 7
    idx[2, :] = -1                       # a query with no valid key -> zeros
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = vggt_sparse.token_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), idx.to(cuda),
                                             status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    want = oracle.token_sparse_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                         idx.numpy())
    _check(out, want)
    assert (out[2] == 0).all()
